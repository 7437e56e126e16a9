// Host side of the C ABI declared in include/mockbird_kv.h: context lifetime,
// argument validation, staging for the host-array entry points, and launches.
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "mb_internal.cuh"

using namespace mb;

#define MB_VERSION "mockbird-b200 0.1.0 (sm_100a)"

namespace {

int fail(mb_ctx* c, int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (c) c->last_error = buf;
    return code;
}

int cuda_fail(mb_ctx* c, cudaError_t e, const char* what) {
    return fail(c, e == cudaErrorMemoryAllocation ? MB_ERR_OOM : MB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define CK(call, what)                                        \
    do {                                                      \
        cudaError_t e_ = (call);                              \
        if (e_ != cudaSuccess) return cuda_fail(c, e_, what); \
    } while (0)

// Switch to the context's device for the duration of a call.
struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int check_layer(mb_ctx* c, int layer) {
    if (layer < 0 || layer >= c->cfg.layers)
        return fail(c, MB_ERR_LAYER, "layer %d out of range [0, %d)", layer, c->cfg.layers);
    return MB_OK;
}

int check_batch(mb_ctx* c, int n) {
    if (n < 0 || n > c->cfg.max_batch)
        return fail(c, MB_ERR_ARG, "item count %d out of range [0, %d] (max_batch)", n, c->cfg.max_batch);
    return MB_OK;
}

// Host-side checks of one position (decode.ts:719-724 for the non-wrapping ring).
int check_position(mb_ctx* c, int pos) {
    if (pos < 0 || pos >= c->cfg.max_position)
        return fail(c, MB_ERR_POSITION, "position %d out of range [0, %d)", pos, c->cfg.max_position);
    if (!c->cfg.wrap && pos >= c->cfg.capacity)
        return fail(c, MB_ERR_CAPACITY,
                    "decode position %d exceeds the KV ring (%d slots); it must be sized prefill_rows + "
                    "max_new_frames",
                    pos, c->cfg.capacity);
    return MB_OK;
}

}  // namespace

// Host-side checks of the items of a host-array call: stream range, no stream
// twice, positions (decode.ts:719-724 for the non-wrapping ring).
int mb::check_items_host(mb_ctx* c, int n, const int32_t* streams, const int32_t* positions) {
    std::vector<char> seen(c->cfg.streams, 0);
    for (int i = 0; i < n; i++) {
        const int s = streams[i];
        if (s < 0 || s >= c->cfg.streams)
            return fail(c, MB_ERR_STREAM, "item %d: stream %d out of range [0, %d)", i, s, c->cfg.streams);
        if (seen[s]) return fail(c, MB_ERR_STREAM, "item %d: stream %d appears twice in one call", i, s);
        seen[s] = 1;
        int rc = check_position(c, positions[i]);
        if (rc) return rc;
    }
    return MB_OK;
}

namespace {

// The decode launch of every context entry point: the per-chunk kernel
// (mb_decode.cu), or -- when MOCKBIRD_DECODE_KERNEL=persistent and the call fits
// it -- the persistent stream-K kernel (mb_decode_persist.cu).  Both compute the
// same thing.  overlap_previous: see launch_decode.
// layers: consecutive layers from `layer` in one launch (q and out hold every
// layer's n rows, layer after layer); the persistent kernel runs one launch per layer.
cudaError_t run_decode(mb_ctx* c, bool append, int layer, int n, const int32_t* streams, const int32_t* positions,
                       const float* q, int q_stride, float* out, cudaStream_t st, bool overlap_previous = false,
                       int layers = 1) {
    if (c->persistent && decode_persist_supported(ring_view(c, layer), n, q_stride)) {
        for (int l = 0; l < layers; l++) {
            const cudaError_t e = launch_decode_persist(c->cfg.dtype, append, ring_view(c, layer + l), c->scratch, n,
                                                        streams, positions, q + (size_t)l * n * q_stride, q_stride,
                                                        out + (size_t)l * n * c->cfg.heads * HD, st);
            if (e != cudaSuccess) return e;
        }
        return cudaSuccess;
    }
    return launch_decode(c->cfg.dtype, append, ring_view(c, layer), c->scratch, n, streams, positions, q, q_stride,
                         out, st, overlap_previous, false, layers);
}

}  // namespace

extern "C" {

MB_API const char* mb_version(void) { return MB_VERSION; }

MB_API void mb_config_default(mb_config* cfg) {
    if (!cfg) return;
    cfg->layers = 12;
    cfg->heads = 12;
    cfg->head_dim = 64;
    cfg->capacity = 570;
    cfg->streams = 1;
    cfg->dtype = MB_F32;
    cfg->wrap = 0;
    cfg->max_position = 65536;
    cfg->rope_theta = 10000.0f;
    cfg->device = 0;
    cfg->max_batch = 0;
}

MB_API const char* mb_last_error(const mb_ctx* ctx) { return ctx ? ctx->last_error.c_str() : "null context"; }

MB_API int mb_create(const mb_config* cfg_in, mb_ctx** out) {
    if (!cfg_in || !out) return MB_ERR_ARG;
    *out = nullptr;
    mb_config cfg = *cfg_in;
    if (cfg.max_position <= 0) cfg.max_position = 65536;
    if (cfg.max_batch <= 0) cfg.max_batch = cfg.streams;
    if (cfg.head_dim != HD || cfg.layers <= 0 || cfg.heads <= 0 || cfg.heads > 64 || cfg.capacity <= 0 ||
        cfg.streams <= 0 || cfg.dtype < MB_F32 || cfg.dtype > MB_F16 || cfg.max_batch > 65535 ||
        !(cfg.rope_theta > 0.0f))
        return MB_ERR_ARG;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || cfg.device < 0 || cfg.device >= ndev) return MB_ERR_CUDA;

    mb_ctx* c = new mb_ctx();
    c->cfg = cfg;
    {  // MOCKBIRD_DECODE_KERNEL=persistent selects the persistent decode kernel (A/B measurements)
        const char* k = getenv("MOCKBIRD_DECODE_KERNEL");
        c->persistent = k && strcmp(k, "persistent") == 0;
    }
    c->esize = cfg.dtype == MB_F32 ? 4 : 2;
    DeviceGuard g(cfg.device);
    auto bail = [&](int rc) {
        mb_destroy(c);
        return rc;
    };
    if (!g.ok) return bail(MB_ERR_CUDA);

    const size_t slots = (size_t)cfg.layers * cfg.streams * cfg.capacity;
    c->kv_bytes = slots * 2 * cfg.heads * HD * c->esize;
    if (cudaMalloc(&c->kv, c->kv_bytes) != cudaSuccess) return bail(MB_ERR_OOM);
    if (cudaMalloc(&c->slot_pos, slots * sizeof(int32_t)) != cudaSuccess) return bail(MB_ERR_OOM);
    if (cudaMemset(c->kv, 0, c->kv_bytes) != cudaSuccess) return bail(MB_ERR_CUDA);
    if (cudaMemset(c->slot_pos, 0xFF, slots * sizeof(int32_t)) != cudaSuccess) return bail(MB_ERR_CUDA);

    // RoPE table: angle and cos/sin in fp64, rounded once to fp32
    // (tools/onnx-probe/ref-decode.mjs:111-124 evaluates them in fp64)
    {
        std::vector<float2> tab((size_t)cfg.max_position * 32);
        for (int p = 0; p < cfg.max_position; p++)
            for (int i = 0; i < 32; i++) {
                const double inv = pow((double)cfg.rope_theta, -(2.0 * i) / 64.0);
                const double a = (double)p * inv;
                tab[(size_t)p * 32 + i] = make_float2((float)cos(a), (float)sin(a));
            }
        if (cudaMalloc(&c->rope, tab.size() * sizeof(float2)) != cudaSuccess) return bail(MB_ERR_OOM);
        if (cudaMemcpy(c->rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice) != cudaSuccess)
            return bail(MB_ERR_CUDA);
    }
    if (cudaMalloc(&c->d_err, sizeof(int32_t)) != cudaSuccess) return bail(MB_ERR_OOM);
    if (cudaMemset(c->d_err, 0, sizeof(int32_t)) != cudaSuccess) return bail(MB_ERR_CUDA);

    // split-K scratch: one (m, l, acc[64]) partial per chunk and a ticket per (item, head)
    const int rows = chunk_rows(cfg.dtype);
    c->scratch.max_splits = (cfg.capacity + rows - 1) / rows;
    // (the persistent kernel's units are half a chunk: it may need twice the slots)
    const int part_slots = c->scratch.max_splits > persist_part_stride(cfg.dtype, cfg.capacity)
                               ? c->scratch.max_splits
                               : persist_part_stride(cfg.dtype, cfg.capacity);
    // (one launch may cover every layer: items of all layers at once)
    const size_t items = (size_t)cfg.max_batch * cfg.layers;
    const size_t part_bytes = items * cfg.heads * part_slots * (2 + HD) * sizeof(float);
    const size_t cnt_bytes = items * cfg.heads * sizeof(int32_t);
    c->scratch_bytes = part_bytes + cnt_bytes;
    if (cudaMalloc(&c->scratch.part, part_bytes) != cudaSuccess) return bail(MB_ERR_OOM);
    if (cudaMalloc(&c->scratch.counters, cnt_bytes) != cudaSuccess) return bail(MB_ERR_OOM);
    if (cudaMemset(c->scratch.counters, 0, cnt_bytes) != cudaSuccess) return bail(MB_ERR_CUDA);

    // staging for the host-array entry points
    const size_t hid = (size_t)cfg.heads * HD;
    if (cudaMalloc(&c->d_ids, 2 * cfg.max_batch * sizeof(int32_t)) != cudaSuccess) return bail(MB_ERR_OOM);
    if (cudaMallocHost(&c->h_ids, 2 * cfg.max_batch * sizeof(int32_t)) != cudaSuccess) return bail(MB_ERR_OOM);
    if (cudaMalloc(&c->d_qkv, (size_t)cfg.layers * cfg.max_batch * 3 * hid * sizeof(float)) != cudaSuccess)
        return bail(MB_ERR_OOM);
    if (cudaMalloc(&c->d_out, (size_t)cfg.layers * cfg.max_batch * hid * sizeof(float)) != cudaSuccess)
        return bail(MB_ERR_OOM);
    if (cudaStreamCreateWithFlags(&c->cp_in, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&c->cp_out, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&c->ev_start, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&c->ev_end, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&c->ev_ids, cudaEventDisableTiming) != cudaSuccess)
        return bail(MB_ERR_CUDA);
    if (cudaMallocHost(&c->h_err, sizeof(int32_t)) != cudaSuccess) return bail(MB_ERR_OOM);
    c->ev_in.assign(cfg.layers, nullptr);
    c->ev_done.assign(cfg.layers, nullptr);
    for (int l = 0; l < cfg.layers; l++)
        if (cudaEventCreateWithFlags(&c->ev_in[l], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&c->ev_done[l], cudaEventDisableTiming) != cudaSuccess)
            return bail(MB_ERR_CUDA);
    if (cudaDeviceSynchronize() != cudaSuccess) return bail(MB_ERR_CUDA);
    *out = c;
    return MB_OK;
}

MB_API int mb_destroy(mb_ctx* c) {
    if (!c) return MB_ERR_ARG;
    {
        DeviceGuard g(c->cfg.device);
        void* ptrs[] = {c->kv, c->slot_pos, c->rope, c->d_err, c->scratch.part, c->scratch.counters,
                        c->d_ids, c->d_qkv, c->d_out, c->pf_stage};
        for (void* p : ptrs)
            if (p) cudaFree(p);
        for (auto* evs : {&c->ev_in, &c->ev_done})
            for (cudaEvent_t e : *evs)
                if (e) cudaEventDestroy(e);
        if (c->ev_start) cudaEventDestroy(c->ev_start);
        if (c->ev_end) cudaEventDestroy(c->ev_end);
        if (c->ev_ids) cudaEventDestroy(c->ev_ids);
        if (c->h_err) cudaFreeHost(c->h_err);
        if (c->h_ids) cudaFreeHost(c->h_ids);
        if (c->cp_in) cudaStreamDestroy(c->cp_in);
        if (c->cp_out) cudaStreamDestroy(c->cp_out);
    }
    delete c;
    return MB_OK;
}

MB_API int mb_reset(mb_ctx* c, int32_t stream, void* cuda_stream) {
    if (!c) return MB_ERR_ARG;
    if (stream >= c->cfg.streams) return fail(c, MB_ERR_STREAM, "stream %d out of range", stream);
    DeviceGuard g(c->cfg.device);
    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    CK(launch_reset(c, stream, st), "reset");
    if (stream < 0) {  // a full reset also re-arms the split-K tickets
        CK(cudaMemsetAsync(c->scratch.counters, 0,
                           (size_t)c->cfg.max_batch * c->cfg.layers * c->cfg.heads * sizeof(int32_t), st),
           "reset tickets");
    }
    return MB_OK;
}

MB_API int mb_rope_append(mb_ctx* c, int32_t layer, int32_t n, const int32_t* streams, const int32_t* positions,
                          float* qkv, void* cuda_stream) {
    if (!c) return MB_ERR_ARG;
    int rc;
    if ((rc = check_layer(c, layer)) || (rc = check_batch(c, n))) return rc;
    if (n == 0) return MB_OK;
    if (!streams || !positions || !qkv || !aligned(qkv, 16))
        return fail(c, MB_ERR_ARG, "null or misaligned device pointer");
    DeviceGuard g(c->cfg.device);
    CK(launch_rope_append(c->cfg.dtype, ring_view(c, layer), n, streams, positions, qkv,
                          static_cast<cudaStream_t>(cuda_stream)),
       "rope_append launch");
    return MB_OK;
}

MB_API int mb_attend(mb_ctx* c, int32_t layer, int32_t n, const int32_t* streams, const int32_t* positions,
                     const float* q, int32_t q_stride, float* out, void* cuda_stream) {
    if (!c) return MB_ERR_ARG;
    int rc;
    if ((rc = check_layer(c, layer)) || (rc = check_batch(c, n))) return rc;
    if (n == 0) return MB_OK;
    if (!streams || !positions || !q || !out || !aligned(q, 16) || !aligned(out, 16) || q_stride < c->cfg.heads * HD ||
        (q_stride & 1))
        return fail(c, MB_ERR_ARG, "null/misaligned device pointer or bad q_stride %d", q_stride);
    DeviceGuard g(c->cfg.device);
    CK(run_decode(c, false, layer, n, streams, positions, q, q_stride, out, static_cast<cudaStream_t>(cuda_stream)),
       "attend launch");
    return MB_OK;
}

MB_API int mb_append_attend(mb_ctx* c, int32_t layer, int32_t n, const int32_t* streams, const int32_t* positions,
                            const float* qkv, float* out, void* cuda_stream) {
    if (!c) return MB_ERR_ARG;
    int rc;
    if ((rc = check_layer(c, layer)) || (rc = check_batch(c, n))) return rc;
    if (n == 0) return MB_OK;
    if (!streams || !positions || !qkv || !out || !aligned(qkv, 16) || !aligned(out, 16))
        return fail(c, MB_ERR_ARG, "null or misaligned device pointer");
    DeviceGuard g(c->cfg.device);
    CK(run_decode(c, true, layer, n, streams, positions, qkv, 3 * c->cfg.heads * HD, out,
                  static_cast<cudaStream_t>(cuda_stream)),
       "append_attend launch");
    return MB_OK;
}

MB_API int mb_decode_step(mb_ctx* c, int32_t n, const int32_t* streams, const int32_t* positions, const float* qkv,
                          float* out, void* cuda_stream) {
    if (!c) return MB_ERR_ARG;
    int rc;
    if ((rc = check_batch(c, n))) return rc;
    if (n == 0) return MB_OK;
    if (!streams || !positions || !qkv || !out || !aligned(qkv, 16) || !aligned(out, 16))
        return fail(c, MB_ERR_ARG, "null or misaligned device pointer");
    DeviceGuard g(c->cfg.device);
    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    const size_t hid = (size_t)c->cfg.heads * HD;
    // every layer in one launch: the layers touch disjoint rings
    CK(run_decode(c, true, 0, n, streams, positions, qkv, 3 * (int)hid, out, st, false, c->cfg.layers),
       "append_attend launch");
    return MB_OK;
}

}  // extern "C"

thread_local mb::LaunchPriority mb::launch_priority;

// The status of device rejection bits read back (clearing them on the device).
int mb::report_bits(mb_ctx* c, int32_t bits) {
    if (!bits) return MB_OK;
    CK(cudaMemset(c->d_err, 0, sizeof(int32_t)), "clear device status");
    if (bits & DERR_TIMEOUT)
        return fail(c, MB_ERR_TIMEOUT, "a bounded device-side wait gave up (bits 0x%x)", bits);
    return fail(c, MB_ERR_DEVICE, "a kernel rejected an item:%s%s%s", (bits & DERR_STREAM) ? " stream out of range" : "",
                (bits & DERR_POSITION) ? " position out of range" : "",
                (bits & DERR_CAPACITY) ? " position beyond a non-wrapping ring" : "");
}

extern "C" {

MB_API int mb_sync(mb_ctx* c, void* cuda_stream) {
    if (!c) return MB_ERR_ARG;
    DeviceGuard g(c->cfg.device);
    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    CK(cudaStreamSynchronize(st), "synchronize");
    int32_t bits = 0;
    CK(cudaMemcpy(&bits, c->d_err, sizeof bits, cudaMemcpyDeviceToHost), "read device status");
    return report_bits(c, bits);
}

// The end of a host-array call: the status word rides behind the outputs on
// `copy_st` into pinned memory, so one synchronisation of `st` (which waits for
// `copy_st`) returns both.
// The stream ids and positions of a host-array call, packed into the context's
// page-locked staging (ids, then positions) and copied in with one transfer: the
// caller's arrays are usually pageable, and each pageable copy is staged and
// synchronous on the host.  A call that succeeds synchronises before it returns,
// but one that fails after queueing this copy returns without waiting, so the
// staging is reused only once the event behind the previous copy has completed.
static cudaError_t stage_ids(mb_ctx* c, int n, const int32_t* streams, const int32_t* positions,
                             cudaStream_t st) {
    cudaError_t e = cudaEventSynchronize(c->ev_ids);
    if (e != cudaSuccess) return e;
    memcpy(c->h_ids, streams, n * sizeof(int32_t));
    memcpy(c->h_ids + n, positions, n * sizeof(int32_t));
    e = cudaMemcpyAsync(c->d_ids, c->h_ids, 2 * n * sizeof(int32_t), cudaMemcpyHostToDevice, st);
    return e == cudaSuccess ? cudaEventRecord(c->ev_ids, st) : e;
}

static int finish_host_call(mb_ctx* c, cudaStream_t st, cudaStream_t copy_st) {
    CK(cudaMemcpyAsync(c->h_err, c->d_err, sizeof(int32_t), cudaMemcpyDeviceToHost, copy_st), "read device status");
    if (copy_st != st) {
        CK(cudaEventRecord(c->ev_end, copy_st), "copies done");
        CK(cudaStreamWaitEvent(st, c->ev_end, 0), "copies done");
    }
    CK(cudaStreamSynchronize(st), "synchronize");
    return report_bits(c, *c->h_err);
}

MB_API int mb_append_attend_host(mb_ctx* c, int32_t layer, int32_t n, const int32_t* streams,
                                 const int32_t* positions, const float* qkv, float* out, void* cuda_stream) {
    if (!c) return MB_ERR_ARG;
    int rc;
    if ((rc = check_layer(c, layer)) || (rc = check_batch(c, n))) return rc;
    if (n == 0) return MB_OK;
    if (!streams || !positions || !qkv || !out) return fail(c, MB_ERR_ARG, "null host pointer");
    if ((rc = check_items_host(c, n, streams, positions))) return rc;
    DeviceGuard g(c->cfg.device);
    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    const size_t hid = (size_t)c->cfg.heads * HD;
    CK(stage_ids(c, n, streams, positions, st), "copy streams and positions");
    CK(cudaMemcpyAsync(c->d_qkv, qkv, n * 3 * hid * sizeof(float), cudaMemcpyHostToDevice, st), "copy qkv");
    CK(run_decode(c, true, layer, n, c->d_ids, c->d_ids + n, c->d_qkv, 3 * (int)hid, c->d_out, st),
       "append_attend launch");
    CK(cudaMemcpyAsync(out, c->d_out, n * hid * sizeof(float), cudaMemcpyDeviceToHost, st), "copy out");
    return finish_host_call(c, st, st);
}

// Segments of mb_decode_step_host: runs of consecutive layers [b_s, b_{s+1}),
// each decoded by one launch, its qkv rows copied in as one group before it and
// its context rows copied out as one group after it, on the context's two copy
// streams, so that copies overlap the decode of other segments.  A launch
// boundary costs the tail of a launch, and a copy group is waited for as a
// whole, so the split is chosen by a small model: page-locked copies at ~50 GB/s
// each way (serial per direction), the decode at ~5.5 TB/s of live-window bytes
// per layer, and ~10 us per launch; every split into at most 4 segments is
// tried and the one with the earliest estimated end is kept.
static void host_step_plan(const mb_ctx* c, int n, const int32_t* positions, std::vector<int>& bounds) {
    const int L = c->cfg.layers;
    double window_bytes = 0;  // K and V windows one layer's decode reads
    for (int i = 0; i < n; i++) {
        const int w = positions[i] + 1 < c->cfg.capacity ? positions[i] + 1 : c->cfg.capacity;
        window_bytes += 2.0 * w * c->cfg.heads * HD * (double)c->esize;
    }
    const double hid = (double)c->cfg.heads * HD;
    const double t_layer = window_bytes / 5.5e12, t_launch = 10e-6;
    const double c_in = n * 3 * hid * 4 / 50e9, c_out = n * hid * 4 / 50e9;  // per layer
    auto cost = [&](const std::vector<int>& b) {
        double in_ready = 0, seg_end = 0, out_end = 0;
        for (size_t s = 0; s + 1 < b.size(); s++) {
            const int k = b[s + 1] - b[s];
            in_ready += k * c_in;
            seg_end = (seg_end > in_ready ? seg_end : in_ready) + k * t_layer + t_launch;
            out_end = (out_end > seg_end ? out_end : seg_end) + k * c_out;
        }
        return out_end;
    };
    std::vector<int> best = {0, L}, cand;
    double best_t = cost(best);
    const int maxseg = L < 4 ? L : 4;
    // every composition of L into 2..maxseg parts (cuts at increasing layers)
    for (int parts = 2; parts <= maxseg; parts++) {
        std::vector<int> cut(parts - 1);
        for (int i = 0; i < parts - 1; i++) cut[i] = i + 1;
        while (true) {
            cand.assign(1, 0);
            cand.insert(cand.end(), cut.begin(), cut.end());
            cand.push_back(L);
            const double t = cost(cand);
            if (t < best_t) best_t = t, best = cand;
            int i = parts - 2;
            while (i >= 0 && cut[i] == L - (parts - 1 - i)) i--;
            if (i < 0) break;
            cut[i]++;
            for (int j = i + 1; j < parts - 1; j++) cut[j] = cut[j - 1] + 1;
        }
    }
    bounds = best;
}

MB_API int mb_decode_step_host(mb_ctx* c, int32_t n, const int32_t* streams, const int32_t* positions,
                               const float* qkv, float* out, void* cuda_stream) {
    if (!c) return MB_ERR_ARG;
    int rc;
    if ((rc = check_batch(c, n))) return rc;
    if (n == 0) return MB_OK;
    if (!streams || !positions || !qkv || !out) return fail(c, MB_ERR_ARG, "null host pointer");
    if ((rc = check_items_host(c, n, streams, positions))) return rc;
    DeviceGuard g(c->cfg.device);
    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    const size_t hid = (size_t)c->cfg.heads * HD;
    const size_t in_l = (size_t)n * 3 * hid, out_l = (size_t)n * hid;  // floats per layer
    std::vector<int> bounds;
    host_step_plan(c, n, positions, bounds);
    const size_t segs = bounds.size() - 1;
    // Per segment: its qkv rows copied in on cp_in; its launch on `st` waits for
    // them; its context rows copied out on cp_out once it is done.  Both copy
    // streams start behind the work already queued on `st`, and `st` ends behind them.
    CK(cudaEventRecord(c->ev_start, st), "order copies");
    CK(cudaStreamWaitEvent(c->cp_in, c->ev_start, 0), "order copies");
    CK(cudaStreamWaitEvent(c->cp_out, c->ev_start, 0), "order copies");
    CK(stage_ids(c, n, streams, positions, c->cp_in), "copy streams and positions");
    for (size_t g = 0; g < segs; g++) {
        const size_t l = bounds[g], k = bounds[g + 1] - bounds[g];
        CK(cudaMemcpyAsync(c->d_qkv + l * in_l, qkv + l * in_l, k * in_l * sizeof(float), cudaMemcpyHostToDevice,
                           c->cp_in),
           "copy qkv");
        CK(cudaEventRecord(c->ev_in[g], c->cp_in), "copy qkv");
    }
    for (size_t g = 0; g < segs; g++) {
        const size_t l = bounds[g], k = bounds[g + 1] - bounds[g];
        CK(cudaStreamWaitEvent(st, c->ev_in[g], 0), "wait qkv");
        CK(run_decode(c, true, (int)l, n, c->d_ids, c->d_ids + n, c->d_qkv + l * in_l, 3 * (int)hid,
                      c->d_out + l * out_l, st, false, (int)k),
           "append_attend launch");
        CK(cudaEventRecord(c->ev_done[g], st), "segment done");
        CK(cudaStreamWaitEvent(c->cp_out, c->ev_done[g], 0), "wait segment");
        CK(cudaMemcpyAsync(out + l * out_l, c->d_out + l * out_l, k * out_l * sizeof(float), cudaMemcpyDeviceToHost,
                           c->cp_out),
           "copy out");
    }
    return finish_host_call(c, st, c->cp_out);
}

MB_API int mb_prefill(mb_ctx* c, int32_t layer, int32_t n, const int32_t* streams, int32_t rows, const float* qkv,
                      float* out, void* cuda_stream) {
    if (!c) return MB_ERR_ARG;
    int rc;
    if ((rc = check_layer(c, layer)) || (rc = check_batch(c, n))) return rc;
    if (n == 0) return MB_OK;
    if (rows <= 0) return fail(c, MB_ERR_ARG, "prefill called with no rows");
    if (rows > c->cfg.capacity)
        return fail(c, MB_ERR_CAPACITY, "prefill of %d rows exceeds the ring capacity %d", rows, c->cfg.capacity);
    if (rows > c->cfg.max_position) return fail(c, MB_ERR_POSITION, "prefill rows beyond max_position");
    if (!streams || !qkv || !out || !aligned(qkv, 16) || !aligned(out, 16))
        return fail(c, MB_ERR_ARG, "null or misaligned device pointer");
    DeviceGuard g(c->cfg.device);
    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    // fp32 rings: the stage is the context's own, grown when a call needs more
    // (cudaFree then cudaMalloc, both synchronising the device, so no earlier
    // call still uses the old one); it stays allocated for the next calls
    const size_t stage_bytes = prefill_stage_bytes(c->cfg.dtype, n, c->cfg.heads, rows);
    if (stage_bytes > c->pf_stage_bytes) {
        if (c->pf_stage) CK(cudaFree(c->pf_stage), "prefill stage free");
        c->pf_stage = nullptr;
        c->pf_stage_bytes = 0;
        if (cudaMalloc(&c->pf_stage, stage_bytes) != cudaSuccess) {
            c->pf_stage = nullptr;
            cudaGetLastError();
            return fail(c, MB_ERR_OOM, "prefill stage of %zu bytes", stage_bytes);
        }
        c->pf_stage_bytes = stage_bytes;
    }
    CK(launch_prefill(c->cfg.dtype, ring_view(c, layer), n, streams, rows, qkv, out, c->pf_stage, st),
       "prefill launch");
    return MB_OK;
}

MB_API int mb_gather(mb_ctx* c, int32_t layer, int32_t stream, int32_t position, void* k_out, void* v_out,
                     int32_t* slots_out, void* cuda_stream) {
    if (!c) return MB_ERR_ARG;
    int rc;
    if ((rc = check_layer(c, layer))) return rc;
    if (stream < 0 || stream >= c->cfg.streams) return fail(c, MB_ERR_STREAM, "stream %d out of range", stream);
    if ((rc = check_position(c, position))) return rc;
    if (!k_out || !v_out || !slots_out) return fail(c, MB_ERR_ARG, "null device pointer");
    DeviceGuard g(c->cfg.device);
    CK(launch_gather(c->cfg.dtype, ring_view(c, layer), stream, position, k_out, v_out, slots_out,
                     static_cast<cudaStream_t>(cuda_stream)),
       "gather launch");
    return MB_OK;
}

MB_API int mb_ring_write(mb_ctx* c, int32_t layer, int32_t stream, int32_t first_position, int32_t count,
                         const void* k, const void* v, void* cuda_stream) {
    if (!c) return MB_ERR_ARG;
    int rc;
    if ((rc = check_layer(c, layer))) return rc;
    if (stream < 0 || stream >= c->cfg.streams) return fail(c, MB_ERR_STREAM, "stream %d out of range", stream);
    if (count <= 0 || count > c->cfg.capacity)
        return fail(c, MB_ERR_ARG, "count %d out of range [1, capacity %d]", count, c->cfg.capacity);
    if ((rc = check_position(c, first_position)) || (rc = check_position(c, first_position + count - 1))) return rc;
    if (!k || !v) return fail(c, MB_ERR_ARG, "null device pointer");
    DeviceGuard g(c->cfg.device);
    CK(launch_ring_write(c->cfg.dtype, ring_view(c, layer), stream, first_position, count, k, v,
                         static_cast<cudaStream_t>(cuda_stream)),
       "ring_write launch");
    return MB_OK;
}

MB_API int mb_set_wait_limit(mb_ctx* c, int64_t cycles) {
    if (!c) return MB_ERR_ARG;
    c->wait_probe = cycles < 0;
    c->wait_limit = cycles > 0 ? cycles : cycles < 0 ? -cycles : mb::WAIT_LIMIT;
    return MB_OK;
}

MB_API int mb_ring_info_get(const mb_ctx* c, mb_ring_info* out) {
    if (!c || !out) return MB_ERR_ARG;
    out->kv = c->kv;
    out->slot_pos = c->slot_pos;
    out->kv_bytes = c->kv_bytes;
    out->elem_bytes = c->esize;
    out->scratch_bytes = c->scratch_bytes;
    return MB_OK;
}

}  // extern "C"
