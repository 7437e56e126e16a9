// The decode step around the KV-ring path: the global
// transformer layer of DecodeRunner.runLayer (liyu1981/mockbird,
// src/lib/tts/engine/decode.ts:474-620) for n streams at once, and the final
// LayerNorm of globalStep (decode.ts:749-772).
//
// Per layer: LN1 -> QKV GEMM (+ bias) -> append + RoPE + attention (this
// library's decode kernel) -> c_proj GEMM (+ bias + residual) -> LN2 -> fc_in
// GEMM (+ bias, GELU(tanh), bf16 out) -> fc_out GEMM (+ bias + residual).  The
// GEMMs are this library's tcgen05 kernels (mb_gemm.cu: bf16 weights and
// activations, fp32 accumulation in TMEM, bias / residual / GELU in the
// epilogue; y = b + x W with W [K][N] as the published graph stores it, held
// transposed on the device); LayerNorm (LAYERNORM_1, kernels-decode.ts:168-200:
// eps 1e-5, two passes) is a kernel here; GELU (GELU_TANH, :373-390) is fc_in's
// epilogue.
#include <stdlib.h>
#include <string.h>

#include "mb_decoder.cuh"

namespace {

using bf16 = __nv_bfloat16;

// ---------------------------------------------------------------- kernels

// One warp per row: mean, then the mean squared deviation (the two passes of
// LAYERNORM_1), out = (x - mean) * rsqrt(var + 1e-5) * w + b (mb::dec::ln_load /
// ln_apply).  In place is fine: the row is in registers before it is written.
// Launched as a programmatic dependent of the GEMM before it: nothing global
// is touched before that kernel has completed.
template <typename TO, int PER>
__global__ void layernorm_rows(const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ b,
                               TO* __restrict__ y, int rows, int width) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    float v[PER];
    mb::dec::ln_load<PER>(x + (size_t)row * width, lane, v);
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    mb::dec::ln_apply<TO, PER>(v, w, b, y + (size_t)row * width, width, lane);
}

template <typename TO, int PER>
cudaError_t layernorm_t(const float* x, const float* w, const float* b, TO* y, int rows, int width,
                        cudaStream_t st) {
    const int warps = 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((rows + warps - 1) / warps);
    cfg.blockDim = dim3(32 * warps);
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = mb::with_priority(attr, 1);
    return cudaLaunchKernelEx(&cfg, layernorm_rows<TO, PER>, x, w, b, y, rows, width);
}

template <typename TO>
cudaError_t layernorm(const float* x, const float* w, const float* b, TO* y, int rows, int width, cudaStream_t st) {
    switch (width / 32) {  // width = heads * 64
        case 2: return layernorm_t<TO, 2>(x, w, b, y, rows, width, st);
        case 8: return layernorm_t<TO, 8>(x, w, b, y, rows, width, st);
        case 24: return layernorm_t<TO, 24>(x, w, b, y, rows, width, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

namespace mb {
namespace dec {

int fail(mb_decoder* d, int code, const std::string& msg) {
    if (d && d->ctx) d->ctx->last_error = msg;
    return code;
}

uint16_t f32_to_bf16_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

void transpose_to_bf16(const float* w, int K, int N, uint16_t* out) {
    for (int k = 0; k < K; k++)
        for (int n = 0; n < N; n++) out[(size_t)n * K + k] = f32_to_bf16_bits(w[(size_t)k * N + n]);
}

namespace {
const CUtensorMap* operand_map(mb_decoder* d, const void* base, int k, int rows, int box_rows, int box_kb) {
    const auto key = std::make_tuple(base, k, rows, box_rows, box_kb);
    auto it = d->maps.find(key);
    if (it == d->maps.end()) {
        CUtensorMap m;
        if (!mb::gemm::make_map(&m, base, k, rows, box_rows, box_kb)) return nullptr;
        it = d->maps.emplace(key, m).first;
    }
    return &it->second;
}
}  // namespace

int gemm(mb_decoder* d, int M, int N, int K, const bf16* x, const bf16* Wt, const float* bias, void* y, int ldy,
         int epi, cudaStream_t st, const RingView* ring, const int32_t* streams, const int32_t* positions,
         int x_row0) {
    const auto pkey = std::make_tuple(M, N, K, epi);
    auto pit = d->gemm_plans.find(pkey);
    if (pit == d->gemm_plans.end()) pit = d->gemm_plans.emplace(pkey, mb::gemm::choose(M, N, K, epi)).first;
    const mb::gemm::Plan p = pit->second;
    const CUtensorMap* ta =
        operand_map(d, x, K, d->ctx->cfg.max_batch - x_row0, mb::gemm::a_box_rows(p), mb::gemm::box_kb(p));
    const CUtensorMap* tb = operand_map(d, Wt, K, N, mb::gemm::b_box_rows(p), mb::gemm::box_kb(p));
    if (!ta || !tb) return fail(d, MB_ERR_CUDA, "decoder: GEMM tensor map encoding failed");
    mb::gemm::Args a;
    a.M = M, a.N = N, a.K = K, a.splits = p.splits;
    a.bias = bias, a.y = y, a.ldy = ldy;
    a.err = d->ctx->d_err;
    a.ring = ring ? *ring : RingView{};
    a.streams = streams, a.positions = positions;
    a.ring_dtype = d->ctx->cfg.dtype;
    // a programmatic dependent of the kernel before it (the GEMM loads its first
    // weight tiles while that kernel finishes)
    const cudaError_t e = mb::gemm::launch(*ta, *tb, a, p, epi, st, true);
    if (e != cudaSuccess) return fail(d, MB_ERR_CUDA, std::string("decoder GEMM: ") + cudaGetErrorString(e));
    return MB_OK;
}

namespace {
// The layers and ln_f for items [row0, row0 + n) of the step: `streams`,
// `positions`, `hidden` and `lnf_bf16` already point at row row0; the
// activation buffers and the split-K scratch are offset here.  after_qkv0, when
// non-null, is recorded on `st` right after layer 0's QKV GEMM.
int run_rows(mb_decoder* d, int row0, int n, const int32_t* streams, const int32_t* positions, float* hidden,
             bf16* lnf_bf16, cudaStream_t st, bool ln1_ready, bool qkv_append, cudaEvent_t after_qkv0) {
    mb_ctx* c = d->ctx;
    const int h = d->hid, f = d->ffn;
    bf16* xb = d->xb + (size_t)row0 * h;
    float* qkv = d->qkv + (size_t)row0 * 3 * h;
    bf16* h1 = d->h1 + (size_t)row0 * f;
    Scratch sc = c->scratch;  // partials of these items only: [row0 + item][head][split]
    sc.part += (size_t)row0 * c->cfg.heads * sc.max_splits * (2 + HD);
    int rc = MB_OK;
    cudaError_t e = cudaSuccess;
    for (int l = 0; l < d->layers && rc == MB_OK && e == cudaSuccess; l++) {
        const auto& W = d->L[l];
        if (!(l == 0 && ln1_ready) && (e = layernorm<bf16>(hidden, W.ln1_w, W.ln1_b, xb, n, h, st)) != cudaSuccess)
            break;
        // QKV with RoPE and the ring append in the GEMM's epilogue (the roped q
        // rows land in qkv, the new K/V rows in the ring), or q|k|v stored
        const RingView rv = mb::ring_view(c, l);
        if ((rc = gemm(d, n, 3 * h, h, xb, W.w_attn, W.b_attn, qkv, 3 * h,
                       qkv_append ? mb::gemm::EPI_QKV_RING : mb::gemm::EPI_STORE, st, &rv, streams, positions,
                       row0)))
            break;
        if (l == 0 && after_qkv0 && (e = cudaEventRecord(after_qkv0, st)) != cudaSuccess) break;
        // attention over each window, the new row included (appended here when
        // the GEMM did not); launched without programmatic overlap, since its ring
        // reads start at entry.  The context rows go straight to the bf16 input of
        // the c_proj GEMM
        if ((e = mb::launch_decode(c->cfg.dtype, !qkv_append, rv, sc, n, streams, positions, qkv, 3 * h, xb, st,
                                   false, true)) != cudaSuccess)
            break;
        if ((rc = gemm(d, n, h, h, xb, W.w_proj, W.b_proj, hidden, h, mb::gemm::EPI_ACCUM, st, nullptr, nullptr,
                       nullptr, row0)))
            break;
        if ((e = layernorm<bf16>(hidden, W.ln2_w, W.ln2_b, xb, n, h, st)) != cudaSuccess) break;
        if ((rc = gemm(d, n, f, h, xb, W.w_in, W.b_in, h1, f, mb::gemm::EPI_GELU_BF16, st, nullptr, nullptr, nullptr,
                       row0)))
            break;
        if ((rc = gemm(d, n, h, f, h1, W.w_out, W.b_out, hidden, h, mb::gemm::EPI_ACCUM, st, nullptr, nullptr,
                       nullptr, row0)))
            break;
        e = cudaGetLastError();
    }
    if (rc == MB_OK && e == cudaSuccess)
        e = lnf_bf16 ? layernorm<bf16>(hidden, d->lnf_w, d->lnf_b, lnf_bf16, n, h, st)
                     : layernorm<float>(hidden, d->lnf_w, d->lnf_b, hidden, n, h, st);
    if (rc) return rc;
    if (e != cudaSuccess) return fail(d, MB_ERR_CUDA, std::string("decoder: ") + cudaGetErrorString(e));
    return MB_OK;
}
}  // namespace

int run(mb_decoder* d, int n, const int32_t* streams, const int32_t* positions, float* hidden, bf16* lnf_bf16,
        cudaStream_t st, bool ln1_ready, bool qkv_append, bool split) {
    const int n0 = n / 2;
    if (!split || !d->split || !d->side || n0 < SPLIT_MIN_ROWS)
        return run_rows(d, 0, n, streams, positions, hidden, lnf_bf16, st, ln1_ready, qkv_append, nullptr);
    const int h = d->hid;
    const mb::LaunchPriority saved = mb::launch_priority;
    mb::launch_priority.set = true;
    mb::launch_priority.value = d->prio_high;
    mb::launch_priority.decode_value = d->prio_low;
    int rc = MB_OK;
    cudaError_t e = cudaEventRecord(d->ev_fork, st);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(d->side, d->ev_fork, 0);
    const bool forked = e == cudaSuccess;
    if (!forked) rc = fail(d, MB_ERR_CUDA, std::string("decoder fork: ") + cudaGetErrorString(e));
    if (rc == MB_OK)
        rc = run_rows(d, 0, n0, streams, positions, hidden, lnf_bf16, st, ln1_ready, qkv_append, d->ev_stagger);
    if (rc == MB_OK && (e = cudaStreamWaitEvent(d->side, d->ev_stagger, 0)) != cudaSuccess)
        rc = fail(d, MB_ERR_CUDA, std::string("decoder fork: ") + cudaGetErrorString(e));
    if (rc == MB_OK)
        rc = run_rows(d, n0, n - n0, streams + n0, positions + n0, hidden + (size_t)n0 * h,
                      lnf_bf16 ? lnf_bf16 + (size_t)n0 * h : nullptr, d->side, ln1_ready, qkv_append, nullptr);
    if (forked) {  // the caller's stream ends behind both chains, whatever happened
        e = cudaEventRecord(d->ev_join, d->side);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(st, d->ev_join, 0);
        if (e != cudaSuccess && rc == MB_OK)
            rc = fail(d, MB_ERR_CUDA, std::string("decoder join: ") + cudaGetErrorString(e));
    }
    mb::launch_priority = saved;
    return rc;
}

}  // namespace dec
}  // namespace mb

extern "C" {

MB_API size_t mb_decoder_weight_count(const mb_ctx* c, int32_t ffn) {
    if (!c || ffn <= 0) return 0;
    const size_t h = (size_t)c->cfg.heads * mb::HD, f = (size_t)ffn;
    const size_t per_layer = 2 * h + h * 3 * h + 3 * h + h * h + h + 2 * h + h * f + f + f * h + h;
    return per_layer * c->cfg.layers + 2 * h;
}

MB_API int mb_decoder_destroy(mb_decoder* d) {
    if (!d) return MB_ERR_ARG;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(d->ctx->cfg.device);
    for (auto& kv : d->graphs) cudaGraphExecDestroy(kv.second);
    if (d->cap) cudaStreamDestroy(d->cap);
    if (d->side) cudaStreamDestroy(d->side);
    for (cudaEvent_t ev : {d->ev_fork, d->ev_stagger, d->ev_join})
        if (ev) cudaEventDestroy(ev);
    void* ptrs[] = {d->wmem, d->xb, d->qkv, d->h1, d->g_streams, d->g_positions, d->g_hidden};
    for (void* p : ptrs)
        if (p) cudaFree(p);
    if (prev >= 0) cudaSetDevice(prev);
    delete d;
    return MB_OK;
}

MB_API int mb_decoder_create(mb_ctx* c, int32_t ffn, const float* w, size_t count, mb_decoder** out) {
    if (!c || !w || !out || ffn <= 0 || ffn % 64) return MB_ERR_ARG;
    *out = nullptr;
    const int h = c->cfg.heads * mb::HD;
    if (h / 32 != 2 && h / 32 != 8 && h / 32 != 24) {
        c->last_error = "decoder: hidden width must be 64, 256 or 768";
        return MB_ERR_ARG;
    }
    if (count != mb_decoder_weight_count(c, ffn)) {
        c->last_error = "decoder: weight count does not match layers x (hidden, ffn)";
        return MB_ERR_ARG;
    }
    int prev = -1;
    cudaGetDevice(&prev);
    if (cudaSetDevice(c->cfg.device) != cudaSuccess) return MB_ERR_CUDA;
    mb_decoder* d = new mb_decoder();
    d->ctx = c;
    d->hid = h;
    d->ffn = ffn;
    d->layers = c->cfg.layers;
    auto bail = [&](int rc, const char* msg) {
        c->last_error = msg;
        mb_decoder_destroy(d);
        if (prev >= 0) cudaSetDevice(prev);
        return rc;
    };
    // device image: fp32 vectors first, then bf16 matrices (each block 256-byte aligned)
    // (a matrix [K][N] is stored transposed, W^T [N][K]: the GEMM's K-major B operand)
    struct Blk {
        size_t src, n;
        int K, N;  // K > 0: a matrix
        size_t dst;
    };
    std::vector<Blk> blks;
    size_t src = 0;
    auto add = [&](size_t n, int K = 0, int N = 0) {
        blks.push_back({src, n, K, N, 0});
        src += n;
    };
    for (int l = 0; l < d->layers; l++) {
        add(h), add(h);                                // ln1
        add((size_t)h * 3 * h, h, 3 * h), add(3 * h);  // c_attn
        add((size_t)h * h, h, h), add(h);              // c_proj
        add(h), add(h);                                // ln2
        add((size_t)h * ffn, h, ffn), add(ffn);        // fc_in
        add((size_t)ffn * h, ffn, h), add(h);          // fc_out
    }
    add(h), add(h);  // ln_f
    size_t bytes = 0;
    for (auto& b : blks) {
        b.dst = bytes;
        bytes += ((b.n * (b.K ? 2 : 4)) + 255) & ~size_t(255);
    }
    std::vector<unsigned char> img(bytes, 0);
    for (auto& b : blks) {
        if (b.K) {
            mb::dec::transpose_to_bf16(w + b.src, b.K, b.N, reinterpret_cast<uint16_t*>(img.data() + b.dst));
        } else {
            memcpy(img.data() + b.dst, w + b.src, b.n * 4);
        }
    }
    if (cudaMalloc(&d->wmem, bytes) != cudaSuccess) return bail(MB_ERR_OOM, "decoder: weight allocation failed");
    if (cudaMemcpy(d->wmem, img.data(), bytes, cudaMemcpyHostToDevice) != cudaSuccess)
        return bail(MB_ERR_CUDA, "decoder: weight upload failed");
    auto F = [&](size_t i) { return reinterpret_cast<const float*>((char*)d->wmem + blks[i].dst); };
    auto B = [&](size_t i) { return reinterpret_cast<const bf16*>((char*)d->wmem + blks[i].dst); };
    for (int l = 0; l < d->layers; l++) {
        const size_t o = (size_t)l * 12;
        d->L.push_back({F(o + 0), F(o + 1), F(o + 3), F(o + 5), F(o + 6), F(o + 7), F(o + 9), F(o + 11), B(o + 2),
                        B(o + 4), B(o + 8), B(o + 10)});
    }
    d->lnf_w = F(blks.size() - 2);
    d->lnf_b = F(blks.size() - 1);
    const size_t mb = c->cfg.max_batch;
    if (cudaMalloc(&d->xb, mb * h * sizeof(bf16)) != cudaSuccess ||
        cudaMalloc(&d->qkv, mb * 3 * h * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&d->h1, mb * ffn * sizeof(bf16)) != cudaSuccess || cudaMalloc(&d->g_streams, mb * 4) != cudaSuccess ||
        cudaMalloc(&d->g_positions, mb * 4) != cudaSuccess ||
        cudaMalloc(&d->g_hidden, mb * h * sizeof(float)) != cudaSuccess)
        return bail(MB_ERR_OOM, "decoder: activation allocation failed");
    if (cudaStreamCreateWithFlags(&d->cap, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&d->side, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&d->ev_fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&d->ev_stagger, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&d->ev_join, cudaEventDisableTiming) != cudaSuccess ||
        cudaDeviceGetStreamPriorityRange(&d->prio_low, &d->prio_high) != cudaSuccess)
        return bail(MB_ERR_CUDA, "decoder: stream creation failed");
    {
        const char* v = getenv("MOCKBIRD_DECODER_GRAPH");
        d->use_graph = !(v && strcmp(v, "0") == 0);
        v = getenv("MOCKBIRD_DECODER_SPLIT");
        d->split = !(v && strcmp(v, "0") == 0);
    }
    if (prev >= 0) cudaSetDevice(prev);
    *out = d;
    return MB_OK;
}

}  // extern "C"

namespace {

// One step over the staged inputs (d->g_streams, d->g_positions, d->g_hidden) on
// `st`: a replay of the step captured for this item count, or -- the first step
// of a count, or with graphs off -- the launches themselves (so kernel modules
// are loaded and tensor maps built outside any capture), after which the step is
// captured, without running, for the next calls.
int step_staged(mb_decoder* d, int n, cudaStream_t st) {
    if (!d->use_graph)
        return mb::dec::run(d, n, d->g_streams, d->g_positions, d->g_hidden, nullptr, st, false, true, true);
    auto it = d->graphs.find(n);
    cudaError_t e;
    if (it != d->graphs.end()) {
        e = cudaGraphLaunch(it->second, st);
        return e == cudaSuccess ? MB_OK : mb::dec::fail(d, MB_ERR_CUDA, std::string("decoder graph: ") + cudaGetErrorString(e));
    }
    int rc = mb::dec::run(d, n, d->g_streams, d->g_positions, d->g_hidden, nullptr, st, false, true, true);
    if (rc) return rc;
    cudaGraph_t g = nullptr;
    if ((e = cudaStreamBeginCapture(d->cap, cudaStreamCaptureModeThreadLocal)) != cudaSuccess)
        return mb::dec::fail(d, MB_ERR_CUDA, std::string("decoder capture: ") + cudaGetErrorString(e));
    const int rc2 = mb::dec::run(d, n, d->g_streams, d->g_positions, d->g_hidden, nullptr, d->cap, false, true, true);
    e = cudaStreamEndCapture(d->cap, &g);
    cudaGraphExec_t ex = nullptr;
    // A split step's kernel nodes carry the priorities they were launched with;
    // a one-chain step's graph runs at the priority of the stream it is launched on.
    const bool split = d->split && d->side && n / 2 >= mb::dec::SPLIT_MIN_ROWS;
    if (rc2 == MB_OK && e == cudaSuccess)
        e = cudaGraphInstantiate(&ex, g, split ? cudaGraphInstantiateFlagUseNodePriority : 0);
    if (g) cudaGraphDestroy(g);
    if (rc2 != MB_OK) return rc2;
    if (e != cudaSuccess) return mb::dec::fail(d, MB_ERR_CUDA, std::string("decoder capture: ") + cudaGetErrorString(e));
    d->graphs.emplace(n, ex);
    return MB_OK;
}

struct DevGuard {
    int prev = -1;
    bool ok = true;
    explicit DevGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DevGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

}  // namespace

extern "C" {

MB_API int mb_decoder_step(mb_decoder* d, int32_t n, const int32_t* streams, const int32_t* positions,
                           float* hidden, void* cuda_stream) {
    if (!d) return MB_ERR_ARG;
    mb_ctx* c = d->ctx;
    if (n < 0 || n > c->cfg.max_batch) return mb::dec::fail(d, MB_ERR_ARG, "decoder: item count out of range");
    if (n == 0) return MB_OK;
    if (!streams || !positions || !hidden || (reinterpret_cast<uintptr_t>(hidden) & 15))
        return mb::dec::fail(d, MB_ERR_ARG, "decoder: null or misaligned device pointer");
    DevGuard g(c->cfg.device);
    if (!g.ok) return MB_ERR_CUDA;
    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    if (!d->use_graph) return mb::dec::run(d, n, streams, positions, hidden, nullptr, st, false, true, true);
    // the captured step reads and writes this object's own buffers only
    const size_t hb = (size_t)n * d->hid * sizeof(float);
    cudaError_t e = cudaMemcpyAsync(d->g_streams, streams, n * 4, cudaMemcpyDeviceToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d->g_positions, positions, n * 4, cudaMemcpyDeviceToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d->g_hidden, hidden, hb, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return mb::dec::fail(d, MB_ERR_CUDA, std::string("decoder inputs: ") + cudaGetErrorString(e));
    const int rc = step_staged(d, n, st);
    if (rc) return rc;
    if ((e = cudaMemcpyAsync(hidden, d->g_hidden, hb, cudaMemcpyDeviceToDevice, st)) != cudaSuccess)
        return mb::dec::fail(d, MB_ERR_CUDA, std::string("decoder output: ") + cudaGetErrorString(e));
    return MB_OK;
}

MB_API int mb_decoder_step_host(mb_decoder* d, int32_t n, const int32_t* streams, const int32_t* positions,
                                float* hidden, void* cuda_stream) {
    if (!d) return MB_ERR_ARG;
    mb_ctx* c = d->ctx;
    if (n < 0 || n > c->cfg.max_batch) return mb::dec::fail(d, MB_ERR_ARG, "decoder: item count out of range");
    if (n == 0) return MB_OK;
    if (!streams || !positions || !hidden) return mb::dec::fail(d, MB_ERR_ARG, "decoder: null host pointer");
    int rc = mb::check_items_host(c, n, streams, positions);
    if (rc) return rc;
    DevGuard g(c->cfg.device);
    if (!g.ok) return MB_ERR_CUDA;
    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    // A previous call that failed after queueing its copies may have left them
    // reading the staging; nothing is reused before they are done.
    cudaError_t e = cudaEventSynchronize(c->ev_ids);
    if (e == cudaSuccess) {
        memcpy(c->h_ids, streams, n * sizeof(int32_t));
        memcpy(c->h_ids + n, positions, n * sizeof(int32_t));
        e = cudaMemcpyAsync(d->g_streams, c->h_ids, n * 4, cudaMemcpyHostToDevice, st);
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(d->g_positions, c->h_ids + n, n * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaEventRecord(c->ev_ids, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d->g_hidden, hidden, (size_t)n * d->hid * 4, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return mb::dec::fail(d, MB_ERR_CUDA, std::string("decoder inputs: ") + cudaGetErrorString(e));
    if ((rc = step_staged(d, n, st))) return rc;
    // ln_f of the last layer and the ring's device status word, then one wait
    e = cudaMemcpyAsync(hidden, d->g_hidden, (size_t)n * d->hid * 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(c->h_err, c->d_err, sizeof(int32_t), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return mb::dec::fail(d, MB_ERR_CUDA, std::string("decoder outputs: ") + cudaGetErrorString(e));
    return mb::report_bits(c, *c->h_err);
}

}  // extern "C"
