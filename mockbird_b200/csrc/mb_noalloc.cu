// mb_append_attend_noalloc: the fused decode (append + RoPE + split-K attention)
// for callers that cannot allocate device memory.  The caller owns the ring, the
// RoPE table, the inputs, the outputs and a status word; the split-K partials
// live in one fixed device array defined in this file.
#include <mutex>

#include "mb_internal.cuh"

namespace {

// Scratch of every no-allocation call on a device.  Loaded with the library's
// device code, held until the process exits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[MB_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_addr[kMaxDevices] = {};

// Host code cannot use g_noalloc_scratch as a device address (on the host it
// names a stand-in); look up the device address once per device, with that
// device current.  The address belongs to the device's primary context: a
// cudaDeviceReset while the library is loaded would leave it stale.
int scratch_address(int device, void** out) {
    if (device < 0 || device >= kMaxDevices) return MB_ERR_ARG;
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_addr[device]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return MB_ERR_CUDA;
        g_scratch_addr[device] = p;
    }
    *out = g_scratch_addr[device];
    return MB_OK;
}

size_t round256(size_t b) { return (b + 255) & ~size_t(255); }

}  // namespace

extern "C" MB_API int mb_append_attend_noalloc(const mb_ring_ref* ring, int32_t layer, int32_t n,
                                               const int32_t* streams, const int32_t* positions, const float* qkv,
                                               float* out, void* cuda_stream) {
    if (!ring || !ring->kv || !ring->slot_pos || !ring->rope || !ring->status) return MB_ERR_ARG;
    if (ring->layers <= 0 || ring->heads <= 0 || ring->heads > 64 || ring->capacity <= 0 || ring->streams <= 0 ||
        ring->max_position <= 0 || ring->dtype < MB_F32 || ring->dtype > MB_F16)
        return MB_ERR_ARG;
    if (layer < 0 || layer >= ring->layers) return MB_ERR_LAYER;
    if (n < 0 || n > 65535) return MB_ERR_ARG;
    if (n == 0) return MB_OK;
    // the kernel reads qkv and the ring 16 bytes at a time, the RoPE table as
    // (cos, sin) float2 pairs, and stream ids, positions, slot positions and the
    // status word as int32 (the status by atomics): misaligned pointers are
    // rejected here rather than faulting on the device
    auto mis = [](const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) != 0; };
    if (!streams || !positions || !qkv || !out || mis(qkv, 16) || mis(out, 16) || mis(ring->kv, 16) ||
        mis(ring->rope, 8) || mis(ring->slot_pos, 4) || mis(ring->status, 4) || mis(streams, 4) ||
        mis(positions, 4))
        return MB_ERR_ARG;

    // scratch needed by this call: the split-K partials (written by the decode
    // kernel and read back by its combine kernel within the call)
    const int rows = mb::chunk_rows(ring->dtype);
    const int max_splits = (ring->capacity + rows - 1) / rows;
    const size_t part_bytes = round256((size_t)n * ring->heads * max_splits * (2 + mb::HD) * sizeof(float));
    if (part_bytes > MB_NOALLOC_SCRATCH_BYTES) return MB_ERR_ARG;

    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return MB_ERR_CUDA;
    void* base = nullptr;
    int rc = scratch_address(device, &base);
    if (rc) return rc;

    mb::Scratch sc;
    sc.part = static_cast<float*>(base);
    sc.counters = nullptr;  // the per-chunk decode kernel takes no tickets
    sc.max_splits = max_splits;

    mb::RingView v;
    const size_t esize = ring->dtype == MB_F32 ? 4 : 2;
    const size_t per_layer = (size_t)ring->streams * 2 * ring->heads * (size_t)ring->capacity * mb::HD;
    v.kv = static_cast<char*>(ring->kv) + per_layer * layer * esize;
    v.slot_pos = ring->slot_pos + (size_t)layer * ring->streams * ring->capacity;
    v.rope = reinterpret_cast<const float2*>(ring->rope);
    v.err = ring->status;
    v.streams = ring->streams;
    v.heads = ring->heads;
    v.capacity = ring->capacity;
    v.wrap = ring->wrap;
    v.max_position = ring->max_position;
    v.kv_layer = per_layer;
    v.slot_layer = (size_t)ring->streams * ring->capacity;
    v.wait_limit = mb::WAIT_LIMIT;
    v.wait_probe = 0;

    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    // the array keeps the previous call's contents; every partial the combine
    // reads is written by this call's decode kernel first, so nothing is cleared
    if (mb::launch_decode(ring->dtype, true, v, sc, n, streams, positions, qkv, 3 * ring->heads * mb::HD, out, st) !=
        cudaSuccess)
        return MB_ERR_CUDA;
    return MB_OK;
}
