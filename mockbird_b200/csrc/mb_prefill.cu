// Prefill and ring-maintenance kernels.
//
// Reference semantics (liyu1981/mockbird, src/lib/tts/engine/):
//   ROPE_SPLIT_CACHE   kernels-batch.ts:194-234  (position = row, K/V -> cache, Q roped)
//   ATTENTION_SCORES / ATTENTION_SOFTMAX / ATTENTION_APPLY  kernels-batch.ts:246-350
//     (causal softmax(Q K^T * 0.125) V; the reference materialises [12, S, S]
//      scores and probabilities and applies them with one workgroup per head)
// Here the three attention passes are one flash-style kernel: scores never leave
// the chip.
#include <type_traits>

#include "mb_internal.cuh"

namespace mb {

template <typename T>
struct P2;
template <>
struct P2<float> {
    __device__ static void st(float* p, float2 v) { *reinterpret_cast<float2*>(p) = v; }
    __device__ static float2 ld(const float* p) { return *reinterpret_cast<const float2*>(p); }
    __device__ static float2 rnd(float2 v) { return v; }
};
template <>
struct P2<__nv_bfloat16> {
    __device__ static void st(__nv_bfloat16* p, float2 v) {
        *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(v.x, v.y);
    }
    __device__ static float2 ld(const __nv_bfloat16* p) {
        return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
    }
    __device__ static float2 rnd(float2 v) { return __bfloat1622float2(__floats2bfloat162_rn(v.x, v.y)); }
};
template <>
struct P2<__half> {
    __device__ static void st(__half* p, float2 v) { *reinterpret_cast<__half2*>(p) = __floats2half2_rn(v.x, v.y); }
    __device__ static float2 ld(const __half* p) { return __half22float2(*reinterpret_cast<const __half2*>(p)); }
    __device__ static float2 rnd(float2 v) { return __half22float2(__floats2half2_rn(v.x, v.y)); }
};

// Four consecutive elements in the storage type from two pairs: one 16-byte
// (fp32) or 8-byte (16-bit) store.
template <typename T>
__device__ __forceinline__ void st4(T* p, float2 a, float2 b) {
    if constexpr (sizeof(T) == 4) {
        *reinterpret_cast<float4*>(p) = make_float4(a.x, a.y, b.x, b.y);
    } else {
        T tmp[4];
        P2<T>::st(tmp, a);
        P2<T>::st(tmp + 2, b);
        *reinterpret_cast<uint2*>(p) = *reinterpret_cast<const uint2*>(tmp);
    }
}

// ---------------------------------------------------------------- prefill

// ROPE_SPLIT_CACHE for all rows of n items: grid (ceil(rows / ROPE_ROWS), n),
// heads * 16 threads, each owning 4 consecutive dims (two RoPE pairs) of one head
// in ROPE_ROWS consecutive rows: 16-byte loads of q, k, v and the (cos, sin) pairs.
// K roped and V raw go to slot = row.  For fp32 rings the roped Q, the roped K
// and V also go, each as two bf16 parts (hi = bf16(x), lo = bf16(x - hi)), to
// the stage [6][n][heads][rows][64] (Q hi, Q lo, K hi, K lo, V hi, V lo) that
// the tensor-core attention kernel loads; for 16-bit rings `split` is null and
// the attention kernel ropes Q itself as it loads it.  Block 0 of an item also
// marks the item's slots >= rows empty: a prefill starts an utterance at
// position 0.
constexpr int ROPE_ROWS = 4;

// Four consecutive values as bf16 parts: hi = bf16(x), lo = bf16(x - hi).
__device__ __forceinline__ void split4(float2 a, float2 b, __nv_bfloat16* hi, __nv_bfloat16* lo) {
    const __nv_bfloat162 h0 = __floats2bfloat162_rn(a.x, a.y), h1 = __floats2bfloat162_rn(b.x, b.y);
    const float2 f0 = __bfloat1622float2(h0), f1 = __bfloat1622float2(h1);
    const __nv_bfloat162 l0 = __floats2bfloat162_rn(a.x - f0.x, a.y - f0.y);
    const __nv_bfloat162 l1 = __floats2bfloat162_rn(b.x - f1.x, b.y - f1.y);
    *reinterpret_cast<uint2*>(hi) =
        make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
    *reinterpret_cast<uint2*>(lo) =
        make_uint2(*reinterpret_cast<const uint32_t*>(&l0), *reinterpret_cast<const uint32_t*>(&l1));
}

template <typename T>
__global__ void __launch_bounds__(1024) prefill_rope_kernel(RingView r, const int32_t* __restrict__ streams, int rows,
                                                            const float* __restrict__ qkv,
                                                            __nv_bfloat16* __restrict__ split) {
    // the attention kernel that follows may start its Q prologue now; it reads
    // what this kernel writes only after this grid has completed
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int item = blockIdx.y, r0 = blockIdx.x * ROPE_ROWS;
    const int s = streams[item];
    if (s < 0 || s >= r.streams) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(r.err, DERR_STREAM);
        return;
    }
    const int H = r.heads, HID = H * HD, C = r.capacity;
    const int t = threadIdx.x, h = t >> 4, d4 = (t & 15) * 4;  // head, first of 4 dims
    const int rend = min(r0 + ROPE_ROWS, rows);
    T* kbase = reinterpret_cast<T*>(r.kv) + (((size_t)s * 2 + 0) * H + h) * (size_t)C * HD + d4;
    T* vbase = reinterpret_cast<T*>(r.kv) + (((size_t)s * 2 + 1) * H + h) * (size_t)C * HD + d4;
    // part p of this (item, head): plane p * n * H + item * H + h of the stage
    const size_t plane = (size_t)rows * HD, pstride = (size_t)gridDim.y * H * plane;
    __nv_bfloat16* sbase = sizeof(T) == 4 ? split + ((size_t)item * H + h) * plane + d4 : nullptr;
    for (int row = r0; row < rend; row++) {
        const float* src = qkv + ((size_t)item * rows + row) * 3 * HID + h * HD + d4;
        const float4 cs = *reinterpret_cast<const float4*>(r.rope + (size_t)row * 32 + d4 / 2);
        const float4 k = *reinterpret_cast<const float4*>(src + HID);
        const float4 v = *reinterpret_cast<const float4*>(src + 2 * HID);
        const float2 c0 = make_float2(cs.x, cs.y), c1 = make_float2(cs.z, cs.w);
        const float2 k0 = rope_pair(make_float2(k.x, k.y), c0), k1 = rope_pair(make_float2(k.z, k.w), c1);
        st4(kbase + (size_t)row * HD, k0, k1);
        st4(vbase + (size_t)row * HD, make_float2(v.x, v.y), make_float2(v.z, v.w));
        if constexpr (sizeof(T) == 4) {  // only fp32 rings have a stage (16-bit rings keep 32 registers)
            const float4 q = *reinterpret_cast<const float4*>(src);
            __nv_bfloat16* o = sbase + (size_t)row * HD;
            split4(rope_pair(make_float2(q.x, q.y), c0), rope_pair(make_float2(q.z, q.w), c1), o, o + pstride);
            split4(k0, k1, o + 2 * pstride, o + 3 * pstride);
            split4(make_float2(v.x, v.y), make_float2(v.z, v.w), o + 4 * pstride, o + 5 * pstride);
        }
    }
    if (t < rend - r0) r.slot_pos[(size_t)s * C + r0 + t] = r0 + t;
    if (blockIdx.x == 0)
        for (int j = rows + t; j < C; j += blockDim.x) r.slot_pos[(size_t)s * C + j] = -1;
}

size_t prefill_stage_bytes(int dtype, int n, int heads, int rows) {
    // fp32 rings: Q, K and V as bf16 hi/lo parts; 16-bit rings rope Q in the attention kernel
    return dtype == MB_F32 ? (size_t)6 * n * heads * rows * HD * 2 : 0;
}

template <typename T>
static cudaError_t prefill_t(const RingView& r, int n, const int32_t* streams, int rows, const float* qkv,
                             float* out, void* stage, cudaStream_t st) {
    if (r.heads * 16 > 1024) return cudaErrorInvalidConfiguration;
    constexpr bool F32 = sizeof(T) == 4;
    prefill_rope_kernel<T><<<dim3((rows + ROPE_ROWS - 1) / ROPE_ROWS, n), r.heads * 16, 0, st>>>(
        r, streams, rows, qkv, F32 ? static_cast<__nv_bfloat16*>(stage) : nullptr);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if constexpr (F32)  // split bf16 parts on the tensor cores (mb_prefill_tc.cu)
        return launch_prefill_attn_split(r, n, streams, rows, stage, out, st);
    // 16-bit rings: tensor cores (mb_prefill_tc.cu), Q roped there
    return launch_prefill_attn_tc(std::is_same<T, __nv_bfloat16>::value ? MB_BF16 : MB_F16, r, n, streams, rows,
                                  qkv, out, st);
}

cudaError_t launch_prefill(int dtype, const RingView& r, int n, const int32_t* streams, int rows,
                           const float* qkv, float* out, void* stage, cudaStream_t st) {
    switch (dtype) {
        case MB_F32: return prefill_t<float>(r, n, streams, rows, qkv, out, stage, st);
        case MB_BF16: return prefill_t<__nv_bfloat16>(r, n, streams, rows, qkv, out, stage, st);
        default: return prefill_t<__half>(r, n, streams, rows, qkv, out, stage, st);
    }
}

// ---------------------------------------------------------------- gather / write / reset

// Live window in position order (PrefillRunner.readLayerCache, prefill.ts:644-664,
// generalised to the wrap): grid (W), 256 threads.
template <typename T>
__global__ void gather_kernel(RingView r, int s, int cur, int W, T* k_out, T* v_out, int32_t* slots_out) {
    const int w = blockIdx.x;
    const int H = r.heads, C = r.capacity;
    const int p = cur - W + 1 + w, slot = p % C;
    const bool ok = r.slot_pos[(size_t)s * C + slot] == p;
    if (threadIdx.x == 0) slots_out[w] = ok ? slot : -1;
    for (int e = threadIdx.x; e < H * HD; e += blockDim.x) {
        const int h = e / HD, d = e % HD;
        const T* kb = reinterpret_cast<const T*>(r.kv) + (((size_t)s * 2 + 0) * H + h) * (size_t)C * HD;
        const T* vb = reinterpret_cast<const T*>(r.kv) + (((size_t)s * 2 + 1) * H + h) * (size_t)C * HD;
        const size_t o = ((size_t)h * W + w) * HD + d;
        k_out[o] = ok ? kb[(size_t)slot * HD + d] : T(0.f);
        v_out[o] = ok ? vb[(size_t)slot * HD + d] : T(0.f);
    }
}

// Write rows [heads][count][64] at positions first.. (prefill.ts:610-620 poisonKv).
template <typename T>
__global__ void ring_write_kernel(RingView r, int s, int first, int count, const T* k, const T* v) {
    const int w = blockIdx.x;
    const int H = r.heads, C = r.capacity;
    const int p = first + w, slot = p % C;
    for (int e = threadIdx.x; e < H * HD; e += blockDim.x) {
        const int h = e / HD, d = e % HD;
        T* kb = reinterpret_cast<T*>(r.kv) + (((size_t)s * 2 + 0) * H + h) * (size_t)C * HD;
        T* vb = reinterpret_cast<T*>(r.kv) + (((size_t)s * 2 + 1) * H + h) * (size_t)C * HD;
        const size_t i = ((size_t)h * count + w) * HD + d;
        kb[(size_t)slot * HD + d] = k[i];
        vb[(size_t)slot * HD + d] = v[i];
    }
    if (threadIdx.x == 0) r.slot_pos[(size_t)s * C + slot] = p;
}

template <typename T>
static cudaError_t gather_t(const RingView& r, int stream, int position, void* k_out, void* v_out,
                            int32_t* slots_out, cudaStream_t st) {
    const int W = min(position + 1, r.capacity);
    gather_kernel<T><<<W, 256, 0, st>>>(r, stream, position, W, reinterpret_cast<T*>(k_out),
                                        reinterpret_cast<T*>(v_out), slots_out);
    return cudaGetLastError();
}

cudaError_t launch_gather(int dtype, const RingView& r, int stream, int position, void* k_out, void* v_out,
                          int32_t* slots_out, cudaStream_t st) {
    switch (dtype) {
        case MB_F32: return gather_t<float>(r, stream, position, k_out, v_out, slots_out, st);
        case MB_BF16: return gather_t<__nv_bfloat16>(r, stream, position, k_out, v_out, slots_out, st);
        default: return gather_t<__half>(r, stream, position, k_out, v_out, slots_out, st);
    }
}

template <typename T>
static cudaError_t write_t(const RingView& r, int stream, int first, int count, const void* k, const void* v,
                           cudaStream_t st) {
    ring_write_kernel<T><<<count, 256, 0, st>>>(r, stream, first, count, reinterpret_cast<const T*>(k),
                                                reinterpret_cast<const T*>(v));
    return cudaGetLastError();
}

cudaError_t launch_ring_write(int dtype, const RingView& r, int stream, int first, int count, const void* k,
                              const void* v, cudaStream_t st) {
    switch (dtype) {
        case MB_F32: return write_t<float>(r, stream, first, count, k, v, st);
        case MB_BF16: return write_t<__nv_bfloat16>(r, stream, first, count, k, v, st);
        default: return write_t<__half>(r, stream, first, count, k, v, st);
    }
}

// slot_pos <- -1 for one stream (all layers) or for all streams; int32 -1 is
// the byte pattern 0xFF, so a (2-D) memset does it.
cudaError_t launch_reset(const mb_ctx* c, int stream, cudaStream_t st) {
    const size_t row = (size_t)c->cfg.capacity * sizeof(int32_t);
    if (stream < 0)
        return cudaMemsetAsync(c->slot_pos, 0xFF, row * c->cfg.streams * c->cfg.layers, st);
    return cudaMemset2DAsync(c->slot_pos + (size_t)stream * c->cfg.capacity, row * c->cfg.streams, 0xFF, row,
                             c->cfg.layers, st);
}

}  // namespace mb
