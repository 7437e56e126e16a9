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

__device__ __forceinline__ float2 rope_pair_p(float2 v, float2 cs) {
    return make_float2(__fadd_rn(__fmul_rn(v.x, cs.x), -__fmul_rn(v.y, cs.y)),
                       __fadd_rn(__fmul_rn(v.y, cs.x), __fmul_rn(v.x, cs.y)));
}

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
// K roped and V raw go to slot = row; the roped Q goes to the stage
// [n][heads][rows][64] (rounded to the storage dtype for 16-bit rings: the
// attention kernel consumes Q in that type).  Block 0 of an item also marks the
// item's slots >= rows empty: a prefill starts an utterance at position 0.
constexpr int ROPE_ROWS = 4;

template <typename T>
__global__ void __launch_bounds__(1024) prefill_rope_kernel(RingView r, const int32_t* __restrict__ streams, int rows,
                                                            const float* __restrict__ qkv, T* q_stage) {
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
    T* qbase = q_stage + ((size_t)item * H + h) * rows * HD + d4;
    for (int row = r0; row < rend; row++) {
        const float* src = qkv + ((size_t)item * rows + row) * 3 * HID + h * HD + d4;
        const float4 cs = *reinterpret_cast<const float4*>(r.rope + (size_t)row * 32 + d4 / 2);
        const float4 q = *reinterpret_cast<const float4*>(src);
        const float4 k = *reinterpret_cast<const float4*>(src + HID);
        const float4 v = *reinterpret_cast<const float4*>(src + 2 * HID);
        const float2 c0 = make_float2(cs.x, cs.y), c1 = make_float2(cs.z, cs.w);
        st4(qbase + (size_t)row * HD, rope_pair_p(make_float2(q.x, q.y), c0), rope_pair_p(make_float2(q.z, q.w), c1));
        st4(kbase + (size_t)row * HD, rope_pair_p(make_float2(k.x, k.y), c0), rope_pair_p(make_float2(k.z, k.w), c1));
        st4(vbase + (size_t)row * HD, make_float2(v.x, v.y), make_float2(v.z, v.w));
    }
    if (t < rend - r0) r.slot_pos[(size_t)s * C + r0 + t] = r0 + t;
    if (blockIdx.x == 0)
        for (int j = rows + t; j < C; j += blockDim.x) r.slot_pos[(size_t)s * C + j] = -1;
}

// Causal flash attention on CUDA cores for fp32 rings (kind::f16 tensor cores
// take 16-bit operands; 16-bit rings use mb_prefill_tc.cu): grid (ceil(rows/64),
// heads, n), 128 threads = 64 queries x 2 halves of the head dim.  K/V tiles of 64
// slots are staged in shared memory as fp32; each query keeps its running max /
// sum and 32 accumulators.
template <typename T>
__global__ void __launch_bounds__(128) prefill_attn_simt_kernel(RingView r, const int32_t* __restrict__ streams,
                                                                int rows, const T* __restrict__ q_stage,
                                                                float* __restrict__ out) {
    __shared__ __align__(16) float ks[64][HD];
    __shared__ __align__(16) float vs[64][HD];
    const int qt = blockIdx.x, h = blockIdx.y, item = blockIdx.z, tid = threadIdx.x;
    const int s = streams[item];
    if (s < 0 || s >= r.streams) return;
    const int H = r.heads, C = r.capacity;
    const int qi = qt * 64 + (tid >> 1), half = tid & 1;
    const bool active = qi < rows;
    float q[32];
#pragma unroll
    for (int d = 0; d < 32; d++) q[d] = 0.f;
    if (active) {
        const T* qp = q_stage + (((size_t)item * H + h) * rows + qi) * HD + half * 32;
#pragma unroll
        for (int d = 0; d < 32; d += 2) {
            float2 v = P2<T>::ld(qp + d);
            q[d] = v.x * (SCALE * LOG2E);
            q[d + 1] = v.y * (SCALE * LOG2E);
        }
    }
    float acc[32];
#pragma unroll
    for (int d = 0; d < 32; d++) acc[d] = 0.f;
    float m = -INFINITY, l = 0.f;
    const T* kb = reinterpret_cast<const T*>(r.kv) + (((size_t)s * 2 + 0) * H + h) * (size_t)C * HD;
    const T* vb = reinterpret_cast<const T*>(r.kv) + (((size_t)s * 2 + 1) * H + h) * (size_t)C * HD;
    const int last_key = min(rows, qt * 64 + 64);  // keys [0, last_key) are needed by this tile
    for (int k0 = 0; k0 < last_key; k0 += 64) {
        __syncthreads();
        for (int e = tid * 2; e < 64 * HD; e += 256) {
            const int j = e / HD, d = e % HD;
            float2 kv = make_float2(0.f, 0.f), vv = make_float2(0.f, 0.f);
            if (k0 + j < rows) {
                kv = P2<T>::ld(kb + (size_t)(k0 + j) * HD + d);
                vv = P2<T>::ld(vb + (size_t)(k0 + j) * HD + d);
            }
            ks[j][d] = kv.x;
            ks[j][d + 1] = kv.y;
            vs[j][d] = vv.x;
            vs[j][d + 1] = vv.y;
        }
        __syncthreads();
        // groups of 8 keys: 8 scores, one rescale of the accumulators, then 8
        // exponentials and P.V.  Uniform trip counts (the pair shuffle needs the
        // whole warp); the causal mask key <= query is applied per thread.
        const int jend = min(64, last_key - k0);
        for (int j0 = 0; j0 < jend; j0 += 8) {
            float sc[8];
            float gmax = -INFINITY;
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int j = j0 + u;
                float sdot = 0.f;
                if (j < jend) {
#pragma unroll
                    for (int d = 0; d < 32; d++) sdot = fmaf(q[d], ks[j][half * 32 + d], sdot);
                }
                sdot += __shfl_xor_sync(0xffffffffu, sdot, 1);
                sc[u] = (active && j < jend && k0 + j <= qi) ? sdot : -INFINITY;
                gmax = fmaxf(gmax, sc[u]);
            }
            if (gmax != -INFINITY) {
                const float mn = fmaxf(m, gmax);
                const float corr = exp2f(m - mn);  // 0 on the first live group (m = -inf)
                l *= corr;
#pragma unroll
                for (int d = 0; d < 32; d++) acc[d] *= corr;
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    const float p = exp2f(sc[u] - mn);  // 0 for masked keys
                    l += p;
                    if (j0 + u < jend) {
#pragma unroll
                        for (int d = 0; d < 32; d++) acc[d] = fmaf(p, vs[j0 + u][half * 32 + d], acc[d]);
                    }
                }
                m = mn;
            }
        }
    }
    if (active) {
        float* o = out + ((size_t)item * rows + qi) * H * HD + h * HD + half * 32;
        const float inv = 1.f / l;
#pragma unroll
        for (int d = 0; d < 32; d += 4)
            *reinterpret_cast<float4*>(o + d) = make_float4(acc[d] * inv, acc[d + 1] * inv, acc[d + 2] * inv,
                                                            acc[d + 3] * inv);
    }
}

size_t prefill_stage_bytes(int dtype, int n, int heads, int rows) {
    return (size_t)n * heads * rows * HD * (dtype == MB_F32 ? 4 : 2);
}

template <typename T>
static cudaError_t prefill_t(const RingView& r, int n, const int32_t* streams, int rows, const float* qkv,
                             float* out, void* q_stage, cudaStream_t st) {
    if (r.heads * 16 > 1024) return cudaErrorInvalidConfiguration;
    prefill_rope_kernel<T><<<dim3((rows + ROPE_ROWS - 1) / ROPE_ROWS, n), r.heads * 16, 0, st>>>(
        r, streams, rows, qkv, reinterpret_cast<T*>(q_stage));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if constexpr (sizeof(T) == 2)  // 16-bit rings: tensor cores (mb_prefill_tc.cu)
        return launch_prefill_attn_tc(std::is_same<T, __nv_bfloat16>::value ? MB_BF16 : MB_F16, r, n, streams, rows,
                                      q_stage, out, st);
    prefill_attn_simt_kernel<T><<<dim3((rows + 63) / 64, r.heads, n), 128, 0, st>>>(
        r, streams, rows, reinterpret_cast<const T*>(q_stage), out);
    return cudaGetLastError();
}

cudaError_t launch_prefill(int dtype, const RingView& r, int n, const int32_t* streams, int rows,
                           const float* qkv, float* out, void* q_stage, cudaStream_t st) {
    switch (dtype) {
        case MB_F32: return prefill_t<float>(r, n, streams, rows, qkv, out, q_stage, st);
        case MB_BF16: return prefill_t<__nv_bfloat16>(r, n, streams, rows, qkv, out, q_stage, st);
        default: return prefill_t<__half>(r, n, streams, rows, qkv, out, q_stage, st);
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
