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
// K roped and V raw go to slot = row.  For fp32 rings the roped Q goes to the
// stage [n][heads][rows][64]; for 16-bit rings q_stage is null and the
// tensor-core attention kernel ropes Q itself as it loads it.  Block 0 of an item
// also marks the item's slots >= rows empty: a prefill starts an utterance at
// position 0.
constexpr int ROPE_ROWS = 4;

template <typename T>
__global__ void __launch_bounds__(1024) prefill_rope_kernel(RingView r, const int32_t* __restrict__ streams, int rows,
                                                            const float* __restrict__ qkv, T* q_stage) {
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
    T* qbase = q_stage ? q_stage + ((size_t)item * H + h) * rows * HD + d4 : nullptr;
    for (int row = r0; row < rend; row++) {
        const float* src = qkv + ((size_t)item * rows + row) * 3 * HID + h * HD + d4;
        const float4 cs = *reinterpret_cast<const float4*>(r.rope + (size_t)row * 32 + d4 / 2);
        const float4 k = *reinterpret_cast<const float4*>(src + HID);
        const float4 v = *reinterpret_cast<const float4*>(src + 2 * HID);
        const float2 c0 = make_float2(cs.x, cs.y), c1 = make_float2(cs.z, cs.w);
        if (q_stage) {
            const float4 q = *reinterpret_cast<const float4*>(src);
            st4(qbase + (size_t)row * HD, rope_pair(make_float2(q.x, q.y), c0), rope_pair(make_float2(q.z, q.w), c1));
        }
        st4(kbase + (size_t)row * HD, rope_pair(make_float2(k.x, k.y), c0), rope_pair(make_float2(k.z, k.w), c1));
        st4(vbase + (size_t)row * HD, make_float2(v.x, v.y), make_float2(v.z, v.w));
    }
    if (t < rend - r0) r.slot_pos[(size_t)s * C + r0 + t] = r0 + t;
    if (blockIdx.x == 0)
        for (int j = rows + t; j < C; j += blockDim.x) r.slot_pos[(size_t)s * C + j] = -1;
}

// Causal flash attention on CUDA cores for fp32 rings (kind::f16 tensor cores
// take 16-bit operands, and tf32 would not meet the fp32 tolerance), blocked the
// way a CUDA-core GEMM is: grid (ceil(rows/64), heads, n), 256 threads; thread
// (tq, tk) = (t / 16, t % 16) owns a 4 x 4 block of the 64 x 64 score tile (query
// rows 4tq.., key columns 4tk..) and a 4 x 4 block of the 64 x 64 output (query
// rows 4tq.., dims 4tk..).  Q and K are staged transposed ([dim][row]) and V
// as rows, so each dimension (key) step of QK^T (PV) is two 16-byte shared
// loads and 16 FMAs.  Row maxima and sums reduce over the 16 threads of a
// half-warp; P goes through shared memory transposed ([key][query]).
namespace simt {
constexpr int BQ = 64, BK = 64, LD = 68;  // tile rows; padded row length (floats)
struct Smem {
    float q[HD][LD];   // Q^T, pre-scaled by 0.125 * log2(e)
    float k[HD][LD];   // K^T of the key tile
    float v[BK][LD];   // V rows of the key tile
    float p[BK][LD];   // P^T
};
}  // namespace simt

__global__ void __launch_bounds__(256) prefill_attn_simt_kernel(RingView r, const int32_t* __restrict__ streams,
                                                                int rows, const float* __restrict__ q_stage,
                                                                float* __restrict__ out) {
    using namespace simt;
    extern __shared__ __align__(16) unsigned char simt_raw[];
    Smem& sm = *reinterpret_cast<Smem*>(simt_raw);
    const int qt = blockIdx.x, h = blockIdx.y, item = blockIdx.z, t = threadIdx.x;
    const int s = streams[item];
    if (s < 0 || s >= r.streams) return;
    const int H = r.heads, C = r.capacity, q0 = qt * BQ;
    const int tq = t >> 4, tk = t & 15;
    const float* qg = q_stage + ((size_t)item * H + h) * rows * HD;
    const float* kb = reinterpret_cast<const float*>(r.kv) + (((size_t)s * 2 + 0) * H + h) * (size_t)C * HD;
    const float* vb = reinterpret_cast<const float*>(r.kv) + (((size_t)s * 2 + 1) * H + h) * (size_t)C * HD;

    // Q^T, scaled (rows past `rows` read as 0).  A warp covers 8 rows x 4 chunks
    // of 16 bytes: 64-byte global segments, 2-way conflicts on the transposed stores.
    for (int e = t; e < BQ * HD / 4; e += 256) {
        const int row = ((e >> 5) & 7) * 8 + (e & 7), d = (((e >> 8) * 4) + ((e >> 3) & 3)) * 4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (q0 + row < rows) v = *reinterpret_cast<const float4*>(qg + (size_t)(q0 + row) * HD + d);
        const float sc = SCALE * LOG2E;
        sm.q[d][row] = v.x * sc;
        sm.q[d + 1][row] = v.y * sc;
        sm.q[d + 2][row] = v.z * sc;
        sm.q[d + 3][row] = v.w * sc;
    }
    float o[4][4], m[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        m[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int j = 0; j < 4; j++) o[i][j] = 0.f;
    }
    const int last_key = min(rows, q0 + BQ);  // keys [0, last_key) are needed by this tile
    for (int k0 = 0; k0 < last_key; k0 += BK) {
        __syncthreads();  // the previous tile's K, V and P are consumed (and Q^T is written)
        for (int e = t; e < BK * HD / 4; e += 256) {
            const int j = ((e >> 5) & 7) * 8 + (e & 7), d = (((e >> 8) * 4) + ((e >> 3) & 3)) * 4;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (k0 + j < rows) {
                kv = *reinterpret_cast<const float4*>(kb + (size_t)(k0 + j) * HD + d);
                vv = *reinterpret_cast<const float4*>(vb + (size_t)(k0 + j) * HD + d);
            }
            sm.k[d][j] = kv.x;
            sm.k[d + 1][j] = kv.y;
            sm.k[d + 2][j] = kv.z;
            sm.k[d + 3][j] = kv.w;
            *reinterpret_cast<float4*>(&sm.v[j][d]) = vv;
        }
        __syncthreads();
        // ---- S block: rows 4tq.., keys 4tk..
        float sc[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) sc[i][j] = 0.f;
#pragma unroll 8
        for (int d = 0; d < HD; d++) {
            const float4 qa = *reinterpret_cast<const float4*>(&sm.q[d][4 * tq]);
            const float4 ka = *reinterpret_cast<const float4*>(&sm.k[d][4 * tk]);
            const float qv[4] = {qa.x, qa.y, qa.z, qa.w}, kv[4] = {ka.x, ka.y, ka.z, ka.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) sc[i][j] = fmaf(qv[i], kv[j], sc[i][j]);
        }
        // ---- causal mask (key <= query, key < rows), row maxima over the half-warp
        float mnew[4], corr[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int qi = q0 + 4 * tq + i;
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int kj = k0 + 4 * tk + j;
                if (kj > qi || kj >= rows) sc[i][j] = -INFINITY;
                mx = fmaxf(mx, sc[i][j]);
            }
#pragma unroll
            for (int o2 = 8; o2 > 0; o2 >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o2));
            mnew[i] = fmaxf(m[i], mx);
            // a row with nothing live yet keeps m = -inf: its p and corr stay 0
            corr[i] = mnew[i] == -INFINITY ? 1.f : exp2f(m[i] - mnew[i]);
        }
        // ---- P = 2^(s - m), row sums, P^T to shared memory
        float ps[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float sum = 0.f;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                ps[i][j] = sc[i][j] == -INFINITY ? 0.f : exp2f(sc[i][j] - mnew[i]);
                sum += ps[i][j];
            }
#pragma unroll
            for (int o2 = 8; o2 > 0; o2 >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o2);
            l[i] = l[i] * corr[i] + sum;
            m[i] = mnew[i];
#pragma unroll
            for (int j = 0; j < 4; j++) o[i][j] *= corr[i];
        }
#pragma unroll
        for (int j = 0; j < 4; j++)
            *reinterpret_cast<float4*>(&sm.p[4 * tk + j][4 * tq]) = make_float4(ps[0][j], ps[1][j], ps[2][j], ps[3][j]);
        __syncthreads();
        // ---- O block += P V: rows 4tq.., dims 4tk..
        const int kend = min(BK, last_key - k0);
#pragma unroll 8
        for (int kk = 0; kk < kend; kk++) {
            const float4 pa = *reinterpret_cast<const float4*>(&sm.p[kk][4 * tq]);
            const float4 va = *reinterpret_cast<const float4*>(&sm.v[kk][4 * tk]);
            const float pv[4] = {pa.x, pa.y, pa.z, pa.w}, vv[4] = {va.x, va.y, va.z, va.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) o[i][j] = fmaf(pv[i], vv[j], o[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int qi = q0 + 4 * tq + i;
        if (qi < rows) {
            const float inv = 1.f / l[i];
            *reinterpret_cast<float4*>(out + ((size_t)item * rows + qi) * H * HD + h * HD + 4 * tk) =
                make_float4(o[i][0] * inv, o[i][1] * inv, o[i][2] * inv, o[i][3] * inv);
        }
    }
}

size_t prefill_stage_bytes(int dtype, int n, int heads, int rows) {
    return dtype == MB_F32 ? (size_t)n * heads * rows * HD * 4 : 0;  // 16-bit rings rope Q in the attention kernel
}

template <typename T>
static cudaError_t prefill_t(const RingView& r, int n, const int32_t* streams, int rows, const float* qkv,
                             float* out, void* q_stage, cudaStream_t st) {
    if (r.heads * 16 > 1024) return cudaErrorInvalidConfiguration;
    prefill_rope_kernel<T><<<dim3((rows + ROPE_ROWS - 1) / ROPE_ROWS, n), r.heads * 16, 0, st>>>(
        r, streams, rows, qkv, sizeof(T) == 4 ? reinterpret_cast<T*>(q_stage) : nullptr);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if constexpr (sizeof(T) == 2)  // 16-bit rings: tensor cores (mb_prefill_tc.cu), Q roped there
        return launch_prefill_attn_tc(std::is_same<T, __nv_bfloat16>::value ? MB_BF16 : MB_F16, r, n, streams, rows,
                                      qkv, out, st);
    if constexpr (sizeof(T) == 4) {
        static bool attr_set[64] = {};  // per device
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
        if (!attr_set[dev]) {
            e = cudaFuncSetAttribute(prefill_attn_simt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)sizeof(simt::Smem));
            if (e != cudaSuccess) return e;
            attr_set[dev] = true;
        }
        prefill_attn_simt_kernel<<<dim3((rows + simt::BQ - 1) / simt::BQ, r.heads, n), 256, sizeof(simt::Smem), st>>>(
            r, streams, rows, reinterpret_cast<const float*>(q_stage), out);
    }
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
