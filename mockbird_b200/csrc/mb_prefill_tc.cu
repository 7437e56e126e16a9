// Causal prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM)
// for 16-bit rings: the ATTENTION_SCORES / _SOFTMAX / _APPLY passes of the
// reference (kernels-batch.ts:246-350) as one flash-attention kernel.
//
// One CTA = 128 queries of one (item, head); 8 warps: warps w and w+4 read TMEM
// lanes 32(w%4).. (query rows), w/4 picks the half of the key columns (and of
// the output dims) a thread owns.  Per 128-key tile j (causal: j <= query tile):
//   S = Q K^T   tcgen05.mma kind::f16, M=128 N=128 K=64, fp32 into TMEM cols [0,128)
//   softmax     tcgen05.ld S into registers, row max across the two halves in
//               shared memory, exp2 with four independent partial sums, P (16-bit)
//               written to shared memory in the 128-byte-swizzled K-major layout;
//               tiles with no masked key skip the mask
//   O_j = P V   tcgen05.mma, M=128 N=64 K=128 (V as an MN-major operand), TMEM cols [128,192)
//   O = O*corr + O_j in registers
// At the end O is normalised, staged in the free P buffers (128-byte swizzle)
// and written by two TMA tile stores (rows past the last are clipped).
// The tensor pipe runs the next tile's S behind the current PV: once the softmax
// of tile j has read S_j and written P_j, one thread issues O_j = P_j V_j and then
// S_{j+1} = Q K_{j+1}^T into the same TMEM columns, each with its own commit
// barrier, so S_{j+1} is computed while the CTA reads O_j back.  (Issuing S_{j+1}
// before the softmax of tile j, into a second TMEM buffer, was measured slower:
// it queues in front of PV_j.)  Q, K, V arrive by 3-D TMA tile loads (128-byte
// swizzle, zero fill past the last row, no multicast); K is double-buffered and
// fetched two tiles ahead, V one tile ahead.  96 KB of shared memory and 256
// TMEM columns per CTA: two CTAs share an SM.  Every wait is bounded; a CTA that
// gives up flags MB_ERR_TIMEOUT, waits (bounded) for its copies and MMAs in
// flight, and frees its TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "mb_internal.cuh"
#include "mb_ptx.cuh"

namespace mb {
namespace {

constexpr int BM = 128;                   // queries per CTA (UMMA M)
constexpr int BN = 128;                   // keys per tile
constexpr int TILE = BM * HD * 2;         // [128][64] 16-bit = 16 KB
constexpr uint32_t TMEM_COLS = 256;       // S [0,128) | O tile [128,192)
constexpr uint32_t S_COL = 0, O_COL = 128;
constexpr int NTHREADS = 256;             // 8 warps: (TMEM lane quarter) x (column half)

struct alignas(1024) TcSmem {
    unsigned char q[TILE];
    unsigned char k[2][TILE];             // key tiles j (even j) and j (odd j)
    unsigned char v[TILE];
    unsigned char p[2][TILE];             // P: keys [0,64) and [64,128) as two K-major sub-tiles
    float rmax[2][BM];                    // per column half: row maxima, then row sums
    uint64_t bar_q, bar_k[2], bar_v, bar_s, bar_o;
    uint32_t tmem_base;
};
constexpr size_t SMEM_BYTES = sizeof(TcSmem) + 1024;  // + alignment slack of the dynamic base

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    if constexpr (BF16) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    } else {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// P = 2^(s - m) for this thread's 64 scores (ex2(-inf) = 0 keeps masked keys at
// 0), packed to 16 bits into its row of the 128-byte-swizzled P sub-tile; adds
// to the four partial row sums.  (Computing half of the exponentials on the FMA
// pipe with a polynomial, to unload MUFU, was measured 1.7 % slower here.)
// Scores are raw (unscaled); the scale goes into the exponent's argument, one
// FFMA per score: p = 2^(s * scale - m), m in the scaled (log2) domain.
template <bool BF16>
__device__ __forceinline__ void softmax_pack(const float (&sv)[64], float scale, float m_new, unsigned char* sub,
                                             int row, float& ls0, float& ls1, float& ls2, float& ls3) {
#pragma unroll
    for (int ch = 0; ch < 8; ch++) {
        float pv[8];
#pragma unroll
        for (int e = 0; e < 8; e++) pv[e] = ex2(fmaf(sv[8 * ch + e], scale, -m_new));
        ls0 += pv[0] + pv[4];
        ls1 += pv[1] + pv[5];
        ls2 += pv[2] + pv[6];
        ls3 += pv[3] + pv[7];
        *reinterpret_cast<uint4*>(sub + ((ch ^ (row & 7)) << 4)) =
            make_uint4(pack2<BF16>(pv[0], pv[1]), pack2<BF16>(pv[2], pv[3]), pack2<BF16>(pv[4], pv[5]),
                       pack2<BF16>(pv[6], pv[7]));
    }
}

template <bool BF16>
__global__ void __launch_bounds__(NTHREADS, 2)
    prefill_attn_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tkv,
                           const __grid_constant__ CUtensorMap tout, RingView r, const int32_t* __restrict__ streams,
                           int rows) {
    extern __shared__ unsigned char smem_raw[];
    TcSmem& sm = *reinterpret_cast<TcSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int qt = gridDim.x - 1 - blockIdx.x;  // the longest (most key tiles) first
    const int h = blockIdx.y, item = blockIdx.z;
    const int s = streams[item];
    if (s < 0 || s >= r.streams) return;        // the RoPE/cache kernel has flagged it
    const int H = r.heads, q0 = qt * BM, ntiles = qt + 1;
    const int kplane = (s * 2 + 0) * H + h, vplane = (s * 2 + 1) * H + h, qplane = item * H + h;

    if (warp == 0) tmem_alloc(&sm.tmem_base, TMEM_COLS);
    if (tid == 0) {
        mbar_init(&sm.bar_q, 1);
        mbar_init(&sm.bar_k[0], 1);
        mbar_init(&sm.bar_k[1], 1);
        mbar_init(&sm.bar_v, 1);
        mbar_init(&sm.bar_s, 1);
        mbar_init(&sm.bar_o, 1);
        fence_mbar_init();
        prefetch_tmap(&tq);
        prefetch_tmap(&tkv);
        prefetch_tmap(&tout);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = sm.tmem_base;

    // issue/complete counts per barrier (identical in every thread: the control flow is uniform)
    int k0_issued = 1, k1_issued = ntiles > 1 ? 1 : 0, k0_done = 0, k1_done = 0;  // per key buffer
    int v_issued = 1, v_done = 0, s_issued = 0, s_done = 0, o_issued = 0, o_done = 0;
    if (tid == 0) {
        mbar_expect_tx(&sm.bar_q, TILE);
        tma_load_3d(sm.q, &tq, 0, q0, qplane, &sm.bar_q);
        mbar_expect_tx(&sm.bar_k[0], TILE);
        tma_load_3d(sm.k[0], &tkv, 0, 0, kplane, &sm.bar_k[0]);
        if (ntiles > 1) {
            mbar_expect_tx(&sm.bar_k[1], TILE);
            tma_load_3d(sm.k[1], &tkv, 0, BN, kplane, &sm.bar_k[1]);
        }
        mbar_expect_tx(&sm.bar_v, TILE);
        tma_load_3d(sm.v, &tkv, 0, 0, vplane, &sm.bar_v);
    }

    constexpr uint32_t IDESC_QK = idesc_f16(BF16 ? 1u : 0u, 0u, BM, BN);
    constexpr uint32_t IDESC_PV = idesc_f16(BF16 ? 1u : 0u, 1u, BM, HD);
    const float scale = SCALE * LOG2E;
    // warps w and w+4 share TMEM lanes 32(w%4).. (query rows); w/4 picks the column half
    const int quarter = warp & 3, half = warp >> 2;
    const int row = quarter * 32 + lane;
    const int qg = q0 + row;
    const uint32_t lane_addr = tbase + ((uint32_t)(quarter * 32) << 16);
    float o[HD / 2];
#pragma unroll
    for (int d = 0; d < HD / 2; d++) o[d] = 0.f;
    float m_run = -INFINITY, l_half = 0.f;

    // S_0 = Q K_0^T
    bool ok = __syncthreads_and(mbar_wait(&sm.bar_q, 0, WAIT_LIMIT) && mbar_wait(&sm.bar_k[0], 0, WAIT_LIMIT));
    bool q_done = ok;
    if (ok) {
        k0_done++;
        if (tid == 0) {
            tc_fence_after();
            const uint32_t qa = smem_u32(sm.q), ka = smem_u32(sm.k[0]);
#pragma unroll
            for (int kk = 0; kk < HD / 16; kk++)
                umma_f16(tbase + S_COL, sdesc_sw128(qa + 32 * kk, 16, 1024), sdesc_sw128(ka + 32 * kk, 16, 1024),
                         IDESC_QK, kk > 0);
            umma_commit(&sm.bar_s);
        }
        s_issued++;
    }
    for (int j = 0; j < ntiles && ok; j++) {
        const int k0 = j * BN, kb_ = j & 1;
        // ---- S_j landed in TMEM: its key buffer is free for tile j + 2
        ok = __syncthreads_and(mbar_wait(&sm.bar_s, s_done & 1, WAIT_LIMIT));
        if (!ok) break;
        s_done++;
        if (j + 2 < ntiles) {
            if (tid == 0) {
                mbar_expect_tx(&sm.bar_k[kb_], TILE);
                tma_load_3d(sm.k[kb_], &tkv, 0, k0 + 2 * BN, kplane, &sm.bar_k[kb_]);
            }
            if (kb_) k1_issued++; else k0_issued++;
        }
        tc_fence_after();

        // ---- this thread's 64 scores (keys k0 + 64*half ..), kept in registers
        float sv[64];
        tmem_ld64(lane_addr + S_COL + 64 * half, sv);
        const int kb = k0 + 64 * half;
        const bool full = (k0 + BN <= q0) && (k0 + BN <= rows);  // no key of the tile is masked
        float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
        // row maximum of the raw scores (the scale is positive, so it commutes)
        if (full) {
#pragma unroll
            for (int i = 0; i < 64; i += 4) {
                mx0 = fmaxf(mx0, sv[i]);
                mx1 = fmaxf(mx1, sv[i + 1]);
                mx2 = fmaxf(mx2, sv[i + 2]);
                mx3 = fmaxf(mx3, sv[i + 3]);
            }
        } else {  // causal mask key <= query, and keys < rows: keys kb + i live iff i <= lim
            const int lim = min(qg, rows - 1) - kb;
#pragma unroll
            for (int i = 0; i < 64; i += 4) {
                sv[i] = i <= lim ? sv[i] : -INFINITY;
                sv[i + 1] = i + 1 <= lim ? sv[i + 1] : -INFINITY;
                sv[i + 2] = i + 2 <= lim ? sv[i + 2] : -INFINITY;
                sv[i + 3] = i + 3 <= lim ? sv[i + 3] : -INFINITY;
                mx0 = fmaxf(mx0, sv[i]);
                mx1 = fmaxf(mx1, sv[i + 1]);
                mx2 = fmaxf(mx2, sv[i + 2]);
                mx3 = fmaxf(mx3, sv[i + 3]);
            }
        }
        sm.rmax[half][row] = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
        __syncthreads();
        const float m_tile = fmaxf(sm.rmax[0][row], sm.rmax[1][row]) * scale;
        const float m_new = fmaxf(m_run, m_tile);   // finite: key 0 of tile 0 is never masked
        const float corr = ex2(m_run - m_new);      // 0 on the first tile (m_run = -inf)
        float ls0 = 0.f, ls1 = 0.f, ls2 = 0.f, ls3 = 0.f;
        unsigned char* sub = sm.p[half] + row * 128;  // this half's 64 keys = P sub-tile `half`
        softmax_pack<BF16>(sv, scale, m_new, sub, row, ls0, ls1, ls2, ls3);
        l_half = l_half * corr + ((ls0 + ls1) + (ls2 + ls3));
        m_run = m_new;
        fence_async_smem();
        tc_fence_before();

        // ---- O_j = P_j V_j, then S_{j+1} = Q K_{j+1}^T behind it on the tensor pipe
        const bool more = j + 1 < ntiles;
        const int next_done = kb_ ? k0_done : k1_done;  // completions so far of tile j+1's key buffer
        ok = __syncthreads_and(mbar_wait(&sm.bar_v, v_done & 1, WAIT_LIMIT) &&
                               (!more || mbar_wait(&sm.bar_k[kb_ ^ 1], next_done & 1, WAIT_LIMIT)));
        if (!ok) break;
        v_done++;
        if (more) {
            if (kb_) k0_done++; else k1_done++;
        }
        if (tid == 0) {
            tc_fence_after();
            const uint32_t pa = smem_u32(sm.p[0]), pb = smem_u32(sm.p[1]), va = smem_u32(sm.v);
#pragma unroll
            for (int kk = 0; kk < BN / 16; kk++)
                umma_f16(tbase + O_COL, sdesc_sw128((kk < 4 ? pa : pb) + 32 * (kk & 3), 16, 1024),
                         sdesc_sw128(va + 2048 * kk, TILE, 1024), IDESC_PV, kk > 0);
            umma_commit(&sm.bar_o);
            if (more) {
                const uint32_t qa = smem_u32(sm.q), ka = smem_u32(sm.k[kb_ ^ 1]);
#pragma unroll
                for (int kk = 0; kk < HD / 16; kk++)
                    umma_f16(tbase + S_COL, sdesc_sw128(qa + 32 * kk, 16, 1024),
                             sdesc_sw128(ka + 32 * kk, 16, 1024), IDESC_QK, kk > 0);
                umma_commit(&sm.bar_s);
            }
        }
        o_issued++;
        if (more) s_issued++;
        ok = __syncthreads_and(mbar_wait(&sm.bar_o, o_done & 1, WAIT_LIMIT));
        if (!ok) break;
        o_done++;
        if (more) {  // V consumed: fetch the next tile's values
            if (tid == 0) {
                mbar_expect_tx(&sm.bar_v, TILE);
                tma_load_3d(sm.v, &tkv, 0, k0 + BN, vplane, &sm.bar_v);
            }
            v_issued++;
        }
        tc_fence_after();
        {
            float v[32];
            tmem_ld32(lane_addr + O_COL + 32 * half, v);
#pragma unroll
            for (int i = 0; i < 32; i++) o[i] = fmaf(o[i], corr, v[i]);
        }
        tc_fence_before();  // the next barrier orders this O read before PV_{j+1} overwrites it
    }

    if (ok) {
        // normalise, stage the O tile in the (now free) P buffers -- half `half`
        // of the 64 output dims in sub-tile `half`, 128-byte swizzled -- and store
        // it with two TMA tile stores (rows past `rows` are clipped by the map)
        sm.rmax[half][row] = l_half;  // exchange the two halves' sums
        __syncthreads();
        const float inv = 1.f / (sm.rmax[0][row] + sm.rmax[1][row]);
        unsigned char* dsub = sm.p[half] + row * 128;
#pragma unroll
        for (int c = 0; c < 8; c++)
            *reinterpret_cast<float4*>(dsub + ((c ^ (row & 7)) << 4)) =
                make_float4(o[4 * c] * inv, o[4 * c + 1] * inv, o[4 * c + 2] * inv, o[4 * c + 3] * inv);
        fence_async_smem();
        __syncthreads();
        if (tid == 0) {
            tma_store_3d(&tout, sm.p[0], h * HD, q0, item);
            tma_store_3d(&tout, sm.p[1], h * HD + 32, q0, item);
            bulk_store_drain();
        }
    } else if (tid == 0) {
        // gave up: record it, then let everything in flight land before the
        // shared memory and TMEM of this CTA are released
        atomicOr(r.err, DERR_TIMEOUT);
        if (!q_done) mbar_wait(&sm.bar_q, 0, WAIT_LIMIT);
        for (; k0_done < k0_issued; k0_done++) mbar_wait(&sm.bar_k[0], k0_done & 1, WAIT_LIMIT);
        for (; k1_done < k1_issued; k1_done++) mbar_wait(&sm.bar_k[1], k1_done & 1, WAIT_LIMIT);
        for (; v_done < v_issued; v_done++) mbar_wait(&sm.bar_v, v_done & 1, WAIT_LIMIT);
        for (; s_done < s_issued; s_done++) mbar_wait(&sm.bar_s, s_done & 1, WAIT_LIMIT);
        for (; o_done < o_issued; o_done++) mbar_wait(&sm.bar_o, o_done & 1, WAIT_LIMIT);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_free(tbase, TMEM_COLS);
    }
}

// ---------------------------------------------------------------- host: tensor maps

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 3-D map over [planes][rows][64] 16-bit elements, rows 128 B apart, planes
// `plane_stride` bytes apart; box 128 rows x 64, 128-byte swizzle, zero fill
// past the last row.
bool make_map(CUtensorMap* m, bool bf16, const void* base, int rows, int planes, size_t plane_stride) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)HD, (cuuint64_t)rows, (cuuint64_t)planes};
    cuuint64_t strides[2] = {(cuuint64_t)HD * 2, (cuuint64_t)plane_stride};
    cuuint32_t box[3] = {(cuuint32_t)HD, (cuuint32_t)BN, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
              const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 3-D map over the fp32 output [items][rows][heads*64]: box 32 dims x 128 rows
// (128 bytes wide, the 128-byte swizzle span), one item.
bool make_out_map(CUtensorMap* m, float* out, int rows, int n, int width) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)width, (cuuint64_t)rows, (cuuint64_t)n};
    cuuint64_t strides[2] = {(cuuint64_t)width * 4, (cuuint64_t)rows * width * 4};
    cuuint32_t box[3] = {32, (cuuint32_t)BM, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, out, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool BF16>
cudaError_t launch_tc(const RingView& r, int n, const int32_t* streams, int rows, const void* q_stage, float* out,
                      cudaStream_t st) {
    CUtensorMap tq, tkv, tout;
    if (!make_map(&tq, BF16, q_stage, rows, n * r.heads, (size_t)rows * HD * 2) ||
        !make_map(&tkv, BF16, r.kv, rows, r.streams * 2 * r.heads, (size_t)r.capacity * HD * 2) ||
        !make_out_map(&tout, out, rows, n, r.heads * HD))
        return cudaErrorInvalidValue;
    static bool attr_set[64] = {};  // per device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(prefill_attn_tc_kernel<BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)SMEM_BYTES);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    dim3 grid((rows + BM - 1) / BM, r.heads, n);
    prefill_attn_tc_kernel<BF16><<<grid, NTHREADS, SMEM_BYTES, st>>>(tq, tkv, tout, r, streams, rows);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_prefill_attn_tc(int dtype, const RingView& r, int n, const int32_t* streams, int rows,
                                   const void* q_stage, float* out, cudaStream_t st) {
    return dtype == MB_BF16 ? launch_tc<true>(r, n, streams, rows, q_stage, out, st)
                            : launch_tc<false>(r, n, streams, rows, q_stage, out, st);
}

}  // namespace mb
