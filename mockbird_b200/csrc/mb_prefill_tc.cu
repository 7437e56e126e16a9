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
// Q, K, V arrive by 3-D TMA tile loads (128-byte swizzle, zero fill past the last
// row, no multicast).  K of tile j+1 is fetched as soon as the QK^T MMA of tile j
// has consumed K, V of tile j+1 as soon as the PV MMA has consumed V.  (Issuing
// S_{j+1} = Q K_{j+1}^T ahead, into a second TMEM buffer, was measured slower on
// B200: it queues in front of PV_j on the tensor pipe.)  80 KB of
// shared memory and 256 TMEM columns per CTA: two CTAs share an SM.  Every wait is
// bounded; a CTA that gives up flags MB_ERR_TIMEOUT, waits (bounded) for its
// copies and MMAs in flight, and frees its TMEM.
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
    unsigned char k[TILE];
    unsigned char v[TILE];
    unsigned char p[2][TILE];             // P: keys [0,64) and [64,128) as two K-major sub-tiles
    float rmax[2][BM];                    // per column half: row maxima, then row sums
    uint64_t bar_q, bar_k, bar_v, bar_mma;
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

template <bool BF16>
__global__ void __launch_bounds__(NTHREADS, 2)
    prefill_attn_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tkv,
                           RingView r, const int32_t* __restrict__ streams, int rows, float* __restrict__ out) {
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
        mbar_init(&sm.bar_k, 1);
        mbar_init(&sm.bar_v, 1);
        mbar_init(&sm.bar_mma, 1);
        fence_mbar_init();
        prefetch_tmap(&tq);
        prefetch_tmap(&tkv);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = sm.tmem_base;

    // issue/complete counts per barrier (identical in every thread: the control flow is uniform)
    int k_issued = 1, k_done = 0, v_issued = 1, v_done = 0, mma_issued = 0, mma_done = 0;
    if (tid == 0) {
        mbar_expect_tx(&sm.bar_q, TILE);
        tma_load_3d(sm.q, &tq, 0, q0, qplane, &sm.bar_q);
        mbar_expect_tx(&sm.bar_k, TILE);
        tma_load_3d(sm.k, &tkv, 0, 0, kplane, &sm.bar_k);
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

    bool ok = __syncthreads_and(mbar_wait(&sm.bar_q, 0, WAIT_LIMIT));
    bool q_done = ok;
    for (int j = 0; j < ntiles && ok; j++) {
        const int k0 = j * BN;
        // ---- S = Q K^T
        ok = __syncthreads_and(mbar_wait(&sm.bar_k, k_done & 1, WAIT_LIMIT));
        if (!ok) break;
        k_done++;
        if (tid == 0) {
            tc_fence_after();
            const uint32_t qa = smem_u32(sm.q), ka = smem_u32(sm.k);
#pragma unroll
            for (int kk = 0; kk < HD / 16; kk++)
                umma_f16(tbase + S_COL, sdesc_sw128(qa + 32 * kk, 16, 1024), sdesc_sw128(ka + 32 * kk, 16, 1024),
                         IDESC_QK, kk > 0);
            umma_commit(&sm.bar_mma);
        }
        mma_issued++;
        ok = __syncthreads_and(mbar_wait(&sm.bar_mma, mma_done & 1, WAIT_LIMIT));
        if (!ok) break;
        mma_done++;
        if (tid == 0 && j + 1 < ntiles) {  // K consumed: fetch the next tile's keys
            mbar_expect_tx(&sm.bar_k, TILE);
            tma_load_3d(sm.k, &tkv, 0, k0 + BN, kplane, &sm.bar_k);
        }
        if (j + 1 < ntiles) k_issued++;
        tc_fence_after();

        // ---- this thread's 64 scores (keys k0 + 64*half ..), kept in registers
        float sv[64];
        tmem_ld64(lane_addr + S_COL + 64 * half, sv);
        const int kb = k0 + 64 * half;
        const bool full = (k0 + BN <= q0) && (k0 + BN <= rows);  // no key of the tile is masked
        float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
        if (full) {
#pragma unroll
            for (int i = 0; i < 64; i += 4) {
                sv[i] *= scale;
                sv[i + 1] *= scale;
                sv[i + 2] *= scale;
                sv[i + 3] *= scale;
                mx0 = fmaxf(mx0, sv[i]);
                mx1 = fmaxf(mx1, sv[i + 1]);
                mx2 = fmaxf(mx2, sv[i + 2]);
                mx3 = fmaxf(mx3, sv[i + 3]);
            }
        } else {  // causal mask key <= query, and keys < rows
#pragma unroll
            for (int i = 0; i < 64; i++) {
                const int key = kb + i;
                sv[i] = (key <= qg && key < rows) ? sv[i] * scale : -INFINITY;
            }
#pragma unroll
            for (int i = 0; i < 64; i += 4) {
                mx0 = fmaxf(mx0, sv[i]);
                mx1 = fmaxf(mx1, sv[i + 1]);
                mx2 = fmaxf(mx2, sv[i + 2]);
                mx3 = fmaxf(mx3, sv[i + 3]);
            }
        }
        sm.rmax[half][row] = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
        __syncthreads();
        const float m_tile = fmaxf(sm.rmax[0][row], sm.rmax[1][row]);
        const float m_new = fmaxf(m_run, m_tile);   // finite: key 0 of tile 0 is never masked
        const float corr = ex2(m_run - m_new);      // 0 on the first tile (m_run = -inf)
        float ls0 = 0.f, ls1 = 0.f, ls2 = 0.f, ls3 = 0.f;
        unsigned char* sub = sm.p[half] + row * 128;  // this half's 64 keys = P sub-tile `half`
#pragma unroll
        for (int ch = 0; ch < 8; ch++) {
            const float p0 = ex2(sv[8 * ch + 0] - m_new), p1 = ex2(sv[8 * ch + 1] - m_new);
            const float p2 = ex2(sv[8 * ch + 2] - m_new), p3 = ex2(sv[8 * ch + 3] - m_new);
            const float p4 = ex2(sv[8 * ch + 4] - m_new), p5 = ex2(sv[8 * ch + 5] - m_new);
            const float p6 = ex2(sv[8 * ch + 6] - m_new), p7 = ex2(sv[8 * ch + 7] - m_new);
            ls0 += p0 + p4;
            ls1 += p1 + p5;
            ls2 += p2 + p6;
            ls3 += p3 + p7;
            *reinterpret_cast<uint4*>(sub + ((ch ^ (row & 7)) << 4)) =
                make_uint4(pack2<BF16>(p0, p1), pack2<BF16>(p2, p3), pack2<BF16>(p4, p5), pack2<BF16>(p6, p7));
        }
        l_half = l_half * corr + ((ls0 + ls1) + (ls2 + ls3));
        m_run = m_new;
        fence_async_smem();
        tc_fence_before();

        // ---- O_j = P V
        ok = __syncthreads_and(mbar_wait(&sm.bar_v, v_done & 1, WAIT_LIMIT));
        if (!ok) break;
        v_done++;
        if (tid == 0) {
            tc_fence_after();
            const uint32_t pa = smem_u32(sm.p[0]), pb = smem_u32(sm.p[1]), va = smem_u32(sm.v);
#pragma unroll
            for (int kk = 0; kk < BN / 16; kk++)
                umma_f16(tbase + O_COL, sdesc_sw128((kk < 4 ? pa : pb) + 32 * (kk & 3), 16, 1024),
                         sdesc_sw128(va + 2048 * kk, TILE, 1024), IDESC_PV, kk > 0);
            umma_commit(&sm.bar_mma);
        }
        mma_issued++;
        ok = __syncthreads_and(mbar_wait(&sm.bar_mma, mma_done & 1, WAIT_LIMIT));
        if (!ok) break;
        mma_done++;
        if (tid == 0 && j + 1 < ntiles) {  // V consumed: fetch the next tile's values
            mbar_expect_tx(&sm.bar_v, TILE);
            tma_load_3d(sm.v, &tkv, 0, k0 + BN, vplane, &sm.bar_v);
        }
        if (j + 1 < ntiles) v_issued++;
        tc_fence_after();
        {
            float v[32];
            tmem_ld32(lane_addr + O_COL + 32 * half, v);
#pragma unroll
            for (int i = 0; i < 32; i++) o[i] = fmaf(o[i], corr, v[i]);
        }
        tc_fence_before();
        __syncthreads();  // S, the O tile and P are free for the next tile
    }

    if (ok) {
        sm.rmax[half][row] = l_half;  // exchange the two halves' sums
        __syncthreads();
        if (qg < rows) {
            const float inv = 1.f / (sm.rmax[0][row] + sm.rmax[1][row]);
            float* dst = out + ((size_t)item * rows + qg) * H * HD + h * HD + 32 * half;
#pragma unroll
            for (int d = 0; d < 32; d += 4)
                *reinterpret_cast<float4*>(dst + d) = make_float4(o[d] * inv, o[d + 1] * inv, o[d + 2] * inv,
                                                                  o[d + 3] * inv);
        }
    } else if (tid == 0) {
        // gave up: record it, then let everything in flight land before the
        // shared memory and TMEM of this CTA are released
        atomicOr(r.err, DERR_TIMEOUT);
        if (!q_done) mbar_wait(&sm.bar_q, 0, WAIT_LIMIT);
        for (; k_done < k_issued; k_done++) mbar_wait(&sm.bar_k, k_done & 1, WAIT_LIMIT);
        for (; v_done < v_issued; v_done++) mbar_wait(&sm.bar_v, v_done & 1, WAIT_LIMIT);
        for (; mma_done < mma_issued; mma_done++) mbar_wait(&sm.bar_mma, mma_done & 1, WAIT_LIMIT);
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

template <bool BF16>
cudaError_t launch_tc(const RingView& r, int n, const int32_t* streams, int rows, const void* q_stage, float* out,
                      cudaStream_t st) {
    CUtensorMap tq, tkv;
    if (!make_map(&tq, BF16, q_stage, rows, n * r.heads, (size_t)rows * HD * 2) ||
        !make_map(&tkv, BF16, r.kv, rows, r.streams * 2 * r.heads, (size_t)r.capacity * HD * 2))
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
    prefill_attn_tc_kernel<BF16><<<grid, NTHREADS, SMEM_BYTES, st>>>(tq, tkv, r, streams, rows, out);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_prefill_attn_tc(int dtype, const RingView& r, int n, const int32_t* streams, int rows,
                                   const void* q_stage, float* out, cudaStream_t st) {
    return dtype == MB_BF16 ? launch_tc<true>(r, n, streams, rows, q_stage, out, st)
                            : launch_tc<false>(r, n, streams, rows, q_stage, out, st);
}

}  // namespace mb
