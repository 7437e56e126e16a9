// Causal prefill attention on the 5th-generation tensor cores for 16-bit rings,
// with 64-key tiles and four CTAs per SM: the ATTENTION_SCORES / _SOFTMAX /
// _APPLY passes of the reference (kernels-batch.ts:246-350) as one
// flash-attention kernel.
//
// A work item = 128 queries of one (item, head); 4 warps, thread t owns query
// row t, which is also its TMEM lane.  The grid is four CTAs per SM (at most one
// per work item), each staying resident over several work items: they are
// handed out longest first, round by round, in snake order across the CTAs, so
// the CTAs' totals stay close, and the TMEM allocation, the barriers and the
// tensor-map prefetch are paid once per CTA (5 % faster at config 3 than one CTA
// per item, whose last wave ran part-empty).  The CTA reads its Q rows straight from the fp32
// QKV input and ropes them itself (the RoPE/cache kernel writes only K and V),
// so Q never makes a round trip through HBM.  TMEM holds S (64 columns) and the running O (64
// columns): 128 columns, so four CTAs share an SM's 512, and 48 KB of shared
// memory each.  Per 64-key tile j (causal: keys up to the CTA's last query):
//   S_j = Q K_j^T      tcgen05.mma kind::f16, M=128 N=64 K=64, fp32 in TMEM
//   softmax            tcgen05.ld of the row's 64 scores; the running maximum
//                      moves only when a row's tile maximum exceeds it by more
//                      than 2^8 (then O is rescaled in TMEM and the row sum with
//                      it), so P = 2^(s*scale - m) stays <= 256, exact enough in
//                      16 bits; P written to shared memory, 128-byte swizzled
//   O += P_j V_j       tcgen05.mma, M=128 N=64 K=64 (V as an MN-major operand),
//                      accumulated in TMEM; right behind it S_{j+1}
// K_{j+1} and V_j are fetched (3-D TMA, no multicast) as soon as S_j has landed,
// which also means PV_{j-1} has (the MMAs complete in issue order).  At the end O
// is read back once, normalised, staged in shared memory and written by two TMA
// tile stores.  Every wait is bounded; a CTA that gives up flags MB_ERR_TIMEOUT,
// waits (bounded) for its copies and MMAs in flight, and frees its TMEM.
// (An earlier shape -- 128-key tiles, 8 warps, O in registers, two CTAs per SM --
// was measured 17 % slower: its per-tile chain of dependent steps was the limit,
// and two chains per SM hid too little of it.)
#include <cuda.h>
#include <cudaTypedefs.h>

#include "mb_internal.cuh"
#include "mb_ptx.cuh"

namespace mb {
namespace {

constexpr int BM = 128;                   // queries per CTA (UMMA M)
constexpr int BN = 64;                    // keys per tile
constexpr int QTILE = BM * HD * 2;        // [128][64] 16-bit = 16 KB
constexpr int KTILE = BN * HD * 2;        // [64][64] 16-bit = 8 KB
constexpr uint32_t TMEM_COLS = 128;       // S [0,64) | O [64,128)
constexpr uint32_t S_COL = 0, O_COL = 64;
constexpr int NTHREADS = 128;
constexpr float RESCALE_LOG2 = 8.f;       // the running max moves when a tile's exceeds it by > 2^8

struct alignas(1024) TcSmem {
    unsigned char q[QTILE];
    unsigned char p[QTILE];               // P [128 rows][64 keys]; at the end O dims 0-31
    unsigned char k[KTILE];               // k and v together hold O dims 32-63 at the end
    unsigned char v[KTILE];
    uint64_t bar_k, bar_v, bar_s, bar_o;
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

// One normalised context row (64 fp32) from registers to global memory.
__device__ __forceinline__ void store_row(float* dst, const float* o, float inv) {
#pragma unroll
    for (int c = 0; c < 16; c++)
        reinterpret_cast<float4*>(dst)[c] =
            make_float4(o[4 * c] * inv, o[4 * c + 1] * inv, o[4 * c + 2] * inv, o[4 * c + 3] * inv);
}

// 128-byte-swizzled row of 128 B: 16-byte chunk c of row r sits at chunk c ^ (r % 8)
__device__ __forceinline__ unsigned char* swz(unsigned char* base, int r, int c) {
    return base + r * 128 + ((c ^ (r & 7)) << 4);
}

// Loads of eight row pairs of Q (pairs p0..p0+7 of this warp's 32 rows; the
// half-warp's rows are grow0 + 2p): q dims 4*l16..4*l16+3 and their two (cos,
// sin) pairs; rows past `rows` read as zero.
__device__ __forceinline__ void q_rows_load(const float* qkv_row0, const float2* rope, int grow0, int rows, int l16,
                                            int HID, float4 (&qv)[8], float4 (&cs)[8], int p0) {
#pragma unroll
    for (int u = 0; u < 8; u++) {
        const int gq = grow0 + 2 * (p0 + u);
        qv[u] = cs[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (gq < rows) {
            qv[u] = *reinterpret_cast<const float4*>(qkv_row0 + (size_t)gq * 3 * HID);
            cs[u] = *reinterpret_cast<const float4*>(rope + (size_t)gq * 32 + 2 * l16);
        }
    }
}

// An L2 prefetch of the q rows of pairs p0..p0+7 (no registers held)
__device__ __forceinline__ void q_rows_prefetch(const float* qkv_row0, int grow0, int rows, int HID, int p0) {
#pragma unroll
    for (int u = 0; u < 8; u++) {
        const int gq = grow0 + 2 * (p0 + u);
        if (gq < rows) asm volatile("prefetch.global.L2 [%0];" ::"l"(qkv_row0 + (size_t)gq * 3 * HID));
    }
}

// RoPE of the loaded pairs and their 8-byte stores into the swizzled Q tile
template <bool BF16>
__device__ __forceinline__ void q_rows_store(unsigned char* q, int warp, int lane, const float4 (&qv)[8],
                                             const float4 (&cs)[8], int p0) {
    const int l16 = lane & 15;
#pragma unroll
    for (int u = 0; u < 8; u++) {
        const int rr = warp * 32 + 2 * (p0 + u) + (lane >> 4);
        const float2 a = rope_pair(make_float2(qv[u].x, qv[u].y), make_float2(cs[u].x, cs[u].y));
        const float2 b = rope_pair(make_float2(qv[u].z, qv[u].w), make_float2(cs[u].z, cs[u].w));
        *reinterpret_cast<uint2*>(swz(q, rr, l16 >> 1) + (l16 & 1) * 8) =
            make_uint2(pack2<BF16>(a.x, a.y), pack2<BF16>(b.x, b.y));
    }
}

template <bool BF16>
__global__ void __launch_bounds__(NTHREADS, 4)
    prefill_attn_tc_kernel(const float* __restrict__ qkv, const __grid_constant__ CUtensorMap tkv,
                             const __grid_constant__ CUtensorMap tout, RingView r,
                             const int32_t* __restrict__ streams, int rows, int n, int qtiles) {
    extern __shared__ unsigned char smem_raw[];
    TcSmem& sm = *reinterpret_cast<TcSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5;
    const int H = r.heads;
    // Work items: the query tiles of every (item, head), sorted longest first
    // (item index w: tile qtiles - 1 - w / (heads * n)).  CTA b takes one item per
    // round, in snake order (b in even rounds, G - 1 - b in odd ones), so the
    // CTAs' totals stay close and none is left with a long tile at the end.
    const int G = gridDim.x, W = qtiles * H * n;
    auto work = [&](int rnd) { return rnd * G + ((rnd & 1) ? G - 1 - (int)blockIdx.x : (int)blockIdx.x); };
    int w = work(0);  // < W: the grid is at most W CTAs
    int qt = qtiles - 1 - w / (H * n), h = (w % (H * n)) % H, item = (w % (H * n)) / H;
    int s = streams[item];
    // (query tiles from row 0: laid out from the last row back, as the fp32-ring
    // kernel below has them, this kernel measured 3 % slower)
    int q0 = qt * BM;

    // Q: the CTA's 128 rows come straight from the fp32 QKV input and are roped
    // here (position = row), with the cache kernel's rope_pair so they round
    // exactly as a staged copy would, then stored in 16 bits as the
    // 128-byte-swizzled K-major tile the QK^T MMA reads.  Half a warp per row,
    // lane l16 owning dims 4*l16..4*l16+3 (two RoPE pairs): 256-byte coalesced
    // reads of the row and of its (cos, sin) pairs.  The loads of the first half
    // of the rows, and an L2 prefetch of the second, are issued before the setup
    // below, so their latency overlaps it.
    const int HID = H * HD, lane = tid & 31, l16 = lane & 15;
    const float* qkv_row0 = qkv + (size_t)item * rows * 3 * HID + h * HD + 4 * l16;
    float4 qv[8], cs[8];
    // the first item's Q rows are requested into L2 before the setup (its loads,
    // at the top of the item loop, then find them there)
    q_rows_prefetch(qkv_row0, q0 + warp * 32 + (lane >> 4), rows, HID, 0);
    q_rows_prefetch(qkv_row0, q0 + warp * 32 + (lane >> 4), rows, HID, 8);

    if (warp == 0) tmem_alloc(&sm.tmem_base, TMEM_COLS);
    if (tid == 0) {
        mbar_init(&sm.bar_k, 1);
        mbar_init(&sm.bar_v, 1);
        mbar_init(&sm.bar_s, 1);
        mbar_init(&sm.bar_o, 1);
        fence_mbar_init();
        prefetch_tmap(&tkv);
        prefetch_tmap(&tout);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = sm.tmem_base;

    // issue/complete counts per barrier (identical in every thread: the control
    // flow is uniform); they run on from one work item to the next
    int k_issued = 0, k_done = 0, v_issued = 0, v_done = 0, s_issued = 0, s_done = 0, o_issued = 0, o_done = 0;
    constexpr uint32_t IDESC_QK = idesc_f16(BF16 ? 1u : 0u, 0u, BM, BN);
    constexpr uint32_t IDESC_PV = idesc_f16(BF16 ? 1u : 0u, 1u, BM, HD);
    const float scale = SCALE * LOG2E;
    const int row = tid;
    const uint32_t lane_addr = tbase + ((uint32_t)(warp * 32) << 16);
    bool ok = true, waited = false;  // waited: thread 0 has passed griddepcontrol.wait
    for (int rnd = 0; ok; rnd++) {
    if (rnd > 0) {
        w = work(rnd);
        if (w >= W) break;
        qt = qtiles - 1 - w / (H * n), h = (w % (H * n)) % H, item = (w % (H * n)) / H;
        s = streams[item];
        q0 = qt * BM;
        qkv_row0 = qkv + (size_t)item * rows * 3 * HID + h * HD + 4 * l16;
    }
    if (s < 0 || s >= r.streams) continue;  // the RoPE/cache kernel has flagged it
    q_rows_load(qkv_row0, r.rope, q0 + warp * 32 + (lane >> 4), rows, l16, HID, qv, cs, 0);
    q_rows_prefetch(qkv_row0, q0 + warp * 32 + (lane >> 4), rows, HID, 8);
    const int ntiles = (min(q0 + BM, rows) + BN - 1) / BN;
    const int kplane = (s * 2 + 0) * H + h, vplane = (s * 2 + 1) * H + h;
    const int qg = q0 + row;
    if (tid == 0) {
        // The kernel is a programmatic dependent of the RoPE/cache kernel: the
        // first item's Q loads and the setup may run during that kernel's tail,
        // but the K/V it writes are read only after it has completed.  Thread 0
        // is the only thread that reads or writes global memory between an
        // item's Q load and its end (the K/V loads and the output stores are its
        // TMA copies; it has let the previous item's stores read their staging).
        if (!waited) asm volatile("griddepcontrol.wait;" ::: "memory");
        waited = true;
        mbar_expect_tx(&sm.bar_k, KTILE);
        tma_load_3d(sm.k, &tkv, 0, 0, kplane, &sm.bar_k);
        mbar_expect_tx(&sm.bar_v, KTILE);
        tma_load_3d(sm.v, &tkv, 0, 0, vplane, &sm.bar_v);
    }
    k_issued++;
    v_issued++;
    float m_run = -INFINITY, l_run = 0.f;

    // Q: the first half of the rows roped and stored, then the second half
    // loaded, roped and stored
    q_rows_store<BF16>(sm.q, warp, lane, qv, cs, 0);
    q_rows_load(qkv_row0, r.rope, q0 + warp * 32 + (lane >> 4), rows, l16, HID, qv, cs, 8);
    q_rows_store<BF16>(sm.q, warp, lane, qv, cs, 8);
    fence_async_smem();  // the Q stores, seen by the tensor core

    // S_0 = Q K_0^T
    ok = __syncthreads_and(mbar_wait(&sm.bar_k, k_done & 1, WAIT_LIMIT));
    if (ok) {
        k_done++;
        if (tid == 0) {
            tc_fence_after();
            const uint32_t qa = smem_u32(sm.q), ka = smem_u32(sm.k);
#pragma unroll
            for (int kk = 0; kk < HD / 16; kk++)
                umma_f16(tbase + S_COL, sdesc_sw128(qa + 32 * kk, 16, 1024), sdesc_sw128(ka + 32 * kk, 16, 1024),
                         IDESC_QK, kk > 0);
            umma_commit(&sm.bar_s);
        }
        s_issued++;
    }
    for (int j = 0; j < ntiles && ok; j++) {
        const int k0 = j * BN;
        const bool more = j + 1 < ntiles;
        // ---- S_j landed: K_j is consumed, and so is V_{j-1} (PV_{j-1} was issued before S_j)
        ok = __syncthreads_and(mbar_wait(&sm.bar_s, s_done & 1, WAIT_LIMIT));
        if (!ok) break;
        s_done++;
        if (tid == 0) {
            if (more) {
                mbar_expect_tx(&sm.bar_k, KTILE);
                tma_load_3d(sm.k, &tkv, 0, k0 + BN, kplane, &sm.bar_k);
            }
            if (j > 0) {
                mbar_expect_tx(&sm.bar_v, KTILE);
                tma_load_3d(sm.v, &tkv, 0, k0, vplane, &sm.bar_v);
            }
        }
        if (more) k_issued++;
        if (j > 0) v_issued++;
        tc_fence_after();

        // ---- this row's 64 scores
        float sv[64];
        tmem_ld64(lane_addr + S_COL, sv);
        const bool full = (k0 + BN <= q0) && (k0 + BN <= rows);  // no key of the tile is masked
        float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
        if (full) {
#pragma unroll
            for (int i = 0; i < 64; i += 4) {
                mx0 = fmaxf(mx0, sv[i]);
                mx1 = fmaxf(mx1, sv[i + 1]);
                mx2 = fmaxf(mx2, sv[i + 2]);
                mx3 = fmaxf(mx3, sv[i + 3]);
            }
        } else {  // causal mask key <= query, and keys < rows: keys k0 + i live iff i <= lim
            const int lim = min(qg, rows - 1) - k0;
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
        // the scale is positive, so the maximum of the raw scores scales to the scaled one;
        // tile 0 always moves the maximum (key 0 is live for every row)
        const float m_tile = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * scale;
        const bool grow = m_tile > m_run + RESCALE_LOG2;
        const float m_new = grow ? m_tile : m_run;
        const float corr = grow ? ex2(m_run - m_new) : 1.f;  // 0 on tile 0
        float ls0 = 0.f, ls1 = 0.f, ls2 = 0.f, ls3 = 0.f;
#pragma unroll
        for (int ch = 0; ch < 8; ch++) {
            float pv[8];
#pragma unroll
            for (int e = 0; e < 8; e++) pv[e] = ex2(fmaf(sv[8 * ch + e], scale, -m_new));
            ls0 += pv[0] + pv[4];
            ls1 += pv[1] + pv[5];
            ls2 += pv[2] + pv[6];
            ls3 += pv[3] + pv[7];
            *reinterpret_cast<uint4*>(swz(sm.p, row, ch)) =
                make_uint4(pack2<BF16>(pv[0], pv[1]), pack2<BF16>(pv[2], pv[3]), pack2<BF16>(pv[4], pv[5]),
                           pack2<BF16>(pv[6], pv[7]));
        }
        l_run = l_run * corr + ((ls0 + ls1) + (ls2 + ls3));
        m_run = m_new;
        // O of the earlier tiles follows a moved maximum (PV_{j-1} has landed; the
        // scores are dead here, which keeps the registers for O)
        if (j > 0 && __any_sync(0xffffffffu, grow)) {  // TMEM access is warp-collective
            float o[64];
            tmem_ld64(lane_addr + O_COL, o);
#pragma unroll
            for (int i = 0; i < 64; i++) o[i] *= corr;
            tmem_st64(lane_addr + O_COL, o);
        }
        fence_async_smem();
        tc_fence_before();

        // ---- O += P_j V_j, then S_{j+1} = Q K_{j+1}^T behind it on the tensor pipe
        ok = __syncthreads_and(mbar_wait(&sm.bar_v, v_done & 1, WAIT_LIMIT) &&
                               (!more || mbar_wait(&sm.bar_k, k_done & 1, WAIT_LIMIT)));
        if (!ok) break;
        v_done++;
        if (more) k_done++;
        if (tid == 0) {
            tc_fence_after();
            const uint32_t pa = smem_u32(sm.p), va = smem_u32(sm.v);
#pragma unroll
            for (int kk = 0; kk < BN / 16; kk++)
                umma_f16(tbase + O_COL, sdesc_sw128(pa + 32 * kk, 16, 1024), sdesc_sw128(va + 2048 * kk, KTILE, 1024),
                         IDESC_PV, j > 0 || kk > 0);
            if (more) {
                const uint32_t qa = smem_u32(sm.q), ka = smem_u32(sm.k);
#pragma unroll
                for (int kk = 0; kk < HD / 16; kk++)
                    umma_f16(tbase + S_COL, sdesc_sw128(qa + 32 * kk, 16, 1024),
                             sdesc_sw128(ka + 32 * kk, 16, 1024), IDESC_QK, kk > 0);
                umma_commit(&sm.bar_s);
            } else {
                umma_commit(&sm.bar_o);
            }
        }
        if (more)
            s_issued++;
        else
            o_issued++;
    }
    if (ok) {  // the last PV: O is final
        ok = __syncthreads_and(mbar_wait(&sm.bar_o, o_done & 1, WAIT_LIMIT));
        if (ok) o_done++;
    }

    if (ok) {
        // normalise, stage O (dims 0-31 in the P buffer, 32-63 in the K and V
        // buffers, 128-byte swizzled) and write it with two TMA tile stores
        tc_fence_after();
        float o[64];
        tmem_ld64(lane_addr + O_COL, o);
        const float inv = 1.f / l_run;
#pragma unroll
        for (int c = 0; c < 8; c++)
            *reinterpret_cast<float4*>(swz(sm.p, row, c)) =
                make_float4(o[4 * c] * inv, o[4 * c + 1] * inv, o[4 * c + 2] * inv, o[4 * c + 3] * inv);
#pragma unroll
        for (int c = 0; c < 8; c++)
            *reinterpret_cast<float4*>(swz(sm.k, row, c)) =
                make_float4(o[32 + 4 * c] * inv, o[33 + 4 * c] * inv, o[34 + 4 * c] * inv, o[35 + 4 * c] * inv);
        fence_async_smem();
        __syncthreads();
        if (tid == 0) {
            tma_store_3d(&tout, sm.p, h * HD, q0, item);
            tma_store_3d(&tout, sm.k, h * HD + 32, q0, item);
            bulk_store_drain();
        }
    }
    }  // work items
    if (!ok && tid == 0) {
        // gave up: record it, then let everything in flight land before the
        // shared memory and TMEM of this CTA are released
        atomicOr(r.err, DERR_TIMEOUT);
        for (; k_done < k_issued; k_done++) mbar_wait(&sm.bar_k, k_done & 1, WAIT_LIMIT);
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

// 3-D map over [planes][rows][64] 16-bit elements (rows 128 B apart, planes
// `plane_stride` bytes apart); box `box_rows` x 64, 128-byte swizzle, zero fill
// past the last row.
bool make_map(CUtensorMap* m, bool bf16, const void* base, int rows, int planes, size_t plane_stride, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)HD, (cuuint64_t)rows, (cuuint64_t)planes};
    cuuint64_t strides[2] = {(cuuint64_t)HD * 2, (cuuint64_t)plane_stride};
    cuuint32_t box[3] = {(cuuint32_t)HD, (cuuint32_t)box_rows, 1};
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
cudaError_t launch_tc(const RingView& r, int n, const int32_t* streams, int rows, const float* qkv, float* out,
                        cudaStream_t st) {
    CUtensorMap tkv, tout;
    if (!make_map(&tkv, BF16, r.kv, rows, r.streams * 2 * r.heads, (size_t)r.capacity * HD * 2, BN) ||
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
    // four CTAs per SM (the TMEM limit), each over several query tiles
    static int sms[64] = {};  // per device
    if (!sms[dev] && (e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
        return e;
    const int qtiles = (rows + BM - 1) / BM, work = qtiles * r.heads * n;
    // programmatic dependent of the RoPE/cache kernel launched just before it
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(work < 4 * sms[dev] ? work : 4 * sms[dev]);
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, prefill_attn_tc_kernel<BF16>, (const float*)qkv, tkv, tout, r, streams, rows, n,
                              qtiles);
}


// ---------------------------------------------------------------- fp32 rings: split operands
//
// fp32 rings on the same tensor cores: every fp32 operand x is carried as two
// bf16 parts, hi = bf16(x) and lo = bf16(x - hi), and each product as
// hi*hi + hi*lo + lo*hi (the lo*lo term, ~2^-18 of the product, is dropped), all
// accumulated in fp32 in TMEM: ~2^-17 relative error per product, against 2^-9
// for plain bf16 operands.  The RoPE/cache kernel writes the parts of the roped
// Q, the roped K and V into a stage [6][items][heads][rows][64] bf16 (Q hi, Q
// lo, K hi, K lo, V hi, V lo) next to the fp32 ring, and this kernel loads them
// by TMA.  The softmax splits P the same way.  Otherwise the kernel is the
// 16-bit one above: one CTA = 128 queries of an (item, head), 64-key tiles, S
// and O in TMEM, PV_j then S_{j+1} back to back on the tensor pipe; 12 MMAs per
// product instead of 4, and twice the shared memory (two CTAs per SM, each
// resident over several work items as in the 16-bit kernel).
struct alignas(1024) X3Smem {
    unsigned char qh[QTILE], ql[QTILE];   // Q parts
    unsigned char ph[QTILE], pl[QTILE];   // P parts; at the end O (dims 0-31 over ph, 32-63 over pl)
    unsigned char kh[KTILE], kl[KTILE];   // K_j parts
    unsigned char vh[KTILE], vl[KTILE];   // V_j parts
    uint64_t bar_q, bar_k, bar_v, bar_s, bar_o;
    uint32_t tmem_base;
};
constexpr size_t X3_SMEM_BYTES = sizeof(X3Smem) + 1024;

// Two products' worth of P parts: hi = bf16(p), lo = bf16(p - hi), packed in pairs.
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

// D (+)= A B over three part products: A_hi B_hi + A_hi B_lo + A_lo B_hi, K = 16
// per instruction, `steps` instructions along K; A K-major, B K-major (S) or
// MN-major (PV) with the given per-step offsets.
__device__ __forceinline__ void umma_x3(uint32_t d, uint32_t ah, uint32_t al, uint32_t bh, uint32_t bl, int steps,
                                        uint32_t a_step, uint32_t b_step, uint32_t b_lbo, uint32_t idesc,
                                        bool accumulate) {
    for (int kk = 0; kk < steps; kk++) {
        const uint64_t dah = sdesc_sw128(ah + a_step * kk, 16, 1024), dal = sdesc_sw128(al + a_step * kk, 16, 1024);
        const uint64_t dbh = sdesc_sw128(bh + b_step * kk, b_lbo, 1024),
                       dbl = sdesc_sw128(bl + b_step * kk, b_lbo, 1024);
        umma_f16(d, dah, dbh, idesc, (accumulate || kk > 0) ? 1u : 0u);
        umma_f16(d, dah, dbl, idesc, 1u);
        umma_f16(d, dal, dbh, idesc, 1u);
    }
}

__global__ void __launch_bounds__(NTHREADS, 2)
    prefill_attn_x3_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tkv,
                           const __grid_constant__ CUtensorMap tout, RingView r, const int32_t* __restrict__ streams,
                           int rows, float* __restrict__ out, int n, int qtiles) {
    extern __shared__ unsigned char smem_raw[];
    X3Smem& sm = *reinterpret_cast<X3Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5;
    const int H = r.heads, np = n * H;
    // persistent over the work items as the 16-bit kernel (longest first, snake order)
    const int G = gridDim.x, W = qtiles * np;
    auto work = [&](int rnd) { return rnd * G + ((rnd & 1) ? G - 1 - (int)blockIdx.x : (int)blockIdx.x); };
    // Query tiles are laid out from the end: tile qt > 0 covers rows [q0, q0 + 128)
    // ending at `rows`, and tile 0 the remainder [0, q_end), so the partial tile
    // is the one with the fewest keys (444 rows: 1 + 3 + 5 + 7 key tiles, not
    // 2 + 4 + 6 + 7 with the partial tile last; 3-4 % faster here)
    const int first = rows - (qtiles - 1) * BM;  // rows of tile 0: 1..128

    if (warp == 0) tmem_alloc(&sm.tmem_base, TMEM_COLS);
    if (tid == 0) {
        mbar_init(&sm.bar_q, 1);
        mbar_init(&sm.bar_k, 1);
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

    int q_issued = 0, q_done = 0, k_issued = 0, k_done = 0, v_issued = 0, v_done = 0, s_issued = 0, s_done = 0,
        o_issued = 0, o_done = 0;
    constexpr uint32_t IDESC_QK = idesc_f16(1u, 0u, BM, BN);
    constexpr uint32_t IDESC_PV = idesc_f16(1u, 1u, BM, HD);
    const float scale = SCALE * LOG2E;
    const int row = tid;
    const uint32_t lane_addr = tbase + ((uint32_t)(warp * 32) << 16);
    const uint32_t qha = smem_u32(sm.qh), qla = smem_u32(sm.ql), pha = smem_u32(sm.ph), pla = smem_u32(sm.pl);
    const uint32_t kha = smem_u32(sm.kh), kla = smem_u32(sm.kl), vha = smem_u32(sm.vh), vla = smem_u32(sm.vl);
    bool ok = true, waited = false;  // waited: thread 0 has passed griddepcontrol.wait
    for (int rnd = 0; ok; rnd++) {
    const int w = work(rnd);
    if (w >= W) break;
    const int qt = qtiles - 1 - w / np, h = (w % np) % H, item = (w % np) / H;
    const int s = streams[item];
    if (s < 0 || s >= r.streams) continue;  // the RoPE/cache kernel has flagged it
    const int q0 = qt == 0 ? 0 : first + (qt - 1) * BM, q_end = qt == 0 ? first : q0 + BM;
    const int ntiles = (q_end + BN - 1) / BN;
    // planes of the stage: part p of (item, head) is plane p * n * H + item * H + h
    const int pq = item * H + h;
    if (tid == 0) {
        // a programmatic dependent of the RoPE/cache kernel, which writes the
        // stage; the previous item's stores have read their staging (drained)
        if (!waited) asm volatile("griddepcontrol.wait;" ::: "memory");
        waited = true;
        mbar_expect_tx(&sm.bar_q, 2 * QTILE);
        tma_load_3d(sm.qh, &tq, 0, q0, 0 * np + pq, &sm.bar_q);
        tma_load_3d(sm.ql, &tq, 0, q0, 1 * np + pq, &sm.bar_q);
        mbar_expect_tx(&sm.bar_k, 2 * KTILE);
        tma_load_3d(sm.kh, &tkv, 0, 0, 2 * np + pq, &sm.bar_k);
        tma_load_3d(sm.kl, &tkv, 0, 0, 3 * np + pq, &sm.bar_k);
        mbar_expect_tx(&sm.bar_v, 2 * KTILE);
        tma_load_3d(sm.vh, &tkv, 0, 0, 4 * np + pq, &sm.bar_v);
        tma_load_3d(sm.vl, &tkv, 0, 0, 5 * np + pq, &sm.bar_v);
    }
    q_issued++;
    k_issued++;
    v_issued++;
    const int qg = q0 + row;
    float m_run = -INFINITY, l_run = 0.f;

    // S_0 = Q K_0^T
    ok = __syncthreads_and(mbar_wait(&sm.bar_q, q_done & 1, WAIT_LIMIT) &&
                           mbar_wait(&sm.bar_k, k_done & 1, WAIT_LIMIT));
    if (ok) {
        q_done++;
        k_done++;
        if (tid == 0) {
            tc_fence_after();
            umma_x3(tbase + S_COL, qha, qla, kha, kla, HD / 16, 32, 32, 16, IDESC_QK, false);
            umma_commit(&sm.bar_s);
        }
        s_issued++;
    }
    for (int j = 0; j < ntiles && ok; j++) {
        const int k0 = j * BN;
        const bool more = j + 1 < ntiles;
        // ---- S_j landed: K_j is consumed, and so is V_{j-1} (PV_{j-1} was issued before S_j)
        ok = __syncthreads_and(mbar_wait(&sm.bar_s, s_done & 1, WAIT_LIMIT));
        if (!ok) break;
        s_done++;
        if (tid == 0) {
            if (more) {
                mbar_expect_tx(&sm.bar_k, 2 * KTILE);
                tma_load_3d(sm.kh, &tkv, 0, k0 + BN, 2 * np + pq, &sm.bar_k);
                tma_load_3d(sm.kl, &tkv, 0, k0 + BN, 3 * np + pq, &sm.bar_k);
            }
            if (j > 0) {
                mbar_expect_tx(&sm.bar_v, 2 * KTILE);
                tma_load_3d(sm.vh, &tkv, 0, k0, 4 * np + pq, &sm.bar_v);
                tma_load_3d(sm.vl, &tkv, 0, k0, 5 * np + pq, &sm.bar_v);
            }
        }
        if (more) k_issued++;
        if (j > 0) v_issued++;
        tc_fence_after();

        // ---- this row's 64 scores (the 16-bit kernel's softmax, P split into parts)
        float sv[64];
        tmem_ld64(lane_addr + S_COL, sv);
        const bool full = (k0 + BN <= q0) && (k0 + BN <= rows);
        float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
        if (!full) {
            const int lim = min(qg, rows - 1) - k0;
#pragma unroll
            for (int i = 0; i < 64; i++) sv[i] = i <= lim ? sv[i] : -INFINITY;
        }
#pragma unroll
        for (int i = 0; i < 64; i += 4) {
            mx0 = fmaxf(mx0, sv[i]);
            mx1 = fmaxf(mx1, sv[i + 1]);
            mx2 = fmaxf(mx2, sv[i + 2]);
            mx3 = fmaxf(mx3, sv[i + 3]);
        }
        const float m_tile = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * scale;
        const bool grow = m_tile > m_run + RESCALE_LOG2;
        const float m_new = grow ? m_tile : m_run;
        const float corr = grow ? ex2(m_run - m_new) : 1.f;
        float ls0 = 0.f, ls1 = 0.f, ls2 = 0.f, ls3 = 0.f;
#pragma unroll
        for (int ch = 0; ch < 8; ch++) {
            float pv[8];
#pragma unroll
            for (int e = 0; e < 8; e++) pv[e] = ex2(fmaf(sv[8 * ch + e], scale, -m_new));
            ls0 += pv[0] + pv[4];
            ls1 += pv[1] + pv[5];
            ls2 += pv[2] + pv[6];
            ls3 += pv[3] + pv[7];
            uint32_t hi[4], lo[4];
#pragma unroll
            for (int e = 0; e < 4; e++) split2(pv[2 * e], pv[2 * e + 1], hi[e], lo[e]);
            *reinterpret_cast<uint4*>(swz(sm.ph, row, ch)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            *reinterpret_cast<uint4*>(swz(sm.pl, row, ch)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
        l_run = l_run * corr + ((ls0 + ls1) + (ls2 + ls3));
        m_run = m_new;
        if (j > 0 && __any_sync(0xffffffffu, grow)) {
            float o[64];
            tmem_ld64(lane_addr + O_COL, o);
#pragma unroll
            for (int i = 0; i < 64; i++) o[i] *= corr;
            tmem_st64(lane_addr + O_COL, o);
        }
        fence_async_smem();
        tc_fence_before();

        // ---- O += P_j V_j, then S_{j+1} = Q K_{j+1}^T behind it
        ok = __syncthreads_and(mbar_wait(&sm.bar_v, v_done & 1, WAIT_LIMIT) &&
                               (!more || mbar_wait(&sm.bar_k, k_done & 1, WAIT_LIMIT)));
        if (!ok) break;
        v_done++;
        if (more) k_done++;
        if (tid == 0) {
            tc_fence_after();
            umma_x3(tbase + O_COL, pha, pla, vha, vla, BN / 16, 32, 2048, KTILE, IDESC_PV, j > 0);
            if (more) {
                umma_x3(tbase + S_COL, qha, qla, kha, kla, HD / 16, 32, 32, 16, IDESC_QK, false);
                umma_commit(&sm.bar_s);
            } else {
                umma_commit(&sm.bar_o);
            }
        }
        if (more)
            s_issued++;
        else
            o_issued++;
    }
    if (ok) {
        ok = __syncthreads_and(mbar_wait(&sm.bar_o, o_done & 1, WAIT_LIMIT));
        if (ok) o_done++;
    }

    if (ok && q_end - q0 < BM) {
        tc_fence_after();
        float o[64];
        tmem_ld64(lane_addr + O_COL, o);
        if (row < q_end - q0) store_row(out + ((size_t)item * rows + q0 + row) * H * HD + h * HD, o, 1.f / l_run);
    } else if (ok) {
        // normalise, stage O (dims 0-31 over ph, 32-63 over pl, 128-byte
        // swizzled) and write it with two TMA tile stores
        tc_fence_after();
        float o[64];
        tmem_ld64(lane_addr + O_COL, o);
        const float inv = 1.f / l_run;
#pragma unroll
        for (int c = 0; c < 8; c++)
            *reinterpret_cast<float4*>(swz(sm.ph, row, c)) =
                make_float4(o[4 * c] * inv, o[4 * c + 1] * inv, o[4 * c + 2] * inv, o[4 * c + 3] * inv);
#pragma unroll
        for (int c = 0; c < 8; c++)
            *reinterpret_cast<float4*>(swz(sm.pl, row, c)) =
                make_float4(o[32 + 4 * c] * inv, o[33 + 4 * c] * inv, o[34 + 4 * c] * inv, o[35 + 4 * c] * inv);
        fence_async_smem();
        __syncthreads();
        if (tid == 0) {
            tma_store_3d(&tout, sm.ph, h * HD, q0, item);
            tma_store_3d(&tout, sm.pl, h * HD + 32, q0, item);
            bulk_store_drain();
        }
        __syncthreads();  // the staging is free again before the next item's P parts
    }
    }  // work items
    if (!ok && tid == 0) {
        atomicOr(r.err, DERR_TIMEOUT);
        for (; q_done < q_issued; q_done++) mbar_wait(&sm.bar_q, q_done & 1, WAIT_LIMIT);
        for (; k_done < k_issued; k_done++) mbar_wait(&sm.bar_k, k_done & 1, WAIT_LIMIT);
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

cudaError_t launch_x3(const RingView& r, int n, const int32_t* streams, int rows, const void* stage, float* out,
                      cudaStream_t st) {
    CUtensorMap tq, tkv, tout;
    const int planes = 6 * n * r.heads;
    const size_t pstride = (size_t)rows * HD * 2;
    if (!make_map(&tq, true, stage, rows, planes, pstride, BM) ||
        !make_map(&tkv, true, stage, rows, planes, pstride, BN) || !make_out_map(&tout, out, rows, n, r.heads * HD))
        return cudaErrorInvalidValue;
    static bool attr_set[64] = {};  // per device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(prefill_attn_x3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)X3_SMEM_BYTES);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    // two CTAs per SM (the shared-memory limit), each over several query tiles
    static int sms[64] = {};  // per device
    if (!sms[dev] && (e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
        return e;
    const int qtiles = (rows + BM - 1) / BM, work = qtiles * r.heads * n;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(work < 2 * sms[dev] ? work : 2 * sms[dev]);
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = X3_SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, prefill_attn_x3_kernel, tq, tkv, tout, r, streams, rows, out, n, qtiles);
}

}  // namespace

cudaError_t launch_prefill_attn_tc(int dtype, const RingView& r, int n, const int32_t* streams, int rows,
                                     const float* qkv, float* out, cudaStream_t st) {
    return dtype == MB_BF16 ? launch_tc<true>(r, n, streams, rows, qkv, out, st)
                            : launch_tc<false>(r, n, streams, rows, qkv, out, st);
}

cudaError_t launch_prefill_attn_split(const RingView& r, int n, const int32_t* streams, int rows, const void* stage,
                                      float* out, cudaStream_t st) {
    return launch_x3(r, n, streams, rows, stage, out, st);
}

}  // namespace mb
