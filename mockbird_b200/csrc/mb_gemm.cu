// Batched-stream GEMMs of the decode step on the 5th-generation tensor cores.
//
// The reference runs every projection of a decode step as a GEMV, one lane per
// output column with a serial K loop (GEMV, liyu1981/mockbird
// src/lib/tts/engine/kernels-decode.ts:127-142: y = b + x W, W [K][N]).  With n
// streams decoding together the same weights serve n rows, so here each
// projection is one GEMM y[n][N] = x[n][K] W[K][N] on tcgen05:
//   * W is stored transposed at upload (W^T [N][K], K-major), the activations
//     x [n][K] are bf16 rows; both arrive by TMA (128-byte swizzle, no
//     multicast; boxes of three or four K blocks) into a two-stage ring;
//   * one thread issues TMA, one thread issues tcgen05.mma (kind::f16, bf16 in,
//     fp32 accumulate, M = 128 rows, N = 32, 64 or 128 columns) into TMEM,
//     releasing each stage with tcgen05.commit;
//   * four warps read the accumulator back (warp w owns TMEM lanes 32w..32w+31,
//     i.e. rows) into a shared-memory tile, and the epilogue then walks that tile
//     row-contiguously: + bias, the residual add of c_proj and fc_out, or
//     GELU(tanh) with a bf16 store for fc_in (GELU_TANH, kernels-decode.ts:373-390),
//     so no separate bias, residual or GELU pass touches memory.
// At decode batch sizes (a few hundred rows) the operand traffic from L2, not
// the tensor pipe, bounds these GEMMs, and every output tile re-reads its rows of
// x.  So tiles are wide and K is split over the CTAs of one thread-block
// cluster: each CTA multiplies a slice of K, the partial tiles meet in
// distributed shared memory, and each CTA of the cluster sums its share of the
// rows over all partials in split order -- the same order on every run, with no
// global workspace.
// Every mbarrier wait is bounded; a CTA that gives up flags DERR_TIMEOUT, lets
// its copies and MMAs in flight land, frees its TMEM, and its cluster writes
// nothing.
#include <cudaTypedefs.h>

#include <map>
#include <mutex>
#include <tuple>

#include "mb_gemm.cuh"
#include "mb_internal.cuh"
#include "mb_ptx.cuh"

namespace mb {
namespace gemm {
namespace {

constexpr int NTHREADS = 128;
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int MAX_SPLITS = 8;         // the portable cluster size

// Stages of the CTA-pair kernel's ring (one K block per stage).
constexpr int RING_STAGES = 6;

// One-CTA kernel: a ring stage is one TMA box of x and one of W^T, KB K blocks
// deep each, and the ring holds two stages.  Measured on B200 (one thread
// keeping a ring full, data in L2): a box costs the SM about the same time
// whatever its size, so one K block per box moved 20-32 KB per ~640 cycles with
// the MMAs running, and three to four K blocks per box ~330-400 cycles per K
// block -- near the bound of shared memory itself, which every K block crosses
// twice (TMA writes 16 KB of x and BN x 128 B of W^T, the MMAs read them).  A
// deeper ring of the same boxes was no faster.
template <int BN>
struct Shape {
    static constexpr int KB = kb_per_box(BN);         // K blocks per box
    static constexpr int B_BYTES = BN * BK * 2;       // one K block of W^T rows
    static constexpr int A_STAGE = KB * A_BYTES;      // x: KB tiles [128][64]
    static constexpr int STAGE = KB * (A_BYTES + B_BYTES);  // then W^T: KB tiles [BN][64]
    static constexpr int STAGES = 2;
    static constexpr uint32_t TMEM_COLS = BN;         // a power of two >= 32
    static constexpr int TS = BN + 4;                 // row stride (floats) of the staged output tile
    static constexpr int BAR_OFF = STAGES * STAGE;    // barriers, TMEM address, then the bias
    static constexpr int BAR_BYTES = ((8 * (2 * STAGES + 1) + 4) + 127) / 128 * 128;
    static constexpr int SMEM = BAR_OFF + BAR_BYTES + BN * 4 + 1024;  // + alignment slack of the dynamic base
    static_assert(STAGE % 1024 == 0 && A_STAGE % 1024 == 0 && B_BYTES % 1024 == 0, "swizzle-atom alignment");
    static_assert(BM * TS * 4 <= STAGES * STAGE, "the output tile is staged in the stage ring");
    static_assert(SMEM <= 227 * 1024, "shared memory per CTA");
};

__device__ __forceinline__ float tanh_fast(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// GELU, tanh approximation (GELU_TANH); the MUFU tanh's ~2^-11 relative error is
// below the bf16 rounding of the stored result.
__device__ __forceinline__ float gelu_tanh(float a) {
    const float inner = 0.7978845608028654f * (a + 0.044715f * a * a * a);
    return 0.5f * a * (1.f + tanh_fast(inner));
}

__device__ __forceinline__ uint32_t bf16x2(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// The address in the cluster's shared window of `local` in CTA `rank`.
__device__ __forceinline__ uint32_t peer_addr(const void* local, uint32_t rank) {
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(local)), "r"(rank));
    return a;
}

// 16 bytes from the shared memory of a CTA of the cluster.  Issued without a
// compiler memory barrier, so a thread's loads of several partials go out
// together; they are ordered after the cluster barrier that precedes them.
__device__ __forceinline__ float4 ld_peer4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr));
    return v;
}

__device__ __forceinline__ int ld_peer_int(uint32_t addr) {
    int v;
    asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
    return v;
}

// Every thread of every CTA of the cluster; shared-memory writes before it are
// visible to the whole cluster after it.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// The two halves of a cluster-wide barrier, issued apart so its latency can hide
// behind the work between them (every thread of every CTA arrives, then waits).
__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// The epilogue of 4 consecutive columns n..n+3 of row m: v = acc (summed over
// the splits), b = their bias (zero without one).
template <int EPI>
__device__ __forceinline__ void finish4(const Args& a, int m, int n, float4 v, float4 b) {
    v.x += b.x, v.y += b.y, v.z += b.z, v.w += b.w;
    if constexpr (EPI == EPI_QKV_RING) {
        const RingView& r = a.ring;
        const int hid = r.heads * HD, part = n / hid, w = n - part * hid;  // part 0 q, 1 k, 2 v
        const int s = a.streams[m], pos = a.positions[m];
        const bool ok = s >= 0 && s < r.streams && pos >= 0 && pos < r.max_position && (r.wrap || pos < r.capacity);
        if (part < 2 && ok) {  // the two RoPE pairs of dims w .. w + 3 (the same arithmetic as the decode kernel)
            const float2* cs = r.rope + (size_t)pos * 32 + ((w & (HD - 1)) >> 1);
            const float2 lo = rope_pair(make_float2(v.x, v.y), cs[0]), hi = rope_pair(make_float2(v.z, v.w), cs[1]);
            v = make_float4(lo.x, lo.y, hi.x, hi.y);
        }
        if (part == 0) {
            *reinterpret_cast<float4*>(reinterpret_cast<float*>(a.y) + (size_t)m * a.ldy + n) = v;
        } else if (ok) {
            const int head = w / HD, slot = pos % r.capacity;
            const size_t off = (((size_t)s * 2 + (part - 1)) * r.heads + head) * (size_t)r.capacity * HD +
                               (size_t)slot * HD + (w & (HD - 1));
            if (a.ring_dtype == MB_F32) {
                *reinterpret_cast<float4*>(static_cast<float*>(r.kv) + off) = v;
            } else if (a.ring_dtype == MB_BF16) {
                *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(r.kv) + off) =
                    make_uint2(bf16x2(v.x, v.y), bf16x2(v.z, v.w));
            } else {
                const __half2 h0 = __floats2half2_rn(v.x, v.y), h1 = __floats2half2_rn(v.z, v.w);
                *reinterpret_cast<uint2*>(static_cast<__half*>(r.kv) + off) =
                    make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
            }
        }
        if (n == 0 && ok) r.slot_pos[(size_t)s * r.capacity + pos % r.capacity] = pos;
    } else if constexpr (EPI == EPI_GELU_BF16) {
        *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(a.y) + (size_t)m * a.ldy + n) =
            make_uint2(bf16x2(gelu_tanh(v.x), gelu_tanh(v.y)), bf16x2(gelu_tanh(v.z), gelu_tanh(v.w)));
    } else {
        float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(a.y) + (size_t)m * a.ldy + n);
        if constexpr (EPI == EPI_ACCUM) {
            const float4 r = *dst;
            v.x += r.x, v.y += r.y, v.z += r.z, v.w += r.w;
        }
        *dst = v;
    }
}

// grid (N / BN, ceil(M / 128), splits), clusters of (1, 1, splits), 128 threads.
// With splits > 1, CTA `split` of a cluster multiplies K blocks
// [split * kb / splits, (split + 1) * kb / splits), stages its partial tile in its
// shared memory, and after a cluster barrier sums rows
// [split * 128 / splits, (split + 1) * 128 / splits) of the tile over the
// partials of every CTA of the cluster, read in split order.
template <int BN, int EPI>
__global__ void __launch_bounds__(NTHREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, Args a) {
    using S = Shape<BN>;
    constexpr int STAGES = S::STAGES, KB = S::KB;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                         ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + S::BAR_OFF);
    uint64_t* empty = full + STAGES;
    uint64_t* done = empty + STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    float* sbias = reinterpret_cast<float*>(sm + S::BAR_OFF + S::BAR_BYTES);
    __shared__ int s_fail;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nt = blockIdx.x, mt = blockIdx.y, split = blockIdx.z;  // split = the CTA's rank in its cluster
    const int n0 = nt * BN, m0 = mt * BM;
    const int kb_total = a.K / BK;
    const int kb0 = split * kb_total / a.splits, kb1 = (split + 1) * kb_total / a.splits;
    const int nkb = kb1 - kb0;  // >= 1: the host keeps at least one K block per split
    const int nch = (nkb + KB - 1) / KB;          // boxes of KB K blocks (ring stages) this CTA multiplies
    const int pre = nch < STAGES ? nch : STAGES;  // stages whose weight boxes load before the wait

    int fills[STAGES] = {};  // producer: loads issued per stage
    if (tid == 0) {
        // ---- TMA producer.  Its barriers first; the weight boxes of the first
        // stages do not depend on the kernel before this one, so they are
        // requested at once, ahead of the TMEM allocation and the block barrier.
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
        s_fail = 0;
        prefetch_tmap(&ta);
        prefetch_tmap(&tb);
        for (int c = 0; c < pre; c++) {
            mbar_expect_tx(&full[c], S::STAGE);
            tma_load_3d(sm + c * S::STAGE + S::A_STAGE, &tb, 0, n0, kb0 + c * KB, &full[c]);
        }
    } else if (warp == 1) {
        tmem_alloc(tmem_slot, S::TMEM_COLS);
    } else if (warp >= 2) {
        // the bias (a weight: no kernel writes it) into shared memory while the tiles are in flight
        for (int c = tid - 64; c < BN; c += 64) sbias[c] = a.bias ? a.bias[n0 + c] : 0.f;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tmem_slot;

    if (tid == 0) {
        // the activation boxes after the kernel ahead has finished (programmatic
        // dependent launch).  A box may reach past this CTA's K range: the K
        // blocks of the next split (read, never multiplied) or past K (zero fill).
        asm volatile("griddepcontrol.wait;" ::: "memory");
        for (int c = 0; c < pre; c++) {
            tma_load_3d(sm + c * S::STAGE, &ta, 0, m0, kb0 + c * KB, &full[c]);
            fills[c]++;
        }
        // stage c % STAGES again once the MMAs reading it have completed
        for (int c = pre; c < nch; c++) {
            const int s = c % STAGES;
            if (!mbar_wait(&empty[s], ((c / STAGES) - 1) & 1, WAIT_LIMIT)) {
                atomicOr(&s_fail, 1);
                break;
            }
            unsigned char* st = sm + s * S::STAGE;
            mbar_expect_tx(&full[s], S::STAGE);
            tma_load_3d(st + S::A_STAGE, &tb, 0, n0, kb0 + c * KB, &full[s]);
            tma_load_3d(st, &ta, 0, m0, kb0 + c * KB, &full[s]);
            fills[s]++;
        }
    } else if (tid == 32) {
        // ---- MMA issuer: D[128 x BN] (+)= A[128 x 64] B[BN x 64]^T per K block, 4 MMAs of K = 16
        constexpr uint32_t IDESC = idesc_f16(1u, 0u, BM, BN);
        for (int c = 0; c < nch; c++) {
            const int s = c % STAGES;
            if (!mbar_wait(&full[s], (c / STAGES) & 1, WAIT_LIMIT)) {
                atomicOr(&s_fail, 1);
                break;
            }
            tc_fence_after();
            const uint32_t base = smem_u32(sm + s * S::STAGE);
            const int nq = min(KB, nkb - c * KB);  // the box's K blocks inside this CTA's range
            for (int q = 0; q < nq; q++) {
                const uint32_t aa = base + q * A_BYTES, ba = base + S::A_STAGE + q * S::B_BYTES;
#pragma unroll
                for (int kk = 0; kk < BK / 16; kk++)
                    umma_f16(tbase, sdesc_sw128(aa + 32 * kk, 16, 1024), sdesc_sw128(ba + 32 * kk, 16, 1024), IDESC,
                             (c > 0 || q > 0 || kk > 0) ? 1u : 0u);
            }
            umma_commit(&empty[s]);
        }
        umma_commit(done);  // arrives once every MMA issued above has completed
    }
    // The other lanes of the producer and MMA warps wait here, at a warp barrier,
    // instead of polling the accumulator barrier beside their working lane.
    __syncwarp();
    // (the producer has waited for the kernel ahead already; every thread does
    // before the epilogue's global accesses)
    asm volatile("griddepcontrol.wait;" ::: "memory");

    // ---- the accumulator
    if (!mbar_wait(done, 0, WAIT_LIMIT)) atomicOr(&s_fail, 1);
    tc_fence_after();
    // TMEM -> the stage ring (free now: every MMA has completed), as a [128][BN]
    // fp32 tile with rows TS floats apart (16-byte stores of the 8 lanes of a
    // shared-memory phase land in distinct bank quads).  A CTA that gave up
    // stages garbage, never stored: its cluster writes nothing.
    float* tile = reinterpret_cast<float*>(sm);
    {
        const int r = warp * 32 + lane;
        const uint32_t taddr = tbase + ((uint32_t)(warp * 32) << 16);
#pragma unroll
        for (int c = 0; c < BN; c += 16) {
            float v[16];
            tmem_ld16(taddr + c, v);  // warp-collective
#pragma unroll
            for (int j = 0; j < 16; j += 4)
                *reinterpret_cast<float4*>(tile + r * S::TS + c + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        }
    }
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    __syncthreads();

    // ---- epilogue: row-contiguous, BN / 4 threads per row, 16-byte pieces
    constexpr int TPR = BN / 4, RPP = NTHREADS / TPR;  // threads per row, rows per pass
    const int cq = (tid % TPR) * 4, rq = tid / TPR;
    const float4 b4 = *reinterpret_cast<const float4*>(sbias + cq);
    bool good = s_fail == 0;
    if (a.splits == 1) {
        if (good) {
#pragma unroll 4
            for (int rr = rq; rr < BM; rr += RPP)
                if (m0 + rr < a.M)
                    finish4<EPI>(a, m0 + rr, n0 + cq, *reinterpret_cast<const float4*>(tile + rr * S::TS + cq), b4);
        }
    } else {
        cluster_sync();  // every partial tile (and every CTA's s_fail) is in place
        uint32_t peer_tile[MAX_SPLITS];
#pragma unroll
        for (int sp = 0; sp < MAX_SPLITS; sp++) {
            peer_tile[sp] = 0;
            if (sp < a.splits) {
                peer_tile[sp] = peer_addr(tile, (uint32_t)sp);
                good = good && ld_peer_int(peer_addr(&s_fail, (uint32_t)sp)) == 0;
            }
        }
        const int r_lo = split * BM / a.splits, r_hi = (split + 1) * BM / a.splits;
        if (good) {
            // two rows per round: every partial of both is requested before any is summed
            for (int rr = r_lo + rq; rr < r_hi; rr += 2 * RPP) {
                const int r2 = rr + RPP;
                const uint32_t o1 = (uint32_t)(rr * S::TS + cq) * 4, o2 = (uint32_t)(r2 * S::TS + cq) * 4;
                float4 p1[MAX_SPLITS], p2[MAX_SPLITS];
#pragma unroll
                for (int sp = 0; sp < MAX_SPLITS; sp++) {
                    if (sp < a.splits) {
                        p1[sp] = ld_peer4(peer_tile[sp] + o1);
                        if (r2 < r_hi) p2[sp] = ld_peer4(peer_tile[sp] + o2);
                    }
                }
                float4 v1 = p1[0], v2 = p2[0];
#pragma unroll
                for (int sp = 1; sp < MAX_SPLITS; sp++) {
                    if (sp < a.splits) {
                        v1.x += p1[sp].x, v1.y += p1[sp].y, v1.z += p1[sp].z, v1.w += p1[sp].w;
                        v2.x += p2[sp].x, v2.y += p2[sp].y, v2.z += p2[sp].z, v2.w += p2[sp].w;
                    }
                }
                if (m0 + rr < a.M) finish4<EPI>(a, m0 + rr, n0 + cq, v1, b4);
                if (r2 < r_hi && m0 + r2 < a.M) finish4<EPI>(a, m0 + r2, n0 + cq, v2, b4);
            }
        }
        cluster_sync();  // no CTA leaves while the others still read its tile
    }
    if (s_fail && tid == 0) {
        // gave up here: record it, then let every load issued land before the
        // shared memory is released (the MMAs have completed: `done` follows them)
        atomicOr(a.err, DERR_TIMEOUT);
        for (int s = 0; s < STAGES; s++)
            if (fills[s] > 0) mbar_wait(&full[s], (fills[s] - 1) & 1, WAIT_LIMIT);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_free(tbase, S::TMEM_COLS);
    }
}

// ---------------------------------------------------------------- CTA pairs

template <int BN>
struct PairShape {
    static constexpr int A_H = 64 * BK * 2;            // this CTA's 64 rows of x per K block: 8 KB
    static constexpr int B_H = (BN / 2) * BK * 2;      // its BN/2 rows of W^T per K block
    static constexpr int STAGE = A_H + B_H;            // multiple of 1024 (swizzle-atom alignment)
    static constexpr int STAGES = RING_STAGES;
    static constexpr uint32_t TMEM_COLS = BN / 2 < 32 ? 32 : BN / 2;
    static constexpr int TS = BN + 4;                  // row stride (floats) of the staged 64-row tile
    static constexpr int BAR_OFF = STAGES * STAGE;
    static constexpr int BAR_BYTES = ((8 * (3 * STAGES + 1) + 4) + 127) / 128 * 128;
    // at least 120 KB: one CTA per SM, so that the pairs spread over the SMs
    static constexpr int SMEM_NEED = BAR_OFF + BAR_BYTES + BN * 4 + 1024;
    static constexpr int SMEM = SMEM_NEED < 120 * 1024 ? 120 * 1024 : SMEM_NEED;
    static_assert(STAGE % 1024 == 0, "stage alignment");
    static_assert(64 * TS * 4 <= STAGES * STAGE, "the output rows are staged in the stage ring");
    static_assert(SMEM <= 227 * 1024, "shared memory per CTA");
};

// grid (2 * N / BN, ceil(M / 128)), clusters of (2, 1, 1), 128 threads.  A CTA
// pair computes the 128 x BN output tile at rows m0.., columns n0..: CTA r (its
// rank in the cluster) loads rows m0 + 64 r .. + 63 of x and rows
// n0 + r BN/2 .. of W^T, and the even CTA issues tcgen05.mma.cta_group::2
// (M = 128, N = BN) over both CTAs' tiles; each CTA's TMEM receives its own 64
// output rows, columns [0, BN/2) in lanes 0-63 and [BN/2, BN) in lanes 64-127.
// So each CTA streams 64 + BN/2 operand rows per K block where an unpaired
// 128 x BN/2 tile would stream 128 + BN/2.
// Stage protocol: the even CTA's producer waits for the stage to be free (its
// `empty`, committed by the MMAs), sets the stage's byte count for both CTAs on
// its `full`, signals the odd CTA's `go` for that stage, and loads its halves;
// the odd CTA loads its halves only after `go`, so no copy is ever in flight that
// the even CTA does not account for; both CTAs' copies complete on the even
// CTA's `full`.  The MMAs' completion is multicast to both CTAs' `done`.
template <int BN, int EPI>
__global__ void __launch_bounds__(NTHREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, Args a) {
    using S = PairShape<BN>;
    constexpr int STAGES = S::STAGES;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                         ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + S::BAR_OFF);
    uint64_t* empty = full + STAGES;
    uint64_t* go = empty + STAGES;
    uint64_t* done = go + STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    float* sbias = reinterpret_cast<float*>(sm + S::BAR_OFF + S::BAR_BYTES);
    __shared__ int s_fail;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster_rank();
    const bool lead = rank == 0;
    const int n0 = (blockIdx.x >> 1) * BN, m0 = blockIdx.y * BM;
    const int a_row = m0 + 64 * (int)rank, b_row = n0 + (BN / 2) * (int)rank;
    const int nkb = a.K / BK;
    const int pre = nkb < STAGES ? nkb : STAGES;

    if (warp == 0) tmem_alloc_pair(tmem_slot, S::TMEM_COLS);
    if (tid == 32) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            mbar_init(&go[s], 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
        s_fail = 0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // both CTAs' barriers exist before either touches the other's
    cluster_arrive();
    cluster_wait();
    const uint32_t tbase = *tmem_slot;

    int fills[STAGES] = {};  // even CTA's producer: fills accounted per stage (both CTAs' bytes)
    const uint32_t full0 = peer_addr(full, 0);  // the even CTA's `full` barriers, in the cluster window
    if (tid == 0) {
        prefetch_tmap(&ta);
        prefetch_tmap(&tb);
        if (lead) {
            const uint32_t peer_go = peer_addr(go, 1);
            // stages of the first K blocks: weight tiles before waiting for the kernel ahead
            for (int i = 0; i < pre; i++) {
                mbar_expect_tx(&full[i], 2 * S::STAGE);
                mbar_arrive_remote(peer_go + i * 8);
                tma_load_3d_pair(sm + i * S::STAGE + S::A_H, &tb, 0, b_row, i, full0 + i * 8);
                fills[i]++;
            }
            asm volatile("griddepcontrol.wait;" ::: "memory");
            for (int i = 0; i < pre; i++) tma_load_3d_pair(sm + i * S::STAGE, &ta, 0, a_row, i, full0 + i * 8);
            for (int i = pre; i < nkb; i++) {
                const int s = i % STAGES;
                if (!mbar_wait(&empty[s], ((i / STAGES) - 1) & 1, WAIT_LIMIT)) {
                    atomicOr(&s_fail, 1);
                    break;
                }
                mbar_expect_tx(&full[s], 2 * S::STAGE);
                mbar_arrive_remote(peer_go + s * 8);
                unsigned char* st = sm + s * S::STAGE;
                tma_load_3d_pair(st + S::A_H, &tb, 0, b_row, i, full0 + s * 8);
                tma_load_3d_pair(st, &ta, 0, a_row, i, full0 + s * 8);
                fills[s]++;
            }
        } else {
            for (int i = 0; i < nkb; i++) {
                const int s = i % STAGES;
                if (!mbar_wait(&go[s], (i / STAGES) & 1, WAIT_LIMIT)) {
                    atomicOr(&s_fail, 1);
                    break;
                }
                unsigned char* st = sm + s * S::STAGE;
                tma_load_3d_pair(st + S::A_H, &tb, 0, b_row, i, full0 + s * 8);
                if (i == 0) asm volatile("griddepcontrol.wait;" ::: "memory");
                tma_load_3d_pair(st, &ta, 0, a_row, i, full0 + s * 8);
            }
        }
    } else if (tid == 32 && lead) {
        // ---- MMA issuer of the pair: D[128 x BN] (+)= A[128 x 64] B[BN x 64]^T per stage
        constexpr uint32_t IDESC = idesc_f16(1u, 0u, 2 * 64, BN);
        for (int i = 0; i < nkb; i++) {
            const int s = i % STAGES;
            if (!mbar_wait(&full[s], (i / STAGES) & 1, WAIT_LIMIT)) {
                atomicOr(&s_fail, 1);
                break;
            }
            tc_fence_after();
            const uint32_t aa = smem_u32(sm + s * S::STAGE), ba = aa + S::A_H;
#pragma unroll
            for (int kk = 0; kk < BK / 16; kk++)
                umma_f16_pair(tbase, sdesc_sw128(aa + 32 * kk, 16, 1024), sdesc_sw128(ba + 32 * kk, 16, 1024), IDESC,
                              (i > 0 || kk > 0) ? 1u : 0u);
            umma_commit_pair(&empty[s]);
        }
        umma_commit_pair_mc(done, 0x3);  // both CTAs: every MMA issued above has completed
    } else if (warp >= 2) {
        for (int c = tid - 64; c < BN; c += 64) sbias[c] = a.bias ? a.bias[n0 + c] : 0.f;
    }
    __syncwarp();
    asm volatile("griddepcontrol.wait;" ::: "memory");

    // ---- this CTA's 64 rows: warp w reads lanes 32w..32w+31, i.e. rows (w & 1) * 32 + lane
    // and the column half (w >> 1)
    if (!mbar_wait(done, 0, WAIT_LIMIT)) atomicOr(&s_fail, 1);
    tc_fence_after();
    float* tile = reinterpret_cast<float*>(sm);
    {
        const int r = (warp & 1) * 32 + lane, c0 = (warp >> 1) * (BN / 2);
        const uint32_t taddr = tbase + ((uint32_t)(warp * 32) << 16);
#pragma unroll
        for (int c = 0; c < BN / 2; c += 16) {
            float v[16];
            tmem_ld16(taddr + c, v);  // warp-collective
#pragma unroll
            for (int j = 0; j < 16; j += 4)
                *reinterpret_cast<float4*>(tile + r * S::TS + c0 + c + j) =
                    make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        }
    }
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    tc_fence_before();
    cluster_arrive();  // this CTA is done with its TMEM (the pair frees it together below)
    __syncthreads();
    constexpr int TPR = BN / 4, RPP = NTHREADS / TPR;
    const int cq = (tid % TPR) * 4, rq = tid / TPR;
    const float4 b4 = *reinterpret_cast<const float4*>(sbias + cq);
    if (s_fail == 0) {
#pragma unroll 4
        for (int rr = rq; rr < 64; rr += RPP)
            if (a_row + rr < a.M)
                finish4<EPI>(a, a_row + rr, n0 + cq, *reinterpret_cast<const float4*>(tile + rr * S::TS + cq), b4);
    } else if (tid == 0) {
        atomicOr(a.err, DERR_TIMEOUT);
        // the even CTA lets every copy it accounted for (its own and the odd CTA's) land
        for (int s = 0; s < STAGES; s++)
            if (fills[s] > 0) mbar_wait(&full[s], (fills[s] - 1) & 1, WAIT_LIMIT);
    }
    cluster_wait();
    tc_fence_after();
    if (warp == 0) tmem_free_pair(tbase, S::TMEM_COLS);
}

template <int BN, int EPI>
cudaError_t prepare_pair(int dev) {
    static bool attr_set[64] = {};
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemm_pair_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             PairShape<BN>::SMEM);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    return cudaSuccess;
}

template <int BN>
void config_pair(cudaLaunchConfig_t& cfg, cudaLaunchAttribute (&attr)[3], const Args& a, cudaStream_t st, bool pdl) {
    cfg = {};
    cfg.gridDim = dim3(2 * (a.N / BN), (a.M + BM - 1) / BM, 1);
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = PairShape<BN>::SMEM;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = with_priority(attr, pdl ? 2 : 1);
}

template <int BN, int EPI>
cudaError_t launch_pair_t(const CUtensorMap& ta, const CUtensorMap& tb, const Args& a, cudaStream_t st, bool pdl) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = prepare_pair<BN, EPI>(dev);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[3];
    config_pair<BN>(cfg, attr, a, st, pdl);
    return cudaLaunchKernelEx(&cfg, gemm_pair_kernel<BN, EPI>, ta, tb, a);
}

template <int BN>
cudaError_t launch_pair_bn(const CUtensorMap& ta, const CUtensorMap& tb, const Args& a, int epi, cudaStream_t st,
                           bool pdl) {
    switch (epi) {
        case EPI_STORE: return launch_pair_t<BN, EPI_STORE>(ta, tb, a, st, pdl);
        case EPI_ACCUM: return launch_pair_t<BN, EPI_ACCUM>(ta, tb, a, st, pdl);
        case EPI_GELU_BF16: return launch_pair_t<BN, EPI_GELU_BF16>(ta, tb, a, st, pdl);
        case EPI_QKV_RING: return launch_pair_t<BN, EPI_QKV_RING>(ta, tb, a, st, pdl);
        default: return cudaErrorInvalidValue;
    }
}

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

template <int BN>
void config(cudaLaunchConfig_t& cfg, cudaLaunchAttribute (&attr)[3], const Args& a, int splits, cudaStream_t st,
            bool pdl) {
    cfg = {};
    cfg.gridDim = dim3(a.N / BN, (a.M + BM - 1) / BM, splits);
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = Shape<BN>::SMEM;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = splits;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = with_priority(attr, pdl ? 2 : 1);
}

template <int BN, int EPI>
cudaError_t prepare(int dev) {
    static bool attr_set[64] = {};  // per device
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        cudaError_t e =
            cudaFuncSetAttribute(gemm_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, Shape<BN>::SMEM);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    return cudaSuccess;
}

template <int BN, int EPI>
cudaError_t launch_t(const CUtensorMap& ta, const CUtensorMap& tb, const Args& a, cudaStream_t st, bool pdl) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = prepare<BN, EPI>(dev);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[3];
    config<BN>(cfg, attr, a, a.splits, st, pdl);
    return cudaLaunchKernelEx(&cfg, gemm_kernel<BN, EPI>, ta, tb, a);
}

// Clusters of `splits` CTAs of the (BN, EPI) kernel that fit on the device at once.
template <int BN, int EPI>
int active_clusters(int splits) {
    static std::mutex mu;
    static std::map<std::tuple<int, int>, int> cache;  // (device, splits)
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find({dev, splits});
    if (it != cache.end()) return it->second;
    int n = 0;
    if (prepare<BN, EPI>(dev) == cudaSuccess) {
        Args a{};
        a.M = BM, a.N = BN, a.K = BK * splits, a.splits = splits;
        cudaLaunchConfig_t cfg;
        cudaLaunchAttribute attr[3];
        config<BN>(cfg, attr, a, splits, nullptr, false);
        cfg.numAttrs = 1;  // the cluster shape only
        if (cudaOccupancyMaxActiveClusters(&n, gemm_kernel<BN, EPI>, &cfg) != cudaSuccess) n = 0;
    }
    cudaGetLastError();  // a failed query leaves no error behind for the next call
    cache[{dev, splits}] = n;
    return n;
}

template <int BN>
int active_clusters_bn(int epi, int splits) {
    switch (epi) {
        case EPI_STORE: return active_clusters<BN, EPI_STORE>(splits);
        case EPI_ACCUM: return active_clusters<BN, EPI_ACCUM>(splits);
        case EPI_QKV_RING: return active_clusters<BN, EPI_QKV_RING>(splits);
        default: return active_clusters<BN, EPI_GELU_BF16>(splits);
    }
}

int active_clusters_of(int bn, int epi, int splits) {
    return bn == 128 ? active_clusters_bn<128>(epi, splits)
                     : bn == 64 ? active_clusters_bn<64>(epi, splits) : active_clusters_bn<32>(epi, splits);
}

template <int BN>
cudaError_t launch_bn(const CUtensorMap& ta, const CUtensorMap& tb, const Args& a, int epi, cudaStream_t st,
                      bool pdl) {
    switch (epi) {
        case EPI_STORE: return launch_t<BN, EPI_STORE>(ta, tb, a, st, pdl);
        case EPI_ACCUM: return launch_t<BN, EPI_ACCUM>(ta, tb, a, st, pdl);
        case EPI_GELU_BF16: return launch_t<BN, EPI_GELU_BF16>(ta, tb, a, st, pdl);
        case EPI_QKV_RING: return launch_t<BN, EPI_QKV_RING>(ta, tb, a, st, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

// Cost of a plan in SM cycles, calibrated on B200 launches of these kernels at
// 256 rows: a CTA's K blocks cost about (128 + bn) x 128 bytes of shared-memory
// traffic each way (TMA writes, the MMAs read; whole boxes are written), at
// ~128 bytes per cycle; a split adds about 4 000 cycles of cluster barriers and
// distributed-shared-memory latency, plus the partials each CTA reads (about 20
// bytes per cycle).  CTA pairs (cta_group::2) are not chosen: at 256 rows they
// measured 1.5-2x slower than the best one-CTA plan (QKV 11.9 vs 7.2 us), and
// are reached only by an explicit request (mb_gemm_bf16 with splits = -1).
Plan choose(int M, int N, int K, int epi) {
    const int m_tiles = (M + BM - 1) / BM, kb = K / BK;
    Plan best{32, 1, 0};
    double best_cost = -1;
    auto consider = [&](Plan p, double cost) {
        if (best_cost < 0 || cost < best_cost) best_cost = cost, best = p;
    };
    for (int bn : {128, 64, 32}) {
        if (N % bn) continue;
        const int tiles = m_tiles * (N / bn);  // one cluster per output tile
        for (int s = 1; s <= MAX_SPLITS && s <= kb; s++) {
            // one wave: every cluster resident at once
            const int fit = active_clusters_of(bn, epi, s);
            if (fit <= 0 || tiles > fit) break;
            const int k_blocks = (kb + s - 1) / s, box = kb_per_box(bn);
            const int written = (k_blocks + box - 1) / box * box;
            double cost = (double)(BM + bn) * BK * 2 * (written + k_blocks) / 128.0;
            if (s > 1) cost += 4000.0 + (double)BM * bn * 4 * (s - 1) / s / 20.0;
            consider(Plan{bn, s, 0}, cost);
        }
    }
    return best;  // nothing fits one wave (very large M): 32-wide tiles, no split
}

bool make_map(CUtensorMap* m, const void* base, int k, int rows, int box_rows, int box_kb) {
    auto fn = encode_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) || k % BK || box_kb < 1) return false;
    cuuint64_t dims[3] = {(cuuint64_t)BK, (cuuint64_t)rows, (cuuint64_t)(k / BK)};
    cuuint64_t strides[2] = {(cuuint64_t)k * 2, (cuuint64_t)BK * 2};
    cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)box_rows, (cuuint32_t)box_kb};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t launch(const CUtensorMap& ta, const CUtensorMap& tb, const Args& a, const Plan& p, int epi,
                   cudaStream_t st, bool pdl) {
    if (a.M <= 0 || a.K % BK || a.N % p.bn || p.splits < 1 || p.splits > MAX_SPLITS || a.K / BK < p.splits ||
        (p.pair && p.splits != 1))
        return cudaErrorInvalidValue;
    Args b = a;
    b.splits = p.splits;
    if (p.pair) {
        switch (p.bn) {
            case 128: return launch_pair_bn<128>(ta, tb, b, epi, st, pdl);
            case 64: return launch_pair_bn<64>(ta, tb, b, epi, st, pdl);
            case 32: return launch_pair_bn<32>(ta, tb, b, epi, st, pdl);
            default: return cudaErrorInvalidValue;
        }
    }
    switch (p.bn) {
        case 128: return launch_bn<128>(ta, tb, b, epi, st, pdl);
        case 64: return launch_bn<64>(ta, tb, b, epi, st, pdl);
        case 32: return launch_bn<32>(ta, tb, b, epi, st, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace gemm
}  // namespace mb

// ---------------------------------------------------------------- C ABI

extern "C" {

MB_API int mb_gemm_bf16(int32_t m, int32_t n, int32_t k, const void* x, const void* wt, const float* bias, void* y,
                        int32_t epi, int32_t bn, int32_t splits, int32_t* status, void* cuda_stream) {
    using namespace mb::gemm;
    if (m < 0 || n <= 0 || k <= 0 || k % BK || n % 32 || epi < EPI_STORE || epi > EPI_GELU_BF16) return MB_ERR_ARG;
    if ((bn != 0 && bn != 32 && bn != 64 && bn != 128) || splits < -1 || splits > MAX_SPLITS ||
        (bn == 0) != (splits == 0) || (bn && n % bn) || splits > k / BK)
        return MB_ERR_ARG;
    if (m == 0) return MB_OK;
    auto mis = [](const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) != 0; };
    if (!x || !wt || !y || !status || mis(x, 16) || mis(wt, 16) || mis(y, 16) || mis(bias, 16) || mis(status, 4))
        return MB_ERR_ARG;
    const Plan p = bn ? (splits < 0 ? Plan{bn, 1, 1} : Plan{bn, splits, 0}) : choose(m, n, k, epi);
    CUtensorMap ta, tb;
    if (!make_map(&ta, x, k, m, a_box_rows(p), box_kb(p)) || !make_map(&tb, wt, k, n, b_box_rows(p), box_kb(p)))
        return MB_ERR_CUDA;
    Args a;
    a.M = m, a.N = n, a.K = k, a.splits = p.splits;
    a.bias = bias, a.y = y, a.ldy = n;
    a.err = status;
    return launch(ta, tb, a, p, epi, static_cast<cudaStream_t>(cuda_stream), false) == cudaSuccess ? MB_OK
                                                                                                    : MB_ERR_CUDA;
}

}  // extern "C"
