// Persistent, pipelined flash-decode (append + RoPE + attention): the hot path.
//
// Same results as decode_kernel (mb_decode.cu) -- reference semantics
// ROPE_SPLIT_RING/_CODEC + ATTEND_RING/_CODEC, kernels-decode.ts:216-327, 590-714 --
// organised for bandwidth:
//   * one CTA per SM: producer warp(s) and consumer warps; every consumer warp
//     is an independent stream-K worker.  All (item, head, chunk) units of the
//     launch (8 KB of K + 8 KB of V each) form one sequence, cut into #workers
//     contiguous equal shares: balance within one unit, whatever the windows;
//   * lane 0 of a producer warp streams each of its workers' units into that
//     worker's ring of stages with 1-D bulk copies (no multicast): the K and V chunk, the
//     chunk's slot positions, and -- at a window's first unit -- the query row and
//     RoPE row, and in the chunk holding the new slot the new k / v rows;
//   * a consumer warp needs no block barrier: lane = slot for the scores (rotated
//     16-byte reads, conflict-free), warp shuffles for max / sum, lane = 2 dims for
//     P.V, an online-softmax merge into a running (m, l, acc) per window.  A window
//     wholly inside the worker's share is finished in registers; one cut by a
//     share boundary publishes a partial, and the last worker to take the window's
//     ticket combines.
// All waits are bounded; a worker that gives up flags MB_ERR_TIMEOUT and the
// producer drains every copy in flight before the CTA exits.
#include "mb_internal.cuh"
#include "mb_ptx.cuh"

namespace mb {
namespace {

#ifndef MB_PERSIST_NW
#define MB_PERSIST_NW 4
#endif
#ifndef MB_PERSIST_NP
#define MB_PERSIST_NP 4
#endif
#ifndef MB_PERSIST_NS
#define MB_PERSIST_NS 3
#endif
#ifndef MB_PERSIST_UNIT
#define MB_PERSIST_UNIT 8192
#endif
#ifndef MB_PERSIST_NMAX
#define MB_PERSIST_NMAX 1024
#endif
constexpr int NW = MB_PERSIST_NW;          // consumer warps (workers) per CTA
constexpr int NP = MB_PERSIST_NP;          // producer warps; producer p feeds workers p, p+NP, ...
constexpr int NS = MB_PERSIST_NS;          // stages per worker
constexpr int NTHREADS = 32 * (NW + NP);
constexpr int NMAX = MB_PERSIST_NMAX;      // items a launch may hold (prologue arrays in shared memory)
constexpr int UNIT_BYTES = MB_PERSIST_UNIT;  // K (and V) bytes per unit

template <typename T>
struct Shape {
    static constexpr int E = sizeof(T);
    static constexpr int ROWS = UNIT_BYTES / (HD * E);  // 32 (fp32) / 64 (16-bit) slots per unit
    static constexpr int RPL = (ROWS + 31) / 32;        // slots per lane
    static constexpr int RB = HD * E;                   // bytes per slot row
    static constexpr int VPR = RB / 16;                 // 16-byte vectors per row
};

struct alignas(128) Stage {
    unsigned char k[UNIT_BYTES];
    unsigned char v[UNIT_BYTES];
    int32_t sp[UNIT_BYTES / 128];  // slot positions of the unit's rows
    float q[HD];           // raw query row (window start only)
    float cs[HD];          // RoPE (cos, sin) row at the query position
    float kn[HD];          // raw new key row (unit holding the new slot)
    float vn[HD];          // new value row
};

struct Smem {
    Stage st[NW][NS];
    int32_t pos[NMAX];
    int32_t str[NMAX];
    int32_t prefix[NMAX + 1];       // units before item i (heads x chunks)
    alignas(16) float qs[NW][HD];   // roped query of each worker's current window
    uint64_t full[NW][NS], empty[NW][NS];
    int32_t consumed[NW];
    int32_t scan[8];
};

__device__ __forceinline__ float2 rope2(float2 v, float2 cs) {
    return make_float2(__fadd_rn(__fmul_rn(v.x, cs.x), -__fmul_rn(v.y, cs.y)),
                       __fadd_rn(__fmul_rn(v.y, cs.x), __fmul_rn(v.x, cs.y)));
}

template <typename T>
struct St2;
template <>
struct St2<float> {
    __device__ static void st(float* p, float2 v) { *reinterpret_cast<float2*>(p) = v; }
    __device__ static float2 ld(const float* p) { return *reinterpret_cast<const float2*>(p); }
};
template <>
struct St2<__nv_bfloat16> {
    __device__ static void st(__nv_bfloat16* p, float2 v) {
        *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(v.x, v.y);
    }
    __device__ static float2 ld(const __nv_bfloat16* p) {
        return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
    }
};
template <>
struct St2<__half> {
    __device__ static void st(__half* p, float2 v) { *reinterpret_cast<__half2*>(p) = __floats2half2_rn(v.x, v.y); }
    __device__ static float2 ld(const __half* p) { return __half22float2(*reinterpret_cast<const __half2*>(p)); }
};

// dot of one 16-byte vector of a stored row (vector index v) with the query
template <typename T>
__device__ __forceinline__ float dot_vec(uint4 raw, const float4* q4, int v, float acc) {
    if constexpr (sizeof(T) == 4) {
        const float4 kf = *reinterpret_cast<const float4*>(&raw);
        const float4 qf = q4[v];
        acc = fmaf(kf.x, qf.x, acc);
        acc = fmaf(kf.y, qf.y, acc);
        acc = fmaf(kf.z, qf.z, acc);
        return fmaf(kf.w, qf.w, acc);
    } else {
        const float4 qa = q4[2 * v], qb = q4[2 * v + 1];
        const uint32_t* w = reinterpret_cast<const uint32_t*>(&raw);
        const float2 a = St2<T>::ld(reinterpret_cast<const T*>(&w[0]));
        const float2 b = St2<T>::ld(reinterpret_cast<const T*>(&w[1]));
        const float2 c = St2<T>::ld(reinterpret_cast<const T*>(&w[2]));
        const float2 d = St2<T>::ld(reinterpret_cast<const T*>(&w[3]));
        acc = fmaf(a.x, qa.x, acc);
        acc = fmaf(a.y, qa.y, acc);
        acc = fmaf(b.x, qa.z, acc);
        acc = fmaf(b.y, qa.w, acc);
        acc = fmaf(c.x, qb.x, acc);
        acc = fmaf(c.y, qb.y, acc);
        acc = fmaf(d.x, qb.z, acc);
        return fmaf(d.y, qb.w, acc);
    }
}

struct Cursor {
    int item, head, chunk, nsplit;
};

__device__ __forceinline__ int nsplit_of(int pos, int C, int rows_per_unit) {
    return (min(pos + 1, C) + rows_per_unit - 1) / rows_per_unit;
}

__device__ __forceinline__ int64_t share_start(int64_t w, int64_t total, int64_t workers) {
    return w * total / workers;
}

// the worker whose (non-empty) share holds unit u
__device__ __forceinline__ int64_t worker_of(int64_t u, int64_t total, int64_t workers) {
    int64_t w = (u * workers) / total;
    while (w + 1 < workers && share_start(w + 1, total, workers) <= u) w++;
    while (w > 0 && share_start(w, total, workers) > u) w--;
    return w;
}

// The shares holding units of the window [ws, we), from the one holding ws to
// the one holding we-1 (empty shares never appear).  A part is stored at the
// offset of its first unit in the window, so slots are unique.
struct PartWalk {
    int64_t ws, we, total, workers, w;
    __device__ PartWalk(int64_t ws_, int64_t we_, int64_t total_, int64_t workers_)
        : ws(ws_), we(we_), total(total_), workers(workers_), w(worker_of(ws_, total_, workers_)) {}
    __device__ int offset() const {
        const int64_t st = share_start(w, total, workers);
        return (int)((st > ws ? st : ws) - ws);
    }
    __device__ bool next() {
        const int64_t nx = share_start(w + 1, total, workers);
        if (nx >= we) return false;
        w = worker_of(nx, total, workers);
        return true;
    }
};

// A worker's walk over its units (the same in the producer and the consumer).
template <int ROWS>
struct Walker {
    const Smem* sm;
    int n, H, C;
    Cursor c;
    __device__ void start(int64_t u) {
        int lo = 0, hi = n - 1;  // the last item with prefix <= u holds unit u
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (sm->prefix[mid] <= u) lo = mid;
            else hi = mid - 1;
        }
        c.item = lo;
        c.nsplit = nsplit_of(sm->pos[lo], C, ROWS);
        const int rem = (int)(u - sm->prefix[lo]);
        c.head = rem / c.nsplit;
        c.chunk = rem % c.nsplit;
    }
    __device__ void advance() {
        if (++c.chunk == c.nsplit) {
            c.chunk = 0;
            if (++c.head == H) {
                c.head = 0;
                do {
                    c.item++;
                } while (c.item < n && sm->prefix[c.item + 1] == sm->prefix[c.item]);
                if (c.item < n) c.nsplit = nsplit_of(sm->pos[c.item], C, ROWS);
            }
        }
    }
};

template <typename T, bool APPEND>
__global__ void __launch_bounds__(NTHREADS, 1)
    decode_persist_kernel(RingView r, Scratch sc, int part_stride, int n, const int32_t* __restrict__ streams,
                          const int32_t* __restrict__ positions, const float* __restrict__ q_in, int q_stride,
                          float* __restrict__ out) {
    using S = Shape<T>;
    constexpr int ROWS = S::ROWS, RPL = S::RPL, RB = S::RB, VPR = S::VPR;
    extern __shared__ unsigned char smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int C = r.capacity, H = r.heads, HID = H * HD;

    // ---- prologue: positions, streams and the unit prefix over items (every CTA)
    constexpr int PER = (NMAX + NTHREADS - 1) / NTHREADS;
    int local[PER];
    int lsum = 0;
    const int i0 = tid * PER;
#pragma unroll
    for (int k = 0; k < PER; k++) {
        const int i = i0 + k;
        int units = 0;
        if (i < n) {
            const int s = streams[i], p = positions[i];
            int bad = 0;
            if (s < 0 || s >= r.streams) bad |= DERR_STREAM;
            if (p < 0 || p >= r.max_position) bad |= DERR_POSITION;
            else if (!r.wrap && p >= C) bad |= DERR_CAPACITY;
            if (bad && blockIdx.x == 0) atomicOr(r.err, bad);
            sm.pos[i] = p;
            sm.str[i] = s;
            units = bad ? 0 : H * nsplit_of(p, C, ROWS);
        }
        local[k] = units;
        lsum += units;
    }
    int incl = lsum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) sm.scan[warp] = incl;
    if (tid == 0) {
        for (int w = 0; w < NW; w++) {
            sm.consumed[w] = 0;
            for (int s = 0; s < NS; s++) {
                mbar_init(&sm.full[w][s], 1);
                mbar_init(&sm.empty[w][s], 1);
            }
        }
        fence_mbar_init();
    }
    __syncthreads();
    int run = incl - lsum;
    for (int w = 0; w < warp; w++) run += sm.scan[w];
#pragma unroll
    for (int k = 0; k < PER; k++) {
        const int i = i0 + k;
        if (i < n) sm.prefix[i] = run;
        run += local[k];
    }
    if (tid == NTHREADS - 1) sm.prefix[n] = run;
    __syncthreads();
    const int64_t total = sm.prefix[n];
    if (total == 0) return;
    const int64_t workers = (int64_t)gridDim.x * NW;

    if (warp < NP) {
        // ================================================================ producer
        if (lane != 0) return;
        Walker<ROWS> wk[NW];
        int nunits[NW], issued[NW], maxu = 0;
        for (int w = warp; w < NW; w += NP) {
            const int64_t gw = (int64_t)blockIdx.x * NW + w;
            const int64_t ub = share_start(gw, total, workers);
            nunits[w] = (int)(share_start(gw + 1, total, workers) - ub);
            issued[w] = 0;
            maxu = max(maxu, nunits[w]);
            wk[w].sm = &sm;
            wk[w].n = n;
            wk[w].H = H;
            wk[w].C = C;
            if (nunits[w] > 0) wk[w].start(ub);
        }
        bool stop = false;
        for (int k = 0; k < maxu && !stop; k++) {
            for (int w = warp; w < NW; w += NP) {
                if (k >= nunits[w]) continue;
                const int s = k % NS;
                if (k >= NS && !mbar_wait(&sm.empty[w][s], ((k / NS) - 1) & 1, WAIT_LIMIT)) {
                    atomicOr(r.err, DERR_TIMEOUT);
                    stop = true;
                    break;
                }
                const Cursor& c = wk[w].c;
                const int pos = sm.pos[c.item], sid = sm.str[c.item];
                const int count = min(pos + 1, C);
                const int j0 = c.chunk * ROWS, rows = min(ROWS, count - j0);
                const int newslot = pos % C;
                const bool has_new = APPEND && newslot >= j0 && newslot < j0 + rows;
                const bool first = c.chunk == 0 || k == 0;
                const uint32_t kv_bytes = (uint32_t)rows * RB;
                const uint32_t sp_bytes = (uint32_t)((rows + 3) & ~3) * 4;
                const uint32_t extra = (first ? 2u : 0u) + (has_new ? (first ? 2u : 3u) : 0u);
                Stage& stg = sm.st[w][s];
                mbar_expect_tx(&sm.full[w][s], 2 * kv_bytes + sp_bytes + extra * HD * 4);
                const T* kb = reinterpret_cast<const T*>(r.kv) + (((size_t)sid * 2 + 0) * H + c.head) * (size_t)C * HD;
                const T* vb = reinterpret_cast<const T*>(r.kv) + (((size_t)sid * 2 + 1) * H + c.head) * (size_t)C * HD;
                bulk_g2s(stg.k, kb + (size_t)j0 * HD, kv_bytes, &sm.full[w][s]);
                bulk_g2s(stg.v, vb + (size_t)j0 * HD, kv_bytes, &sm.full[w][s]);
                bulk_g2s(stg.sp, r.slot_pos + (size_t)sid * C + j0, sp_bytes, &sm.full[w][s]);
                const float* row = q_in + (size_t)c.item * q_stride;
                const float* csrow = reinterpret_cast<const float*>(r.rope) + (size_t)pos * HD;
                if (first) {
                    bulk_g2s(stg.q, row + c.head * HD, HD * 4, &sm.full[w][s]);
                    bulk_g2s(stg.cs, csrow, HD * 4, &sm.full[w][s]);
                }
                if (has_new) {
                    if (!first) bulk_g2s(stg.cs, csrow, HD * 4, &sm.full[w][s]);
                    bulk_g2s(stg.kn, row + HID + c.head * HD, HD * 4, &sm.full[w][s]);
                    bulk_g2s(stg.vn, row + 2 * HID + c.head * HD, HD * 4, &sm.full[w][s]);
                }
                issued[w] = k + 1;
                wk[w].advance();
            }
        }
        // drain: every copy issued must land before the CTA exits
        for (int w = warp; w < NW; w += NP)
            for (int kk = max(0, issued[w] - NS); kk < issued[w]; kk++) {
                if (kk < *(volatile int32_t*)&sm.consumed[w]) continue;
                mbar_wait(&sm.full[w][kk % NS], (kk / NS) & 1, WAIT_LIMIT);
            }
        return;
    }

    // ==================================================================== consumer warp = worker
    const int w = warp - NP;
    const int64_t gw = (int64_t)blockIdx.x * NW + w;
    const int64_t u_begin = share_start(gw, total, workers), u_end = share_start(gw + 1, total, workers);
    const int nunits = (int)(u_end - u_begin);
    if (nunits == 0) return;
    Walker<ROWS> wk;
    wk.sm = &sm;
    wk.n = n;
    wk.H = H;
    wk.C = C;
    wk.start(u_begin);
    float* qs = sm.qs[w];
    float a0 = 0.f, a1 = 0.f;  // this lane's two output dims of the running window
    float m_run = -INFINITY, l_run = 0.f;
    int64_t win_start = -1;

    for (int k = 0; k < nunits; k++) {
        const Cursor& c = wk.c;
        const int s = k % NS;
        Stage& stg = sm.st[w][s];
        const bool got = __all_sync(0xffffffffu, mbar_wait(&sm.full[w][s], (k / NS) & 1, WAIT_LIMIT));
        if (!got) {
            if (lane == 0) atomicOr(r.err, DERR_TIMEOUT);
            break;
        }
        const int pos = sm.pos[c.item];
        const int count = min(pos + 1, C);
        const int j0 = c.chunk * ROWS, rows = min(ROWS, count - j0);
        const int newslot = pos % C;
        const bool has_new = APPEND && newslot >= j0 && newslot < j0 + rows;
        if (c.chunk == 0 || k == 0) {  // a window starts: its roped query
            win_start = sm.prefix[c.item] + (int64_t)c.head * c.nsplit;
            m_run = -INFINITY;
            l_run = 0.f;
            a0 = a1 = 0.f;
            float2 qv = make_float2(stg.q[2 * lane], stg.q[2 * lane + 1]);
            if (APPEND) qv = rope2(qv, make_float2(stg.cs[2 * lane], stg.cs[2 * lane + 1]));
            qs[2 * lane] = qv.x;
            qs[2 * lane + 1] = qv.y;
        }
        if (has_new) {  // the append: rope k, store K/V, substitute the row on chip
            const int sid = sm.str[c.item];
            T* kb = reinterpret_cast<T*>(r.kv) + (((size_t)sid * 2 + 0) * H + c.head) * (size_t)C * HD;
            T* vb = reinterpret_cast<T*>(r.kv) + (((size_t)sid * 2 + 1) * H + c.head) * (size_t)C * HD;
            const float2 kr = rope2(make_float2(stg.kn[2 * lane], stg.kn[2 * lane + 1]),
                                    make_float2(stg.cs[2 * lane], stg.cs[2 * lane + 1]));
            const float2 vv = make_float2(stg.vn[2 * lane], stg.vn[2 * lane + 1]);
            St2<T>::st(kb + (size_t)newslot * HD + 2 * lane, kr);
            St2<T>::st(vb + (size_t)newslot * HD + 2 * lane, vv);
            St2<T>::st(reinterpret_cast<T*>(stg.k + (newslot - j0) * RB) + 2 * lane, kr);
            St2<T>::st(reinterpret_cast<T*>(stg.v + (newslot - j0) * RB) + 2 * lane, vv);
            if (lane == 0) {
                stg.sp[newslot - j0] = pos;
                if (c.head == 0) r.slot_pos[(size_t)sid * C + newslot] = pos;
            }
        }
        __syncwarp();

        // ---- scores: lane owns slots lane (+32); rotated 16-byte reads
        const float4* q4 = reinterpret_cast<const float4*>(qs);
        float sv[RPL];
        float m = -INFINITY;
#pragma unroll
        for (int rr = 0; rr < RPL; rr++) {
            const int j = lane + 32 * rr;
            bool live = false;
            if (j < rows) {
                const int stored = stg.sp[j];
                live = stored >= 0 && pos - stored >= 0 && pos - stored < C;
            }
            float dot = 0.f;
            if (live) {
                const uint4* kp = reinterpret_cast<const uint4*>(stg.k + j * RB);
#pragma unroll
                for (int kk = 0; kk < VPR; kk++) {
                    const int v = (kk + lane) & (VPR - 1);
                    dot = dot_vec<T>(kp[v], q4, v, dot);
                }
            }
            sv[rr] = live ? dot * (SCALE * LOG2E) : -INFINITY;
            m = fmaxf(m, sv[rr]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float p[RPL], l = 0.f;
#pragma unroll
        for (int rr = 0; rr < RPL; rr++) {
            p[rr] = sv[rr] == -INFINITY ? 0.f : exp2f(sv[rr] - m);
            l += p[rr];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);

        // ---- P.V: lane owns dims 2*lane, 2*lane+1; p of slot j comes from lane j % 32
        float b0 = 0.f, b1 = 0.f;
#pragma unroll
        for (int rr = 0; rr < RPL; rr++) {
            const int jend = min(32, rows - 32 * rr);
#pragma unroll 8
            for (int jj = 0; jj < 32; jj++) {
                const float pj = __shfl_sync(0xffffffffu, p[rr], jj);
                if (jj < jend) {
                    const float2 vv =
                        St2<T>::ld(reinterpret_cast<const T*>(stg.v + (32 * rr + jj) * RB) + 2 * lane);
                    b0 = fmaf(pj, vv.x, b0);
                    b1 = fmaf(pj, vv.y, b1);
                }
            }
        }
        __syncwarp();
        if (lane == 0) {  // the stage is no longer read: hand it back to the producer
            sm.consumed[w] = k + 1;
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&sm.empty[w][s])) : "memory");
        }
        // ---- merge into the window's running state
        if (m != -INFINITY) {
            const float M = fmaxf(m_run, m);
            const float wa = exp2f(m_run - M), wb = exp2f(m - M);
            a0 = a0 * wa + b0 * wb;
            a1 = a1 * wa + b1 * wb;
            l_run = l_run * wa + l * wb;
            m_run = M;
        }
        // ---- window finished here?  (its last unit, or the end of this worker's share)
        if (c.chunk == c.nsplit - 1 || k == nunits - 1) {
            const int64_t win_end = win_start + c.nsplit;
            float* dst = out + (size_t)c.item * HID + c.head * HD + 2 * lane;
            if (win_start >= u_begin && win_end <= u_end) {
                const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
                *reinterpret_cast<float2*>(dst) = make_float2(a0 * inv, a1 * inv);
            } else {
                int nparts = 1;
                for (PartWalk pw(win_start, win_end, total, workers); pw.next();) nparts++;
                const int my_off = (int)((u_begin > win_start ? u_begin : win_start) - win_start);
                float* pbase = sc.part + ((size_t)c.item * H + c.head) * part_stride * (2 + HD);
                float* mine = pbase + (size_t)my_off * (2 + HD);
                mine[2 + 2 * lane] = a0;
                mine[3 + 2 * lane] = a1;
                if (lane == 0) {
                    mine[0] = m_run;
                    mine[1] = l_run;
                }
                __syncwarp();
                int ticket = 0;
                if (lane == 0) {
                    __threadfence();
                    ticket = atomicAdd(&sc.counters[(size_t)c.item * H + c.head], 1);
                }
                ticket = __shfl_sync(0xffffffffu, ticket, 0);
                if (ticket == nparts - 1) {
                    __threadfence();
                    float Mx = -INFINITY;
                    {
                        PartWalk pw(win_start, win_end, total, workers);
                        do Mx = fmaxf(Mx, __ldcg(pbase + (size_t)pw.offset() * (2 + HD)));
                        while (pw.next());
                    }
                    float L = 0.f, o0 = 0.f, o1 = 0.f;
                    PartWalk pw(win_start, win_end, total, workers);
                    do {
                        const float* q = pbase + (size_t)pw.offset() * (2 + HD);
                        const float mq = __ldcg(q);
                        if (mq != -INFINITY) {
                            const float wt = exp2f(mq - Mx);
                            L = fmaf(__ldcg(q + 1), wt, L);
                            o0 = fmaf(__ldcg(q + 2 + 2 * lane), wt, o0);
                            o1 = fmaf(__ldcg(q + 3 + 2 * lane), wt, o1);
                        }
                    } while (pw.next());
                    const float inv = L > 0.f ? 1.f / L : 0.f;
                    *reinterpret_cast<float2*>(dst) = make_float2(o0 * inv, o1 * inv);
                    if (lane == 0) sc.counters[(size_t)c.item * H + c.head] = 0;
                }
            }
        }
        wk.advance();
    }
}

int sm_count(int dev) {
    static int cache[64] = {};
    if (dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = v > 0 ? v : 148;
    }
    return cache[dev];
}

template <typename T, bool APPEND>
cudaError_t launch_t(const RingView& r, const Scratch& s, int n, const int32_t* streams, const int32_t* positions,
                     const float* q, int q_stride, float* out, cudaStream_t st) {
    static bool attr_set[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    const size_t bytes = sizeof(Smem) + 128;
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(decode_persist_kernel<T, APPEND>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)bytes);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    const int part_stride = persist_part_stride(sizeof(T) == 4 ? MB_F32 : MB_BF16, r.capacity);
    decode_persist_kernel<T, APPEND><<<sm_count(dev), NTHREADS, bytes, st>>>(r, s, part_stride, n, streams, positions,
                                                                              q, q_stride, out);
    return cudaGetLastError();
}

}  // namespace

int persist_part_stride(int dtype, int capacity) {
    const int rows = UNIT_BYTES / (HD * (dtype == MB_F32 ? 4 : 2));
    return (capacity + rows - 1) / rows;
}

bool decode_persist_supported(const RingView& r, int n, int q_stride) {
    return n > 0 && n <= NMAX && (r.capacity % 4) == 0 && (q_stride % 4) == 0;
}

cudaError_t launch_decode_persist(int dtype, bool append, const RingView& r, const Scratch& s, int n,
                                  const int32_t* streams, const int32_t* positions, const float* q, int q_stride,
                                  float* out, cudaStream_t st) {
    switch (dtype) {
        case MB_F32:
            return append ? launch_t<float, true>(r, s, n, streams, positions, q, q_stride, out, st)
                          : launch_t<float, false>(r, s, n, streams, positions, q, q_stride, out, st);
        case MB_BF16:
            return append ? launch_t<__nv_bfloat16, true>(r, s, n, streams, positions, q, q_stride, out, st)
                          : launch_t<__nv_bfloat16, false>(r, s, n, streams, positions, q, q_stride, out, st);
        default:
            return append ? launch_t<__half, true>(r, s, n, streams, positions, q, q_stride, out, st)
                          : launch_t<__half, false>(r, s, n, streams, positions, q, q_stride, out, st);
    }
}

}  // namespace mb
