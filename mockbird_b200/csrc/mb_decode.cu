// Decode-side kernels: append + RoPE into the ring, and split-K flash-decode
// attention over the live window, fused into one launch for the hot path.
//
// Reference semantics (liyu1981/mockbird, src/lib/tts/engine/):
//   ROPE_SPLIT_RING  kernels-decode.ts:216-241 / ROPE_SPLIT_CODEC :679-714
//   ATTEND_RING      kernels-decode.ts:254-327 / ATTEND_RING_CODEC :590-667
// The reference runs one 64-lane workgroup per head with a serial 64-FMA dot per
// lane and six barriers per 64-slot tile.  Here every (item, head) window is cut
// into 16 KB chunks of K and V; each CTA pulls its chunk into shared memory with
// two bulk copies (cp.async.bulk, no multicast), scores it with bank-conflict-
// free rotated 16-byte reads, and leaves an (m, l, acc[64]) partial with plain
// stores.  A small kernel launched right behind it (a programmatic dependent)
// folds each window's partials (online-softmax rescale) and writes the context
// row.  No tensor cores: one query per head is a GEMV.
#include "mb_internal.cuh"
#include "mb_ptx.cuh"

namespace mb {


// ---------------------------------------------------------------- storage types

template <typename T>
struct Store;
template <>
struct Store<float> {
    __device__ static float2 load2(const float* p) { return *reinterpret_cast<const float2*>(p); }
    __device__ static void store2(float* p, float2 v) { *reinterpret_cast<float2*>(p) = v; }
    __device__ static float2 round2(float2 v) { return v; }
};
template <>
struct Store<__nv_bfloat16> {
    __device__ static float2 load2(const __nv_bfloat16* p) {
        return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
    }
    __device__ static void store2(__nv_bfloat16* p, float2 v) {
        *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(v.x, v.y);
    }
    __device__ static float2 round2(float2 v) { return __bfloat1622float2(__floats2bfloat162_rn(v.x, v.y)); }
};
template <>
struct Store<__half> {
    __device__ static float2 load2(const __half* p) { return __half22float2(*reinterpret_cast<const __half2*>(p)); }
    __device__ static void store2(__half* p, float2 v) {
        *reinterpret_cast<__half2*>(p) = __floats2half2_rn(v.x, v.y);
    }
    __device__ static float2 round2(float2 v) { return __half22float2(__floats2half2_rn(v.x, v.y)); }
};

// dot of 8 consecutive stored elements (one 16-byte vector) with q[0..7]
__device__ __forceinline__ float dot8(uint4 raw, const float4* q2, float acc, __nv_bfloat16*) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
    float4 qa = q2[0], qb = q2[1];
    float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
    float2 c = __bfloat1622float2(h[2]), d = __bfloat1622float2(h[3]);
    acc = fmaf(a.x, qa.x, acc); acc = fmaf(a.y, qa.y, acc);
    acc = fmaf(b.x, qa.z, acc); acc = fmaf(b.y, qa.w, acc);
    acc = fmaf(c.x, qb.x, acc); acc = fmaf(c.y, qb.y, acc);
    acc = fmaf(d.x, qb.z, acc); acc = fmaf(d.y, qb.w, acc);
    return acc;
}
__device__ __forceinline__ float dot8(uint4 raw, const float4* q2, float acc, __half*) {
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
    float4 qa = q2[0], qb = q2[1];
    float2 a = __half22float2(h[0]), b = __half22float2(h[1]);
    float2 c = __half22float2(h[2]), d = __half22float2(h[3]);
    acc = fmaf(a.x, qa.x, acc); acc = fmaf(a.y, qa.y, acc);
    acc = fmaf(b.x, qa.z, acc); acc = fmaf(b.y, qa.w, acc);
    acc = fmaf(c.x, qb.x, acc); acc = fmaf(c.y, qb.y, acc);
    acc = fmaf(d.x, qb.z, acc); acc = fmaf(d.y, qb.w, acc);
    return acc;
}

// Validate one item against the ring; on failure record why (every thread of
// the CTA evaluates the same condition, so the early return is uniform).
__device__ __forceinline__ bool item_ok(const RingView& r, int s, int pos) {
    int bad = 0;
    if (s < 0 || s >= r.streams) bad |= DERR_STREAM;
    if (pos < 0 || pos >= r.max_position) bad |= DERR_POSITION;
    else if (!r.wrap && pos >= r.capacity) bad |= DERR_CAPACITY;
    if (bad && threadIdx.x == 0) atomicOr(r.err, bad);
    return bad == 0;
}

// ---------------------------------------------------------------- append (a1/a3)

// One CTA per item, one thread per (head, pair): Q roped in place, K roped and V
// copied into slot pos % C, slot_pos[slot] = pos.
template <typename T>
__global__ void __launch_bounds__(384) rope_append_kernel(RingView r, const int32_t* __restrict__ streams,
                                                          const int32_t* __restrict__ positions, float* qkv) {
    const int item = blockIdx.x;
    const int s = streams[item], pos = positions[item];
    if (!item_ok(r, s, pos)) return;
    const int H = r.heads, HID = H * HD, C = r.capacity, slot = pos % C;
    float* row = qkv + (size_t)item * 3 * HID;
    for (int t = threadIdx.x; t < H * 32; t += blockDim.x) {
        const int h = t >> 5, i = t & 31;
        const float2 cs = r.rope[(size_t)pos * 32 + i];
        float2 q = *reinterpret_cast<const float2*>(row + h * HD + 2 * i);
        float2 k = *reinterpret_cast<const float2*>(row + HID + h * HD + 2 * i);
        float2 v = *reinterpret_cast<const float2*>(row + 2 * HID + h * HD + 2 * i);
        *reinterpret_cast<float2*>(row + h * HD + 2 * i) = rope_pair(q, cs);
        T* kd = reinterpret_cast<T*>(r.kv) + (((size_t)s * 2 + 0) * H + h) * (size_t)C * HD + (size_t)slot * HD + 2 * i;
        T* vd = reinterpret_cast<T*>(r.kv) + (((size_t)s * 2 + 1) * H + h) * (size_t)C * HD + (size_t)slot * HD + 2 * i;
        Store<T>::store2(kd, rope_pair(k, cs));
        Store<T>::store2(vd, v);
    }
    if (threadIdx.x == 0) r.slot_pos[(size_t)s * C + slot] = pos;
}

// ---------------------------------------------------------------- decode attention

template <typename T>
struct DecodeShape {
    static constexpr int E = sizeof(T);
    static constexpr int ROWS = 16384 / (HD * E);  // slots per chunk: 64 (f32) / 128 (16-bit)
    static constexpr int TPR = E / 2;              // score threads per slot: 2 (f32) / 1 (16-bit)
    static constexpr int ROW_BYTES = HD * E;
};

// grid (max_splits, heads, n * layers), 128 threads: blockIdx.z = layer * n +
// item, layers consecutive from r's.  APPEND: q_in is the raw qkv row (stride
// q_stride) and this launch also appends K/V; otherwise q_in holds an
// already-roped query.
// One context value of the output row: fp32, or bf16 when the caller feeds it
// straight into a bf16 GEMM (the decoder step).
__device__ __forceinline__ void store_ctx(void* out, bool bf16, size_t i, float v) {
    if (bf16)
        reinterpret_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
    else
        reinterpret_cast<float*>(out)[i] = v;
}

template <typename T, bool APPEND>
__global__ void __launch_bounds__(128) decode_kernel(RingView r, Scratch sc, const int32_t* __restrict__ streams,
                                                     const int32_t* __restrict__ positions,
                                                     const float* __restrict__ q_in, int q_stride, void* out,
                                                     int out_bf16, int pf_dist, int n) {
    using S = DecodeShape<T>;
    constexpr int ROWS = S::ROWS, TPR = S::TPR, RB = S::ROW_BYTES;
    __shared__ __align__(128) unsigned char sk[ROWS * RB];
    __shared__ __align__(128) unsigned char sv[ROWS * RB];
    __shared__ __align__(16) float qs[HD];
    __shared__ float ps[ROWS];
    __shared__ float red[4][HD];
    __shared__ float wmax[4], wsum[4];
    __shared__ __align__(8) uint64_t bar[3];  // K chunk, V chunk, and one nothing signals (wait probe)

    const int c = blockIdx.x, h = blockIdx.y, z = blockIdx.z, tid = threadIdx.x;
    const int layer = z / n, item = z - layer * n;
    const int lane = tid & 31, warp = tid >> 5;
    const int s = streams[item], pos = positions[item];
    if (!item_ok(r, s, pos)) return;
    const int C = r.capacity, H = r.heads, HID = H * HD;
    // this CTA's layer: its ring, slot positions, q rows and output rows
    r.kv = reinterpret_cast<T*>(r.kv) + (size_t)layer * r.kv_layer;
    r.slot_pos += (size_t)layer * r.slot_layer;
    q_in += (size_t)layer * n * q_stride;
    const int count = min(pos + 1, C);
    const int nsplit = (count + ROWS - 1) / ROWS;
    if (c >= nsplit) return;
    const int j0 = c * ROWS, rows = min(ROWS, count - j0);
    const int newslot = pos % C;
    const bool has_new = APPEND && newslot >= j0 && newslot < j0 + rows;

    T* kbase = reinterpret_cast<T*>(r.kv) + (((size_t)s * 2 + 0) * H + h) * (size_t)C * HD;
    T* vbase = reinterpret_cast<T*>(r.kv) + (((size_t)s * 2 + 1) * H + h) * (size_t)C * HD;

    // The K and V chunk go in flight first: the issuing thread initialised the
    // barriers itself; the others meet them only after the barrier below.  In
    // the chunk holding the new slot the copies skip that row (rows [0, jn) and
    // (jn, rows)): the appending threads write it into shared memory themselves,
    // so it never races the ring store of the same row.
    const int jn = has_new ? newslot - j0 : -1;  // chunk row of the new slot, or none
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        mbar_init(&bar[2], 1);
        fence_mbar_init();
        const uint32_t bytes = (uint32_t)(has_new ? rows - 1 : rows) * RB;
        const int a = has_new ? jn : rows;          // first segment [0, a)
        const int b = has_new ? jn + 1 : rows;      // second segment [b, rows)
        mbar_expect_tx(&bar[0], bytes);
        if (a > 0) bulk_g2s(sk, kbase + (size_t)j0 * HD, (uint32_t)a * RB, &bar[0]);
        if (b < rows) bulk_g2s(sk + b * RB, kbase + (size_t)(j0 + b) * HD, (uint32_t)(rows - b) * RB, &bar[0]);
        mbar_expect_tx(&bar[1], bytes);
        if (a > 0) bulk_g2s(sv, vbase + (size_t)j0 * HD, (uint32_t)a * RB, &bar[1]);
        if (b < rows) bulk_g2s(sv + b * RB, vbase + (size_t)(j0 + b) * HD, (uint32_t)(rows - b) * RB, &bar[1]);
    }

    // An idle thread asks L2 for the chunk of the CTA pf_dist places later in
    // launch order (part of a wave of resident CTAs ahead), so that CTA's bulk
    // copies find it there.  Every byte still comes from HBM once.
    if (pf_dist > 0 && tid == 64) {
        const unsigned gx = gridDim.x, gy = gridDim.y;
        const unsigned t = blockIdx.x + gx * (blockIdx.y + gy * blockIdx.z) + (unsigned)pf_dist;
        if (t < gx * gy * gridDim.z) {
            const int c2 = (int)(t % gx), h2 = (int)((t / gx) % gy), z2 = (int)(t / (gx * gy));
            const int l2 = z2 / n, it2 = z2 - l2 * n;
            const int s2 = streams[it2], p2 = positions[it2];
            if (s2 >= 0 && s2 < r.streams && p2 >= 0) {
                const int count2 = min(p2 + 1, C), j2 = c2 * ROWS;
                if (j2 < count2) {
                    const uint32_t bytes2 = (uint32_t)min(ROWS, count2 - j2) * RB;
                    const T* kv2 = reinterpret_cast<const T*>(r.kv) + ((ptrdiff_t)l2 - layer) * (ptrdiff_t)r.kv_layer;
                    const T* k2 = kv2 + (((size_t)s2 * 2 + 0) * H + h2) * (size_t)C * HD;
                    const T* v2 = kv2 + (((size_t)s2 * 2 + 1) * H + h2) * (size_t)C * HD;
                    bulk_prefetch_l2(k2 + (size_t)j2 * HD, bytes2);
                    bulk_prefetch_l2(v2 + (size_t)j2 * HD, bytes2);
                }
            }
        }
    }

    // query (roped here when appending) and, in the chunk holding the new slot,
    // the new K/V row: written to the ring and to its row of the staged chunk
    const float* row = q_in + (size_t)item * q_stride;
    if (tid < 32) {
        float2 qv = *reinterpret_cast<const float2*>(row + h * HD + 2 * tid);
        if (APPEND) qv = rope_pair(qv, r.rope[(size_t)pos * 32 + tid]);
        qs[2 * tid] = qv.x;
        qs[2 * tid + 1] = qv.y;
    } else if (has_new && tid < 64) {
        if constexpr (APPEND) {  // has_new implies APPEND
            const int i = tid - 32;
            const float2 kv = *reinterpret_cast<const float2*>(row + HID + h * HD + 2 * i);
            const float2 vv = *reinterpret_cast<const float2*>(row + 2 * HID + h * HD + 2 * i);
            const float2 kr = rope_pair(kv, r.rope[(size_t)pos * 32 + i]);
            Store<T>::store2(kbase + (size_t)newslot * HD + 2 * i, kr);
            Store<T>::store2(vbase + (size_t)newslot * HD + 2 * i, vv);
            Store<T>::store2(reinterpret_cast<T*>(sk + jn * RB) + 2 * i, kr);
            Store<T>::store2(reinterpret_cast<T*>(sv + jn * RB) + 2 * i, vv);
        }
    }
    if (has_new && h == 0 && tid == 64) r.slot_pos[(size_t)s * C + newslot] = pos;

    // liveness of this thread's score slot (kernels-decode.ts:622-623)
    const int rr = tid / TPR, part = tid % TPR;
    bool live = false;
    if (rr < rows) {
        const int j = j0 + rr;
        const int stored = (has_new && j == newslot) ? pos : r.slot_pos[(size_t)s * C + j];
        live = stored >= 0 && pos - stored >= 0 && pos - stored < C;
    }

    __syncthreads();  // barriers initialised; qs and the new row written

    // ---- K chunk landed?  Each thread waits for itself (bounded; a copy that
    // never lands reads as an empty chunk, and the CTA agrees on that below)
    // (with the wait probe on, this wait and the V chunk's target the barrier
    // nothing signals, so they run out after r.wait_limit cycles)
    bool ok = mbar_wait(&bar[r.wait_probe ? 2 : 0], 0, r.wait_limit);
    if (!ok) live = false;

    // ---- scores: slot rr, 128 bytes per thread, 16-byte vectors read in a
    // per-slot rotated order so the 8 threads of a shared-memory phase hit 8
    // different bank quads
    float dot = 0.f;
    if (live) {
        const uint4* kp = reinterpret_cast<const uint4*>(sk + rr * RB + part * 128);
        const float4* q4 = reinterpret_cast<const float4*>(qs);
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int v = (k + rr + 4 * part) & 7;
            const uint4 raw = kp[v];
            if constexpr (sizeof(T) == 4) {
                const float4 kf = *reinterpret_cast<const float4*>(&raw);
                const float4 qf = q4[part * 8 + v];
                dot = fmaf(kf.x, qf.x, dot);
                dot = fmaf(kf.y, qf.y, dot);
                dot = fmaf(kf.z, qf.z, dot);
                dot = fmaf(kf.w, qf.w, dot);
            } else {
                dot = dot8(raw, q4 + 2 * v, dot, static_cast<T*>(nullptr));
            }
        }
    }
    if (TPR == 2) dot += __shfl_xor_sync(0xffffffffu, dot, 1);
    const float sc2 = live ? dot * (SCALE * LOG2E) : -INFINITY;  // log2-domain score

    float m = sc2;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) wmax[warp] = m;
    ok = __syncthreads_and(ok);
    if (!ok) {
        if (tid == 0) atomicOr(r.err, DERR_TIMEOUT);
        live = false;
    }
    m = fmaxf(fmaxf(wmax[0], wmax[1]), fmaxf(wmax[2], wmax[3]));
    const float p = live ? exp2f(sc2 - m) : 0.f;
    if (part == 0 && rr < ROWS) ps[rr] = p;
    float l = (part == 0) ? p : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) wsum[warp] = l;

    // ---- V chunk (this barrier also publishes ps and wsum)
    const bool okv = __syncthreads_and(mbar_wait(&bar[r.wait_probe ? 2 : 1], 0, r.wait_limit));
    if (ok && !okv && tid == 0) atomicOr(r.err, DERR_TIMEOUT);
    ok = ok && okv;
    // A CTA that gave up still lets both of its copies land (at the default
    // bound) before it can exit, so none writes into a released CTA.
    if (!ok && tid == 0) {
        mbar_wait(&bar[0], 0, WAIT_LIMIT);
        mbar_wait(&bar[1], 0, WAIT_LIMIT);
    }
    l = wsum[0] + wsum[1] + wsum[2] + wsum[3];

    // ---- P.V: warp w takes slots w, w+4, ...; lane owns dims 2*lane, 2*lane+1
    float a0 = 0.f, a1 = 0.f;
    if (ok) {
        for (int j = warp; j < rows; j += 4) {
            const float pj = ps[j];
            const float2 vv = Store<T>::load2(reinterpret_cast<const T*>(sv + j * RB) + 2 * lane);
            a0 = fmaf(pj, vv.x, a0);
            a1 = fmaf(pj, vv.y, a1);
        }
    }
    red[warp][2 * lane] = a0;
    red[warp][2 * lane + 1] = a1;
    __syncthreads();
    float acc = 0.f;
    if (tid < HD) acc = red[0][tid] + red[1][tid] + red[2][tid] + red[3][tid];

    // Programmatic dependent launch: the split-K scratch is shared by every launch,
    // so it (and the output) is touched only once the previous launch has
    // completed; dependents are released only after that, so a chain of launches
    // never reaches further back than one kernel.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const size_t dst = ((size_t)layer * n + item) * HID + h * HD;
    if (nsplit == 1) {
        if (tid < HD) store_ctx(out, out_bf16, dst + tid, l > 0.f ? acc / l : 0.f);
        return;
    }

    // ---- split-K: publish the partial and exit.  fold_kernel, launched right
    // behind this kernel, combines the partials of every window once they are
    // all written (its griddepcontrol.wait orders them), so no CTA waits on a
    // fence or a ticket here.
    float* mine = sc.part + (((size_t)z * H + h) * sc.max_splits + c) * (2 + HD);
    if (tid < HD) mine[2 + tid] = acc;
    if (tid == 0) {
        mine[0] = m;
        mine[1] = l;
    }
}

// The split-K combine: one warp per (item, head) window of more than one chunk.
// Lane l reads split l's (m, l) (and every 32nd after it), the warp reduces the
// maximum and the weighted sum, and lane l then sums dims 2l, 2l+1 of every
// split's acc with that split's weight 2^(m_c - M), the loads of a batch of
// splits in flight together.  Launched as a programmatic dependent of the decode
// kernel: griddepcontrol.wait returns once that kernel has completed and its
// partials are visible.  Dependents are released right away: the next decode
// launch touches the scratch and the output only after its own wait, which
// returns only once this kernel has completed.
// grid (ceil(heads / 4), n * layers), 128 threads: blockIdx.y = layer * n + item.
__global__ void __launch_bounds__(128) fold_kernel(RingView r, Scratch sc, const int32_t* __restrict__ streams,
                                                   const int32_t* __restrict__ positions, void* out, int out_bf16,
                                                   int rows_per_chunk, int n) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    constexpr int PS = 2 + HD;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.x * 4 + warp, z = blockIdx.y;
    const int layer = z / n, item = z - layer * n;
    const int H = r.heads;
    if (h >= H) return;
    const int s = streams[item], pos = positions[item];
    // an item the decode kernel rejected (and flagged) has no partials
    if (s < 0 || s >= r.streams || pos < 0 || pos >= r.max_position || (!r.wrap && pos >= r.capacity)) return;
    const int count = min(pos + 1, r.capacity);
    const int nsplit = (count + rows_per_chunk - 1) / rows_per_chunk;
    if (nsplit <= 1) return;  // the decode kernel wrote the row itself
    const float* base = sc.part + ((size_t)z * H + h) * sc.max_splits * PS;

    float m0 = -INFINITY, l0 = 0.f;  // split `lane`
    if (lane < nsplit) {
        m0 = __ldcg(base + (size_t)lane * PS);
        l0 = __ldcg(base + (size_t)lane * PS + 1);
    }
    float M = m0;
    for (int cc = lane + 32; cc < nsplit; cc += 32) M = fmaxf(M, __ldcg(base + (size_t)cc * PS));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float w0 = m0 == -INFINITY ? 0.f : exp2f(m0 - M);
    float L = l0 * w0;
    for (int cc = lane + 32; cc < nsplit; cc += 32) {
        const float mc = __ldcg(base + (size_t)cc * PS), lc = __ldcg(base + (size_t)cc * PS + 1);
        L = fmaf(lc, mc == -INFINITY ? 0.f : exp2f(mc - M), L);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);

    float a0 = 0.f, a1 = 0.f;
    for (int cb = 0; cb < nsplit; cb += 32) {
        float w = w0;
        if (cb > 0) {
            const int cc = cb + lane;
            const float mc = cc < nsplit ? __ldcg(base + (size_t)cc * PS) : -INFINITY;
            w = mc == -INFINITY ? 0.f : exp2f(mc - M);
        }
        const int nb = min(32, nsplit - cb);
#pragma unroll 8
        for (int k = 0; k < nb; k++) {
            const float wk = __shfl_sync(0xffffffffu, w, k);
            const float2 a = __ldcg(reinterpret_cast<const float2*>(base + (size_t)(cb + k) * PS + 2) + lane);
            a0 = fmaf(a.x, wk, a0);
            a1 = fmaf(a.y, wk, a1);
        }
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    const size_t dst = ((size_t)layer * n + item) * H * HD + h * HD + 2 * lane;
    store_ctx(out, out_bf16, dst, a0 * inv);
    store_ctx(out, out_bf16, dst + 1, a1 * inv);
}

// ---------------------------------------------------------------- small rings (capacity <= 32)

// The same computation for rings of at most 32 slots (the local head's 17-slot
// ring): one warp per (item, head), lane j scores slot j, warp shuffles for the
// softmax, lane l owns dims 2l, 2l+1 of the query, the new row and the context.
// No staging in shared memory and no split-K: a window is at most 32 slots.
// grid (ceil(heads / 4), n * layers), 128 threads: blockIdx.y = layer * n + item.
template <typename T, bool APPEND>
__global__ void __launch_bounds__(128) decode_small_kernel(RingView r, const int32_t* __restrict__ streams,
                                                           const int32_t* __restrict__ positions,
                                                           const float* __restrict__ q_in, int q_stride, void* out,
                                                           int out_bf16, int n) {
    __shared__ __align__(16) float qs[4][HD];  // the warp's roped query
    __shared__ __align__(16) float kn[4][HD];  // the warp's new K row (storage-rounded)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int layer = blockIdx.y / n, item = blockIdx.y - layer * n;
    const int h = blockIdx.x * 4 + warp;
    const int s = streams[item], pos = positions[item];
    if (!item_ok(r, s, pos)) return;  // uniform over the CTA
    r.kv = reinterpret_cast<T*>(r.kv) + (size_t)layer * r.kv_layer;
    r.slot_pos += (size_t)layer * r.slot_layer;
    q_in += (size_t)layer * n * q_stride;
    const int C = r.capacity, H = r.heads, HID = H * HD;
    const bool head_ok = h < H;
    const int count = min(pos + 1, C), newslot = pos % C;
    const float* row = q_in + (size_t)item * q_stride;
    const T* kbase = reinterpret_cast<const T*>(r.kv) + (((size_t)s * 2 + 0) * H + (head_ok ? h : 0)) * (size_t)C * HD;
    const T* vbase = reinterpret_cast<const T*>(r.kv) + (((size_t)s * 2 + 1) * H + (head_ok ? h : 0)) * (size_t)C * HD;

    // The reads that depend only on (s, pos) go out together, before the first
    // store: the q, k, v of the new row and the K row and stored position of
    // slot `lane`.  The new slot's old K row and position are read too and
    // replaced by the on-chip ones.
    constexpr int NV = HD * (int)sizeof(T) / 16;  // 16-byte pieces of a row
    uint4 raw[NV];
    int stored = -1;
    float2 qv = make_float2(0.f, 0.f), kin = qv, vin = qv, cs = qv;
    if (head_ok) {
        qv = *reinterpret_cast<const float2*>(row + h * HD + 2 * lane);
        if (APPEND) {
            cs = r.rope[(size_t)pos * 32 + lane];
            kin = *reinterpret_cast<const float2*>(row + HID + h * HD + 2 * lane);
            vin = *reinterpret_cast<const float2*>(row + 2 * HID + h * HD + 2 * lane);
        }
        if (lane < count) {
            const uint4* kp = reinterpret_cast<const uint4*>(kbase + (size_t)lane * HD);
#pragma unroll
            for (int v = 0; v < NV; v++) raw[v] = kp[v];
            stored = r.slot_pos[(size_t)s * C + lane];
        }
    }

    float2 vnew = make_float2(0.f, 0.f);
    if (head_ok) {
        if (APPEND) {
            qv = rope_pair(qv, cs);
            const float2 kr = rope_pair(kin, cs);
            Store<T>::store2(const_cast<T*>(kbase) + (size_t)newslot * HD + 2 * lane, kr);
            Store<T>::store2(const_cast<T*>(vbase) + (size_t)newslot * HD + 2 * lane, vin);
            const float2 kq = Store<T>::round2(kr);
            kn[warp][2 * lane] = kq.x;
            kn[warp][2 * lane + 1] = kq.y;
            vnew = Store<T>::round2(vin);
            if (h == 0 && lane == 0) r.slot_pos[(size_t)s * C + newslot] = pos;
        }
        qs[warp][2 * lane] = qv.x;
        qs[warp][2 * lane + 1] = qv.y;
    }
    __syncwarp();

    // ---- lane j: the score of slot j (kernels-decode.ts:622-623 liveness)
    float sc = -INFINITY;
    if (head_ok && lane < count) {
        if (APPEND && lane == newslot) stored = pos;
        if (stored >= 0 && pos - stored >= 0 && pos - stored < C) {
            float dot = 0.f;
            if (APPEND && lane == newslot) {
#pragma unroll 16
                for (int d = 0; d < HD; d++) dot = fmaf(kn[warp][d], qs[warp][d], dot);
            } else {
                const float4* q4 = reinterpret_cast<const float4*>(qs[warp]);
#pragma unroll
                for (int v = 0; v < NV; v++) {
                    if constexpr (sizeof(T) == 4) {
                        const float4 kf = *reinterpret_cast<const float4*>(&raw[v]);
                        const float4 qf = q4[v];
                        dot = fmaf(kf.x, qf.x, dot);
                        dot = fmaf(kf.y, qf.y, dot);
                        dot = fmaf(kf.z, qf.z, dot);
                        dot = fmaf(kf.w, qf.w, dot);
                    } else {
                        dot = dot8(raw[v], q4 + 2 * v, dot, static_cast<T*>(nullptr));
                    }
                }
            }
            sc = dot * (SCALE * LOG2E);
        }
    }
    float m = sc;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float p = sc == -INFINITY ? 0.f : exp2f(sc - m);
    float l = p;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);

    // ---- P.V: lane owns dims 2 lane, 2 lane + 1 (rows of dead slots have p = 0;
    // every row read is inside the ring, so the loads need no guard)
    float a0 = 0.f, a1 = 0.f;
#pragma unroll 4
    for (int j = 0; j < count; j++) {
        const float pj = __shfl_sync(0xffffffffu, p, j);
        const float2 vv = (APPEND && j == newslot) ? vnew : Store<T>::load2(vbase + (size_t)j * HD + 2 * lane);
        a0 = fmaf(pj, vv.x, a0);
        a1 = fmaf(pj, vv.y, a1);
    }
    // outputs only once the previous launch (programmatic dependent launch) has completed
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (head_ok) {
        const size_t dst = ((size_t)layer * n + item) * HID + h * HD + 2 * lane;
        const float inv = l > 0.f ? 1.f / l : 0.f;
        store_ctx(out, out_bf16, dst, a0 * inv);
        store_ctx(out, out_bf16, dst + 1, a1 * inv);
    }
}

// ---------------------------------------------------------------- launchers

template <typename T>
static cudaError_t rope_append_t(const RingView& r, int n, const int32_t* streams, const int32_t* positions,
                                 float* qkv, cudaStream_t st) {
    rope_append_kernel<T><<<n, 384, 0, st>>>(r, streams, positions, qkv);
    return cudaGetLastError();
}

cudaError_t launch_rope_append(int dtype, const RingView& r, int n, const int32_t* streams,
                               const int32_t* positions, float* qkv, cudaStream_t st) {
    switch (dtype) {
        case MB_F32: return rope_append_t<float>(r, n, streams, positions, qkv, st);
        case MB_BF16: return rope_append_t<__nv_bfloat16>(r, n, streams, positions, qkv, st);
        default: return rope_append_t<__half>(r, n, streams, positions, qkv, st);
    }
}

// CTAs between a CTA and the one whose chunk it prefetches into L2 (0: none).
// 1.5 x the SM count (222 on a B200): measured best on the config-2 ring (8
// chunks per window: +3.6 % at full windows) and on config 4 (16 chunks: +1.2 %).
// Off for rings of more than 16 chunks: with long, uneven windows most CTAs a
// fixed distance ahead exit empty, and config 5 (32 chunks) lost 0.4-1.1 %.
// MOCKBIRD_DECODE_PREFETCH=<distance> overrides the choice.
static int decode_prefetch_distance(int max_splits) {
    static const int forced = [] {
        const char* v = getenv("MOCKBIRD_DECODE_PREFETCH");
        return v ? atoi(v) : -1;
    }();
    if (forced >= 0) return forced;
    if (max_splits > 16) return 0;
    static int sms[64] = {};  // per device
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (!sms[dev] && cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        sms[dev] = 0;
        return 0;
    }
    return sms[dev] * 3 / 2;
}

template <typename T>
static cudaError_t decode_t(bool append, const RingView& r, const Scratch& s, int n, const int32_t* streams,
                            const int32_t* positions, const float* q, int q_stride, void* out, cudaStream_t st,
                            bool overlap_previous, bool out_bf16, int layers) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(s.max_splits, r.heads, n * layers);
    cfg.blockDim = dim3(128);
    cfg.stream = st;
    const int ob = out_bf16 ? 1 : 0;
    if (r.capacity <= 32) {  // a window fits one warp
        cfg.gridDim = dim3((r.heads + 3) / 4, n * layers);
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = with_priority(attr, overlap_previous ? 1 : 0, true);
        if (append)
            return cudaLaunchKernelEx(&cfg, decode_small_kernel<T, true>, r, streams, positions, q, q_stride, out, ob,
                                      n);
        return cudaLaunchKernelEx(&cfg, decode_small_kernel<T, false>, r, streams, positions, q, q_stride, out, ob,
                                  n);
    }
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = with_priority(attr, overlap_previous ? 1 : 0, true);
    const int pf = decode_prefetch_distance(s.max_splits);
    cudaError_t e = append ? cudaLaunchKernelEx(&cfg, decode_kernel<T, true>, r, s, streams, positions, q, q_stride,
                                                out, ob, pf, n)
                           : cudaLaunchKernelEx(&cfg, decode_kernel<T, false>, r, s, streams, positions, q, q_stride,
                                                out, ob, pf, n);
    if (e != cudaSuccess || s.max_splits <= 1) return e;
    // the split-K combine, always a programmatic dependent of the decode launch
    cudaLaunchConfig_t fcfg = {};
    fcfg.gridDim = dim3((r.heads + 3) / 4, n * layers);
    fcfg.blockDim = dim3(128);
    fcfg.stream = st;
    cudaLaunchAttribute fattr[2];
    fattr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    fattr[0].val.programmaticStreamSerializationAllowed = 1;
    fcfg.attrs = fattr;
    fcfg.numAttrs = with_priority(fattr, 1);
    return cudaLaunchKernelEx(&fcfg, fold_kernel, r, s, streams, positions, out, ob, DecodeShape<T>::ROWS, n);
}

cudaError_t launch_decode(int dtype, bool append, const RingView& r, const Scratch& s, int n,
                          const int32_t* streams, const int32_t* positions, const float* q, int q_stride,
                          void* out, cudaStream_t st, bool overlap_previous, bool out_bf16, int layers) {
    switch (dtype) {
        case MB_F32:
            return decode_t<float>(append, r, s, n, streams, positions, q, q_stride, out, st, overlap_previous,
                                   out_bf16, layers);
        case MB_BF16:
            return decode_t<__nv_bfloat16>(append, r, s, n, streams, positions, q, q_stride, out, st,
                                           overlap_previous, out_bf16, layers);
        default:
            return decode_t<__half>(append, r, s, n, streams, positions, q, q_stride, out, st, overlap_previous,
                                    out_bf16, layers);
    }
}

}  // namespace mb
