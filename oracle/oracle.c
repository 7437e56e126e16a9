/*
 * oracle.c -- CPU restatement of the reference's KV-ring / RoPE / attention path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker, never the product:
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg (and its
 * `--impl reference` arm) may load it.  The product path (mockbird_b200) never
 * links, imports or calls anything here, and has no CPU fallback.
 *
 * What it restates (paths are inside the reference project liyu1981/mockbird):
 *   - ROPE_SPLIT_RING   src/lib/tts/engine/kernels-decode.ts:216-241   (orc_rope_split_ring)
 *   - ROPE_SPLIT_CODEC  src/lib/tts/engine/kernels-decode.ts:679-714   (wrapping slot = pos % C,
 *                                                                        slots[slot] = pos)
 *   - ATTEND_RING       src/lib/tts/engine/kernels-decode.ts:254-327   (orc_attend_ring, mode 0)
 *   - ATTEND_RING_CODEC src/lib/tts/engine/kernels-decode.ts:590-667   (live-slot mask)
 *   - attend()          tools/onnx-probe/ref-decode.mjs:138-160        (orc_attend_ring, mode 1, fp64)
 *   - ROPE_SPLIT_CACHE  src/lib/tts/engine/kernels-batch.ts:194-234    (orc_prefill)
 *   - ATTENTION_SCORES / _SOFTMAX / _APPLY kernels-batch.ts:246-350    (orc_prefill)
 *   - ring reset        src/lib/tts/engine/codec.ts:279-282 (slots <- -1)
 *   - RoPE table        tools/onnx-probe/ref-decode.mjs:111-124 (inv_freq and angles in fp64)
 *
 * Conventions (docs/moss-tts-runtime-analysis.md:929-977):
 *   q | k | v split of the fused 2304-wide row; head-major [12][64] inside each;
 *   out[2i]   = v[2i]  *c - v[2i+1]*s
 *   out[2i+1] = v[2i+1]*c + v[2i]  *s        c,s = cos/sin(pos * theta^(-2i/64))
 *   scale 0.125, masked score -3e38, K stored after RoPE, V raw.
 *
 * Ring layout (the B200 library's, restated here so the bytes can be compared):
 *   kv[layer][stream][kv(0=K,1=V)][head][slot][64]  in the storage dtype
 *   slot_pos[layer][stream][slot]  int32, -1 = empty
 *
 * Rounding points (so that gathered cache bytes are bit-exact with the GPU):
 *   - cos/sin table: double angle, double cos/sin, rounded once to fp32;
 *   - rotation in fp32 as two products and one add, no fused multiply-add
 *     (this file is compiled with -ffp-contract=off);
 *   - K and V rounded to the storage dtype (round-to-nearest-even) when stored.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_HD 64
#define ORC_NEG (-3.0e38f)

enum { ORC_F32 = 0, ORC_BF16 = 1, ORC_F16 = 2 };

typedef struct {
    int32_t layers;
    int32_t streams;
    int32_t heads;
    int32_t capacity;
    int32_t dtype;
    int32_t wrap;
} orc_geom;

/* ---------------------------------------------------------------- storage */

static inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}
static inline uint16_t f32_to_f16(float f) {
    _Float16 h = (_Float16)f;
    uint16_t u;
    memcpy(&u, &h, 2);
    return u;
}
static inline float f16_to_f32(uint16_t u) {
    _Float16 h;
    memcpy(&h, &u, 2);
    return (float)h;
}

static inline size_t esize(int dtype) { return dtype == ORC_F32 ? 4 : 2; }

/* round an fp32 value to the storage dtype and back */
static inline float round_to(int dtype, float x) {
    if (dtype == ORC_BF16) return bf16_to_f32(f32_to_bf16(x));
    if (dtype == ORC_F16) return f16_to_f32(f32_to_f16(x));
    return x;
}

static inline void store_elem(int dtype, void* base, size_t idx, float x) {
    if (dtype == ORC_F32) ((float*)base)[idx] = x;
    else if (dtype == ORC_BF16) ((uint16_t*)base)[idx] = f32_to_bf16(x);
    else ((uint16_t*)base)[idx] = f32_to_f16(x);
}
static inline float load_elem(int dtype, const void* base, size_t idx) {
    if (dtype == ORC_F32) return ((const float*)base)[idx];
    if (dtype == ORC_BF16) return bf16_to_f32(((const uint16_t*)base)[idx]);
    return f16_to_f32(((const uint16_t*)base)[idx]);
}

/* element offset of kv[layer][stream][which][head][slot][0] */
static inline size_t kv_off(const orc_geom* g, int layer, int stream, int which, int head, int slot) {
    return (((((size_t)layer * g->streams + stream) * 2 + which) * g->heads + head) * (size_t)g->capacity +
            (size_t)slot) * ORC_HD;
}
static inline size_t sp_off(const orc_geom* g, int layer, int stream) {
    return ((size_t)layer * g->streams + stream) * (size_t)g->capacity;
}

size_t orc_kv_elems(const orc_geom* g) {
    return (size_t)g->layers * g->streams * 2 * g->heads * (size_t)g->capacity * ORC_HD;
}

/* ---------------------------------------------------------------- rope */

/* tab[p*64 + 2i] = cos(p * theta^(-2i/64)), tab[p*64 + 2i + 1] = sin(...), p in [0, P).
 * ref-decode.mjs:111 computes invFreq and the angle in fp64; the product stores
 * fp32 values, so each is rounded once. */
void orc_rope_table(int32_t P, double theta, float* tab) {
    for (int32_t p = 0; p < P; p++) {
        for (int i = 0; i < ORC_HD / 2; i++) {
            double inv = pow(theta, -(2.0 * i) / (double)ORC_HD);
            double ang = (double)p * inv;
            tab[(size_t)p * ORC_HD + 2 * i] = (float)cos(ang);
            tab[(size_t)p * ORC_HD + 2 * i + 1] = (float)sin(ang);
        }
    }
}

/* One 64-wide head: kernels-decode.ts:220-232 (partner = -v[d+1] for even d,
 * +v[d-1] for odd d), computed from the original values (the WGSL reads the
 * partner before the in-place write). */
static inline void rope_head(const float* v, const float* cs, float* out) {
    for (int i = 0; i < ORC_HD / 2; i++) {
        float c = cs[2 * i], s = cs[2 * i + 1];
        float a = v[2 * i], b = v[2 * i + 1];
        float ac = a * c, bs = b * s, bc = b * c, as = a * s;
        out[2 * i] = ac - bs;
        out[2 * i + 1] = bc + as;
    }
}

void orc_rope_rows(int32_t rows, int32_t heads, const float* in, int32_t in_stride, const int32_t* positions,
                   const float* tab, float* out, int32_t out_stride) {
    for (int32_t r = 0; r < rows; r++)
        for (int h = 0; h < heads; h++)
            rope_head(in + (size_t)r * in_stride + h * ORC_HD, tab + (size_t)positions[r] * ORC_HD,
                      out + (size_t)r * out_stride + h * ORC_HD);
}

/* ---------------------------------------------------------------- ring state */

/* codec.ts:279-282: every slot reads as empty (-1).  stream < 0: all streams. */
void orc_reset(const orc_geom* g, int32_t* slot_pos, int32_t stream) {
    for (int l = 0; l < g->layers; l++)
        for (int s = 0; s < g->streams; s++) {
            if (stream >= 0 && s != stream) continue;
            int32_t* sp = slot_pos + sp_off(g, l, s);
            for (int j = 0; j < g->capacity; j++) sp[j] = -1;
        }
}

/*
 * ROPE_SPLIT_RING / ROPE_SPLIT_CODEC for n independent streams of one layer.
 * Item i appends the fused row qkv[i][2304] of stream streams[i] at absolute
 * position positions[i]: Q is roped in place in the row (kernels-decode.ts:229-232),
 * K roped into the key ring and V copied into the value ring at slot pos % C
 * (kernels-decode.ts:709-712), and slot_pos[slot] = pos.
 * Returns 0, or -1 when a position does not fit a non-wrapping ring
 * (decode.ts:719-724).
 */
int orc_rope_split_ring(const orc_geom* g, void* kv, int32_t* slot_pos, const float* tab, int32_t layer, int32_t n,
                        const int32_t* streams, const int32_t* positions, float* qkv) {
    const int HID = g->heads * ORC_HD;
    for (int i = 0; i < n; i++)
        if (positions[i] < 0 || (!g->wrap && positions[i] >= g->capacity)) return -1;
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; i++) {
        int s = streams[i], pos = positions[i];
        int slot = pos % g->capacity;
        float* row = qkv + (size_t)i * 3 * HID;
        const float* cs = tab + (size_t)pos * ORC_HD;
        for (int h = 0; h < g->heads; h++) {
            float q[ORC_HD], k[ORC_HD];
            rope_head(row + h * ORC_HD, cs, q);
            rope_head(row + HID + h * ORC_HD, cs, k);
            memcpy(row + h * ORC_HD, q, sizeof q);
            size_t ko = kv_off(g, layer, s, 0, h, slot), vo = kv_off(g, layer, s, 1, h, slot);
            for (int d = 0; d < ORC_HD; d++) {
                store_elem(g->dtype, kv, ko + d, k[d]);
                store_elem(g->dtype, kv, vo + d, row[2 * HID + h * ORC_HD + d]);
            }
        }
        slot_pos[sp_off(g, layer, s) + slot] = pos;
    }
    return 0;
}

/* live iff stored >= 0 and 0 <= cur - stored < C  (kernels-decode.ts:622-623) */
static inline int slot_live(int32_t stored, int32_t cur, int32_t C) {
    return stored >= 0 && cur - stored >= 0 && cur - stored < C;
}

/* The window scanned for a query at position cur: slots [0, min(cur + 1, C)).
 * Without a wrap these are exactly the reference's valid slots [0, pos + 1)
 * (decode.ts:537-545); once the ring has wrapped it is every slot, as in
 * ATTEND_RING_CODEC. */
static inline int window_count(int32_t cur, int32_t C) { return cur + 1 < C ? cur + 1 : C; }

/* ATTEND_RING_CODEC restated lane-for-lane in fp32: 64-slot tiles in slot order,
 * tree reductions for the tile max and sum in the WGSL's order, online rescale. */
static void attend_head_mirror(const orc_geom* g, const void* kv, size_t kbase, size_t vbase, const int32_t* sp,
                               int32_t cur, const float* q, float* out) {
    const int C = g->capacity, count = window_count(cur, C);
    float acc[ORC_HD], tile[64], red[64];
    int live[64];
    float runMax = ORC_NEG, runSum = 0.0f;
    for (int d = 0; d < ORC_HD; d++) acc[d] = 0.0f;
    for (int base = 0; base < count; base += 64) {
        for (int d = 0; d < 64; d++) {
            int j = base + d;
            float s = ORC_NEG;
            live[d] = (j < count) && slot_live(sp[j], cur, C);
            if (live[d]) {
                float dot = 0.0f;
                for (int i = 0; i < ORC_HD; i++) dot = dot + q[i] * load_elem(g->dtype, kv, kbase + (size_t)j * ORC_HD + i);
                s = dot * 0.125f;
            }
            tile[d] = s;
            red[d] = s;
        }
        for (int t = 32; t > 0; t >>= 1)
            for (int d = 0; d < t; d++) red[d] = fmaxf(red[d], red[d + t]);
        float newMax = fmaxf(runMax, red[0]);
        float corr = expf(runMax - newMax);
        for (int d = 0; d < 64; d++) {
            float e = live[d] ? expf(tile[d] - newMax) : 0.0f;
            tile[d] = e;
            red[d] = e;
        }
        for (int t = 32; t > 0; t >>= 1)
            for (int d = 0; d < t; d++) red[d] = red[d] + red[d + t];
        runSum = runSum * corr + red[0];
        runMax = newMax;
        int stop = base + 64 < count ? base + 64 : count;
        for (int d = 0; d < ORC_HD; d++) {
            float a = acc[d] * corr;
            for (int jj = base; jj < stop; jj++)
                if (live[jj - base]) a = a + tile[jj - base] * load_elem(g->dtype, kv, vbase + (size_t)jj * ORC_HD + d);
            acc[d] = a;
        }
    }
    /* an empty window (nothing live) yields 0; the reference would divide 0/0,
       but its engine always appends the query's own slot first */
    for (int d = 0; d < ORC_HD; d++) out[d] = runSum > 0.0f ? acc[d] / runSum : 0.0f;
}

/* ref-decode.mjs:138-160 in fp64 over the live window in POSITION order. */
static void attend_head_f64(const orc_geom* g, const void* kv, size_t kbase, size_t vbase, const int32_t* sp,
                            int32_t cur, const float* q, float* out) {
    const int C = g->capacity, count = window_count(cur, C);
    double* sc = (double*)malloc(sizeof(double) * (size_t)count);
    int* sl = (int*)malloc(sizeof(int) * (size_t)count);
    int m = 0;
    double mx = -INFINITY;
    for (int p = cur - count + 1; p <= cur; p++) {
        int slot = p % C;
        if (!slot_live(sp[slot], cur, C) || sp[slot] != p) continue;
        double s = 0.0;
        for (int i = 0; i < ORC_HD; i++) s += (double)q[i] * (double)load_elem(g->dtype, kv, kbase + (size_t)slot * ORC_HD + i);
        sc[m] = s * 0.125;
        sl[m] = slot;
        if (sc[m] > mx) mx = sc[m];
        m++;
    }
    double sum = 0.0;
    for (int j = 0; j < m; j++) {
        sc[j] = exp(sc[j] - mx);
        sum += sc[j];
    }
    for (int d = 0; d < ORC_HD; d++) {
        double acc = 0.0;
        for (int j = 0; j < m; j++) acc += (sc[j] / sum) * (double)load_elem(g->dtype, kv, vbase + (size_t)sl[j] * ORC_HD + d);
        out[d] = m ? (float)acc : 0.0f;
    }
    free(sc);
    free(sl);
}

/*
 * Decode attention of n queries (one per stream) against layer `layer`'s rings.
 * q[i] is the ROPED query row (stride q_stride floats; head-major [heads][64]).
 * mode 0: the WGSL tile mirror in fp32 (ATTEND_RING / ATTEND_RING_CODEC);
 * mode 1: the fp64 reference (ref-decode.mjs attend).
 */
void orc_attend_ring(const orc_geom* g, const void* kv, const int32_t* slot_pos, int32_t layer, int32_t n,
                     const int32_t* streams, const int32_t* positions, const float* q, int32_t q_stride, float* ctx,
                     int32_t mode) {
    const int HID = g->heads * ORC_HD;
#pragma omp parallel for collapse(2) schedule(dynamic, 4)
    for (int i = 0; i < n; i++)
        for (int h = 0; h < g->heads; h++) {
            int s = streams[i];
            size_t kb = kv_off(g, layer, s, 0, h, 0), vb = kv_off(g, layer, s, 1, h, 0);
            const int32_t* sp = slot_pos + sp_off(g, layer, s);
            const float* qh = q + (size_t)i * q_stride + h * ORC_HD;
            float* o = ctx + (size_t)i * HID + h * ORC_HD;
            if (mode == 1) attend_head_f64(g, kv, kb, vb, sp, positions[i], qh, o);
            else attend_head_mirror(g, kv, kb, vb, sp, positions[i], qh, o);
        }
}

/* The reference's decode order for one layer: ropeSplitRing then attendRing
 * (decode.ts:527-552).  qkv rows are updated in place (roped Q), ctx [n][768]. */
int orc_append_attend(const orc_geom* g, void* kv, int32_t* slot_pos, const float* tab, int32_t layer, int32_t n,
                      const int32_t* streams, const int32_t* positions, float* qkv, float* ctx, int32_t mode) {
    int rc = orc_rope_split_ring(g, kv, slot_pos, tab, layer, n, streams, positions, qkv);
    if (rc) return rc;
    orc_attend_ring(g, kv, slot_pos, layer, n, streams, positions, qkv, 3 * g->heads * ORC_HD, ctx, mode);
    return 0;
}

/*
 * Gather the live window of (layer, stream) for a query at position cur, in
 * POSITION order: row w holds position cur - W + 1 + w, W = min(cur + 1, C).
 * k_out / v_out: [heads][W][64] in the storage dtype (raw bytes); slots_out[w]
 * = the slot that holds that position, or -1 when the slot holds another
 * position (a hole).  Rows of holes are zero.  Returns W.
 */
int32_t orc_gather(const orc_geom* g, const void* kv, const int32_t* slot_pos, int32_t layer, int32_t stream,
                   int32_t cur, void* k_out, void* v_out, int32_t* slots_out) {
    const int C = g->capacity, W = window_count(cur, C);
    const size_t es = esize(g->dtype);
    const int32_t* sp = slot_pos + sp_off(g, layer, stream);
    for (int w = 0; w < W; w++) {
        int p = cur - W + 1 + w, slot = p % C;
        int ok = sp[slot] == p;
        slots_out[w] = ok ? slot : -1;
        for (int h = 0; h < g->heads; h++) {
            size_t dst = ((size_t)h * W + w) * ORC_HD * es;
            if (ok) {
                memcpy((char*)k_out + dst, (const char*)kv + kv_off(g, layer, stream, 0, h, slot) * es, ORC_HD * es);
                memcpy((char*)v_out + dst, (const char*)kv + kv_off(g, layer, stream, 1, h, slot) * es, ORC_HD * es);
            } else {
                memset((char*)k_out + dst, 0, ORC_HD * es);
                memset((char*)v_out + dst, 0, ORC_HD * es);
            }
        }
    }
    return W;
}

/*
 * Causal prefill of `rows` positions (0..rows-1) for n streams of one layer:
 * ROPE_SPLIT_CACHE (kernels-batch.ts:194-234) writes roped K and raw V to slots
 * 0..rows-1 and ropes Q in place; then ATTENTION_SCORES / _SOFTMAX / _APPLY
 * (kernels-batch.ts:246-350) in fp32 over the stored (storage-rounded) K and V.
 * q_round != 0 rounds the roped Q to the storage dtype before the scores, the
 * rounding point of a tensor-core kernel that reads Q in that dtype.
 * qkv: [n][rows][2304] (Q roped in place), ctx: [n][rows][768].
 * Returns 0, or -1 if rows exceeds the capacity.
 */
int orc_prefill(const orc_geom* g, void* kv, int32_t* slot_pos, const float* tab, int32_t layer, int32_t n,
                const int32_t* streams, int32_t rows, float* qkv, float* ctx, int32_t q_round) {
    const int HID = g->heads * ORC_HD;
    if (rows <= 0 || rows > g->capacity) return -1;
    /* ROPE_SPLIT_CACHE: position = row */
#pragma omp parallel for collapse(2) schedule(static)
    for (int i = 0; i < n; i++)
        for (int r = 0; r < rows; r++) {
            int s = streams[i];
            float* row = qkv + ((size_t)i * rows + r) * 3 * HID;
            const float* cs = tab + (size_t)r * ORC_HD;
            for (int h = 0; h < g->heads; h++) {
                float q[ORC_HD], k[ORC_HD];
                rope_head(row + h * ORC_HD, cs, q);
                rope_head(row + HID + h * ORC_HD, cs, k);
                for (int d = 0; d < ORC_HD; d++) row[h * ORC_HD + d] = q_round ? round_to(g->dtype, q[d]) : q[d];
                size_t ko = kv_off(g, layer, s, 0, h, r), vo = kv_off(g, layer, s, 1, h, r);
                for (int d = 0; d < ORC_HD; d++) {
                    store_elem(g->dtype, kv, ko + d, k[d]);
                    store_elem(g->dtype, kv, vo + d, row[2 * HID + h * ORC_HD + d]);
                }
            }
            slot_pos[sp_off(g, layer, s) + r] = r;
        }
    /* scores -> softmax -> apply, per (stream, head, query) */
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
    for (int i = 0; i < n; i++)
        for (int h = 0; h < g->heads; h++) {
            int s = streams[i];
            size_t kb = kv_off(g, layer, s, 0, h, 0), vb = kv_off(g, layer, s, 1, h, 0);
            float* sc = (float*)malloc(sizeof(float) * (size_t)rows);
            float lane[256];
            for (int q0 = 0; q0 < rows; q0++) {
                const float* qv = qkv + ((size_t)i * rows + q0) * 3 * HID + h * ORC_HD;
                float best = -1e30f;
                for (int j = 0; j <= q0; j++) {
                    float dot = 0.0f;
                    for (int d = 0; d < ORC_HD; d++) dot = dot + qv[d] * load_elem(g->dtype, kv, kb + (size_t)j * ORC_HD + d);
                    sc[j] = dot * 0.125f;
                    best = fmaxf(best, sc[j]);
                }
                /* ATTENTION_SOFTMAX: 256 strided lane sums, then a tree */
                for (int l = 0; l < 256; l++) lane[l] = 0.0f;
                for (int j = 0; j <= q0; j++) {
                    sc[j] = expf(sc[j] - best);
                    lane[j % 256] = lane[j % 256] + sc[j];
                }
                for (int t = 128; t > 0; t >>= 1)
                    for (int l = 0; l < t; l++) lane[l] = lane[l] + lane[l + t];
                float total = lane[0];
                for (int j = 0; j <= q0; j++) sc[j] = sc[j] / total;
                /* ATTENTION_APPLY */
                float* o = ctx + ((size_t)i * rows + q0) * HID + h * ORC_HD;
                for (int d = 0; d < ORC_HD; d++) {
                    float acc = 0.0f;
                    for (int j = 0; j <= q0; j++) acc = acc + sc[j] * load_elem(g->dtype, kv, vb + (size_t)j * ORC_HD + d);
                    o[d] = acc;
                }
            }
            free(sc);
        }
    return 0;
}

/* storage conversions exposed for the tests (round-to-nearest-even) */
void orc_round_to(int32_t dtype, const float* in, float* out, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = round_to(dtype, in[i]);
}

/*
 * The PRNG of tests/gpu/kernels.test.mjs:22-30 exactly as JavaScript evaluates it:
 * `seed >> 17` is an ARITHMETIC shift of the int32 view (sign bits shift in),
 * and the draw is (seed / 0xffffffff) * 2 - 1 in fp64, stored to a Float32Array.
 * Advances *state by n draws and writes them to out (out may be NULL to skip).
 */
void orc_xorshift_js(uint32_t* state, int64_t n, float* out) {
    uint32_t x = *state;
    for (int64_t i = 0; i < n; i++) {
        x ^= x << 13;
        uint32_t t = (x >> 17) | ((x & 0x80000000u) ? 0xFFFF8000u : 0u);
        x ^= t;
        x ^= x << 5;
        if (out) out[i] = (float)(((double)x / 4294967295.0) * 2.0 - 1.0);
    }
    *state = x;
}

/* The same draws before the Float32Array store: the tests scale some draws in
 * fp64 first (`rnd() * 0.1`, kernels.test.mjs:98, :176-178), so the stored value
 * is the fp32 rounding of the scaled double, not a scaled fp32 draw. */
void orc_xorshift_js_f64(uint32_t* state, int64_t n, double* out) {
    uint32_t x = *state;
    for (int64_t i = 0; i < n; i++) {
        x ^= x << 13;
        uint32_t t = (x >> 17) | ((x & 0x80000000u) ? 0xFFFF8000u : 0u);
        x ^= t;
        x ^= x << 5;
        out[i] = ((double)x / 4294967295.0) * 2.0 - 1.0;
    }
    *state = x;
}
