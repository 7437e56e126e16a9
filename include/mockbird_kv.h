/*
 * mockbird_kv.h -- C ABI of the B200 KV-ring / RoPE / attention library.
 *
 * Drop-in for the KV-cache/attention dispatch of the reference's WebGPU engine
 * (liyu1981/mockbird, src/lib/tts/engine/).  Every entry point names the
 * reference interface it replaces.  Plain pointers and sizes only: device
 * pointers are CUDA device addresses, `cuda_stream` is a cudaStream_t (NULL =
 * the legacy default stream), host pointers are ordinary process memory.
 *
 * Geometry.  One context owns, on one GPU, the rings of `streams` independent
 * synthesis streams for `layers` layers:
 *     kv[layer][stream][0=K,1=V][head][slot][64]   storage dtype (f32/bf16/f16)
 *     slot_pos[layer][stream][slot]                 int32 absolute position, -1 = empty
 * A query at position p attends the live slots among [0, min(p + 1, capacity)):
 * slot j is live iff slot_pos[j] >= 0 and 0 <= p - slot_pos[j] < capacity
 * (kernels-decode.ts:622-623).  Appends go to slot p % capacity
 * (kernels-decode.ts:709); K is stored after RoPE, V raw.
 *
 * Row layouts (head-major, kernels-decode.ts:216-241):
 *     qkv row  [3][heads][64] f32   (q | k | v, 2304 floats at 12 heads)
 *     ctx row  [heads][64]    f32
 *
 * Errors.  Every call returns an mb_status; mb_last_error() holds the text.
 * Checks a kernel makes on device data (a stream id or position read from a
 * device array) are reported by the next mb_sync() as MB_ERR_DEVICE; the
 * offending item is skipped, never dereferenced.
 *
 * Threading.  A context is not thread-safe; calls are asynchronous on the
 * given CUDA stream unless documented as blocking.  One item per stream per
 * call: two items with the same stream id in one call race.
 */
#ifndef MOCKBIRD_KV_H
#define MOCKBIRD_KV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define MB_API __attribute__((visibility("default")))
#else
#define MB_API
#endif

typedef struct mb_ctx mb_ctx;

enum mb_dtype { MB_F32 = 0, MB_BF16 = 1, MB_F16 = 2 };

enum mb_status {
    MB_OK = 0,
    MB_ERR_ARG = 1,      /* null pointer, bad size, bad config field            */
    MB_ERR_STREAM = 2,   /* stream index out of range, or repeated in one call  */
    MB_ERR_LAYER = 3,    /* layer index out of range                            */
    MB_ERR_POSITION = 4, /* position < 0 or >= max_position                     */
    MB_ERR_CAPACITY = 5, /* position >= capacity on a non-wrapping ring
                            (decode.ts:719-724), or prefill rows > capacity     */
    MB_ERR_CUDA = 6,     /* a CUDA runtime call failed                          */
    MB_ERR_DEVICE = 7,   /* a kernel rejected an item (see mb_last_error)       */
    MB_ERR_OOM = 8,      /* device allocation failed                            */
    MB_ERR_TIMEOUT = 9   /* a bounded device-side wait gave up                  */
};

typedef struct mb_config {
    int32_t layers;       /* transformer layers with a ring (12)                        */
    int32_t heads;        /* attention heads (12)                                       */
    int32_t head_dim;     /* must be 64                                                 */
    int32_t capacity;     /* ring slots per (layer, stream); gpu.ts:300-306 maxSlots   */
    int32_t streams;      /* independent stream rings in this context                   */
    int32_t dtype;        /* enum mb_dtype of the ring storage                          */
    int32_t wrap;         /* 1: slot = position % capacity (codec.ts ring semantics);
                             0: position >= capacity is MB_ERR_CAPACITY (global ring)  */
    int32_t max_position; /* positions must be < this (RoPE table rows); 0 -> 65536     */
    float rope_theta;     /* RoPE base, 10000 (docs/moss-tts-runtime-analysis.md:929)  */
    int32_t device;       /* CUDA device ordinal                                        */
    int32_t max_batch;    /* largest item count per call; 0 -> streams                  */
} mb_config;

/* Device addresses and strides of a context's state (for tests and tools). */
typedef struct mb_ring_info {
    void* kv;              /* kv[layer][stream][2][head][slot][64]  */
    int32_t* slot_pos;     /* slot_pos[layer][stream][slot]         */
    size_t kv_bytes;
    size_t elem_bytes;     /* 4 (f32) or 2 (bf16/f16)               */
    size_t scratch_bytes;  /* split-K partials + counters           */
} mb_ring_info;

/* Fill `cfg` with the reference's global-ring geometry: 12 layers, 12 heads,
 * 64 dims, capacity 570 (gpu.ts:362), fp32, no wrap, theta 10000, device 0. */
MB_API void mb_config_default(mb_config* cfg);

/* Allocate the rings (all slots empty), the RoPE table and the split-K scratch
 * on cfg->device.  Replaces the KV parts of createGpuEngineFor (gpu.ts:316-388):
 * the PrefillRunner kv buffer (prefill.ts:156-160) and the CodecRunner ring +
 * slot array (codec.ts:204-245). */
MB_API int mb_create(const mb_config* cfg, mb_ctx** out);

/* Free everything the context owns.  GpuTtsEngine.dispose (gpu.ts:283-291). */
MB_API int mb_destroy(mb_ctx* ctx);

/* Mark every slot of `stream` (all streams if stream < 0) empty, all layers.
 * WgpuTtsEngineImpl.reset (gpu.ts:237-242) / CodecRunner.resetRings (codec.ts:279-282). */
MB_API int mb_reset(mb_ctx* ctx, int32_t stream, void* cuda_stream);

/* ROPE_SPLIT_RING / ROPE_SPLIT_CODEC (kernels-decode.ts:216-241, 679-714),
 * dispatched at decode.ts:527-535: for each of n items, rope Q IN PLACE in the
 * qkv row, rope K into the key ring and copy V into the value ring at slot
 * position % capacity, and record the position in slot_pos.
 * streams, positions: device int32[n]; qkv: device f32 [n][3*heads*64]. */
MB_API int mb_rope_append(mb_ctx* ctx, int32_t layer, int32_t n, const int32_t* streams,
                          const int32_t* positions, float* qkv, void* cuda_stream);

/* ATTEND_RING / ATTEND_RING_CODEC (kernels-decode.ts:254-327, 590-667),
 * dispatched at decode.ts:536-552: one already-roped query per item against the
 * item's live window, scale 0.125.  q: device f32, row i at q + i*q_stride
 * (q_stride = 3*heads*64 reads the Q block of a roped qkv row);
 * out: device f32 [n][heads*64]. */
MB_API int mb_attend(mb_ctx* ctx, int32_t layer, int32_t n, const int32_t* streams,
                     const int32_t* positions, const float* q, int32_t q_stride, float* out,
                     void* cuda_stream);

/* The hot path: mb_rope_append followed by mb_attend in ONE decode launch
 * (decode.ts:527-552 for n streams at once), plus a small combine launch behind
 * it when windows exceed one split-K chunk (64 fp32 / 128 16-bit slots).  qkv
 * is read-only here (the roped Q stays on chip); out: device f32 [n][heads*64]. */
MB_API int mb_append_attend(mb_ctx* ctx, int32_t layer, int32_t n, const int32_t* streams,
                            const int32_t* positions, const float* qkv, float* out,
                            void* cuda_stream);

/* mb_append_attend for every layer of one decode step: the layer loop of
 * DecodeRunner.globalStep (decode.ts:735-748), all layers in ONE decode launch
 * (they touch disjoint rings) and one combine launch.
 * qkv: device f32 [layers][n][3*heads*64]; out: device f32 [layers][n][heads*64]. */
MB_API int mb_decode_step(mb_ctx* ctx, int32_t n, const int32_t* streams, const int32_t* positions,
                          const float* qkv, float* out, void* cuda_stream);

/* mb_append_attend with HOST arrays: copies streams/positions/qkv in, runs,
 * copies out and waits for the result (the per-layer readback of
 * DecodeRunner, decode.ts:450-463).  Validates every item on the host first. */
MB_API int mb_append_attend_host(mb_ctx* ctx, int32_t layer, int32_t n, const int32_t* streams,
                                 const int32_t* positions, const float* qkv, float* out,
                                 void* cuda_stream);

/* One global decode step for n streams through ALL layers, HOST arrays:
 * qkv [layers][n][3*heads*64], out [layers][n][heads*64]; the layers run in a
 * few launches of consecutive layers, whose rows are copied in and out as groups
 * on the context's own copy streams, overlapping the other launches' decode;
 * returns once `out` is complete -- the granularity of DecodeRunner.globalStep
 * (decode.ts:712-775: one submit, one readback). */
MB_API int mb_decode_step_host(mb_ctx* ctx, int32_t n, const int32_t* streams, const int32_t* positions,
                               const float* qkv, float* out, void* cuda_stream);

/* Causal prefill of positions 0..rows-1 of n streams for one layer:
 * ROPE_SPLIT_CACHE + ATTENTION_SCORES/_SOFTMAX/_APPLY (kernels-batch.ts:194-350,
 * dispatched at prefill.ts:424-462).  The item's slots >= rows are marked empty
 * first (a prefill starts an utterance).  qkv: device f32 [n][rows][3*heads*64]
 * (read-only), out: device f32 [n][rows][heads*64].  rows <= capacity.
 * fp32 rings also use a stage of 6 * n * heads * rows * 128 bytes: the bf16
 * hi/lo parts of Q, K and V that the tensor-core attention reads.  The context
 * keeps it and grows it when a call needs more (a cudaFree / cudaMalloc pair,
 * which synchronise the device; make the largest call first, outside any stream
 * capture).  Like the decode scratch it is shared by the context's calls:
 * prefill calls on one context run in order on one stream. */
MB_API int mb_prefill(mb_ctx* ctx, int32_t layer, int32_t n, const int32_t* streams, int32_t rows,
                      const float* qkv, float* out, void* cuda_stream);

/* The live window of (layer, stream) for a query at `position`, in POSITION
 * order: W = min(position + 1, capacity) rows, row w = position - W + 1 + w.
 * k_out, v_out: device [heads][W][64] in the storage dtype; slots_out: device
 * int32[W], the slot holding that position or -1 (its rows are zero).
 * PrefillRunner.readLayerCache (prefill.ts:644-664), generalised to the wrap. */
MB_API int mb_gather(mb_ctx* ctx, int32_t layer, int32_t stream, int32_t position, void* k_out,
                     void* v_out, int32_t* slots_out, void* cuda_stream);

/* Write `count` rows of already-roped K and raw V, [heads][count][64] in the
 * storage dtype (device pointers), at positions first_position.. of (layer,
 * stream), recording the positions.  The writeBuffer of PrefillRunner.poisonKv
 * (prefill.ts:610-620); also restores a gathered window. */
MB_API int mb_ring_write(mb_ctx* ctx, int32_t layer, int32_t stream, int32_t first_position, int32_t count,
                         const void* k, const void* v, void* cuda_stream);

/* Wait for `cuda_stream` and report device-side rejections (then clear them). */
MB_API int mb_sync(mb_ctx* ctx, void* cuda_stream);

/* Failure detection.  No counterpart in the reference, whose WebGPU queue has no
 * timeouts (its warm-up checks, gpu.ts:201-234, only catch wrong results).  The
 * decode kernels of this context wait for their K/V chunks at most `cycles` SM
 * clock cycles (0 restores the default, about 2 s); a wait that runs out skips
 * the chunk, lets its copies land (at the default bound), and the next mb_sync
 * reports MB_ERR_TIMEOUT.  A negative value is the test of that path: the waits
 * then target a barrier that nothing signals and run out after -cycles cycles,
 * on every launch, until the bound is set again.  Applies to launches queued
 * after the call. */
MB_API int mb_set_wait_limit(mb_ctx* ctx, int64_t cycles);

/* ---------------------------------------------------------------------------
 * The decode step around the path: the whole global
 * transformer layer of DecodeRunner.runLayer (decode.ts:474-620) for n streams
 * at once -- LN1 -> QKV GEMM -> append + RoPE + attention -> c_proj GEMM +
 * residual -> LN2 -> fc_in GEMM + GELU(tanh) -> fc_out GEMM + residual -- and
 * the final LayerNorm, over a context's rings.  The GEMMs (mb_gemm_bf16 below,
 * bf16 weights, fp32 accumulation on the tensor cores, bias / residual / GELU in
 * their epilogues), LayerNorm (eps 1e-5) and the attention are this library's
 * kernels.
 * ------------------------------------------------------------------------- */

typedef struct mb_decoder mb_decoder;

/* Weights as one host array of fp32 in the order of the published graph, per
 * layer (matrices [K][N] row-major, y = b + x W, docs analysis :651):
 *   ln1_w[H*64] ln1_b[H*64] c_attn_w[H*64][3*H*64] c_attn_b[3*H*64]
 *   c_proj_w[H*64][H*64] c_proj_b[H*64] ln2_w[H*64] ln2_b[H*64]
 *   fc_in_w[H*64][ffn] fc_in_b[ffn] fc_out_w[ffn][H*64] fc_out_b[H*64]
 * then ln_f_w[H*64] ln_f_b[H*64].  Matrices are stored on the device as bf16.
 * `count` must equal mb_decoder_weight_count(ctx, ffn). */
MB_API size_t mb_decoder_weight_count(const mb_ctx* ctx, int32_t ffn);
MB_API int mb_decoder_create(mb_ctx* ctx, int32_t ffn, const float* host_weights, size_t count, mb_decoder** out);
MB_API int mb_decoder_destroy(mb_decoder* dec);

/* One global decode step for n streams: hidden [n][H*64] fp32 (device) holds the
 * embedded rows on entry and ln_f of the last layer on return
 * (DecodeRunner.globalStep, decode.ts:712-775, without the embedding).  Each
 * stream appends at its position in every layer's ring.  From 128 items on, the
 * second half of the items runs on a stream the decoder owns, forked from
 * `cuda_stream` and joined back to it by events: work queued on `cuda_stream`
 * after the call still starts only once the whole step is done. */
MB_API int mb_decoder_step(mb_decoder* dec, int32_t n, const int32_t* streams, const int32_t* positions,
                           float* hidden, void* cuda_stream);

/* mb_decoder_step with HOST arrays -- the call DecodeRunner.globalStep makes
 * (decode.ts:712-775: the embedded row written in, one submit of every layer,
 * one readback of the ln_f row, decode.ts:774; gpu.ts:244 decodeStep): streams
 * and positions [n] are checked on the host (range, duplicates, positions as
 * mb_append_attend_host does), hidden [n][H*64] fp32 holds the embedded rows on
 * entry and ln_f of the last layer on return; one synchronisation, and the
 * ring's device status is reported as by mb_sync. */
MB_API int mb_decoder_step_host(mb_decoder* dec, int32_t n, const int32_t* streams, const int32_t* positions,
                                float* hidden, void* cuda_stream);

/* GEMV (kernels-decode.ts:127-142: y = b + x W with W [K][N] row-major), the
 * projection kernel of DecodeRunner.runLayer (decode.ts:517-526, 553-619), for
 * m rows (streams) at once on the tensor cores -- the GEMM the decoder step runs
 * for each of its projections, on the current device:
 *   x    device bf16 [m][k]          (activation rows)
 *   wt   device bf16 [n][k]          (W transposed: row j holds column j of W)
 *   bias device f32 [n] or NULL
 *   y    epi 0: device f32 [m][n] = x W + bias
 *        epi 1: device f32 [m][n] += x W + bias      (the residual add)
 *        epi 2: device bf16 [m][n] = gelu_tanh(x W + bias)   (GELU_TANH, :373-390)
 * fp32 accumulation; k a multiple of 64, n of 32; every pointer 16-byte aligned
 * (status 4-byte).  bn, splits: 0, 0 = the library's plan; else bn (32, 64 or
 * 128, dividing n) output columns per CTA and K split over `splits` (1..8, at
 * most k / 64) CTAs of a thread-block cluster, whose partials are summed in a
 * fixed order; splits = -1: a pair of CTAs per 128 x bn tile (one tcgen05 MMA
 * over both, each CTA loading half of the rows of x and of W^T).  status: device int32 the kernel ORs 8 into when a bounded wait
 * gives up.  Async on cuda_stream. */
MB_API int mb_gemm_bf16(int32_t m, int32_t n, int32_t k, const void* x, const void* wt, const float* bias, void* y,
                        int32_t epi, int32_t bn, int32_t splits, int32_t* status, void* cuda_stream);

/* ---------------------------------------------------------------------------
 * Local head: the 17 sequential steps that turn one global hidden state into one
 * frame of 16 audio codes, for n streams at once.  Replaces
 * DecodeRunner.nextFrame (src/lib/tts/engine/decode.ts:788-939) and its
 * clearSeen (decode.ts:275-280); the per-step kernels it replaces are
 * EMBED_ROW_LOCAL, the layer of runLayer, LAYERNORM_1 (ln_f), TEXT_HEAD_DECIDE,
 * the audio-head GEMV and ARGMAX_PENALTY (kernels-decode.ts:96-124, 428-535).
 *
 *   step 0      x = the global hidden state -> continue iff
 *               ln_f(x)·text_head[:, assistant_slot] >= ln_f(x)·text_head[:, audio_end]
 *   step 1      x = wte[assistant_slot]     -> token 0 = argmax over audio head 0
 *   step 2+i    x = audio_emb_i[token i]     -> token i+1 = argmax over audio head i+1
 *
 * Each step runs the local transformer's one layer over the local ring at
 * position = step, then ln_f.  The argmax is greedy with the repetition penalty
 * over the codes already emitted on that channel since the stream's last clear:
 * a seen logit s becomes s / penalty when s >= 0 and s * penalty when s < 0;
 * ties go to the lowest id.  As in the reference's GPU path, all 17 steps run
 * (and set seen bits) even when the frame says stop.
 * ------------------------------------------------------------------------- */

typedef struct mb_local_head mb_local_head;

typedef struct mb_local_config {
    int32_t ffn;              /* FFN width of the local layer (3072) */
    int32_t codes;            /* codebook size (CODES = 1024, decode.ts:48): 128, 256, 512, 1024 or 2048 */
    int32_t channels;         /* codebooks per frame (n_vq = 16), 1..64; a frame takes channels + 1 steps */
    float repetition_penalty; /* audio_repetition_penalty (1.2 in the published defaults) */
} mb_local_config;

/* Weights as one host array of fp32:
 *   the local layer and ln_f, in mb_decoder_create's order for a one-layer ring
 *     (mb_decoder_weight_count(local_ring, ffn) values)
 *   wte_slot[H*64]                  the wte row of audio_assistant_slot_token_id
 *   text_cols[2][H*64]              text head columns audio_end_token_id, then
 *                                   audio_assistant_slot_token_id
 *   audio_emb[channels-1][codes][H*64]   the audio embedding tables 0..channels-2
 *   audio_head[channels][H*64][codes]    the audio heads ([K][N] row-major, no bias)
 * `local_ring` must have one layer, capacity and max_position >= channels + 1;
 * its `streams` are the streams whose seen masks the head keeps, its max_batch
 * bounds n.  The layer and head matrices are stored on the device as bf16.
 * mb_local_head_weight_count returns 0 for a ring the head cannot use. */
MB_API size_t mb_local_head_weight_count(const mb_ctx* local_ring, const mb_local_config* cfg);
MB_API int mb_local_head_create(mb_ctx* local_ring, const mb_local_config* cfg, const float* host_weights,
                                size_t count, mb_local_head** out);
MB_API int mb_local_head_destroy(mb_local_head* head);

/* Zero the seen masks of one stream (or of every stream when stream = -1): a new
 * utterance starts clean (clearSeen, decode.ts:275-280).  Async on cuda_stream. */
MB_API int mb_local_head_clear(mb_local_head* head, int32_t stream, void* cuda_stream);

/* One frame for n streams.  Device pointers: streams [n] (distinct ring stream
 * ids), hidden [n][H*64] fp32 (the global step's ln_f output; not modified),
 * tokens [n][channels] int32 out, cont [n] int32 out (1 = continue, 0 = the
 * utterance ends: nextFrame's null), logits [n][channels][codes] fp32 out or NULL
 * (every channel's logits before the penalty, for tests).  Async on cuda_stream. */
MB_API int mb_local_head_frame(mb_local_head* head, int32_t n, const int32_t* streams, const float* hidden,
                               int32_t* tokens, int32_t* cont, float* logits, void* cuda_stream);

/* mb_local_head_frame with HOST arrays, as DecodeRunner.nextFrame takes the
 * hidden row from the host and reads the stop flag and the tokens back
 * (decode.ts:788, 933-935): streams [n] are checked on the host (range,
 * duplicates), hidden [n][H*64] is copied in, the frame runs, tokens
 * [n][channels] and cont [n] are copied out with the ring's device status word,
 * and the call returns once they are in place (one synchronisation). */
MB_API int mb_local_head_frame_host(mb_local_head* head, int32_t n, const int32_t* streams, const float* hidden,
                                    int32_t* tokens, int32_t* cont, void* cuda_stream);

/* ARGMAX_PENALTY alone (kernels-decode.ts:428-485), on the current device: for
 * each of n rows, token = the penalised argmax of logits [n][codes] under the
 * row's seen mask seen [n][codes/32] (bit j of word j/32), whose bit is then
 * set.  Device pointers, logits 16-byte aligned; codes 128, 256, 512, 1024 or
 * 2048. */
MB_API int mb_argmax_penalty(int32_t n, int32_t codes, const float* logits, uint32_t* seen, float penalty,
                             int32_t* tokens, void* cuda_stream);

/* ---------------------------------------------------------------------------
 * No-allocation entry point.  No counterpart in the reference: the reference
 * allocates its GPU buffers once per engine and never hands that job to callers.
 *
 * Some callers cannot call cudaMalloc: a host application whose device memory
 * is already owned by another allocator (a framework's caching pool, a game or
 * audio engine's arena) where an extra cudaMalloc can fail or fragment, or a
 * real-time audio thread that must not block on the device-wide synchronisation
 * that cudaMalloc/cudaFree may imply.  Such a caller owns every buffer itself and
 * describes its ring with an mb_ring_ref; the entry point below allocates
 * nothing.  The split-K scratch of the decode kernel lives in a fixed,
 * file-scope device array of MB_NOALLOC_SCRATCH_BYTES that every GPU which
 * loads this library holds until the process exits.
 * ------------------------------------------------------------------------- */

/* Maximum scratch of mb_append_attend_noalloc: a call needs
 * n * heads * ceil(capacity / chunk) * 66 * 4 bytes of partials (chunk = 64 slots
 * for fp32, 128 for 16-bit storage), rounded up to 256 bytes; larger calls are
 * rejected with MB_ERR_ARG. */
#define MB_NOALLOC_SCRATCH_BYTES (8u << 20)

/* A ring in caller-owned device memory, laid out as a context's (see above). */
typedef struct mb_ring_ref {
    void* kv;              /* kv[layers][streams][2][heads][capacity][64], storage dtype, 16-byte aligned */
    int32_t* slot_pos;     /* slot_pos[layers][streams][capacity], -1 = empty                          */
    const float* rope;     /* [max_position][32][2]: cos, sin of p * theta^(-2i/64), angle and
                              cos/sin in fp64, each rounded once to fp32                              */
    int32_t* status;       /* device int32; kernel rejections are OR-ed in (1 stream, 2 position,
                              4 beyond a non-wrapping ring, 8 timeout); the caller reads and clears it */
    int32_t layers, heads, capacity, streams, dtype, wrap, max_position;
} mb_ring_ref;

/* mb_append_attend on a caller-owned ring, allocating nothing.  Same inputs,
 * outputs and results as mb_append_attend; scratch comes from the library's
 * fixed device array.  The first call on each device looks that array up
 * (cudaGetSymbolAddress, with the caller's current device), so make that first
 * call before any stream capture.  Every call shares the one array and keeps
 * its partials there until the call's combine kernel has read them: calls that
 * overlap on the GPU (other streams, other threads) race and must be serialised
 * by the caller.  Uses the current CUDA device, in its primary context; the looked-up
 * address stays cached for the life of the process, so do not reset the device
 * (cudaDeviceReset) while using this entry point.  Returns MB_ERR_ARG for bad
 * arguments -- null or misaligned pointers (qkv, out and kv 16-byte aligned,
 * rope 8-byte, streams, positions, slot_pos and status 4-byte) -- or for a call
 * that needs more than MB_NOALLOC_SCRATCH_BYTES of scratch. */
MB_API int mb_append_attend_noalloc(const mb_ring_ref* ring, int32_t layer, int32_t n, const int32_t* streams,
                                    const int32_t* positions, const float* qkv, float* out, void* cuda_stream);

/* Device addresses and sizes of the context's state. */
MB_API int mb_ring_info_get(const mb_ctx* ctx, mb_ring_info* out);

/* Text of the last error on this context ("" if none). */
MB_API const char* mb_last_error(const mb_ctx* ctx);

/* Library version string. */
MB_API const char* mb_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MOCKBIRD_KV_H */
