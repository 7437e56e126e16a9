// The local head: the 17 sequential steps that turn one global hidden state into
// one frame of 16 audio codes (DecodeRunner.nextFrame, liyu1981/mockbird
// src/lib/tts/engine/decode.ts:788-939; CPU form tools/onnx-probe/ref-decode.mjs
// :236-283 and :380-410), for n streams at once.
//
//   step 0      x = the global hidden state   -> continue/stop from two columns
//                                                 of the text head (TEXT_HEAD_DECIDE)
//   step 1      x = wte[assistant_slot]        -> argmax over audio head 0
//   step 2+i    x = audio_emb_i[token_i]       -> argmax over audio head i+1
//
// Every step runs the local transformer's single layer over a 17-slot KV ring at
// position = step, then ln_f.  The argmax is greedy with the HuggingFace
// repetition penalty over the codes already emitted on that channel in this
// utterance (ARGMAX_PENALTY, kernels-decode.ts:428-485): a per-stream,
// per-channel 1024-bit seen mask kept on the device.  Tokens never leave the
// device between steps.
//
// The layer is the decoder machinery of mb_decoder.cu (this library's tcgen05
// GEMMs with bf16 weights and fp32 accumulation, its LayerNorm and fused append +
// RoPE + attention kernels).  The 16 audio heads [768][1024] are bf16 GEMMs
// without bias (the graph's bare MatMul, decode.ts:875); the embeddings, the two
// text-head columns and everything between the GEMMs stay fp32.
//
// One frame is ~220 launches of small kernels, so by default it is captured once
// per batch size into a CUDA graph and replayed (MOCKBIRD_LOCAL_GRAPH=0 turns
// that off); the graph reads and writes only this object's own buffers.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <map>
#include <vector>
#include <utility>

#include "mb_decoder.cuh"

namespace {

using bf16 = __nv_bfloat16;

// x[i] = the step's input row (EMBED_ROW_LOCAL, kernels-decode.ts:96-124, modes
// 1 and 2; mode "hidden" is the writeBuffer of decode.ts:792), and then the local
// layer's LN1 of it, one warp per item: the row goes to x (fp32, the residual
// stream) and LN1(row) to xb (bf16, the QKV GEMM's input), so the layer starts
// at its GEMM.  Same arithmetic as the separate LayerNorm (mb::dec::ln_apply).
// Tokens come from argmax_penalty_kernel and are always in [0, codes); the clamp
// only keeps a corrupted token from addressing outside the table.
template <int PER>
__global__ void local_embed_ln_kernel(int n, int step, int h, int channels, int codes, const float* __restrict__ hin,
                                      const float* __restrict__ wte_slot, const float* __restrict__ emb,
                                      const int32_t* __restrict__ tokens, const float* __restrict__ ln_w,
                                      const float* __restrict__ ln_b, float* __restrict__ x,
                                      __nv_bfloat16* __restrict__ xb) {
    const int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (i >= n) return;
    const float* src;
    if (step == 0) {
        src = hin + (size_t)i * h;
    } else if (step == 1) {
        src = wte_slot;
    } else {
        const int ch = step - 2;
        int tok = tokens[(size_t)i * channels + ch];
        tok = min(max(tok, 0), codes - 1);
        src = emb + ((size_t)ch * codes + tok) * h;
    }
    float v[PER];
    mb::dec::ln_load<PER>(src, lane, v);
    mb::dec::ln_store<PER>(x + (size_t)i * h, lane, v);
    mb::dec::ln_apply<__nv_bfloat16, PER>(v, ln_w, ln_b, xb + (size_t)i * h, h, lane);
}

// TEXT_HEAD_DECIDE (kernels-decode.ts:487-535): the dot products of ln_f(x) with
// the text head's audio_end and assistant_slot columns; continue iff
// assistant >= end.  One warp per item.
__global__ void local_decide_kernel(int n, int h, const float* __restrict__ x, const float* __restrict__ cols,
                                    int32_t* __restrict__ cont) {
    const int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (i >= n) return;
    const float* xr = x + (size_t)i * h;
    float end = 0.f, asst = 0.f;
    for (int d = lane; d < h; d += 32) {
        end = fmaf(xr[d], cols[d], end);
        asst = fmaf(xr[d], cols[h + d], asst);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        end += __shfl_xor_sync(0xffffffffu, end, o);
        asst += __shfl_xor_sync(0xffffffffu, asst, o);
    }
    if (lane == 0) cont[i] = asst >= end ? 1 : 0;
}

// ARGMAX_PENALTY (kernels-decode.ts:428-485) for one row per warp.  A logit
// whose bit is set in the row's seen mask becomes s / penalty (s >= 0) or
// s * penalty (s < 0); the winner is the largest value, ties to the lowest id,
// starting from (-1e30, id 0) as the reference does; its bit is then set.
// Lane l scans its contiguous ids [l*codes/32, (l+1)*codes/32) in order with a
// strict > (all of its loads issued up front), and the warp reduces under the
// order (value desc, id asc) -- the same total-order maximum as the reference's
// strided scan and tree, so the same winner.
// Row i: logits + i*codes; mask = seen + row_sel(i) * seen_row_words + ch * codes/32
// (row_sel(i) = streams[i] when `streams` is given, else i; rows whose stream is
// outside [0, n_seen_rows) get token 0 and leave the masks alone -- the ring's
// own kernel reports such a stream); token -> tokens[i*tok_stride + ch].
// The next step's input, built by the warp that has just chosen the token: row
// emb[ch][token] to x and the local layer's LN1 of it to xb (the next step of
// the frame embeds channel ch's token, and local_embed_ln_kernel does the same
// for the other steps).
struct EmbedNext {
    const float* emb;  // [channels - 1][codes][h]
    const float *ln_w, *ln_b;
    float* x;
    __nv_bfloat16* xb;
    int h;
};

template <int PER, int HPER>  // ids per lane = codes / 32, a multiple of 4; HPER = h / 32, 0: no EmbedNext
__global__ void argmax_penalty_kernel(int n, int codes, const float* __restrict__ logits, uint32_t* __restrict__ seen,
                                      const int32_t* __restrict__ streams, int n_seen_rows, int seen_row_words, int ch,
                                      float penalty, int32_t* __restrict__ tokens, int tok_stride, EmbedNext en) {
    const int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (i >= n) return;
    const int row = streams ? streams[i] : i;
    const bool ok = row >= 0 && row < n_seen_rows;
    uint32_t* mask = seen + (size_t)(ok ? row : 0) * seen_row_words + (size_t)ch * (codes >> 5);
    const float4* lg = reinterpret_cast<const float4*>(logits + (size_t)i * codes + lane * PER);
    float v[PER];
#pragma unroll
    for (int k = 0; k < PER / 4; k++) {
        const float4 q = lg[k];
        v[4 * k] = q.x, v[4 * k + 1] = q.y, v[4 * k + 2] = q.z, v[4 * k + 3] = q.w;
    }
    const int j0 = lane * PER;
    float best = -1e30f;
    int idx = 0;
#pragma unroll
    for (int w = 0; w < PER / 32 + (PER % 32 != 0); w++) {
        const int jw = j0 + 32 * w;  // this lane's ids jw .. jw+31 share one mask word when PER >= 32
        const uint32_t bits = ok ? mask[jw >> 5] : 0u;
#pragma unroll
        for (int e = 0; e < (PER < 32 ? PER : 32); e++) {
            const int j = jw + e;
            float s = v[32 * w + e];
            if ((bits >> (j & 31)) & 1u) s = s >= 0.f ? s / penalty : s * penalty;
            if (s > best) {
                best = s;
                idx = j;
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > best || (ov == best && oi < idx)) {
            best = ov;
            idx = oi;
        }
    }
    if (lane == 0) {
        tokens[(size_t)i * tok_stride + ch] = ok ? idx : 0;
        if (ok) mask[idx >> 5] |= 1u << (idx & 31);
    }
    if constexpr (HPER > 0) {  // every lane holds the reduced (best, idx)
        const int tok = ok ? idx : 0;
        float x[HPER];
        mb::dec::ln_load<HPER>(en.emb + ((size_t)ch * codes + tok) * en.h, lane, x);
        mb::dec::ln_store<HPER>(en.x + (size_t)i * en.h, lane, x);
        mb::dec::ln_apply<__nv_bfloat16, HPER>(x, en.ln_w, en.ln_b, en.xb + (size_t)i * en.h, en.h, lane);
    }
}

// Launches the argmax for `codes` in {128, 256, 512, 1024, 2048} (ids per lane a
// multiple of 4); other sizes are rejected by the callers' checks.
// next: when non-null, the same launch also builds the next step's input (EmbedNext).
template <int HPER>
cudaError_t launch_argmax_h(int n, int codes, const float* logits, uint32_t* seen, const int32_t* streams,
                            int n_seen_rows, int seen_row_words, int ch, float penalty, int32_t* tokens,
                            int tok_stride, const EmbedNext& en, cudaStream_t st) {
    const int warps = 2, blocks = (n + warps - 1) / warps;
#define MB_ARGMAX(PER)                                                                                              \
    argmax_penalty_kernel<PER, HPER><<<blocks, 32 * warps, 0, st>>>(n, codes, logits, seen, streams, n_seen_rows, \
                                                                      seen_row_words, ch, penalty, tokens,          \
                                                                      tok_stride, en)
    switch (codes) {
        case 128: MB_ARGMAX(4); break;
        case 256: MB_ARGMAX(8); break;
        case 512: MB_ARGMAX(16); break;
        case 1024: MB_ARGMAX(32); break;
        case 2048: MB_ARGMAX(64); break;
        default: return cudaErrorInvalidValue;
    }
#undef MB_ARGMAX
    return cudaGetLastError();
}

cudaError_t launch_argmax(int n, int codes, const float* logits, uint32_t* seen, const int32_t* streams,
                          int n_seen_rows, int seen_row_words, int ch, float penalty, int32_t* tokens, int tok_stride,
                          cudaStream_t st, const EmbedNext* next = nullptr) {
    if (!next)
        return launch_argmax_h<0>(n, codes, logits, seen, streams, n_seen_rows, seen_row_words, ch, penalty, tokens,
                                  tok_stride, EmbedNext{}, st);
    switch (next->h / 32) {
        case 2:
            return launch_argmax_h<2>(n, codes, logits, seen, streams, n_seen_rows, seen_row_words, ch, penalty,
                                      tokens, tok_stride, *next, st);
        case 8:
            return launch_argmax_h<8>(n, codes, logits, seen, streams, n_seen_rows, seen_row_words, ch, penalty,
                                      tokens, tok_stride, *next, st);
        case 24:
            return launch_argmax_h<24>(n, codes, logits, seen, streams, n_seen_rows, seen_row_words, ch, penalty,
                                       tokens, tok_stride, *next, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

struct mb_local_head {
    mb_ctx* ctx = nullptr;       // the local ring (one layer, >= channels + 1 slots)
    mb_decoder* dec = nullptr;   // the local transformer layer + ln_f
    int h = 0, codes = 0, channels = 0, max_batch = 0, seen_words = 0;
    float penalty = 1.f;
    void* wmem = nullptr;        // wte_slot [h] | cols [2][h] | emb [(channels-1)][codes][h] (fp32) | heads (bf16)
    const float *wte_slot = nullptr, *cols = nullptr, *emb = nullptr;
    const bf16* heads = nullptr; // [channels][codes][h]: each audio head transposed (the GEMM's K-major operand)
    float* hin = nullptr;        // [max_batch][h] staged global hidden states
    float* x = nullptr;          // [max_batch][h] the step's residual stream
    bf16* hb = nullptr;          // [max_batch][h] ln_f output, head GEMM input
    float* lg = nullptr;         // [max_batch][codes] one channel's logits
    float* lg_all = nullptr;     // [max_batch][channels][codes] when the caller asks for logits
    int32_t* tok = nullptr;      // [max_batch][channels]
    int32_t* cont = nullptr;     // [max_batch]
    int32_t* ids = nullptr;      // [max_batch] staged stream ids
    int32_t* pos = nullptr;      // [channels + 1][max_batch], row s all = s
    uint32_t* seen = nullptr;    // [ring streams][channels][codes / 32]
    bool use_graph = true;
    cudaStream_t cap = nullptr;  // capture stream
    std::map<std::pair<int, int>, cudaGraphExec_t> graphs;  // (n, logits wanted) -> frame
};

namespace {

int lfail(mb_local_head* lh, int code, const std::string& msg) {
    if (lh && lh->ctx) lh->ctx->last_error = msg;
    return code;
}

size_t dec_count(const mb_ctx* c, int ffn) { return mb_decoder_weight_count(c, ffn); }

// The whole frame on `st`, over this object's buffers only (graph-capturable).
int enqueue_frame(mb_local_head* lh, int n, bool want_logits, cudaStream_t st) {
    const int h = lh->h, steps = lh->channels + 1;
    const int warps = 4, wblocks = (n + warps - 1) / warps;
    bool input_ready = false;  // x and xb already hold this step's input (built by the previous argmax)
    for (int step = 0; step < steps; step++) {
        if (!input_ready) {
            const int eb = (n + 1) / 2;  // two warps (items) per block
            const float *w1 = lh->dec->L[0].ln1_w, *b1 = lh->dec->L[0].ln1_b;
            switch (h / 32) {
                case 2:
                    local_embed_ln_kernel<2><<<eb, 64, 0, st>>>(n, step, h, lh->channels, lh->codes, lh->hin,
                                                                lh->wte_slot, lh->emb, lh->tok, w1, b1, lh->x,
                                                                lh->dec->xb);
                    break;
                case 8:
                    local_embed_ln_kernel<8><<<eb, 64, 0, st>>>(n, step, h, lh->channels, lh->codes, lh->hin,
                                                                lh->wte_slot, lh->emb, lh->tok, w1, b1, lh->x,
                                                                lh->dec->xb);
                    break;
                default:
                    local_embed_ln_kernel<24><<<eb, 64, 0, st>>>(n, step, h, lh->channels, lh->codes, lh->hin,
                                                                 lh->wte_slot, lh->emb, lh->tok, w1, b1, lh->x,
                                                                 lh->dec->xb);
                    break;
            }
        }
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return lfail(lh, MB_ERR_CUDA, std::string("local head: ") + cudaGetErrorString(e));
        int rc = mb::dec::run(lh->dec, n, lh->ids, lh->pos + (size_t)step * lh->max_batch, lh->x,
                              step == 0 ? nullptr : lh->hb, st, /*ln1_ready=*/true, /*qkv_append=*/false);
        if (rc) return rc;
        if (step == 0) {
            local_decide_kernel<<<wblocks, 32 * warps, 0, st>>>(n, h, lh->x, lh->cols, lh->cont);
        } else {
            const int ch = step - 1;
            rc = mb::dec::gemm(lh->dec, n, lh->codes, h, lh->hb, lh->heads + (size_t)ch * h * lh->codes, nullptr,
                               lh->lg, lh->codes, mb::gemm::EPI_STORE, st);
            if (rc) return rc;
            // steps before the last also embed the chosen tokens for the next step
            const EmbedNext next{lh->emb, lh->dec->L[0].ln1_w, lh->dec->L[0].ln1_b, lh->x, lh->dec->xb, h};
            const bool fuse = step < lh->channels;
            e = launch_argmax(n, lh->codes, lh->lg, lh->seen, lh->ids, lh->ctx->cfg.streams, lh->seen_words, ch,
                              lh->penalty, lh->tok, lh->channels, st, fuse ? &next : nullptr);
            input_ready = fuse;
            if (e != cudaSuccess)
                return lfail(lh, MB_ERR_CUDA, std::string("local head argmax: ") + cudaGetErrorString(e));
            if (want_logits) {
                const size_t row = (size_t)lh->codes * sizeof(float);
                e = cudaMemcpy2DAsync(lh->lg_all + (size_t)ch * lh->codes, row * lh->channels, lh->lg, row, row, n,
                                      cudaMemcpyDeviceToDevice, st);
                if (e != cudaSuccess)
                    return lfail(lh, MB_ERR_CUDA, std::string("local head: ") + cudaGetErrorString(e));
            }
        }
        e = cudaGetLastError();
        if (e != cudaSuccess) return lfail(lh, MB_ERR_CUDA, std::string("local head: ") + cudaGetErrorString(e));
    }
    return MB_OK;
}

// Replays the captured frame for (n, want_logits).  The first frame of a key runs
// directly on `st` (so every kernel module is loaded and every GEMM plan built
// outside a capture) and is then captured, without running, for the next calls.
int launch_frame(mb_local_head* lh, int n, bool want_logits, cudaStream_t st) {
    const auto key = std::make_pair(n, want_logits ? 1 : 0);
    auto it = lh->graphs.find(key);
    if (it == lh->graphs.end()) {
        int rc = enqueue_frame(lh, n, want_logits, st);
        if (rc) return rc;
        cudaGraph_t g = nullptr;
        cudaError_t e = cudaStreamBeginCapture(lh->cap, cudaStreamCaptureModeThreadLocal);
        if (e != cudaSuccess) return lfail(lh, MB_ERR_CUDA, std::string("local head capture: ") + cudaGetErrorString(e));
        rc = enqueue_frame(lh, n, want_logits, lh->cap);
        e = cudaStreamEndCapture(lh->cap, &g);
        if (rc) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        if (e != cudaSuccess) return lfail(lh, MB_ERR_CUDA, std::string("local head capture: ") + cudaGetErrorString(e));
        cudaGraphExec_t ex = nullptr;
        e = cudaGraphInstantiate(&ex, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess)
            return lfail(lh, MB_ERR_CUDA, std::string("local head graph: ") + cudaGetErrorString(e));
        lh->graphs.emplace(key, ex);
        return MB_OK;
    }
    const cudaError_t e = cudaGraphLaunch(it->second, st);
    if (e != cudaSuccess) return lfail(lh, MB_ERR_CUDA, std::string("local head graph: ") + cudaGetErrorString(e));
    return MB_OK;
}

struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

}  // namespace

extern "C" {

MB_API size_t mb_local_head_weight_count(const mb_ctx* c, const mb_local_config* cfg) {
    if (!c || !cfg || cfg->ffn <= 0 || cfg->codes <= 0 || cfg->channels <= 0) return 0;
    const int steps = cfg->channels + 1;
    if (c->cfg.layers != 1 || c->cfg.capacity < steps || c->cfg.max_position < steps) return 0;
    const size_t h = (size_t)c->cfg.heads * mb::HD, codes = (size_t)cfg->codes, ch = (size_t)cfg->channels;
    return dec_count(c, cfg->ffn) + h + 2 * h + (ch - 1) * codes * h + ch * h * codes;
}

MB_API int mb_local_head_destroy(mb_local_head* lh) {
    if (!lh) return MB_ERR_ARG;
    DeviceGuard g(lh->ctx->cfg.device);
    for (auto& kv : lh->graphs) cudaGraphExecDestroy(kv.second);
    if (lh->cap) cudaStreamDestroy(lh->cap);
    void* ptrs[] = {lh->wmem, lh->hin, lh->x, lh->hb, lh->lg, lh->lg_all, lh->tok, lh->cont, lh->ids, lh->pos,
                    lh->seen};
    for (void* p : ptrs)
        if (p) cudaFree(p);
    if (lh->dec) mb_decoder_destroy(lh->dec);
    delete lh;
    return MB_OK;
}

MB_API int mb_local_head_create(mb_ctx* c, const mb_local_config* cfg, const float* w, size_t count,
                                mb_local_head** out) {
    if (!c || !cfg || !w || !out) return MB_ERR_ARG;
    *out = nullptr;
    const int steps = cfg->channels + 1;
    if (!(cfg->codes == 128 || cfg->codes == 256 || cfg->codes == 512 || cfg->codes == 1024 || cfg->codes == 2048) ||
        cfg->channels <= 0 || cfg->channels > 64 ||
        !(cfg->repetition_penalty > 0.f) || !isfinite(cfg->repetition_penalty)) {
        c->last_error = "local head: codes must be 128, 256, 512, 1024 or 2048, channels in [1, 64], penalty > 0";
        return MB_ERR_ARG;
    }
    if (c->cfg.layers != 1 || c->cfg.capacity < steps || c->cfg.max_position < steps) {
        c->last_error = "local head: the ring must have one layer and at least channels + 1 slots and positions";
        return MB_ERR_ARG;
    }
    if (count != mb_local_head_weight_count(c, cfg)) {
        c->last_error = "local head: weight count does not match (layer, ffn, codes, channels)";
        return MB_ERR_ARG;
    }
    DeviceGuard g(c->cfg.device);
    if (!g.ok) return MB_ERR_CUDA;
    mb_local_head* lh = new mb_local_head();
    lh->ctx = c;
    lh->h = c->cfg.heads * mb::HD;
    lh->codes = cfg->codes;
    lh->channels = cfg->channels;
    lh->penalty = cfg->repetition_penalty;
    lh->max_batch = c->cfg.max_batch;
    lh->seen_words = cfg->channels * (cfg->codes / 32);
    {
        const char* v = getenv("MOCKBIRD_LOCAL_GRAPH");
        lh->use_graph = !(v && strcmp(v, "0") == 0);
    }
    auto bail = [&](int rc, const char* msg) {
        if (msg) c->last_error = msg;
        mb_local_head_destroy(lh);
        return rc;
    };
    const size_t nd = dec_count(c, cfg->ffn);
    int rc = mb_decoder_create(c, cfg->ffn, w, nd, &lh->dec);
    if (rc) return bail(rc, nullptr);
    const size_t h = lh->h, codes = lh->codes, ch = lh->channels, mbat = lh->max_batch;
    // device image: fp32 wte_slot | cols | emb, then the bf16 heads (256-byte aligned)
    const size_t n_f32 = h + 2 * h + (ch - 1) * codes * h;
    const size_t f32_bytes = (n_f32 * 4 + 255) & ~size_t(255);
    const size_t n_heads = ch * h * codes;
    const size_t bytes = f32_bytes + n_heads * 2;
    std::vector<unsigned char> img(bytes, 0);
    memcpy(img.data(), w + nd, n_f32 * 4);
    uint16_t* hb16 = reinterpret_cast<uint16_t*>(img.data() + f32_bytes);
    for (size_t c2 = 0; c2 < ch; c2++)  // each head [h][codes] stored transposed, [codes][h]
        mb::dec::transpose_to_bf16(w + nd + n_f32 + c2 * h * codes, (int)h, (int)codes, hb16 + c2 * h * codes);

    if (cudaMalloc(&lh->wmem, bytes) != cudaSuccess) return bail(MB_ERR_OOM, "local head: weight allocation failed");
    if (cudaMemcpy(lh->wmem, img.data(), bytes, cudaMemcpyHostToDevice) != cudaSuccess)
        return bail(MB_ERR_CUDA, "local head: weight upload failed");
    lh->wte_slot = reinterpret_cast<const float*>(lh->wmem);
    lh->cols = lh->wte_slot + h;
    lh->emb = lh->cols + 2 * h;
    lh->heads = reinterpret_cast<const bf16*>((char*)lh->wmem + f32_bytes);
    std::vector<int32_t> pos((size_t)steps * mbat);
    for (int s = 0; s < steps; s++)
        for (size_t i = 0; i < mbat; i++) pos[(size_t)s * mbat + i] = s;
    const size_t seen_bytes = (size_t)c->cfg.streams * lh->seen_words * 4;
    if (cudaMalloc(&lh->hin, mbat * h * 4) != cudaSuccess || cudaMalloc(&lh->x, mbat * h * 4) != cudaSuccess ||
        cudaMalloc(&lh->hb, mbat * h * 2) != cudaSuccess || cudaMalloc(&lh->lg, mbat * codes * 4) != cudaSuccess ||
        cudaMalloc(&lh->tok, mbat * ch * 4) != cudaSuccess || cudaMalloc(&lh->cont, mbat * 4) != cudaSuccess ||
        cudaMalloc(&lh->ids, mbat * 4) != cudaSuccess || cudaMalloc(&lh->pos, pos.size() * 4) != cudaSuccess ||
        cudaMalloc(&lh->seen, seen_bytes) != cudaSuccess)
        return bail(MB_ERR_OOM, "local head: buffer allocation failed");
    if (cudaMemcpy(lh->pos, pos.data(), pos.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemset(lh->seen, 0, seen_bytes) != cudaSuccess || cudaMemset(lh->tok, 0, mbat * ch * 4) != cudaSuccess)
        return bail(MB_ERR_CUDA, "local head: buffer initialisation failed");
    if (cudaStreamCreateWithFlags(&lh->cap, cudaStreamNonBlocking) != cudaSuccess)
        return bail(MB_ERR_CUDA, "local head: stream creation failed");
    *out = lh;
    return MB_OK;
}

MB_API int mb_local_head_clear(mb_local_head* lh, int32_t stream, void* cuda_stream) {
    if (!lh) return MB_ERR_ARG;
    const int streams = lh->ctx->cfg.streams;
    if (stream < -1 || stream >= streams) return lfail(lh, MB_ERR_STREAM, "local head: stream out of range");
    DeviceGuard g(lh->ctx->cfg.device);
    if (!g.ok) return MB_ERR_CUDA;
    const size_t row = (size_t)lh->seen_words * 4;
    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    const cudaError_t e = stream < 0 ? cudaMemsetAsync(lh->seen, 0, row * streams, st)
                                     : cudaMemsetAsync(lh->seen + (size_t)stream * lh->seen_words, 0, row, st);
    if (e != cudaSuccess) return lfail(lh, MB_ERR_CUDA, std::string("local head: ") + cudaGetErrorString(e));
    return MB_OK;
}

MB_API int mb_local_head_frame(mb_local_head* lh, int32_t n, const int32_t* streams, const float* hidden,
                               int32_t* tokens, int32_t* cont, float* logits, void* cuda_stream) {
    if (!lh) return MB_ERR_ARG;
    if (n < 0 || n > lh->max_batch) return lfail(lh, MB_ERR_ARG, "local head: item count out of range");
    if (n == 0) return MB_OK;
    if (!streams || !hidden || !tokens || !cont)
        return lfail(lh, MB_ERR_ARG, "local head: null device pointer");
    DeviceGuard g(lh->ctx->cfg.device);
    if (!g.ok) return MB_ERR_CUDA;
    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    const size_t h = lh->h, ch = lh->channels, codes = lh->codes;
    if (logits && !lh->lg_all && cudaMalloc(&lh->lg_all, (size_t)lh->max_batch * ch * codes * 4) != cudaSuccess)
        return lfail(lh, MB_ERR_OOM, "local head: logits buffer allocation failed");
    cudaError_t e = cudaMemcpyAsync(lh->ids, streams, (size_t)n * 4, cudaMemcpyDeviceToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(lh->hin, hidden, (size_t)n * h * 4, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return lfail(lh, MB_ERR_CUDA, std::string("local head inputs: ") + cudaGetErrorString(e));
    const int rc = lh->use_graph ? launch_frame(lh, n, logits != nullptr, st) : enqueue_frame(lh, n, logits != nullptr, st);
    if (rc) return rc;
    e = cudaMemcpyAsync(tokens, lh->tok, (size_t)n * ch * 4, cudaMemcpyDeviceToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(cont, lh->cont, (size_t)n * 4, cudaMemcpyDeviceToDevice, st);
    if (e == cudaSuccess && logits)
        e = cudaMemcpyAsync(logits, lh->lg_all, (size_t)n * ch * codes * 4, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return lfail(lh, MB_ERR_CUDA, std::string("local head outputs: ") + cudaGetErrorString(e));
    return MB_OK;
}

MB_API int mb_local_head_frame_host(mb_local_head* lh, int32_t n, const int32_t* streams, const float* hidden,
                                    int32_t* tokens, int32_t* cont, void* cuda_stream) {
    if (!lh) return MB_ERR_ARG;
    if (n < 0 || n > lh->max_batch) return lfail(lh, MB_ERR_ARG, "local head: item count out of range");
    if (n == 0) return MB_OK;
    if (!streams || !hidden || !tokens || !cont) return lfail(lh, MB_ERR_ARG, "local head: null host pointer");
    mb_ctx* c = lh->ctx;
    std::vector<char> seen(c->cfg.streams, 0);
    for (int i = 0; i < n; i++) {
        const int s = streams[i];
        if (s < 0 || s >= c->cfg.streams) return lfail(lh, MB_ERR_STREAM, "local head: stream id out of range");
        if (seen[s]) return lfail(lh, MB_ERR_STREAM, "local head: a stream appears twice in one call");
        seen[s] = 1;
    }
    DeviceGuard g(c->cfg.device);
    if (!g.ok) return MB_ERR_CUDA;
    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    const size_t h = lh->h, ch = lh->channels;
    cudaError_t e = cudaMemcpyAsync(lh->ids, streams, (size_t)n * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(lh->hin, hidden, (size_t)n * h * 4, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return lfail(lh, MB_ERR_CUDA, std::string("local head inputs: ") + cudaGetErrorString(e));
    const int rc = lh->use_graph ? launch_frame(lh, n, false, st) : enqueue_frame(lh, n, false, st);
    if (rc) return rc;
    // the frame's tokens, the stop flags and the ring's device status word, then one wait
    e = cudaMemcpyAsync(tokens, lh->tok, (size_t)n * ch * 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(cont, lh->cont, (size_t)n * 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(c->h_err, c->d_err, sizeof(int32_t), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return lfail(lh, MB_ERR_CUDA, std::string("local head outputs: ") + cudaGetErrorString(e));
    const int32_t bits = *c->h_err;
    if (!bits) return MB_OK;
    if (cudaMemset(c->d_err, 0, sizeof(int32_t)) != cudaSuccess)
        return lfail(lh, MB_ERR_CUDA, "local head: clearing the device status failed");
    if (bits & mb::DERR_TIMEOUT) return lfail(lh, MB_ERR_TIMEOUT, "local head: a bounded device-side wait gave up");
    return lfail(lh, MB_ERR_DEVICE, "local head: a kernel rejected an item");
}

MB_API int mb_argmax_penalty(int32_t n, int32_t codes, const float* logits, uint32_t* seen, float penalty,
                             int32_t* tokens, void* cuda_stream) {
    if (n < 0 || !(codes == 128 || codes == 256 || codes == 512 || codes == 1024 || codes == 2048) ||
        !(penalty > 0.f) || !isfinite(penalty))
        return MB_ERR_ARG;
    if (n == 0) return MB_OK;
    if (!logits || !seen || !tokens || (reinterpret_cast<uintptr_t>(logits) & 15)) return MB_ERR_ARG;
    return launch_argmax(n, codes, logits, seen, nullptr, n, codes / 32, 0, penalty, tokens, 1,
                         static_cast<cudaStream_t>(cuda_stream)) == cudaSuccess
               ? MB_OK
               : MB_ERR_CUDA;
}

}  // extern "C"
