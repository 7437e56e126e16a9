// The transformer-layer machinery shared by the global decode step
// (mb_decoder.cu) and the local 17-step head (mb_local.cu): weights on the
// device, the tensor maps of this library's tcgen05 GEMMs (mb_gemm.cu), and the
// per-layer sequence of DecodeRunner.runLayer (liyu1981/mockbird,
// src/lib/tts/engine/decode.ts:474-620).
#pragma once

#include <map>
#include <string>
#include <tuple>
#include <vector>

#include "mb_gemm.cuh"
#include "mb_internal.cuh"

struct mb_decoder {
    using bf16 = __nv_bfloat16;
    mb_ctx* ctx = nullptr;
    int hid = 0, ffn = 0, layers = 0;
    struct Layer {
        const float *ln1_w, *ln1_b, *b_attn, *b_proj, *ln2_w, *ln2_b, *b_in, *b_out;
        const bf16 *w_attn, *w_proj, *w_in, *w_out;  // transposed: W^T [N][K], K-major
    };
    std::vector<Layer> L;
    const float *lnf_w = nullptr, *lnf_b = nullptr;
    void* wmem = nullptr;      // all weights, one allocation
    bf16* xb = nullptr;        // [max_batch][hid] GEMM input (LayerNorm output, context rows)
    float* qkv = nullptr;      // [max_batch][3*hid]
    bf16* h1 = nullptr;        // [max_batch][ffn] GELU(fc_in) output, fc_out's input
    // tensor maps of the GEMM operands, built once per (base, k, rows, box rows, box K blocks),
    // and the GEMM plans, once per (M, N, K, epilogue)
    std::map<std::tuple<const void*, int, int, int, int>, CUtensorMap> maps;
    std::map<std::tuple<int, int, int, int>, mb::gemm::Plan> gemm_plans;
    // mb_decoder_step replays one captured step per item count over staged inputs
    bool use_graph = true;
    cudaStream_t cap = nullptr;
    int32_t *g_streams = nullptr, *g_positions = nullptr;  // [max_batch]
    float* g_hidden = nullptr;                              // [max_batch][hid]
    std::map<int, cudaGraphExec_t> graphs;
    // A step of at least 2 * SPLIT_MIN_ROWS items runs as two half-batch chains:
    // the second on `side`, forked from and joined to the caller's stream by
    // events, started once the first has launched its layer-0 QKV GEMM
    // (mb::dec::run).  MOCKBIRD_DECODER_SPLIT=0 keeps one chain.
    bool split = true;
    cudaStream_t side = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_stagger = nullptr, ev_join = nullptr;
    int prio_high = 0, prio_low = 0;  // the device's greatest and least stream priority
};

namespace mb {
namespace dec {

using bf16 = __nv_bfloat16;

// Records `msg` as the context's last error and returns `code`.
int fail(mb_decoder* d, int code, const std::string& msg);

// fp32 -> bf16 bits, round to nearest even (NaN stays NaN).
uint16_t f32_to_bf16_bits(float f);

// y = x[M][K] (bf16, rows K apart) * W (given transposed, Wt [N][K] bf16) with
// fp32 accumulation on the tensor cores (mb_gemm.cu), then the epilogue `epi`
// (mb::gemm::Epi) with bias[N] when non-null: y fp32 [M][ldy] (store or +=), or
// bf16 [M][ldy] after GELU(tanh).  x and Wt must be buffers whose tensor maps
// this decoder may cache: x one of its own activation buffers (max_batch rows),
// Wt a weight matrix it owns.
// EPI_QKV_RING also takes the layer's ring and the rows' stream ids and positions.
// x_row0: x starts that many rows into its buffer (the tensor map then spans the
// max_batch - x_row0 rows left in it).
int gemm(mb_decoder* d, int M, int N, int K, const bf16* x, const bf16* Wt, const float* bias, void* y, int ldy,
         int epi, cudaStream_t st, const RingView* ring = nullptr, const int32_t* streams = nullptr,
         const int32_t* positions = nullptr, int x_row0 = 0);

// W [K][N] fp32 (host, row-major) -> W^T [N][K] as bf16 bits, the layout the GEMM reads.
void transpose_to_bf16(const float* w, int K, int N, uint16_t* out);

// The layers of mb_decoder_step on `hidden` [n][hid], then ln_f: into `lnf_bf16`
// [n][hid] (bf16) when it is non-null, else into `hidden` in place (fp32).
// ln1_ready: the caller has already written layer 0's LN1 of `hidden` into
// d->xb (bf16), so that LayerNorm is skipped.
// qkv_append: RoPE and the ring append run in the QKV GEMM's epilogue
// (EPI_QKV_RING) and the decode kernel only attends; otherwise the GEMM stores
// q|k|v and the decode kernel ropes and appends (the local head: its GEMMs are
// latency-bound, and the epilogue's position and RoPE-table loads cost it more
// than the separate append does, 279k against 295k frames/s).
// split: with d->split on and at least 2 * SPLIT_MIN_ROWS items, the items run as
// two half-batch chains on `st` and d->side, the second started after the
// first's layer-0 QKV GEMM, every GEMM, LayerNorm and combine launched at the
// device's greatest priority and the decode attention at its least, so that one
// half's latency-bound GEMMs run while the other half's HBM-bound decode does.
// Each chain has its own rows of the activation buffers and of the split-K
// scratch.
// Arguments are the caller's to check; the current device must be the context's.
constexpr int SPLIT_MIN_ROWS = 64;
int run(mb_decoder* d, int n, const int32_t* streams, const int32_t* positions, float* hidden, bf16* lnf_bf16,
        cudaStream_t st, bool ln1_ready = false, bool qkv_append = true, bool split = false);

// ---- LayerNorm of one row by one warp (LAYERNORM_1: mean, then the mean squared
// deviation, out = (x - mean) * rsqrt(var + 1e-5) * w + b), width = 32 * PER.
// The row sits in registers between ln_load and ln_apply, so a kernel may also
// store it (ln_store) or take it from elsewhere.

// lane's PER values: columns 4 lane + 128 k .. + 3 when PER % 4 == 0 (16-byte
// loads), else lane + 32 i
template <int PER>
__device__ __forceinline__ void ln_load(const float* xr, int lane, float (&v)[PER]) {
    if constexpr (PER % 4 == 0) {
#pragma unroll
        for (int k = 0; k < PER / 4; k++) {
            const float4 q = *reinterpret_cast<const float4*>(xr + 4 * lane + 128 * k);
            v[4 * k] = q.x, v[4 * k + 1] = q.y, v[4 * k + 2] = q.z, v[4 * k + 3] = q.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < PER; i++) v[i] = xr[lane + 32 * i];
    }
}

// the row back to memory in ln_load's layout (fp32)
template <int PER>
__device__ __forceinline__ void ln_store(float* yr, int lane, const float (&v)[PER]) {
    if constexpr (PER % 4 == 0) {
#pragma unroll
        for (int k = 0; k < PER / 4; k++)
            *reinterpret_cast<float4*>(yr + 4 * lane + 128 * k) =
                make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
    } else {
#pragma unroll
        for (int i = 0; i < PER; i++) yr[lane + 32 * i] = v[i];
    }
}

template <typename TO, int PER>
__device__ __forceinline__ void ln_apply(const float (&v)[PER], const float* __restrict__ w,
                                         const float* __restrict__ b, TO* yr, int width, int lane) {
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < PER; i++) sum += v[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float mean = sum / (float)width;
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < PER; i++) {
        const float d = v[i] - mean;
        sq += d * d;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    const float inv = rsqrtf(sq / (float)width + 1e-5f);
    if constexpr (PER % 4 == 0) {  // 16-byte weight/bias loads, 4-element stores
#pragma unroll
        for (int k = 0; k < PER / 4; k++) {
            const int c = 4 * lane + 128 * k;
            const float4 wk = *reinterpret_cast<const float4*>(w + c), bk = *reinterpret_cast<const float4*>(b + c);
            const float r0 = (v[4 * k] - mean) * inv * wk.x + bk.x, r1 = (v[4 * k + 1] - mean) * inv * wk.y + bk.y;
            const float r2 = (v[4 * k + 2] - mean) * inv * wk.z + bk.z, r3 = (v[4 * k + 3] - mean) * inv * wk.w + bk.w;
            if constexpr (sizeof(TO) == 4) {
                *reinterpret_cast<float4*>(yr + c) = make_float4(r0, r1, r2, r3);
            } else {
                const __nv_bfloat162 lo = __floats2bfloat162_rn(r0, r1), hi = __floats2bfloat162_rn(r2, r3);
                uint2 u;
                u.x = *reinterpret_cast<const uint32_t*>(&lo);
                u.y = *reinterpret_cast<const uint32_t*>(&hi);
                *reinterpret_cast<uint2*>(yr + c) = u;
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < PER; i++) {
            const int c = lane + 32 * i;
            yr[c] = (TO)((v[i] - mean) * inv * w[c] + b[c]);
        }
    }
}


}  // namespace dec
}  // namespace mb
