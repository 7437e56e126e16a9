// The transformer-layer machinery shared by the global decode step
// (mb_decoder.cu) and the local 17-step head (mb_local.cu): weights on the
// device, cuBLASLt GEMM plans, and the per-layer sequence of DecodeRunner.runLayer
// (liyu1981/mockbird, src/lib/tts/engine/decode.ts:474-620).
#pragma once

#include <cublasLt.h>

#include <map>
#include <string>
#include <tuple>
#include <vector>

#include "mb_internal.cuh"

struct mb_decoder {
    using bf16 = __nv_bfloat16;
    mb_ctx* ctx = nullptr;
    int hid = 0, ffn = 0, layers = 0;
    struct Layer {
        const float *ln1_w, *ln1_b, *b_attn, *b_proj, *ln2_w, *ln2_b, *b_in, *b_out;
        const bf16 *w_attn, *w_proj, *w_in, *w_out;
    };
    std::vector<Layer> L;
    const float *lnf_w = nullptr, *lnf_b = nullptr;
    void* wmem = nullptr;      // all weights, one allocation
    bf16* xb = nullptr;        // [max_batch][max(hid, ffn)] GEMM input
    float* qkv = nullptr;      // [max_batch][3*hid]
    float* h1 = nullptr;       // [max_batch][ffn]
    cublasLtHandle_t lt = nullptr;
    void* workspace = nullptr;
    size_t ws_bytes = 32u << 20;
    struct Plan {  // one GEMM shape: descriptors and the chosen algorithm, built once
        cublasLtMatmulDesc_t op = nullptr;
        cublasLtMatrixLayout_t a = nullptr, b = nullptr, c = nullptr;
        cublasLtMatmulAlgo_t algo{};
    };
    std::map<std::tuple<int, int, int, int>, Plan> plans;  // (M, N, K, has bias)
    // mb_decoder_step replays one captured step per item count over staged inputs
    bool use_graph = true;
    cudaStream_t cap = nullptr;
    int32_t *g_streams = nullptr, *g_positions = nullptr;  // [max_batch]
    float* g_hidden = nullptr;                              // [max_batch][hid]
    std::map<int, cudaGraphExec_t> graphs;
};

namespace mb {
namespace dec {

using bf16 = __nv_bfloat16;

// Records `msg` as the context's last error and returns `code`.
int fail(mb_decoder* d, int code, const std::string& msg);

// fp32 -> bf16 bits, round to nearest even (NaN stays NaN).
uint16_t f32_to_bf16_bits(float f);

// y[M][N] (fp32, row-major) = x[M][K] (bf16) * W[K][N] (bf16) (+ bias[N] when
// non-null) (+ y when accumulate).  cuBLASLt, fp32 accumulation.
int gemm(mb_decoder* d, int M, int N, int K, const bf16* x, const bf16* W, const float* bias, float* y,
         bool accumulate, cudaStream_t st);

// The layers of mb_decoder_step on `hidden` [n][hid], then ln_f: into `lnf_bf16`
// [n][hid] (bf16) when it is non-null, else into `hidden` in place (fp32).
// Arguments are the caller's to check; the current device must be the context's.
int run(mb_decoder* d, int n, const int32_t* streams, const int32_t* positions, float* hidden, bf16* lnf_bf16,
        cudaStream_t st);

// y = bf16(x), n elements.
cudaError_t to_bf16(const float* x, bf16* y, size_t n, cudaStream_t st);

}  // namespace dec
}  // namespace mb
