// The decode step around the KV-ring path: the global
// transformer layer of DecodeRunner.runLayer (liyu1981/mockbird,
// src/lib/tts/engine/decode.ts:474-620) for n streams at once, and the final
// LayerNorm of globalStep (decode.ts:749-772).
//
// Per layer: LN1 -> QKV GEMM -> append + RoPE + attention (this library's decode
// kernel) -> c_proj GEMM + residual -> LN2 -> fc_in GEMM -> GELU(tanh) -> fc_out
// GEMM + residual.  The four GEMMs are plain library GEMMs (cuBLASLt, bf16
// weights and activations, fp32 accumulation, bias and residual in the
// epilogue: y = b + x W, W [K][N] row-major as the published graph stores it);
// LayerNorm (LAYERNORM_1, kernels-decode.ts:168-200: eps 1e-5, two passes) and
// GELU (GELU_TANH, kernels-decode.ts:373-390) are kernels here.
#include <stdlib.h>
#include <string.h>

#include "mb_decoder.cuh"

namespace {

using bf16 = __nv_bfloat16;

// ---------------------------------------------------------------- kernels

// One warp per row: mean, then the mean squared deviation (the two passes of
// LAYERNORM_1), out = (x - mean) * rsqrt(var + 1e-5) * w + b (mb::dec::ln_load /
// ln_apply).  In place is fine: the row is in registers before it is written.
template <typename TO, int PER>
__global__ void layernorm_rows(const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ b,
                               TO* __restrict__ y, int rows, int width) {
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    float v[PER];
    mb::dec::ln_load<PER>(x + (size_t)row * width, lane, v);
    mb::dec::ln_apply<TO, PER>(v, w, b, y + (size_t)row * width, width, lane);
}

// tanh on the MUFU unit (tanh.approx.f32, max relative error about 2^-11): the
// result is rounded to bf16 (2^-8) right after, so the approximation is below
// the output's own resolution.
__device__ __forceinline__ float tanh_fast(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// GELU, tanh approximation (GELU_TANH), fp32 in -> bf16 out, 4 elements a thread
// (n a multiple of 4, both pointers 16-byte aligned)
__global__ void gelu_tanh_to_bf16(const float* __restrict__ x, bf16* __restrict__ y, size_t n) {
    const size_t n4 = n / 4;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const float4 v = reinterpret_cast<const float4*>(x)[i];
        float r[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const float a = r[k];
            const float inner = 0.7978845608028654f * (a + 0.044715f * a * a * a);
            r[k] = 0.5f * a * (1.f + tanh_fast(inner));
        }
        const __nv_bfloat162 lo = __floats2bfloat162_rn(r[0], r[1]), hi = __floats2bfloat162_rn(r[2], r[3]);
        uint2 packed;
        packed.x = *reinterpret_cast<const uint32_t*>(&lo);
        packed.y = *reinterpret_cast<const uint32_t*>(&hi);
        reinterpret_cast<uint2*>(y)[i] = packed;
    }
}

__global__ void to_bf16_kernel(const float* __restrict__ x, bf16* __restrict__ y, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = __float2bfloat16_rn(x[i]);
}

template <typename TO>
cudaError_t layernorm(const float* x, const float* w, const float* b, TO* y, int rows, int width, cudaStream_t st) {
    const int warps = 2, blocks = (rows + warps - 1) / warps;
    switch (width / 32) {  // width = heads * 64
        case 2: layernorm_rows<TO, 2><<<blocks, 32 * warps, 0, st>>>(x, w, b, y, rows, width); break;
        case 8: layernorm_rows<TO, 8><<<blocks, 32 * warps, 0, st>>>(x, w, b, y, rows, width); break;
        case 24: layernorm_rows<TO, 24><<<blocks, 32 * warps, 0, st>>>(x, w, b, y, rows, width); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

constexpr int CVT_BLOCKS = 2 * 148;

}  // namespace

namespace mb {
namespace dec {

int fail(mb_decoder* d, int code, const std::string& msg) {
    if (d && d->ctx) d->ctx->last_error = msg;
    return code;
}

uint16_t f32_to_bf16_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

cudaError_t to_bf16(const float* x, bf16* y, size_t n, cudaStream_t st) {
    to_bf16_kernel<<<CVT_BLOCKS, 256, 0, st>>>(x, y, n);
    return cudaGetLastError();
}

int gemm(mb_decoder* d, int M, int N, int K, const bf16* x, const bf16* W, const float* bias, float* y,
         bool accumulate, cudaStream_t st) {
    // column-major view: y^T [N x M] = W^T [N x K] * x^T [K x M]
    cublasStatus_t s = CUBLAS_STATUS_SUCCESS;
    const bool has_bias = bias != nullptr;
    const auto key = std::make_tuple(M, N, K, has_bias ? 1 : 0);
    auto it = d->plans.find(key);
    if (it == d->plans.end()) {
        mb_decoder::Plan p;
        cublasLtEpilogue_t epi = has_bias ? CUBLASLT_EPILOGUE_BIAS : CUBLASLT_EPILOGUE_DEFAULT;
        cudaDataType_t bias_t = CUDA_R_32F;
        s = cublasLtMatmulDescCreate(&p.op, CUBLAS_COMPUTE_32F, CUDA_R_32F);
        if (s == CUBLAS_STATUS_SUCCESS)
            s = cublasLtMatmulDescSetAttribute(p.op, CUBLASLT_MATMUL_DESC_EPILOGUE, &epi, sizeof epi);
        if (s == CUBLAS_STATUS_SUCCESS && has_bias)
            s = cublasLtMatmulDescSetAttribute(p.op, CUBLASLT_MATMUL_DESC_BIAS_DATA_TYPE, &bias_t, sizeof bias_t);
        if (s == CUBLAS_STATUS_SUCCESS && has_bias)
            s = cublasLtMatmulDescSetAttribute(p.op, CUBLASLT_MATMUL_DESC_BIAS_POINTER, &bias, sizeof bias);
        if (s == CUBLAS_STATUS_SUCCESS) s = cublasLtMatrixLayoutCreate(&p.a, CUDA_R_16BF, N, K, N);
        if (s == CUBLAS_STATUS_SUCCESS) s = cublasLtMatrixLayoutCreate(&p.b, CUDA_R_16BF, K, M, K);
        if (s == CUBLAS_STATUS_SUCCESS) s = cublasLtMatrixLayoutCreate(&p.c, CUDA_R_32F, N, M, N);
        cublasLtMatmulPreference_t pref = nullptr;
        if (s == CUBLAS_STATUS_SUCCESS) s = cublasLtMatmulPreferenceCreate(&pref);
        if (s == CUBLAS_STATUS_SUCCESS)
            s = cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &d->ws_bytes,
                                                     sizeof d->ws_bytes);
        cublasLtMatmulHeuristicResult_t res = {};
        int found = 0;
        if (s == CUBLAS_STATUS_SUCCESS)
            s = cublasLtMatmulAlgoGetHeuristic(d->lt, p.op, p.a, p.b, p.c, p.c, pref, 1, &res, &found);
        if (pref) cublasLtMatmulPreferenceDestroy(pref);
        if (s == CUBLAS_STATUS_SUCCESS && found == 0) s = CUBLAS_STATUS_NOT_SUPPORTED;
        if (s != CUBLAS_STATUS_SUCCESS) {
            if (p.c) cublasLtMatrixLayoutDestroy(p.c);
            if (p.b) cublasLtMatrixLayoutDestroy(p.b);
            if (p.a) cublasLtMatrixLayoutDestroy(p.a);
            if (p.op) cublasLtMatmulDescDestroy(p.op);
            return fail(d, MB_ERR_CUDA, std::string("cuBLASLt setup failed: ") + cublasLtGetStatusString(s));
        }
        p.algo = res.algo;
        it = d->plans.emplace(key, p).first;
    }
    mb_decoder::Plan& p = it->second;
    if (has_bias) s = cublasLtMatmulDescSetAttribute(p.op, CUBLASLT_MATMUL_DESC_BIAS_POINTER, &bias, sizeof bias);
    const float alpha = 1.f, beta = accumulate ? 1.f : 0.f;
    if (s == CUBLAS_STATUS_SUCCESS)
        s = cublasLtMatmul(d->lt, p.op, &alpha, W, p.a, x, p.b, &beta, y, p.c, y, p.c, &p.algo, d->workspace,
                           d->ws_bytes, st);
    if (s != CUBLAS_STATUS_SUCCESS)
        return fail(d, MB_ERR_CUDA, std::string("cuBLASLt matmul failed: ") + cublasLtGetStatusString(s));
    return MB_OK;
}

int run(mb_decoder* d, int n, const int32_t* streams, const int32_t* positions, float* hidden, bf16* lnf_bf16,
        cudaStream_t st, bool ln1_ready) {
    mb_ctx* c = d->ctx;
    const int h = d->hid, f = d->ffn;
    int rc = MB_OK;
    cudaError_t e = cudaSuccess;
    for (int l = 0; l < d->layers && rc == MB_OK && e == cudaSuccess; l++) {
        const auto& W = d->L[l];
        if (!(l == 0 && ln1_ready) && (e = layernorm<bf16>(hidden, W.ln1_w, W.ln1_b, d->xb, n, h, st)) != cudaSuccess)
            break;
        if ((rc = gemm(d, n, 3 * h, h, d->xb, W.w_attn, W.b_attn, d->qkv, false, st))) break;
        // the context rows go straight to the bf16 input of the c_proj GEMM
        if ((e = mb::launch_decode(c->cfg.dtype, true, mb::ring_view(c, l), c->scratch, n, streams, positions, d->qkv,
                                   3 * h, d->xb, st, false, true)) != cudaSuccess)
            break;
        if ((rc = gemm(d, n, h, h, d->xb, W.w_proj, W.b_proj, hidden, true, st))) break;
        if ((e = layernorm<bf16>(hidden, W.ln2_w, W.ln2_b, d->xb, n, h, st)) != cudaSuccess) break;
        if ((rc = gemm(d, n, f, h, d->xb, W.w_in, W.b_in, d->h1, false, st))) break;
        gelu_tanh_to_bf16<<<CVT_BLOCKS, 256, 0, st>>>(d->h1, d->xb, (size_t)n * f);
        if ((rc = gemm(d, n, h, f, d->xb, W.w_out, W.b_out, hidden, true, st))) break;
        e = cudaGetLastError();
    }
    if (rc == MB_OK && e == cudaSuccess)
        e = lnf_bf16 ? layernorm<bf16>(hidden, d->lnf_w, d->lnf_b, lnf_bf16, n, h, st)
                     : layernorm<float>(hidden, d->lnf_w, d->lnf_b, hidden, n, h, st);
    if (rc) return rc;
    if (e != cudaSuccess) return fail(d, MB_ERR_CUDA, std::string("decoder: ") + cudaGetErrorString(e));
    return MB_OK;
}

}  // namespace dec
}  // namespace mb

extern "C" {

MB_API size_t mb_decoder_weight_count(const mb_ctx* c, int32_t ffn) {
    if (!c || ffn <= 0) return 0;
    const size_t h = (size_t)c->cfg.heads * mb::HD, f = (size_t)ffn;
    const size_t per_layer = 2 * h + h * 3 * h + 3 * h + h * h + h + 2 * h + h * f + f + f * h + h;
    return per_layer * c->cfg.layers + 2 * h;
}

MB_API int mb_decoder_destroy(mb_decoder* d) {
    if (!d) return MB_ERR_ARG;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(d->ctx->cfg.device);
    for (auto& kv : d->graphs) cudaGraphExecDestroy(kv.second);
    if (d->cap) cudaStreamDestroy(d->cap);
    void* ptrs[] = {d->wmem, d->xb, d->qkv, d->h1, d->workspace, d->g_streams, d->g_positions, d->g_hidden};
    for (void* p : ptrs)
        if (p) cudaFree(p);
    for (auto& kv : d->plans) {
        cublasLtMatrixLayoutDestroy(kv.second.c);
        cublasLtMatrixLayoutDestroy(kv.second.b);
        cublasLtMatrixLayoutDestroy(kv.second.a);
        cublasLtMatmulDescDestroy(kv.second.op);
    }
    if (d->lt) cublasLtDestroy(d->lt);
    if (prev >= 0) cudaSetDevice(prev);
    delete d;
    return MB_OK;
}

MB_API int mb_decoder_create(mb_ctx* c, int32_t ffn, const float* w, size_t count, mb_decoder** out) {
    if (!c || !w || !out || ffn <= 0 || ffn % 64) return MB_ERR_ARG;
    *out = nullptr;
    const int h = c->cfg.heads * mb::HD;
    if (h / 32 != 2 && h / 32 != 8 && h / 32 != 24) {
        c->last_error = "decoder: hidden width must be 64, 256 or 768";
        return MB_ERR_ARG;
    }
    if (count != mb_decoder_weight_count(c, ffn)) {
        c->last_error = "decoder: weight count does not match layers x (hidden, ffn)";
        return MB_ERR_ARG;
    }
    int prev = -1;
    cudaGetDevice(&prev);
    if (cudaSetDevice(c->cfg.device) != cudaSuccess) return MB_ERR_CUDA;
    mb_decoder* d = new mb_decoder();
    d->ctx = c;
    d->hid = h;
    d->ffn = ffn;
    d->layers = c->cfg.layers;
    auto bail = [&](int rc, const char* msg) {
        c->last_error = msg;
        mb_decoder_destroy(d);
        if (prev >= 0) cudaSetDevice(prev);
        return rc;
    };
    // device image: fp32 vectors first, then bf16 matrices (each block 256-byte aligned)
    struct Blk {
        size_t src, n;
        bool mat;
        size_t dst;
    };
    std::vector<Blk> blks;
    size_t src = 0;
    auto add = [&](size_t n, bool mat) {
        blks.push_back({src, n, mat, 0});
        src += n;
    };
    for (int l = 0; l < d->layers; l++) {
        add(h, false), add(h, false);                    // ln1
        add((size_t)h * 3 * h, true), add(3 * h, false);  // c_attn
        add((size_t)h * h, true), add(h, false);          // c_proj
        add(h, false), add(h, false);                    // ln2
        add((size_t)h * ffn, true), add(ffn, false);      // fc_in
        add((size_t)ffn * h, true), add(h, false);        // fc_out
    }
    add(h, false), add(h, false);  // ln_f
    size_t bytes = 0;
    for (auto& b : blks) {
        b.dst = bytes;
        bytes += ((b.n * (b.mat ? 2 : 4)) + 255) & ~size_t(255);
    }
    std::vector<unsigned char> img(bytes, 0);
    for (auto& b : blks) {
        if (b.mat) {
            uint16_t* o = reinterpret_cast<uint16_t*>(img.data() + b.dst);
            for (size_t i = 0; i < b.n; i++) o[i] = mb::dec::f32_to_bf16_bits(w[b.src + i]);
        } else {
            memcpy(img.data() + b.dst, w + b.src, b.n * 4);
        }
    }
    if (cudaMalloc(&d->wmem, bytes) != cudaSuccess) return bail(MB_ERR_OOM, "decoder: weight allocation failed");
    if (cudaMemcpy(d->wmem, img.data(), bytes, cudaMemcpyHostToDevice) != cudaSuccess)
        return bail(MB_ERR_CUDA, "decoder: weight upload failed");
    auto F = [&](size_t i) { return reinterpret_cast<const float*>((char*)d->wmem + blks[i].dst); };
    auto B = [&](size_t i) { return reinterpret_cast<const bf16*>((char*)d->wmem + blks[i].dst); };
    for (int l = 0; l < d->layers; l++) {
        const size_t o = (size_t)l * 12;
        d->L.push_back({F(o + 0), F(o + 1), F(o + 3), F(o + 5), F(o + 6), F(o + 7), F(o + 9), F(o + 11), B(o + 2),
                        B(o + 4), B(o + 8), B(o + 10)});
    }
    d->lnf_w = F(blks.size() - 2);
    d->lnf_b = F(blks.size() - 1);
    const size_t mb = c->cfg.max_batch, wide = (size_t)(ffn > h ? ffn : h);
    if (cudaMalloc(&d->xb, mb * wide * sizeof(bf16)) != cudaSuccess ||
        cudaMalloc(&d->qkv, mb * 3 * h * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&d->h1, mb * ffn * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&d->workspace, d->ws_bytes) != cudaSuccess || cudaMalloc(&d->g_streams, mb * 4) != cudaSuccess ||
        cudaMalloc(&d->g_positions, mb * 4) != cudaSuccess ||
        cudaMalloc(&d->g_hidden, mb * h * sizeof(float)) != cudaSuccess)
        return bail(MB_ERR_OOM, "decoder: activation allocation failed");
    if (cublasLtCreate(&d->lt) != CUBLAS_STATUS_SUCCESS) return bail(MB_ERR_CUDA, "decoder: cublasLtCreate failed");
    if (cudaStreamCreateWithFlags(&d->cap, cudaStreamNonBlocking) != cudaSuccess)
        return bail(MB_ERR_CUDA, "decoder: stream creation failed");
    {
        const char* v = getenv("MOCKBIRD_DECODER_GRAPH");
        d->use_graph = !(v && strcmp(v, "0") == 0);
    }
    if (prev >= 0) cudaSetDevice(prev);
    *out = d;
    return MB_OK;
}

MB_API int mb_decoder_step(mb_decoder* d, int32_t n, const int32_t* streams, const int32_t* positions,
                           float* hidden, void* cuda_stream) {
    if (!d) return MB_ERR_ARG;
    mb_ctx* c = d->ctx;
    if (n < 0 || n > c->cfg.max_batch) return mb::dec::fail(d, MB_ERR_ARG, "decoder: item count out of range");
    if (n == 0) return MB_OK;
    if (!streams || !positions || !hidden || (reinterpret_cast<uintptr_t>(hidden) & 15))
        return mb::dec::fail(d, MB_ERR_ARG, "decoder: null or misaligned device pointer");
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != c->cfg.device && cudaSetDevice(c->cfg.device) != cudaSuccess) return MB_ERR_CUDA;
    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    int rc = MB_OK;
    if (!d->use_graph) {
        rc = mb::dec::run(d, n, streams, positions, hidden, nullptr, st);
    } else {
        // One captured step per item count, over inputs staged into this object's
        // buffers; the first step of a count runs directly (kernel modules loaded,
        // GEMM plans built outside any capture) and is then captured for the next.
        const size_t hb = (size_t)n * d->hid * sizeof(float);
        cudaError_t e = cudaMemcpyAsync(d->g_streams, streams, n * 4, cudaMemcpyDeviceToDevice, st);
        if (e == cudaSuccess) e = cudaMemcpyAsync(d->g_positions, positions, n * 4, cudaMemcpyDeviceToDevice, st);
        if (e == cudaSuccess) e = cudaMemcpyAsync(d->g_hidden, hidden, hb, cudaMemcpyDeviceToDevice, st);
        auto it = d->graphs.find(n);
        if (e != cudaSuccess) {
            rc = mb::dec::fail(d, MB_ERR_CUDA, std::string("decoder inputs: ") + cudaGetErrorString(e));
        } else if (it != d->graphs.end()) {
            e = cudaGraphLaunch(it->second, st);
            if (e != cudaSuccess) rc = mb::dec::fail(d, MB_ERR_CUDA, std::string("decoder graph: ") + cudaGetErrorString(e));
        } else {
            rc = mb::dec::run(d, n, d->g_streams, d->g_positions, d->g_hidden, nullptr, st);
            cudaGraph_t g = nullptr;
            if (rc == MB_OK && (e = cudaStreamBeginCapture(d->cap, cudaStreamCaptureModeThreadLocal)) != cudaSuccess)
                rc = mb::dec::fail(d, MB_ERR_CUDA, std::string("decoder capture: ") + cudaGetErrorString(e));
            if (rc == MB_OK) {
                const int rc2 = mb::dec::run(d, n, d->g_streams, d->g_positions, d->g_hidden, nullptr, d->cap);
                e = cudaStreamEndCapture(d->cap, &g);
                cudaGraphExec_t ex = nullptr;
                if (rc2 == MB_OK && e == cudaSuccess) e = cudaGraphInstantiate(&ex, g, 0);
                if (g) cudaGraphDestroy(g);
                if (rc2 != MB_OK)
                    rc = rc2;
                else if (e != cudaSuccess)
                    rc = mb::dec::fail(d, MB_ERR_CUDA, std::string("decoder capture: ") + cudaGetErrorString(e));
                else
                    d->graphs.emplace(n, ex);
            }
        }
        if (rc == MB_OK && (e = cudaMemcpyAsync(hidden, d->g_hidden, hb, cudaMemcpyDeviceToDevice, st)) != cudaSuccess)
            rc = mb::dec::fail(d, MB_ERR_CUDA, std::string("decoder output: ") + cudaGetErrorString(e));
    }
    if (prev >= 0 && prev != c->cfg.device) cudaSetDevice(prev);
    return rc;
}

}  // extern "C"
