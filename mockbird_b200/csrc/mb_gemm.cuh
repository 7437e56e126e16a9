// Batched-stream GEMMs of the decode step on the 5th-generation tensor cores
// (mb_gemm.cu): y = x W (+ bias) with one activation row per stream.  They
// replace the GEMV dispatches of DecodeRunner.runLayer (liyu1981/mockbird,
// src/lib/tts/engine/decode.ts:517-526 QKV, :553-619 c_proj, fc_in, fc_out;
// GEMV, kernels-decode.ts:127-142: y = b + x W, W [K][N] row-major) and the
// audio-head GEMV of nextFrame (decode.ts:788-939), for all streams at once.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "mb_internal.cuh"

namespace mb {
namespace gemm {

// What the epilogue does with acc = x W (fp32) of each output element.
enum Epi : int {
    EPI_STORE = 0,      // y (fp32)  = acc + bias
    EPI_ACCUM = 1,      // y (fp32) += acc + bias      (the residual add of c_proj / fc_out)
    EPI_GELU_BF16 = 2,  // y (bf16)  = gelu_tanh(acc + bias)   (fc_in, GELU_TANH)
    // The QKV projection of a decode step with RoPE and the ring append in its
    // epilogue: the q columns [0, hid) are roped at the row's position and stored
    // fp32 at y (the decode kernel's query input); the k columns are roped and,
    // with the v columns, rounded to the ring's storage type and stored at slot
    // position % capacity of the row's stream, whose slot position is recorded
    // (ROPE_SPLIT_RING / ROPE_SPLIT_CODEC, kernels-decode.ts:216-241, 679-714).
    EPI_QKV_RING = 3,
};

constexpr int BM = 128;  // rows (streams) per tile: the UMMA M, one TMEM lane per row
constexpr int BK = 64;   // K per stage: one 128-byte swizzle row of bf16

// Tile width and split of K for one GEMM shape, chosen on the host: the fewest
// bytes per CTA (its operand tiles, plus the partial tiles it reads from the
// other CTAs of its cluster) with all CTAs resident in one wave.
struct Plan {
    int bn;        // 32, 64 or 128 output columns per CTA (per CTA pair when `pair`)
    int splits;    // K split over this many CTAs of one thread-block cluster (1..8)
    int pair = 0;  // 1: a CTA pair (tcgen05 cta_group::2) per 128 x bn tile, K unsplit
};
// The tensor-map boxes a plan loads: x rows per CTA, W^T rows per CTA, and K
// blocks per box.  A TMA box costs about the same SM time whatever its size, so
// the one-CTA kernel fetches several K blocks per box (3-D view of the matrix).
inline int a_box_rows(const Plan& p) { return p.pair ? BM / 2 : BM; }
inline int b_box_rows(const Plan& p) { return p.pair ? p.bn / 2 : p.bn; }
constexpr int kb_per_box(int bn) { return bn == 128 ? 3 : 4; }  // one-CTA kernel (two stages of boxes)
inline int box_kb(const Plan& p) { return p.pair ? 1 : kb_per_box(p.bn); }
Plan choose(int M, int N, int K, int epi);

struct Args {
    int M, N, K;           // K a multiple of 64, N a multiple of the plan's bn
    int splits;
    const float* bias;     // [N] or null
    void* y;               // fp32 [M][ldy] (EPI_STORE / EPI_ACCUM) or bf16 [M][ldy] (EPI_GELU_BF16)
    int ldy;
    int* err;              // device status word: DERR_TIMEOUT is OR-ed in when a bounded wait gives up
    // EPI_QKV_RING only: the layer's ring (its kv, slot_pos and rope), the row's
    // stream id and position, and the ring's storage type (MB_F32 / MB_BF16 /
    // MB_F16).  A row whose stream or position the ring rejects appends nothing
    // (the decode kernel that follows flags it).
    RingView ring;
    const int32_t* streams;
    const int32_t* positions;
    int ring_dtype;
};

// Tensor map of a K-major bf16 matrix [rows][k] (rows k*2 bytes apart, 16-byte
// aligned base) viewed as [k / 64][rows][64]: dims (64, rows, k / 64), strides
// (k*2, 128) bytes; box 64 x box_rows x box_kb, 128-byte swizzle, zero fill past
// the last row and the last K block.  A box lands in shared memory as box_kb
// consecutive [box_rows][64] tiles, each swizzled as a 2-D box of its own would be.
bool make_map(CUtensorMap* m, const void* base, int k, int rows, int box_rows, int box_kb);

// ta: x [M][K] bf16 (box a_box_rows(plan) x box_kb(plan)); tb: W^T [N][K] bf16
// (box b_box_rows(plan) x box_kb(plan)).
// pdl: launch as a programmatic dependent of the previous kernel on `st` (the
// kernel waits for it before its first read of x or access of y).
cudaError_t launch(const CUtensorMap& ta, const CUtensorMap& tb, const Args& a, const Plan& p, int epi,
                   cudaStream_t st, bool pdl);

}  // namespace gemm
}  // namespace mb
