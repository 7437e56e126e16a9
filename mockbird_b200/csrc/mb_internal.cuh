// Internal declarations shared by the library's translation units.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "mockbird_kv.h"

namespace mb {

constexpr int HD = 64;                  // head dim (kernels-decode.ts: 64 lanes per head)
constexpr float SCALE = 0.125f;         // literal attention scale (docs analysis :846)
constexpr float LOG2E = 1.4426950408889634f;
// Bound of every device-side wait, in SM clock cycles (~2 s at 1.9 GHz; a bulk
// copy takes microseconds): a wait that runs out flags DERR_TIMEOUT.
constexpr long long WAIT_LIMIT = 4000000000LL;

// device-side rejection bits, reported by mb_sync
enum : int32_t {
    DERR_STREAM = 1,
    DERR_POSITION = 2,
    DERR_CAPACITY = 4,
    DERR_TIMEOUT = 8,
};

// Everything a kernel needs to address one layer of the rings.
struct RingView {
    void* kv;             // base of kv[layer]: [stream][2][head][slot][64]
    int32_t* slot_pos;    // base of slot_pos[layer]: [stream][slot]
    const float2* rope;   // [max_position][32] (cos, sin)
    int32_t* err;         // device rejection bits
    int32_t streams, heads, capacity, wrap, max_position;
    size_t kv_layer;      // elements of kv per layer (a launch over several layers steps by it)
    size_t slot_layer;    // elements of slot_pos per layer
    long long wait_limit; // bound of the decode kernel's waits for its K/V chunk (cycles)
    int32_t wait_probe;   // 1: those waits target a barrier nothing signals (they run out; tests)
};

struct Scratch {
    float* part;          // [max_batch][heads][max_splits][2 + 64]
    int32_t* counters;    // [max_batch][heads], zero between launches
    int32_t max_splits;
};

}  // namespace mb

struct mb_ctx {
    mb_config cfg;
    size_t esize = 4;
    size_t kv_bytes = 0;
    void* kv = nullptr;
    int32_t* slot_pos = nullptr;
    float2* rope = nullptr;
    int32_t* d_err = nullptr;
    mb::Scratch scratch{};
    size_t scratch_bytes = 0;
    // staging for the host-array entry points
    int32_t* d_ids = nullptr;  // [2][max_batch]: a call's stream ids, then its positions
    int32_t* h_ids = nullptr;  // page-locked staging of the same, one copy per call
    cudaEvent_t ev_ids = nullptr;  // recorded behind the copy out of h_ids
    float* d_qkv = nullptr;   // [layers][max_batch][3*H*64]
    float* d_out = nullptr;   // [layers][max_batch][H*64]
    // mb_prefill's stage on fp32 rings (bf16 hi/lo parts of Q, K, V), grown on demand
    void* pf_stage = nullptr;
    size_t pf_stage_bytes = 0;
    // mb_decode_step_host's copy pipeline: inputs in and outputs out in groups of
    // layers on their own streams, so that the copies overlap the decode of others
    cudaStream_t cp_in = nullptr, cp_out = nullptr;
    std::vector<cudaEvent_t> ev_in, ev_done;  // per copy group: inputs landed / last layer decoded
    cudaEvent_t ev_start = nullptr, ev_end = nullptr;
    int32_t* h_err = nullptr;  // pinned copy of d_err, read by the host-array entry points
    bool persistent = false;  // decode with the persistent stream-K kernel (when it applies) instead
    long long wait_limit = mb::WAIT_LIMIT;  // mb_set_wait_limit
    bool wait_probe = false;                // mb_set_wait_limit with a negative bound
    std::string last_error;
};

namespace mb {

inline RingView ring_view(const mb_ctx* c, int layer) {
    RingView v;
    size_t per_layer = (size_t)c->cfg.streams * 2 * c->cfg.heads * (size_t)c->cfg.capacity * HD;
    v.kv = (char*)c->kv + per_layer * layer * c->esize;
    v.slot_pos = c->slot_pos + (size_t)layer * c->cfg.streams * c->cfg.capacity;
    v.kv_layer = per_layer;
    v.slot_layer = (size_t)c->cfg.streams * c->cfg.capacity;
    v.rope = c->rope;
    v.err = c->d_err;
    v.streams = c->cfg.streams;
    v.heads = c->cfg.heads;
    v.capacity = c->cfg.capacity;
    v.wrap = c->cfg.wrap;
    v.max_position = c->cfg.max_position;
    v.wait_limit = c->wait_limit;
    v.wait_probe = c->wait_probe ? 1 : 0;
    return v;
}

// RoPE of one (even, odd) pair: out = (a c - b s, b c + a s) with every product
// and sum rounded separately (no FMA), so every kernel that ropes a row (decode
// append, prefill cache, prefill Q) rounds it the same way and the stored K
// matches a CPU restatement bit for bit (kernels-decode.ts:220-232; partner
// -v[d+1] / +v[d-1]).
__device__ __forceinline__ float2 rope_pair(float2 v, float2 cs) {
    return make_float2(__fadd_rn(__fmul_rn(v.x, cs.x), -__fmul_rn(v.y, cs.y)),
                       __fadd_rn(__fmul_rn(v.y, cs.x), __fmul_rn(v.x, cs.y)));
}

// rows of one split-K chunk: 16 KB of K (and 16 KB of V) per chunk
inline int chunk_rows(int dtype) { return dtype == MB_F32 ? 64 : 128; }

// launchers (mb_decode.cu / mb_prefill.cu); return the launch's cudaError_t
cudaError_t launch_rope_append(int dtype, const RingView& r, int n, const int32_t* streams,
                               const int32_t* positions, float* qkv, cudaStream_t st);
// overlap_previous: launch with programmatic dependent launch, allowed only when
// the previous kernel on the stream is a decode launch of a DIFFERENT layer
// (consecutive layers of one decode step): this launch's ring reads and append
// may then run before that kernel has finished.
// out_bf16: write the context rows as bf16 (out then points to __nv_bfloat16).
// layers: the launch covers this many consecutive layers from r's (the same n
// items in each): q and out of layer l at q + l*n*q_stride, out + l*n*heads*64;
// the scratch must hold n * layers items.
cudaError_t launch_decode(int dtype, bool append, const RingView& r, const Scratch& s, int n,
                          const int32_t* streams, const int32_t* positions, const float* q, int q_stride,
                          void* out, cudaStream_t st, bool overlap_previous = false, bool out_bf16 = false,
                          int layers = 1);
bool decode_persist_supported(const RingView& r, int n, int q_stride);
int persist_part_stride(int dtype, int capacity);  // split-K partial slots per (item, head)
cudaError_t launch_decode_persist(int dtype, bool append, const RingView& r, const Scratch& s, int n,
                                  const int32_t* streams, const int32_t* positions, const float* q, int q_stride,
                                  float* out, cudaStream_t st);
// stage: prefill_stage_bytes(dtype, n, heads, rows) bytes of device memory (none for 16-bit rings)
cudaError_t launch_prefill(int dtype, const RingView& r, int n, const int32_t* streams, int rows,
                           const float* qkv, float* out, void* stage, cudaStream_t st);
size_t prefill_stage_bytes(int dtype, int n, int heads, int rows);
cudaError_t launch_prefill_attn_tc(int dtype, const RingView& r, int n, const int32_t* streams, int rows,
                                   const float* qkv, float* out, cudaStream_t st);
// fp32 rings: the attention over the bf16 hi/lo parts of Q, K and V that the
// RoPE/cache kernel wrote to `stage` ([6][n][heads][rows][64]).
cudaError_t launch_prefill_attn_split(const RingView& r, int n, const int32_t* streams, int rows, const void* stage,
                                      float* out, cudaStream_t st);
cudaError_t launch_gather(int dtype, const RingView& r, int stream, int position, void* k_out, void* v_out,
                          int32_t* slots_out, cudaStream_t st);
cudaError_t launch_ring_write(int dtype, const RingView& r, int stream, int first, int count, const void* k,
                              const void* v, cudaStream_t st);
cudaError_t launch_reset(const mb_ctx* c, int stream, cudaStream_t st);

// host-array entry points (mb_api.cu): checks of the items on the host, and the
// status of the device rejection bits a call read back (cleared on the device;
// the message goes to the context's last error)
int check_items_host(mb_ctx* c, int n, const int32_t* streams, const int32_t* positions);
int report_bits(mb_ctx* c, int32_t bits);

// Execution priority (cudaLaunchAttributePriority) of the kernels this thread
// launches while `set`: `value` for every kernel but the decode attention, which
// gets `decode_value`.  Unset, a launch carries no priority and runs at its
// stream's.  The decoder step sets it around its two half-batch chains so that
// one half's GEMMs and LayerNorms are dispatched ahead of the other half's
// pending decode CTAs (mb_decoder.cu).
struct LaunchPriority {
    bool set = false;
    int value = 0, decode_value = 0;
};
extern thread_local LaunchPriority launch_priority;
// Appends the priority attribute (when set) after the `n` attributes in `attrs`
// (room for one more); returns the new count.
inline unsigned int with_priority(cudaLaunchAttribute* attrs, unsigned int n, bool decode = false) {
    if (!launch_priority.set) return n;
    attrs[n].id = cudaLaunchAttributePriority;
    attrs[n].val.priority = decode ? launch_priority.decode_value : launch_priority.value;
    return n + 1;
}

}  // namespace mb
