// Launch arguments, workspace layout and kernel entry points of the routed
// MoE layer.  Internal to the library (the public C ABI is include/ornith_moe_b200.h).
#pragma once
#include "moe_common.cuh"

namespace ornith {

// Workspace of one layer call, all offsets 256-byte aligned.  Rows of the
// intermediate buffers are "routes": r < R = 8T are routed slots (token r/8,
// slot r%8), r = R + t is the shared expert's row for token t.
struct Workspace {
    size_t xq, xs, xsum;          // token activations: int8 [T,2048] (permuted), fp16 [T,8], i32 [T,8]
    size_t middle;                // fp32 [R+T, 512] SiLU*up
    size_t mq, ms, msum;          // middle activations: int8 [R+T,512], fp16 [R+T,2], i32 [R+T,2]
    size_t route_out;             // fp32 [R+T, 2048] per-route down projections
    size_t final_f32;             // fp32 [T, 2048] combined sum before bf16 rounding (diagnostic)
    size_t counts, offsets, routes, cursors, active;  // routing plan
    size_t ctrl;                  // counters of the fused kernels
    size_t topk_w, topk_ids, logit;  // router outputs of the from-logits entry point
    // tensor-core prefill path (only when Tcap > kDecodeMaxT)
    size_t rowpos, slot_tiles, mtiles, n_mtiles;
    size_t agate, agate_sa, agate_sum;  // gate activation tiles [MT][8][32 KB] + per-row scale/sum
    size_t adown, adown_sa, adown_sum;  // down activation tiles [MT][2][32 KB]
    size_t bytes;
};

constexpr int kCtrlWords = 2048;
// ctrl word layout (uint32), zeroed before every fused launch
constexpr int kCtrlXDone = 0;          // token groups quantised
constexpr int kCtrlGateDone = 32;      // [E+1] gate items finished per expert slot
constexpr int kCtrlReady = 320;        // [E+1] middle of the expert slot quantised
constexpr int kCtrlColDone = 608;      // [64] down items finished per output tile
constexpr int kCtrlAbort = 700;        // any CTA gave up a bounded wait
// first bounded wait that gave up: [tag, cta, warp, x, y, observed], tag 1 = ring
// stage (x = stage, y = slot), 2 = producer slot reuse (x = stage, y = slot),
// 3 = global counter (x = ctrl word, y = target, observed = last value)
constexpr int kCtrlGiveUp = 704;
constexpr int kCtrlClearWords = 712;   // words zeroed before every fused launch

Workspace workspace_layout(int Tcap);

struct LayerArgs {
    const uint16_t* x;
    const float* weights;
    const int32_t* ids;
    const uint32_t* gate_codes;
    const uint32_t* gate_meta;
    const uint32_t* down_codes;
    const uint32_t* down_meta;
    const uint32_t* sgate_codes;  // shared expert (null when absent)
    const uint32_t* sgate_meta;
    const uint32_t* sdown_codes;
    const uint32_t* sdown_meta;
    const uint16_t* shared_logit;   // bf16 bits [T]
    const float* silu_table;        // [65536]
    const uint16_t* sigmoid_table;  // bf16 bits [65536]
    uint16_t* out;
    uint16_t* shared_out;
    uint32_t* flags;
    uint8_t* ws;
    Workspace L;
    int T;
    int a8;
    int shared;
    int shared_all_live;  // shared-slot semantics: every token row is live for the input transform
};

template <class T>
__host__ __device__ __forceinline__ T* ws_at(const LayerArgs& a, size_t off) {
    return reinterpret_cast<T*>(a.ws + off);
}

// Host-side count of kernels this library has enqueued (telemetry for benchmarks).
void count_launches(int n);

// Multi-kernel path, any T <= 8192.
cudaError_t launch_generic(const LayerArgs& a, cudaStream_t stream);
// Slot-ordered combine of route_out into out / shared_out (shared by the paths).
cudaError_t launch_combine(const LayerArgs& a, cudaStream_t stream);
// Tensor-core prefill path (T > kDecodeMaxT; needs a workspace laid out for Tcap > kDecodeMaxT).
cudaError_t launch_prefill(const LayerArgs& a, cudaStream_t stream);
// Fused persistent path for decode batches (T <= kDecodeMaxT).
constexpr int kDecodeMaxT = 32;
bool decode_supported(int T);
cudaError_t launch_decode(const LayerArgs& a, cudaStream_t stream);

}  // namespace ornith
