// Launch arguments, workspace layout and kernel entry points of the routed
// MoE layer.  Internal to the library (the public C ABI is include/ornith_moe_b200.h).
#pragma once
#include "moe_common.cuh"

namespace ornith {

// Workspace of one layer call, all offsets 256-byte aligned.  Rows of the
// intermediate buffers are "routes": r < R = 8T are routed slots (token r/8,
// slot r%8), r = R + t is the shared expert's row for token t.  On the
// tensor-core path (rows_by_position) the rows of middle and route_out are in
// slot-position order instead, so that one 128-route M-tile writes one
// contiguous block; rowpos[r] is then the row of route r.
struct Workspace {
    size_t xq, xs, xsum;          // token activations: int8 [T,2048] (permuted), fp16 [T,8], i32 [T,8]
    size_t middle;                // fp32 [R+T, 512] SiLU*up
    size_t mq, ms, msum;          // middle activations: int8 [R+T,512], fp16 [R+T,2], i32 [R+T,2]
    size_t route_out;             // fp32 [R+T, 2048] per-route down projections
    size_t final_f32;             // fp32 [T, 2048] combined sum before bf16 rounding (diagnostic)
    size_t counts, offsets, routes, cursors, active;  // routing plan
    size_t ctrl;                  // counters of the fused kernels
    size_t topk_w, topk_ids, logit;  // router outputs of the from-logits entry point
    size_t xchg;                  // single-token decode: middle rows as (call number, fp32) words [9][512] u64
    size_t xlogit;                // single-token decode from hidden: router logits as (call number, fp32) words [kD1LogitCopies][256]
    // tensor-core prefill path (only when Tcap > kDecodeMaxT)
    size_t rowpos, slot_tiles, mtiles, n_mtiles;
    size_t pblock;                // per-block expert counts, then bases, both [E+1][kPlanBlocks]
    size_t agate, agate_sa, agate_sum;  // gate activation tiles [MT][8][32 KB] + per-row scale/sum
    size_t adown, adown_sa, adown_sum;  // down activation tiles [MT][2][32 KB]
    size_t bytes;
};

constexpr int kCtrlWords = 2048;
// ctrl word layout (uint32), zeroed before every fused launch
constexpr int kCtrlXDone = 0;          // token groups quantised
constexpr int kCtrlLogitDone = 1;      // shared-expert logits written (fused routing)
constexpr int kCtrlRouteDone = 2;      // tokens routed (fused routing spread over CTAs)
constexpr int kMaxSlots = 320;         // expert slots of the fused decode plan (split slots included)
constexpr int kCtrlGateDone = 32;      // [kMaxSlots][2] gate-item counts per (slot, middle half)
constexpr int kCtrlReady = 672;        // [kMaxSlots] middle-quantisation counts per slot
constexpr int kCtrlColDone = 992;      // [64] down items finished per output tile
constexpr int kCtrlAbort = 1056;       // any CTA gave up a bounded wait
// first bounded wait that gave up: [tag, cta, warp, x, y, observed], tag 1 = ring
// stage (x = stage, y = slot), 2 = producer slot reuse (x = stage, y = slot),
// 3 = global counter (x = ctrl word, y = target, observed = last value)
constexpr int kCtrlGiveUp = 1060;
constexpr int kCtrlClearWords = 1072;  // words zeroed before every fused launch
// Words of the single-token decode kernel, never cleared: every launch tags
// its flags with a call number (epoch) read from kCtrlD1Epoch, so stale words
// of earlier calls never match the current one.  Beyond kCtrlClearWords so
// that the multi-token kernel's clear does not touch them.
constexpr int kCtrlD1Epoch = 1088;     // call number of the last completed launch
constexpr int kCtrlD1Seen = 1104;      // [kD1MaxCtas] a CTA read the epoch of this launch
// Copies of the single-token kernel's router-logit words: every CTA polls
// one of them, so that no line of the exchange is read by more than
// ceil(CTAs / copies) CTAs at once (polls of every CTA on one copy were
// found to serialise on its lines).
constexpr int kD1LogitCopies = 16;
constexpr int kD1MaxCtas = 256;
static_assert(kCtrlD1Seen + kD1MaxCtas <= kCtrlWords, "single-token decode words fit the control block");

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
    // fused routing (decode path of the from-logits entry): when `logits` is
    // set the kernel computes the top-8 ids/weights itself (ids/weights above
    // are then ignored) and stores them to ids_out/weights_out; when
    // `shared_gate_weight` is set it also computes the shared-expert logits
    // into logit_out, which is then what shared_logit points at.
    const float* logits;
    const uint16_t* shared_gate_weight;
    int32_t* ids_out;
    float* weights_out;
    uint16_t* logit_out;
    // router linear inside the single-token kernel (from-hidden entry, T = 1):
    // logits = x . router_weight^T, written to logits_out and routed from
    const uint16_t* router_weight;  // bf16 [256][2048]
    float* logits_out;              // fp32 [256]
    Workspace L;
    int T;
    int a8;
    int shared;
    int shared_all_live;  // shared-slot semantics: every token row is live for the input transform
};

// Router top-8 of one token by one warp (the role of vLLM's topk_softmax with
// renormalisation for this layer): the 8 largest finite logits, ties to the
// lower expert index, softmax over the 8 with the portable exp and a
// sequential sum.  Lanes 0..7 write ids[s] and weights[s]; a token with fewer
// than 8 finite logits gets id -1 / weight 0 in the remaining slots.
// Selection works on order-preserving integer keys (finite logits only, -0
// folded onto +0 so that equal logits have equal keys) with two warp
// reductions per round: the largest key, then the lowest index holding it.
__device__ __forceinline__ uint32_t logit_order_key(float v) {
    uint32_t b = __float_as_uint(v);
    if (b == 0x80000000u) b = 0u;
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float logit_from_key(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}
// The selection rounds stay a rolled loop: in a decode layer this code runs
// once per launch, where a short body that stays in the instruction cache
// beats an unrolled one.
__device__ __forceinline__ void route_topk_warp(const float* l, int lane, int32_t* ids, float* weights,
                                                uint32_t& flags) {
    uint32_t key[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float v = l[lane + 32 * i];
        const bool ok = isfinite(v);
        if (!ok) flags |= kFlagNonfiniteInput;
        key[i] = ok ? logit_order_key(v) : 0u;  // every finite key is >= 0x00800000
    }
    float my_v = 0.f;
    int my_i = -1;
#pragma unroll 1
    for (int s = 0; s < kTop; ++s) {
        const uint32_t lm = max(max(max(key[0], key[1]), max(key[2], key[3])), max(max(key[4], key[5]), max(key[6], key[7])));
        const uint32_t m = __reduce_max_sync(0xffffffffu, lm);
        uint32_t li = 0xffffffffu;
#pragma unroll
        for (int i = 7; i >= 0; --i)
            if (m != 0u && key[i] == m) li = uint32_t(lane + 32 * i);
        const uint32_t idx = __reduce_min_sync(0xffffffffu, li);
        if (m != 0u) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (uint32_t(lane + 32 * i) == idx) key[i] = 0u;
        }
        if (lane == s) {
            my_i = m != 0u ? int(idx) : -1;
            my_v = m != 0u ? logit_from_key(m) : 0.f;
        }
    }
    // slot s = lane (lanes 0..7): exp in parallel, the sum in slot order
    const float top = __shfl_sync(0xffffffffu, my_v, 0);
    const int top_i = __shfl_sync(0xffffffffu, my_i, 0);
    const float mx = top_i >= 0 ? top : 0.f;
    const float ex = (lane < kTop && my_i >= 0) ? portable_exp(__fsub_rn(my_v, mx)) : 0.f;
    // every lane gathers the eight terms first (independent shuffles), then
    // adds them in slot order
    float exs[kTop];
#pragma unroll
    for (int s = 0; s < kTop; ++s) exs[s] = __shfl_sync(0xffffffffu, ex, s);
    float sum = 0.f;
#pragma unroll
    for (int s = 0; s < kTop; ++s) sum = __fadd_rn(sum, exs[s]);
    if (lane < kTop) {
        ids[lane] = my_i;
        weights[lane] = my_i >= 0 ? __fdiv_rn(ex, sum) : 0.f;
    }
}

// Shared-expert gate logit of one token by one warp: fp32 products summed per
// lane in k order (k = lane + 32i), then an xor-tree across lanes, rounded to
// bf16.  Every lane returns the bf16 bits.
__device__ __forceinline__ uint16_t shared_logit_warp(const uint16_t* x, const uint16_t* w, int lane) {
    float acc = 0.f;
    for (int i = 0; i < kH / 32; ++i) {
        const int k = lane + 32 * i;
        acc = __fadd_rn(acc, __fmul_rn(bf16_to_f32(x[k]), bf16_to_f32(w[k])));
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, d));
    return bf16_rne(acc);
}

template <class T>
__host__ __device__ __forceinline__ T* ws_at(const LayerArgs& a, size_t off) {
    return reinterpret_cast<T*>(a.ws + off);
}

// Host-side count of kernels this library has enqueued (telemetry for benchmarks).
void count_launches(int n);

// Multi-kernel path, any T <= 8192.
cudaError_t launch_generic(const LayerArgs& a, cudaStream_t stream);
// Slot-ordered combine of route_out into out / shared_out (shared by the paths).
cudaError_t launch_combine(const LayerArgs& a, cudaStream_t stream, bool by_position = false);
// Hadamard + quantise every token group once into xq / xs / xsum.
cudaError_t launch_quant_tokens(const LayerArgs& a, cudaStream_t stream);
// True when a layer call of T tokens runs the tensor-core path, whose middle
// and route_out rows are in slot-position order (see Workspace).
bool rows_by_position(int T);
// Tensor-core prefill path (T > kDecodeMaxT; needs a workspace laid out for Tcap > kDecodeMaxT).
cudaError_t launch_prefill(const LayerArgs& a, cudaStream_t stream);
// Fused persistent path for decode batches (T <= kDecodeMaxT).
constexpr int kDecodeMaxT = 32;
constexpr int kPlanBlocks = 256;  // most blocks of the prefill routing plan
bool decode_supported(int T);
cudaError_t launch_decode(const LayerArgs& a, cudaStream_t stream);
// Single-token decode kernel (T == 1); returns cudaErrorNotSupported when
// this device or call does not fit it (the caller then runs launch_decode's
// multi-token kernel).
cudaError_t launch_decode_single(const LayerArgs& a, cudaStream_t stream);

}  // namespace ornith
