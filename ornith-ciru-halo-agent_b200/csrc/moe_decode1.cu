// Single-token routed-MoE decode layer (T == 1), sm_100a.
//
// Decode at batch 1 reads about 14.6 MB of packed weights per layer (eight
// routed experts and the shared expert, 1.62 MB each) and does almost no
// arithmetic, so the layer's time is the latency of a short chain of
// dependent steps plus the bytes.  This kernel keeps that chain to three
// steps: route, stream every weight byte of the layer into shared memory at
// once, and one hand-off between CTAs for the intermediate (middle) rows.
// The arithmetic is the reference's (kernels/routed_storage/
// routed_storage_n32_consumer.cpp:22-76 transform and quantisation, :124-161
// projection epilogue, :168-175 SiLU*up, :176-185 combine, :187-306 shared
// slot), operation for operation, as in the multi-token kernel.
//
// One cooperative launch of one CTA per SM (148 on B200), 19 warps:
//  * every CTA routes the token itself (top-8 of the logits, or the caller's
//    ids) and builds the same plan: slot 0 is the shared expert when present,
//    then the distinct routed experts in slot order (an expert named by
//    several slots is one plan slot whose routes share every value, since
//    they see the same token);
//  * gate item (slot k, tile pair p) -> CTA 16k + p: gate tile p and up tile
//    p + 16 over the 8 K-groups (66 KB, four bulk copies); warp 2g + r takes
//    K-group g of tile r; warp 0 sums the eight group terms in order, applies
//    SiLU*up and stores the slot's 32 middle columns as 64-bit words that
//    carry the call number beside the fp32 value;
//  * output tile t (32 columns) -> CTA G-1-t, for every slot (two bulk copies
//    per slot, up to 76 KB): warp 2k + g polls the 256 middle words of slot k,
//    K-group g until all carry this call's number (no separate flag, fence or
//    second read), transforms and quantises them and computes that K-group's
//    down term; the tile's per-slot rows and the slot-ordered combine follow
//    in the same CTA;
//  * the copy warp issues all of the CTA's weight blocks with cp.async.bulk
//    right after routing (the shared expert's, which need no routing, before
//    it).  No cluster multicast.
// Call numbers instead of clears: every CTA reads the last completed call's
// number from the workspace and uses the next one, and CTA 0 publishes it once
// every CTA has read it.  No separate clear launch is needed and words of
// earlier calls never match.
// Every wait is bounded (about one second of %globaltimer), after which the
// kernel raises flag 64, lets its issued copies land and returns.
#include <cstdlib>
#include <cstring>

#include "moe_layer.cuh"

namespace ornith {
namespace {

constexpr int kD1Slots = kTop + 1;          // eight routed experts and the shared expert
constexpr int kD1Compute = 2 * kD1Slots;    // compute warps: one per (slot, K-group) of the down tile
constexpr int kD1Copier = kD1Compute;       // the warp that issues the copies
constexpr int kD1Router = 16;               // routes the token (a compute warp idle until the down tile)
constexpr int kD1Combine = kTop + 1;        // the combine of a down tile (warps 0..8 store the per-route rows)
constexpr int kD1Warps = kD1Compute + 1;
constexpr int kD1Threads = kD1Warps * 32;
constexpr int kD1GateItems = kD1Slots * 16;
constexpr int kD1DownCtas = kH / 32;        // one per 32-column output tile
constexpr uint64_t kD1WaitNs = 1000000000ull;
static_assert(kD1Compute >= 16, "a warp per (K-group, tile) of a gate item");

struct __align__(128) D1Smem {
    uint8_t gate_codes[2][8][4096];         // gate item: [0] gate tile p, [1] up tile p + 16; K-group g
    uint32_t gate_meta[2][8][32];
    uint8_t down_codes[kD1Slots][2][4096];  // this CTA's output tile of every slot, K-groups 0 and 1
    uint32_t down_meta[kD1Slots][2][32];
    uint8_t xq[kH];                         // the token's activations, permuted int8
    uint16_t xraw[kH];                      // the token row as given (bf16)
    uint8_t mq[kD1Slots][2][kG];            // every slot's middle activations
    float terms[8][2][32];                  // gate item: group terms of gate and up
    float dterm[kD1Slots][2][32];           // down tile: group term of every slot and K-group
    uint64_t gbar[8];                       // gate item: K-group g of both tiles
    uint64_t gmbar;                         // gate item: metadata of both tiles
    uint64_t dbar[kD1Slots];
    __half xs[8];
    int32_t xsum[8];
    __half ms[kD1Slots][2];
    int32_t msum[kD1Slots][2];
    uint32_t xflag[8];
    int32_t ids[kTop];
    float wts[kTop];
    int32_t slot_of[kTop];                  // plan slot of each of the token's eight slots (-1: not routed)
    int32_t act_e[kD1Slots];                // expert of each plan slot (kE: the shared expert)
    int32_t nslot;
    uint32_t tag;                           // this launch's call number
    uint32_t issued;                        // bits 0..7: gate K-group barriers, 8: gate metadata, 9 + k: down slot k
    int32_t abort;
    float shared_gate;                      // sigmoid of the shared expert's logit (bf16 table value)
    float rlogits[kE];                      // router logits gathered from every CTA (from-hidden entry)
};

__device__ __forceinline__ uint64_t d1_now() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Optional phase timestamps (%globaltimer ns) per CTA, for latency analysis
// only: compiled in with -DORNITH_DECODE1_TRACE, absent from the default build.
#ifdef ORNITH_DECODE1_TRACE
constexpr int kD1TraceSlots = 20;
__device__ unsigned long long g_d1_trace[kD1MaxCtas][kD1TraceSlots];
#define D1_STAMP(i) (g_d1_trace[blockIdx.x][i] = d1_now())
#else
#define D1_STAMP(i) ((void)0)
#endif

__device__ __forceinline__ void d1_barrier() {
    asm volatile("bar.sync 1, %0;" ::"r"(kD1Compute * 32) : "memory");
}

// Programmatic dependent launch: let the next grid on the stream start
// launching; wait until the previous grid has completed and its memory
// operations are visible (a no-op when the launch did not ask for it).
__device__ __forceinline__ void d1_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void d1_wait_prior_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// The plan hand-off from the routing warp to the copy warp (named barrier 2).
__device__ __forceinline__ void d1_plan_sync() { asm volatile("bar.sync 2, 64;" ::: "memory"); }
__device__ __forceinline__ void d1_plan_arrive() { asm volatile("bar.arrive 2, 64;" ::: "memory"); }
// The call number from the copy warp to the router-logit warps and the
// routing warp (named barrier 4, from-hidden entry only).
constexpr int kD1TagThreads = 4 * 32;
__device__ __forceinline__ void d1_tag_sync() { asm volatile("bar.sync 4, %0;" ::"r"(kD1TagThreads) : "memory"); }
__device__ __forceinline__ void d1_tag_arrive() { asm volatile("bar.arrive 4, %0;" ::"r"(kD1TagThreads) : "memory"); }

// One router logit (gates_projection.py:17-25) by one warp, in the order of
// router_logits_kernel: lane l holds k = 256j + 8l .. 8l+7 for j = 0..7, FMA
// in j then element order, then an xor tree across lanes; every lane returns
// the sum.  The same bits as the separate router launch.
// The weight row is constant, so the caller loads it (router_row_load)
// before waiting for the previous grid; x may come from that grid.
__device__ __forceinline__ void router_row_load(const uint16_t* w_row, int lane, uint4 (&wr)[8]) {
#pragma unroll
    for (int j = 0; j < 8; ++j) wr[j] = __ldg(reinterpret_cast<const uint4*>(w_row + j * 256 + lane * 8));
}
__device__ __forceinline__ float router_logit_warp(const uint16_t* x, const uint4 (&wr)[8], int lane) {
    uint4 xr[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) xr[j] = *reinterpret_cast<const uint4*>(x + j * 256 + lane * 8);
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t xv[4] = {xr[j].x, xr[j].y, xr[j].z, xr[j].w}, wv[4] = {wr[j].x, wr[j].y, wr[j].z, wr[j].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            acc = __fmaf_rn(__uint_as_float(xv[i] << 16), __uint_as_float(wv[i] << 16), acc);
            acc = __fmaf_rn(__uint_as_float(xv[i] & 0xffff0000u), __uint_as_float(wv[i] & 0xffff0000u), acc);
        }
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, d));
    return acc;
}

// The gate item's end from warp 0 to the copy warp (named barrier 3).
__device__ __forceinline__ void d1_gate_done_sync() { asm volatile("bar.sync 3, 64;" ::: "memory"); }
__device__ __forceinline__ void d1_gate_done_arrive() { asm volatile("bar.arrive 3, 64;" ::: "memory"); }

// The shared expert's gate logit of the token: fp32 products summed per lane
// in k order (k = lane + 32i), then an xor tree across lanes, rounded to bf16
// (the order of shared_logit_warp), with the token row read from shared
// memory and the 64 weights of each lane loaded before the sum, so that the
// warp waits for one round trip to memory instead of one per step.
__device__ __forceinline__ uint16_t shared_logit_staged(const uint16_t* xs, const uint16_t* w, int lane) {
    uint16_t wv[kH / 32];
#pragma unroll
    for (int i = 0; i < kH / 32; ++i) wv[i] = w[lane + 32 * i];
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < kH / 32; ++i) acc = __fadd_rn(acc, __fmul_rn(bf16_to_f32(xs[lane + 32 * i]), bf16_to_f32(wv[i])));
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, d));
    return bf16_rne(acc);
}

__device__ __forceinline__ void d1_flag_or(uint32_t* flags, uint32_t f) {
    f = __reduce_or_sync(0xffffffffu, f);
    if (f && (threadIdx.x & 31) == 0) atomicOr(flags, f);
}

__device__ __forceinline__ void d1_give_up(D1Smem& S, uint32_t* flags) {
    atomicOr(flags, uint32_t(kFlagWaitTimeout));
    S.abort = 1;
}

// Bounded wait for the first phase of a copy barrier.
__device__ bool d1_wait_copies(uint64_t* bar, const volatile int32_t* abort) {
    if (mbar_try_wait(bar, 0)) return true;
    const uint64_t t0 = d1_now();
    while (!mbar_try_wait_suspend(bar, 0, 1000u)) {
        if (*abort || d1_now() - t0 > kD1WaitNs) return false;
    }
    return true;
}

// Relaxed (single-copy atomic per 64-bit element) accesses of the exchange words.
__device__ __forceinline__ void ld_relaxed_v2(const unsigned long long* p, unsigned long long& x,
                                              unsigned long long& y) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(x), "=l"(y) : "l"(p) : "memory");
}
__device__ __forceinline__ void st_relaxed_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// The copies of one CTA, one per lane.  Copy i: the gate item's four (gate
// and up tile codes, 32 KB each, and metadata, 1 KB each) when `gate_item`,
// then two per down slot k in [k0, k1) (8 KB of codes and 256 B of metadata
// of output tile `tile`).  mbarrier expect-tx is registered for every barrier
// (lane 0: the gate barrier, lane 1 + k: down slot k) before any copy starts.
__device__ __forceinline__ void issue_copies(const LayerArgs& a, D1Smem& S, int lane, bool gate_item, int ge, int gp,
                                             int k0, int k1, int tile) {
    // expect-tx first: lane 0 the gate metadata, lane 1 + g the gate item's
    // K-group g, lane 9 + k down slot k
    if (gate_item && lane == 0) mbar_arrive_expect_tx(&S.gmbar, 2 * 1024);
    if (gate_item && lane >= 1 && lane < 9) mbar_arrive_expect_tx(&S.gbar[lane - 1], 2 * 4096);
    if (lane >= 9 + k0 && lane < 9 + k1) mbar_arrive_expect_tx(&S.dbar[lane - 9], 8192 + 256);
    __syncwarp();
    int i = lane;
    if (gate_item) {
        // copy 0..1: metadata of the gate and up tiles (1 KB each, all
        // K-groups); copy 2 + 2g + r: K-group g of tile r (4 KB), one barrier
        // per K-group so that its two warps start as soon as it has landed
        if (i < 18) {
            const uint32_t* codes = ge == kE ? a.sgate_codes : a.gate_codes + size_t(ge) * (2 * kI) * (kH / 8);
            const uint32_t* meta = ge == kE ? a.sgate_meta : a.gate_meta + size_t(ge) * (2 * kI) * (kH / kG);
            if (i < 2) {
                bulk_g2s(S.gate_meta[i], meta + size_t(gp + 16 * i) * 8 * 32, 1024, &S.gmbar);
            } else {
                const int g = (i - 2) >> 1, r = (i - 2) & 1;
                bulk_g2s(S.gate_codes[r][g], codes + (size_t(gp + 16 * r) * 8 + g) * 1024, 4096, &S.gbar[g]);
            }
            return;
        }
        i -= 18;
    }
    const int k = k0 + (i >> 1);
    if (i < 0 || k >= k1) return;
    const int e = checked(S.act_e[k], kE + 1, a.flags);
    if ((i & 1) == 0) {
        const uint32_t* codes = e == kE ? a.sdown_codes : a.down_codes + size_t(e) * kH * (kI / 8);
        bulk_g2s(S.down_codes[k], codes + size_t(tile) * 2 * 1024, 8192, &S.dbar[k]);
    } else {
        const uint32_t* meta = e == kE ? a.sdown_meta : a.down_meta + size_t(e) * kH * (kI / kG);
        bulk_g2s(S.down_meta[k], meta + size_t(tile) * 2 * 32, 256, &S.dbar[k]);
    }
}

// Exact integer dot of one column (lane) of a 256-group block with one
// activation row: word j holds k = 8j..8j+7, its even and odd nibbles meet the
// permuted activation bytes in __dp4a.  Four independent chains; the integer
// sum is the same in any order.
__device__ __forceinline__ int block_dot(const uint32_t* blk, const uint4* act, int lane) {
    int c0 = 0, c1 = 0, c2 = 0, c3 = 0;
#pragma unroll 8
    for (int jj = 0; jj < 16; ++jj) {
        const uint4 av = act[jj];
        const uint32_t w0 = blk[(2 * jj) * 32 + lane], w1 = blk[(2 * jj + 1) * 32 + lane];
        c0 = __dp4a(int(w0 & 0x0f0f0f0fu), int(av.x), c0);
        c1 = __dp4a(int((w0 >> 4) & 0x0f0f0f0fu), int(av.y), c1);
        c2 = __dp4a(int(w1 & 0x0f0f0f0fu), int(av.z), c2);
        c3 = __dp4a(int((w1 >> 4) & 0x0f0f0f0fu), int(av.w), c3);
    }
    return (c0 + c1) + (c2 + c3);
}

// The down projection value of slot k for this lane's column: (0 + group-0
// term) + group-1 term, bf16-rounded for the shared expert.
__device__ __forceinline__ float down_value(const D1Smem& S, int k, int lane) {
    float v = __fadd_rn(__fadd_rn(0.f, S.dterm[k][0][lane]), S.dterm[k][1][lane]);
    return S.act_e[k] == kE ? bf16_round_f32(v) : v;
}

template <int QMAX>
__global__ void __launch_bounds__(kD1Threads, 1) decode_single_kernel(const LayerArgs a) {
    extern __shared__ __align__(128) uint8_t d1_raw[];
    D1Smem& S = *reinterpret_cast<D1Smem*>(d1_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int b = blockIdx.x, G = gridDim.x;
    uint32_t* ctrl = ws_at<uint32_t>(a, a.L.ctrl);
    unsigned long long* const xchg = ws_at<unsigned long long>(a, a.L.xchg);
    const bool is_down = b >= G - kD1DownCtas;
    const int tile = G - 1 - b;  // output tile of a down CTA
    uint32_t f = 0;
    // The next layer's launch may begin now: its CTAs take SMs as ours leave
    // them, and run only their prologue (barriers, the shared expert's weight
    // copies) until this grid has completed (programmatic dependent launch).
    d1_launch_dependents();

    if (warp == kD1Copier) {
        if (lane == 0) {
            D1_STAMP(0);
            for (int g = 0; g < 8; ++g) mbar_init(&S.gbar[g], 1);
            mbar_init(&S.gmbar, 1);
            for (int i = 0; i < kD1Slots; ++i) mbar_init(&S.dbar[i], 1);
            fence_barrier_init();
            if (a.shared) S.act_e[0] = kE;  // plan slot 0, before its copies are issued
            S.abort = 0;
        }
        __syncwarp();
        // the shared expert's blocks: constant weights, independent of routing
        // and of the previous grid, so issued before waiting for it
        if (a.shared) issue_copies(a, S, lane, b < 16, kE, b, 0, is_down ? 1 : 0, tile);
        d1_wait_prior_grid();  // everything below may read what the previous grid wrote
        uint32_t tag = 0;
        if (lane == 0) {
            tag = *reinterpret_cast<const volatile uint32_t*>(ctrl + kCtrlD1Epoch) + 1u;
            if (tag == 0u) tag = 1u;  // 0 never tags a call, so never-written words never match
            S.tag = tag;
            // seen: the stored value depends on the epoch read, so the read has
            // completed when any CTA observes it.  Relaxed rather than release:
            // a release here would also wait for this thread's bulk copies.
            st_relaxed_u32(ctrl + kCtrlD1Seen + b, tag);
        }
        __syncwarp();
        if (a.router_weight) d1_tag_arrive();  // the router-logit and routing warps need the call number
        d1_plan_sync();  // the routing warp's plan
        if (lane == 0) D1_STAMP(3);
        const int NA = S.nslot, base = a.shared ? 1 : 0, gk = b / 16;
        const bool has_gate = b < NA * 16;
        const bool routed_gate = has_gate && !(a.shared && gk == 0);
        // the routed gate item first; a CTA that also owns a down tile issues
        // its routed down blocks once the gate item has landed (below), so
        // that the gate bytes, needed first, are not slowed by them
        const bool down_now = is_down && !has_gate;
        issue_copies(a, S, lane, routed_gate, routed_gate ? S.act_e[gk] : 0, b % 16, base, down_now ? NA : base,
                     tile);
        if (lane == 0) {
            S.issued = (has_gate ? 0x1ffu : 0u) | (is_down ? 1u << 9 : 0u) * (a.shared ? 1u : 0u) |
                       (down_now ? ((1u << NA) - 1u) << 9 : 0u);
            D1_STAMP(4);
        }
    } else if (warp == kD1Router) {
        d1_wait_prior_grid();
        // router top-8 (from logits) or the caller's ids, then the plan
        uint32_t rf = 0;
        if (a.router_weight) {
            // the logits come from every CTA's router warps as call-numbered
            // words; a wait that runs out routes nothing (ids -1, flag 64)
            d1_tag_sync();
            const uint32_t tag = S.tag;
            // this CTA's copy of the words; a warp load covers 512 contiguous bytes
            const unsigned long long* src =
                ws_at<unsigned long long>(a, a.L.xlogit) + (b % kD1LogitCopies) * kE + 2 * lane;
            unsigned long long wv[8];
            const uint64_t t0 = d1_now();
            bool got = true;
            for (;;) {
#pragma unroll
                for (int i = 0; i < 4; ++i) ld_relaxed_v2(src + 64 * i, wv[2 * i], wv[2 * i + 1]);
                bool mine = true;
#pragma unroll
                for (int i = 0; i < 8; ++i) mine &= uint32_t(wv[i] >> 32) == tag;
                if (__all_sync(0xffffffffu, mine)) break;
                if (__shfl_sync(0xffffffffu, int(d1_now() - t0 > kD1WaitNs), 0)) {
                    got = false;
                    break;
                }
                __nanosleep(32);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i)
                S.rlogits[64 * (i / 2) + 2 * lane + i % 2] =
                    got ? __uint_as_float(uint32_t(wv[i])) : __uint_as_float(0x7fc00000u);
            if (!got && lane == 0) d1_give_up(S, a.flags);
            if (lane == 0) D1_STAMP(19);
            __syncwarp();
            route_topk_warp(S.rlogits, lane, S.ids, S.wts, rf);
        } else if (a.logits) {
            route_topk_warp(a.logits, lane, S.ids, S.wts, rf);
        } else if (lane < kTop) {
            S.ids[lane] = a.ids[lane];
            S.wts[lane] = a.weights[lane];
        }
        __syncwarp();
        if (lane == 0) D1_STAMP(2);
        const int e = lane < kTop ? S.ids[lane] : -1;
        const bool valid = lane < kTop && id_valid(e);
        if (lane < kTop && !valid && e != -1) rf |= kFlagInvalidId;
        if (b == 0 && a.logits && lane < kTop) {
            a.ids_out[lane] = e;
            a.weights_out[lane] = S.wts[lane];
        }
        const unsigned peers = __match_any_sync(0xffffffffu, valid ? e : -1 - lane);
        const int leader = __ffs(peers) - 1;
        const unsigned heads = __ballot_sync(0xffffffffu, valid && leader == lane);
        const int base = a.shared ? 1 : 0;
        const int slot = base + __popc(heads & ((1u << leader) - 1u));
        if (lane < kTop) S.slot_of[lane] = valid ? slot : -1;
        if (valid && leader == lane) S.act_e[slot] = e;
        if (lane == 0) S.nslot = base + __popc(heads);
        d1_plan_arrive();  // hands the plan to the copy warp
        if (lane == 0) D1_STAMP(1);
        if (b == 0) d1_flag_or(a.flags, rf);  // routing and id flags, once
    } else if (warp < 8) {
        d1_wait_prior_grid();
        // the token's 256-groups: warp g transforms and quantises group g
        const uint4 raw = *reinterpret_cast<const uint4*>(a.x + warp * kG + lane * 8);
        reinterpret_cast<uint4*>(S.xraw)[warp * 32 + lane] = raw;  // for the shared expert's logit
        uint32_t qf = wht_quant<QMAX>(
            __uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xffff0000u), __uint_as_float(raw.y << 16),
            __uint_as_float(raw.y & 0xffff0000u), __uint_as_float(raw.z << 16), __uint_as_float(raw.z & 0xffff0000u),
            __uint_as_float(raw.w << 16), __uint_as_float(raw.w & 0xffff0000u), lane,
            reinterpret_cast<uint2*>(S.xq + warp * kG), S.xs + warp, S.xsum + warp);
        qf = __reduce_or_sync(0xffffffffu, qf);
        if (lane == 0) S.xflag[warp] = qf;
        if (tid == 0) D1_STAMP(5);
    } else if (a.router_weight && (warp == 8 || warp == 9)) {
        // router logits of experts b and b + G (gates_projection.py:17-25):
        // into the caller's logits and, tagged with the call number, into the
        // exchange words every CTA's routing warp reads
        const int e = b + (warp - 8) * G;
        uint4 wr[8];
        if (e < kE) router_row_load(a.router_weight + size_t(e) * kH, lane, wr);
        d1_wait_prior_grid();
        if (lane == 0 && warp == 8) D1_STAMP(16);
        float v = 0.f;
        if (e < kE) v = router_logit_warp(a.x, wr, lane);
        if (lane == 0 && warp == 8) D1_STAMP(17);
        d1_tag_sync();
        if (e < kE && lane < kD1LogitCopies) {
            if (lane == 0) a.logits_out[e] = v;
            st_relaxed_u64(ws_at<unsigned long long>(a, a.L.xlogit) + lane * kE + e,
                           (static_cast<unsigned long long>(S.tag) << 32) | __float_as_uint(v));
        }
        if (lane == 0 && warp == 8) D1_STAMP(18);
    } else {
        d1_wait_prior_grid();
    }
    __syncthreads();

    const int NA = S.nslot;
    const uint32_t tag = S.tag;
    const bool has_gate = b < NA * 16;
    const int gk = b / 16, gp = b % 16;
    if (b == 0 && tid == 0) {
        // the token's input flags count when the token is live
        bool live = a.shared_all_live;
        for (int r = 0; r < kTop; ++r) live |= id_valid(S.ids[r]);
        uint32_t xf = 0;
        for (int g = 0; g < 8; ++g) xf |= S.xflag[g];
        if (live && xf) atomicOr(a.flags, xf);
    }

    if (warp == kD1Copier) {
        // a CTA with a gate item and a down tile: its routed down blocks once
        // the gate item is computed (barrier 3 from warp 0), so that neither
        // the gate bytes nor the gate arithmetic share the CTA's copy engine
        // and shared-memory port with them; they are needed only after the
        // middle rows of every CTA are in
        const int base = a.shared ? 1 : 0;
        if (is_down && has_gate && NA > base) {
            d1_gate_done_sync();
            if (!*reinterpret_cast<const volatile int32_t*>(&S.abort)) {
                issue_copies(a, S, lane, false, 0, 0, base, NA, tile);
                if (lane == 0) atomicOr(&S.issued, ((1u << NA) - 1u) << 9);
            }
        }
    } else if (NA == 0) {
        // every slot padded and no shared expert: the output is zero
        if (b == 0)
            for (int i = tid; i < kH; i += kD1Compute * 32) {
                a.out[i] = 0;
                ws_at<float>(a, a.L.final_f32)[i] = 0.f;
            }
    } else {
        // ---- gate item (slot gk, tile pair gp): warp 2g + r = K-group g of tile r
        if (has_gate) {
            if (warp < 16) {
                const int g = warp >> 1, r = warp & 1;
                if (d1_wait_copies(&S.gbar[g], &S.abort) && d1_wait_copies(&S.gmbar, &S.abort)) {
                    if (lane == 0 && warp == 0) D1_STAMP(6);
                    const uint32_t* blk = reinterpret_cast<const uint32_t*>(S.gate_codes[r][g]);
                    const int dot = block_dot(blk, reinterpret_cast<const uint4*>(S.xq + g * kG), lane);
                    S.terms[g][r][lane] = group_term(__half2float(S.xs[g]), dot, S.xsum[g], S.gate_meta[r][g][lane]);
                    if (lane == 0 && warp == 0) D1_STAMP(7);
                } else if (lane == 0) {
                    d1_give_up(S, a.flags);
                }
            }
            d1_barrier();
            if (tid == 0) D1_STAMP(8);
            if (warp == 0 && !*reinterpret_cast<const volatile int32_t*>(&S.abort)) {
                float gv = 0.f, uv = 0.f;
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    gv = __fadd_rn(gv, S.terms[k][0][lane]);
                    uv = __fadd_rn(uv, S.terms[k][1][lane]);
                }
                float value;
                if (S.act_e[gk] == kE) {
                    gv = bf16_round_f32(gv);
                    uv = bf16_round_f32(uv);
                    if (!isfinite(gv) || !isfinite(uv)) f |= kFlagNonfiniteProjection;
                    value = bf16_round_f32(__fmul_rn(a.silu_table[__float_as_uint(gv) >> 16], uv));
                } else {
                    if (!isfinite(gv) || !isfinite(uv)) f |= kFlagNonfiniteProjection;
                    value = silu_mul(gv, uv);
                }
                if (!isfinite(value)) f |= kFlagNonfiniteMiddle;
                // the slot's 32 middle columns, each word tagged with this call's number
                st_relaxed_u64(xchg + size_t(gk) * kI + gp * 32 + lane,
                               (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(value));
                if (lane == 0) D1_STAMP(9);
            }
            if (warp == 0 && is_down && NA > (a.shared ? 1 : 0)) d1_gate_done_arrive();  // the copy warp's down blocks
        }
        // ---- output tile: warp 2k + g = slot k, K-group g ----------------------
        if (is_down) {
            if (warp == kD1Combine && a.shared) {
                // the shared expert's output gate, sigmoid(logit) from the
                // caller's table, while the middle rows are still being made
                const uint16_t v = a.shared_gate_weight ? shared_logit_staged(S.xraw, a.shared_gate_weight, lane)
                                                        : a.shared_logit[0];
                if (a.shared_gate_weight && lane == 0 && tile == 0) a.logit_out[0] = v;
                const float gate = bf16_to_f32(a.sigmoid_table[v]);
                if (lane == 0) S.shared_gate = gate;
            }
            const int k = warp >> 1, g = warp & 1;
            bool ok = k < NA;
            if (ok) {
                // poll the 256 middle words of (k, g) until all carry this call's number
                const unsigned long long* src = xchg + size_t(k) * kI + g * kG + lane * 8;
                unsigned long long w[8];
                const uint64_t t0 = d1_now();
                for (;;) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) ld_relaxed_v2(src + 2 * i, w[2 * i], w[2 * i + 1]);
                    bool mine = true;
#pragma unroll
                    for (int i = 0; i < 8; ++i) mine &= uint32_t(w[i] >> 32) == tag;
                    if (__all_sync(0xffffffffu, mine)) break;
                    const int stop = __shfl_sync(
                        0xffffffffu, int(*reinterpret_cast<const volatile int32_t*>(&S.abort) != 0 ||
                                         d1_now() - t0 > kD1WaitNs), 0);
                    if (stop) {
                        if (lane == 0) d1_give_up(S, a.flags);
                        ok = false;
                        break;
                    }
                    __nanosleep(32);
                }
                if (ok) {
                    if (lane == 0 && warp == 0) D1_STAMP(10);
                    f |= wht_quant<QMAX>(__uint_as_float(uint32_t(w[0])), __uint_as_float(uint32_t(w[1])),
                                         __uint_as_float(uint32_t(w[2])), __uint_as_float(uint32_t(w[3])),
                                         __uint_as_float(uint32_t(w[4])), __uint_as_float(uint32_t(w[5])),
                                         __uint_as_float(uint32_t(w[6])), __uint_as_float(uint32_t(w[7])), lane,
                                         reinterpret_cast<uint2*>(S.mq[k][g]), &S.ms[k][g], &S.msum[k][g]);
                    __syncwarp();
                    if (lane == 0 && warp == 0) D1_STAMP(11);
                    if (d1_wait_copies(&S.dbar[k], &S.abort)) {
                        if (lane == 0 && warp == 0) D1_STAMP(12);
                        const uint32_t* blk = reinterpret_cast<const uint32_t*>(S.down_codes[k][g]);
                        const int dot = block_dot(blk, reinterpret_cast<const uint4*>(S.mq[k][g]), lane);
                        S.dterm[k][g][lane] =
                            group_term(__half2float(S.ms[k][g]), dot, S.msum[k][g], S.down_meta[k][g][lane]);
                        if (lane == 0 && warp == 0) D1_STAMP(13);
                    } else if (lane == 0) {
                        d1_give_up(S, a.flags);
                    }
                }
            }
            // the combine's per-slot plan into registers before the barrier, so
            // that after it only the down terms are read
            int cslot[kTop];
            float cwt[kTop];
            bool cround[kTop];
            if (warp == kD1Combine) {
#pragma unroll
                for (int sl = 0; sl < kTop; ++sl) {
                    cslot[sl] = id_valid(S.ids[sl]) ? S.slot_of[sl] : -1;
                    cwt[sl] = S.wts[sl];
                    cround[sl] = cslot[sl] >= 0 && S.act_e[cslot[sl]] == kE;
                }
            }
            d1_barrier();
            if (tid == 0) D1_STAMP(14);
            if (!*reinterpret_cast<const volatile int32_t*>(&S.abort)) {
                const int col = tile * 32 + lane;
                float* const route_out = ws_at<float>(a, a.L.route_out);
                if (warp < kTop) {
                    // per-route rows (route order), as the other paths leave them
                    const int kk = S.slot_of[warp];
                    if (kk >= 0) {
                        const float v = down_value(S, kk, lane);
                        if (!isfinite(v)) f |= kFlagNonfiniteProjection;
                        route_out[size_t(warp) * kH + col] = v;
                    }
                } else if (warp == kTop && a.shared) {
                    const float v = down_value(S, 0, lane);
                    if (!isfinite(v)) f |= kFlagNonfiniteProjection;
                    route_out[size_t(kTop) * kH + col] = v;
                } else if (warp == kD1Combine) {
                    // slot-ordered combine of the token (reduce_slots :176-185)
                    float dv[kTop];
#pragma unroll
                    for (int sl = 0; sl < kTop; ++sl) {
                        const int kk = cslot[sl] < 0 ? 0 : cslot[sl];
                        const float v = __fadd_rn(__fadd_rn(0.f, S.dterm[kk][0][lane]), S.dterm[kk][1][lane]);
                        dv[sl] = cround[sl] ? bf16_round_f32(v) : v;  // as down_value
                    }
                    float sum = 0.f;
#pragma unroll
                    for (int sl = 0; sl < kTop; ++sl)
                        if (cslot[sl] >= 0) sum = __fadd_rn(sum, __fmul_rn(dv[sl], cwt[sl]));
                    const uint16_t res = bf16_rne(sum);
                    ws_at<float>(a, a.L.final_f32)[col] = sum;
                    a.out[col] = res;
                    if (!isfinite(sum) || (res & 0x7f80u) == 0x7f80u) f |= kFlagNonfiniteOutput;
                    if (a.shared) {
                        const float sh = __fmul_rn(down_value(S, 0, lane), S.shared_gate);
                        a.shared_out[col] = bf16_rne(sh);
                        if (!isfinite(sh)) f |= kFlagNonfiniteOutput;
                    }
                    if (lane == 0) D1_STAMP(15);
                }
            }
        }
    }
    d1_flag_or(a.flags, f);

    if (b == 0 && warp == kD1Copier) {
        // CTA 0 publishes this call's number once every CTA has read the
        // previous one (bounded wait)
        const uint64_t t0 = d1_now();
        bool done = false;
        for (;;) {
            bool mine = true;
            for (int c = lane; c < G; c += 32) mine &= ld_acquire(ctrl + kCtrlD1Seen + c) == tag;
            done = __all_sync(0xffffffffu, mine);
            if (done || __shfl_sync(0xffffffffu, int(d1_now() - t0 > kD1WaitNs), 0)) break;
            __nanosleep(64);
        }
        if (lane == 0) {
            if (!done) atomicOr(a.flags, uint32_t(kFlagWaitTimeout));
            st_release(ctrl + kCtrlD1Epoch, tag);
        }
    }
    // ---- end: after an abort, let every issued copy land before the CTA exits
    __syncthreads();
    if (tid == 0 && S.abort) {
        const uint64_t t0 = d1_now();
        for (int i = 0; i < 9 + kD1Slots; ++i) {
            if (!(S.issued >> i & 1u)) continue;
            uint64_t* bar = i < 8 ? &S.gbar[i] : i == 8 ? &S.gmbar : &S.dbar[i - 9];
            while (!mbar_try_wait(bar, 0) && d1_now() - t0 < kD1WaitNs) {
            }
        }
    }
}

struct D1Device {
    int sms = 0;
    int max_smem = 0;
    bool attr_set[2] = {false, false};
    int pdl = -1;  // -1: not yet known whether the device takes the launch with programmatic serialization
};
D1Device g_d1[64];

// ORNITH_MOE_B200_DECODE1=0 sends single-token calls to the multi-token
// kernel instead (the tests compare the two).
bool single_disabled() {
    const char* v = getenv("ORNITH_MOE_B200_DECODE1");
    return v && strcmp(v, "0") == 0;
}
// ORNITH_MOE_B200_PDL=0 launches without programmatic dependent launch.
bool pdl_disabled() {
    const char* v = getenv("ORNITH_MOE_B200_PDL");
    return v && strcmp(v, "0") == 0;
}

}  // namespace

cudaError_t launch_decode_single(const LayerArgs& a, cudaStream_t stream) {
    if (a.T != 1 || single_disabled()) return cudaErrorNotSupported;
    int device = 0;
    cudaError_t st = cudaGetDevice(&device);
    if (st != cudaSuccess) return st;
    if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
    D1Device& d = g_d1[device];
    if (d.sms == 0) {
        if ((st = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess) return st;
        if ((st = cudaDeviceGetAttribute(&d.max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, device)) != cudaSuccess)
            return st;
    }
    const size_t smem = sizeof(D1Smem);
    // one CTA per gate item and per output tile, at most kD1MaxCtas seen-words
    if (d.sms < kD1GateItems || d.sms > kD1MaxCtas || size_t(d.max_smem) < smem) return cudaErrorNotSupported;
    if (a.router_weight && 2 * d.sms < kE) return cudaErrorNotSupported;  // two router logits per CTA at most
    const int which = a.a8 ? 0 : 1;
    auto kernel = a.a8 ? decode_single_kernel<127> : decode_single_kernel<7>;
    if (!d.attr_set[which]) {
        if ((st = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem))) != cudaSuccess)
            return st;
        d.attr_set[which] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(d.sms);
    cfg.blockDim = dim3(kD1Threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
    if ((st = cudaStreamIsCapturing(stream, &capturing)) != cudaSuccess) return st;
    // programmatic serialization where the device takes it together with the
    // cooperative launch; the first launch outside a stream capture finds out
    const bool try_pdl = !pdl_disabled() && (d.pdl == 1 || (d.pdl < 0 && capturing == cudaStreamCaptureStatusNone));
    cfg.numAttrs = try_pdl ? 2 : 1;
    count_launches(1);
    st = cudaLaunchKernelEx(&cfg, kernel, a);
    if (try_pdl && d.pdl < 0) {
        d.pdl = st == cudaSuccess ? 1 : 0;
        if (st != cudaSuccess) {
            (void)cudaGetLastError();  // the refused launch left no work behind: launch without it
            cfg.numAttrs = 1;
            st = cudaLaunchKernelEx(&cfg, kernel, a);
        }
    }
    return st;
}

#ifdef ORNITH_DECODE1_TRACE
// Copies the phase timestamps of the last single-token launch (256 x 20 u64)
// and clears them.
extern "C" __attribute__((visibility("default"))) int ornith_moe_b200_decode1_trace(void* dst) {
    cudaError_t st = cudaMemcpyFromSymbol(dst, g_d1_trace, sizeof(g_d1_trace));
    if (st != cudaSuccess) return int(st);
    static unsigned long long zeros[kD1MaxCtas][kD1TraceSlots];
    return int(cudaMemcpyToSymbol(g_d1_trace, zeros, sizeof(zeros)));
}
#endif

}  // namespace ornith
