// Fused persistent routed-MoE layer for decode batches (T <= 32), sm_100a.
//
// One cooperative launch per layer, one CTA per SM.  The arithmetic is the
// reference's (kernels/routed_storage/routed_storage_n32_consumer.cpp:319-351);
// the schedule is B200-specific:
//
//  * every CTA routes the batch itself in shared memory: top-8 ids and
//    weights from the router logits (from-logits entry) or the caller's ids,
//    expert slot counts, offsets and route lists (slot 256 = shared expert),
//    so no routing kernel or global scratch is needed;
//  * work items: gate item (expert slot, tile pair p) = gate tile p + up tile
//    p+16 over the 8 K-groups (66 KB of packed weights); down item (slot,
//    tile t) over the 2 K-groups (8.4 KB).  Items are dealt round-robin over
//    CTAs, gate items first;
//  * a producer warp streams each item's 4 KB (tile, group) weight blocks and
//    128 B metadata into a ring of shared-memory stages with cp.async.bulk
//    (no cluster multicast), gate stages before down stages, so HBM streaming
//    never waits on the compute dependencies below;
//  * the eight consumer warps work one item at a time together.  Gate item:
//    warp w takes K-group w of the gate tile and of the up tile (exact __dp4a
//    integer dots, lane = output column, the fixed fp32 group term), the
//    terms meet in shared memory and, after a CTA barrier, warp w sums the
//    eight group terms of route w in ascending group order and writes
//    SiLU(gate)*up.  The CTA that completes the eighth gate item of an
//    (expert slot, middle half) quantises those middle rows with all eight
//    warps and counts them ready;
//  * down items go four at a time: warp pair q takes item q, one K-group per
//    warp, after a bounded wait for its expert's ready count; the pair sums
//    the two group terms in order and writes the fp32 per-route row.  The
//    warp that finishes the last expert of an output tile performs the
//    slot-ordered combine of that tile.
// Every wait is bounded (about one second of %globaltimer), after which the
// kernel raises flag 64, lets in-flight copies land and returns.
#include "moe_layer.cuh"

namespace ornith {
namespace {

constexpr int kNCW = 8;                       // consumer (dot) warps
constexpr int kEW = 2;                        // epilogue warps (throughput mode)
constexpr int kProd = kNCW + kEW;             // producer warp
constexpr int kWarps = kProd + 1;
constexpr int kThreads = kWarps * 32;
constexpr int kTChunk = 4;                    // routes per throughput-mode gate unit
constexpr int kStageBytes = 4096 + 128;       // one (tile, group) block: codes + metadata
constexpr int kChunk = 8;                     // routes per dot pass
constexpr uint64_t kTimeoutNs = 1000000000ull;
constexpr int kRedundantX = 4;                // T <= 4: every CTA quantises all tokens itself
constexpr uint32_t kGateTarget = 8 * kNCW;    // GateDone[slot][half]: 8 gate items x 8 warps
constexpr uint32_t kReadyTarget = 2 * kNCW;   // Ready[slot]: 2 halves x 8 warps
constexpr int kMaxTasks = 64;                 // middle-quantisation tasks per CTA (one per gate item at most)
// named barriers: 1 = the 8 consumer warps, 2..5 = down pairs, 6/7 = gate
// terms ready in buffer 0/1, 8/9 = buffer 0/1 free again, 10 = consumers and
// epilogue warps, 11 = the two epilogue warps
constexpr int kBarConsumers = 1;
constexpr int kBarTermsReady = 6, kBarTermsFree = 8, kBarDotE = 10, kBarE = 11;
constexpr int kDotEThreads = (kNCW + kEW) * 32;
constexpr int kMinStages = 18;                // ring stages needed: one gate item plus slack
constexpr int kTiles = kH / 32;               // 32-column output tiles of a down projection
// Expert slots with at most this many routes skip the ready handoff: each
// down warp quantises its K-group of the slot's middle rows itself as soon as
// that half's gate items are counted.  Heavier slots (the shared expert and
// hot experts of larger batches) are quantised once by the CTA that completes
// them and released through the ready count.
constexpr int kSelfQuantMax = 4;
constexpr int kSplit = 8;   // routes per slot in the throughput plan (heavier experts are split)
__host__ __device__ inline bool light_slot(int T, int nr) { return T <= 4 && nr <= kSelfQuantMax; }

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Optional phase timestamps (%globaltimer ns) per CTA for latency analysis.
// Compiled in only with -DORNITH_DECODE_TRACE; the default build has none.
#ifdef ORNITH_DECODE_TRACE
constexpr int kTraceCtas = 256, kTraceSlots = 32;
__device__ unsigned long long g_decode_trace[kTraceCtas][kTraceSlots];
#define DECODE_TRACE(i) (g_decode_trace[blockIdx.x][i] = clock64())
#define DECODE_TRACE0(i) (threadIdx.x == 0 ? void(g_decode_trace[blockIdx.x][i] = clock64()) : void(0))
#define DECODE_CLOCK(i) (g_decode_trace[blockIdx.x][i] = now_ns())
#define DECODE_VALUE(i, v) (g_decode_trace[blockIdx.x][i] = (unsigned long long)(v))
#else
#define DECODE_VALUE(i, v) ((void)0)
#define DECODE_TRACE(i) ((void)0)
#define DECODE_TRACE0(i) ((void)0)
#define DECODE_CLOCK(i) ((void)0)
#endif

__device__ __forceinline__ void named_barrier(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void named_barrier_arrive(int id, int threads) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

struct Smem {
    uint8_t* ring;
    uint64_t* full;
    uint64_t* empty;
    int* last_st;     // [nst] last stage issued into each ring slot (-1: none)
    uint8_t* xq;      // [T][2048] permuted int8
    __half* xs;       // [T][8]
    int* xsum;        // [T][8]
    int* ids;         // [R]
    float* wts;       // [R]
    int* cnt;         // [E+1] counts, then placement cursors (plan only, inside tbuf)
    int* off;         // [E+1] (plan only, inside tbuf)
    int* act_e;       // [kMaxSlots] expert of active slot k (kE: shared expert)
    int* act_off;     // [kMaxSlots] first position of the slot's routes
    int* act_cnt;     // [kMaxSlots] routes of the slot
    int* routes;      // [R+T]
    float* tbuf;      // gate: [kNCW][2][kChunk][32] group terms; down: [kNCW][kChunk][256 B] activations
    float* pbuf;      // [kNCW/2][kChunk][32] second-group terms of the down pairs
    __half* dscale;   // [kNCW][kChunk]
    int* dsum;        // [kNCW][kChunk]
    int* tasks;       // [kMaxTasks] posted middle-quantisation tasks (2*slot + half)
    uint32_t* xflag;  // [8 kRedundantX] flags of each token group quantised during routing (plan only, inside tbuf)
    int* wpre;        // [2][kMaxSlots+2] cost prefixes of the slots' gate items and down items (plan only, inside tbuf)
    int* misc;        // [0] abort, [1] final issued count, [2] nact, [3] NA, [4] issued so far, [5] tasks posted,
                      // [6..9] this CTA's gate and down item ranges (throughput mode)
};
// Route number at plan position i; debug builds check the position and the
// route against the plan's 9T rows (8T routes, then T shared-slot rows).
__device__ __forceinline__ int route_at(const LayerArgs& a, const Smem& s, int i) {
    const int rows = a.T * (kTop + 1);
    return checked(s.routes[checked(i, rows, a.flags)], rows, a.flags);
}


__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
static_assert((2 * (kE + 4) + 2 * (kMaxSlots + 2)) * 4 + 8 * kRedundantX * 4 <= kNCW * 2 * kChunk * 32 * 4,
              "plan-only arrays must fit inside tbuf");

// Byte offsets of the shared-memory carve for T tokens and nst ring stages.
struct Carve {
    size_t ring, full, empty, last_st, xq, xs, xsum, ids, wts, act_e, act_off, act_cnt, routes, tbuf, pbuf, dscale,
        dsum, tasks, misc, total;
};
__host__ __device__ inline Carve carve(int T, int nst) {
    Carve c{};
    size_t cur = 0;
    auto add = [&](size_t& f, size_t bytes, size_t al) {
        cur = align_up(cur, al);
        f = cur;
        cur += bytes;
    };
    const size_t R = size_t(T) * kTop;
    add(c.ring, size_t(nst) * kStageBytes, 128);
    add(c.full, size_t(nst) * 8, 8);
    add(c.empty, size_t(nst) * 8, 8);
    add(c.last_st, size_t(nst) * 4, 4);
    add(c.xq, size_t(T) * kH, 16);
    add(c.xs, size_t(T) * 8 * 2, 16);
    add(c.xsum, size_t(T) * 8 * 4, 16);
    add(c.ids, R * 4 + 4, 16);
    add(c.wts, R * 4 + 4, 16);
    add(c.act_e, kMaxSlots * 4, 16);
    add(c.act_off, kMaxSlots * 4, 16);
    add(c.act_cnt, kMaxSlots * 4, 16);
    add(c.routes, (R + T) * 4 + 4, 16);
    add(c.tbuf, size_t(kNCW) * 2 * kChunk * 32 * 4, 16);
    add(c.pbuf, size_t(kNCW / 2) * kChunk * 32 * 4, 16);
    add(c.dscale, size_t(kNCW) * kChunk * 2, 16);
    add(c.dsum, size_t(kNCW) * kChunk * 4, 16);
    add(c.tasks, kMaxTasks * 4, 16);
    add(c.misc, 16 * 4, 16);
    c.total = align_up(cur, 128);
    return c;
}

__device__ __forceinline__ void warp_flag_or(uint32_t* flags, uint32_t f) {
    f = __reduce_or_sync(0xffffffffu, f);
    if (f && (threadIdx.x & 31) == 0) atomicOr(flags, f);
}

// The bounded waits and the give-up path are out of line: they are called
// from many places, and in a decode layer the kernel's code size, not its
// instruction count, sets how long each phase takes to start.

// Raise the abort state (CTA-local and global) and flag 64; the first CTA to
// give up records where (kCtrlGiveUp) for the caller's diagnosis.
__device__ __noinline__ void give_up(uint32_t* flags, int* misc, uint32_t* ctrl, uint32_t tag, uint32_t x, uint32_t y,
                                     uint32_t observed) {
    atomicOr(flags, kFlagWaitTimeout);
    atomicExch(&misc[0], 1);
    if (atomicCAS(ctrl + kCtrlGiveUp, 0u, tag) == 0u) {
        ctrl[kCtrlGiveUp + 1] = blockIdx.x;
        ctrl[kCtrlGiveUp + 2] = threadIdx.x >> 5;
        ctrl[kCtrlGiveUp + 3] = x;
        ctrl[kCtrlGiveUp + 4] = y;
        ctrl[kCtrlGiveUp + 5] = observed;
    }
    atomicExch(ctrl + kCtrlAbort, 1u);
}

// Bounded wait for ring stage `st` to be filled.  Returns false when the
// stage was never issued because the CTA is aborting.
// A slot's barrier parity cannot tell phases two apart, so the warp first
// waits until the producer has published that stage st was issued
// (misc[4] > st); from then on the slot's barrier is at most one phase behind
// and the parity is exact.
__device__ __noinline__ bool wait_stage(uint32_t* flags, int* misc_p, uint64_t* full, uint32_t* ctrl, int st, int nst) {
    const int slot = st % nst;
    const uint32_t parity = uint32_t(st / nst) & 1u;
    volatile int* misc = misc_p;
    uint64_t t0 = 0;
    for (int i = 0;; ++i) {
        if (misc[4] > st && mbar_try_wait(&full[slot], parity)) return true;
        if (misc[0] && st >= misc[1]) return false;
        if (i == 0) t0 = now_ns();
        else if ((i & 63) == 0 && now_ns() - t0 > kTimeoutNs) {
            give_up(flags, misc_p, ctrl, 1u, uint32_t(st), uint32_t(slot), uint32_t(misc[4]));
            // the copy, if it was issued, still lands: wait for it (bounded) before leaving
            if (st < misc[4]) {
                uint64_t t1 = now_ns();
                while (!mbar_try_wait(&full[slot], parity) && now_ns() - t1 < kTimeoutNs) {
                }
            }
            return false;
        }
    }
}

// Bounded wait on a global counter reaching `target` (lane 0 of the warp
// polls; the whole warp calls).
__device__ __noinline__ bool wait_counter(uint32_t* flags, int* misc_p, uint32_t* ctrl, const uint32_t* p,
                                          uint32_t target) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) {
        uint64_t t0 = 0;
        for (int i = 0; ld_acquire(p) < target; ++i) {
            volatile int* misc = misc_p;
            if (misc[0] || ld_acquire(ctrl + kCtrlAbort)) {
                // another CTA gave up: stop issuing here too (the exit drain then runs)
                atomicExch(&misc_p[0], 1);
                ok = 0;
                break;
            }
            if (i == 0) t0 = now_ns();
            else if (now_ns() - t0 > kTimeoutNs) {
                give_up(flags, misc_p, ctrl, 3u, uint32_t(p - ctrl), target, ld_acquire(p));
                ok = 0;
                break;
            }
            if (i > 8) __nanosleep(32);
        }
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    __syncwarp();  // the warp's later reads are ordered after lane 0's acquire
    return ok != 0;
}

__device__ __forceinline__ int token_of(int route, int R) { return route >= R ? route - R : route / kTop; }

// Exact integer dots of a gate stage and an up stage (same K-group) for NRC
// routes; lane = output column.  Word j of a stage holds this column's codes
// for k = 8j..8j+7; the even and odd nibbles meet the permuted activation
// bytes (act[i] = 16 bytes per two words) in __dp4a.  The chains are split by
// nibble parity (and by word parity for one or two routes) for
// instruction-level parallelism; the integer sums are the same in any order.
template <int NRC>
__device__ __forceinline__ void stage_dots2(const uint32_t* __restrict__ bg, const uint32_t* __restrict__ bu,
                                            const uint4* const (&act)[kChunk], int lane, int (&dg)[kChunk],
                                            int (&du)[kChunk]) {
    constexpr int P = NRC <= 2 ? 2 : 1;
    int gl[NRC][P], gh[NRC][P], ul[NRC][P], uh[NRC][P];
#pragma unroll
    for (int i = 0; i < NRC; ++i)
#pragma unroll
        for (int q = 0; q < P; ++q) gl[i][q] = gh[i][q] = ul[i][q] = uh[i][q] = 0;
#pragma unroll 4
    for (int jj = 0; jj < 16; ++jj) {
        const uint32_t g0 = bg[(2 * jj) * 32 + lane], g1 = bg[(2 * jj + 1) * 32 + lane];
        const uint32_t u0 = bu[(2 * jj) * 32 + lane], u1 = bu[(2 * jj + 1) * 32 + lane];
        const int g0l = int(g0 & 0x0f0f0f0fu), g0h = int((g0 >> 4) & 0x0f0f0f0fu);
        const int g1l = int(g1 & 0x0f0f0f0fu), g1h = int((g1 >> 4) & 0x0f0f0f0fu);
        const int u0l = int(u0 & 0x0f0f0f0fu), u0h = int((u0 >> 4) & 0x0f0f0f0fu);
        const int u1l = int(u1 & 0x0f0f0f0fu), u1h = int((u1 >> 4) & 0x0f0f0f0fu);
#pragma unroll
        for (int i = 0; i < NRC; ++i) {
            const uint4 av = act[i][jj];
            gl[i][0] = __dp4a(g0l, int(av.x), gl[i][0]);
            gh[i][0] = __dp4a(g0h, int(av.y), gh[i][0]);
            ul[i][0] = __dp4a(u0l, int(av.x), ul[i][0]);
            uh[i][0] = __dp4a(u0h, int(av.y), uh[i][0]);
            gl[i][P - 1] = __dp4a(g1l, int(av.z), gl[i][P - 1]);
            gh[i][P - 1] = __dp4a(g1h, int(av.w), gh[i][P - 1]);
            ul[i][P - 1] = __dp4a(u1l, int(av.z), ul[i][P - 1]);
            uh[i][P - 1] = __dp4a(u1h, int(av.w), uh[i][P - 1]);
        }
    }
#pragma unroll
    for (int i = 0; i < NRC; ++i) {
        int sg = 0, su = 0;
#pragma unroll
        for (int q = 0; q < P; ++q) {
            sg += gl[i][q] + gh[i][q];
            su += ul[i][q] + uh[i][q];
        }
        dg[i] = sg;
        du[i] = su;
    }
}
// n routes (1..8): act[i] for i >= n repeats a valid row and its dot is unused.
__device__ __forceinline__ void stage_dots2_n(int n, const uint32_t* bg, const uint32_t* bu,
                                              const uint4* const (&act)[kChunk], int lane, int (&dg)[kChunk],
                                              int (&du)[kChunk]) {
    if (n == 1) stage_dots2<1>(bg, bu, act, lane, dg, du);
    else if (n == 2) stage_dots2<2>(bg, bu, act, lane, dg, du);
    else if (n <= 4) stage_dots2<4>(bg, bu, act, lane, dg, du);
    else stage_dots2<8>(bg, bu, act, lane, dg, du);
}

// The same for one stage (down projection).
template <int NRC>
__device__ __forceinline__ void stage_dots1(const uint32_t* __restrict__ blk, const uint4* const (&act)[kChunk],
                                            int lane, int (&dot)[kChunk]) {
    constexpr int P = NRC <= 2 ? 2 : 1;
    int dl[NRC][P], dh[NRC][P];
#pragma unroll
    for (int i = 0; i < NRC; ++i)
#pragma unroll
        for (int q = 0; q < P; ++q) dl[i][q] = dh[i][q] = 0;
#pragma unroll 4
    for (int jj = 0; jj < 16; ++jj) {
        const uint32_t w0 = blk[(2 * jj) * 32 + lane], w1 = blk[(2 * jj + 1) * 32 + lane];
        const int w0l = int(w0 & 0x0f0f0f0fu), w0h = int((w0 >> 4) & 0x0f0f0f0fu);
        const int w1l = int(w1 & 0x0f0f0f0fu), w1h = int((w1 >> 4) & 0x0f0f0f0fu);
#pragma unroll
        for (int i = 0; i < NRC; ++i) {
            const uint4 av = act[i][jj];
            dl[i][0] = __dp4a(w0l, int(av.x), dl[i][0]);
            dh[i][0] = __dp4a(w0h, int(av.y), dh[i][0]);
            dl[i][P - 1] = __dp4a(w1l, int(av.z), dl[i][P - 1]);
            dh[i][P - 1] = __dp4a(w1h, int(av.w), dh[i][P - 1]);
        }
    }
#pragma unroll
    for (int i = 0; i < NRC; ++i) {
        int sd = 0;
#pragma unroll
        for (int q = 0; q < P; ++q) sd += dl[i][q] + dh[i][q];
        dot[i] = sd;
    }
}
__device__ __forceinline__ void stage_dots1_n(int n, const uint32_t* blk, const uint4* const (&act)[kChunk], int lane,
                                              int (&dot)[kChunk]) {
    if (n == 1) stage_dots1<1>(blk, act, lane, dot);
    else if (n == 2) stage_dots1<2>(blk, act, lane, dot);
    else if (n <= 4) stage_dots1<4>(blk, act, lane, dot);
    else stage_dots1<8>(blk, act, lane, dot);
}

// Transform + quantise one 256-group of one token (a dead token's group is
// all zeros and reports no flags).
template <int QMAX>
__device__ __forceinline__ void quant_token_group(const LayerArgs& a, const int* ids, int t, int g, int lane, uint2* q,
                                                  __half* scale, int32_t* sum, uint32_t& f, bool report) {
    bool live = a.shared_all_live;
    if (!live)
        for (int sl = 0; sl < kTop; ++sl) live |= id_valid(ids[t * kTop + sl]);
    uint4 raw = make_uint4(0u, 0u, 0u, 0u);
    if (live) raw = *reinterpret_cast<const uint4*>(a.x + size_t(t) * kH + g * kG + lane * 8);
    const uint32_t qf =
        wht_quant<QMAX>(__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xffff0000u), __uint_as_float(raw.y << 16),
                        __uint_as_float(raw.y & 0xffff0000u), __uint_as_float(raw.z << 16),
                        __uint_as_float(raw.z & 0xffff0000u), __uint_as_float(raw.w << 16),
                        __uint_as_float(raw.w & 0xffff0000u), lane, q, scale, sum);
    if (live && report) f |= qf;
}

// One 256-group of one middle row (fp32 in the workspace, written by other
// CTAs: read through L2), lane l holding elements 8l..8l+7.
__device__ __forceinline__ void load_middle(const LayerArgs& a, int route, int g, int lane, float4& v0, float4& v1) {
    const float* src = ws_at<float>(a, a.L.middle) + size_t(route) * kI + g * kG + lane * 8;
    v0 = ldcg4(src);
    v1 = ldcg4(src + 4);
}
template <int QMAX>
__device__ __forceinline__ uint32_t quant_middle(const float4& v0, const float4& v1, int lane, uint2* q, __half* scale,
                                                 int32_t* sum) {
    return wht_quant<QMAX>(v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w, lane, q, scale, sum);
}

// Hadamard + quantise one 256-group of one middle row into the workspace's
// middle activations.
template <int QMAX>
__device__ __forceinline__ void quant_middle_group(const LayerArgs& a, int route, int g, int lane, uint32_t& f) {
    float4 v0, v1;
    load_middle(a, route, g, lane, v0, v1);
    f |= quant_middle<QMAX>(v0, v1, lane, ws_at<uint2>(a, a.L.mq) + (size_t(route) * kI + g * kG) / 8,
                            ws_at<__half>(a, a.L.ms) + route * 2 + g, ws_at<int32_t>(a, a.L.msum) + route * 2 + g);
}

// Throughput mode (T > 4): gate items (16 per slot) and down items (64 per
// slot) are dealt to CTAs in contiguous, cost-balanced ranges of the
// slot-major item order, so that a CTA mostly owns whole (slot, middle half)
// groups and long runs of one slot's down tiles.  Relative cost of an item of
// a slot with nr routes: a gate item streams 66 KB and runs 2 x 16 x 8 dp4a
// per route and lane, a down item streams 8 KB with a fixed per-tile overhead.
// The fixed parts are build-time settings (-DORNITH_DECODE_GATE_COST=…,
// -DORNITH_DECODE_DOWN_COST=…) so that variant builds can measure other
// balances between weight bytes and per-route work; the default is 3 and 4.
#ifndef ORNITH_DECODE_GATE_COST
#define ORNITH_DECODE_GATE_COST 3
#endif
#ifndef ORNITH_DECODE_DOWN_COST
#define ORNITH_DECODE_DOWN_COST 4
#endif
static_assert(ORNITH_DECODE_GATE_COST >= 1 && ORNITH_DECODE_DOWN_COST >= 1, "item costs are positive");
__host__ __device__ inline int gate_cost(int nr) { return ORNITH_DECODE_GATE_COST + nr; }
__host__ __device__ inline int down_cost(int nr) { return ORNITH_DECODE_DOWN_COST + nr; }
// First item (slot-major index, per_slot items per slot) whose cost prefix is
// at least `target`; W[k] = cost of all items of slots < k, W[NA] = total.
__device__ __forceinline__ int first_item(const int* W, int NA, int per_slot, int target) {
    int lo = 0, hi = NA;  // largest k with W[k] <= target
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (W[mid] <= target) lo = mid;
        else hi = mid - 1;
    }
    if (lo >= NA) return NA * per_slot;
    const int wk = (W[lo + 1] - W[lo]) / per_slot;
    const int pidx = (target - W[lo] + wk - 1) / wk;
    return pidx >= per_slot ? (lo + 1) * per_slot : lo * per_slot + pidx;
}
__device__ __forceinline__ int range_start(const int* W, int NA, int per_slot, int b, int G) {
    const long long total = W[NA];
    return first_item(W, NA, per_slot, int((total * b + G - 1) / G));
}

// ---- throughput-mode pieces shared by the consumer and epilogue warps ----

constexpr uint32_t kGateTargetThr = 8;   // split (slot, half): one count per gate item
constexpr uint32_t kReadyTargetThr = 2;  // one count per quantised half
constexpr int kHeavyTask = 8;            // halves with more routes are quantised by all warps after the items
// gate terms of unit buffer `buf`, K-group g, role (0 gate, 1 up), route i of the unit
__device__ __forceinline__ int term_index(int buf, int g, int role, int i, int lane) {
    return (((buf * 8 + g) * 2 + role) * kTChunk + i) * 32 + lane;
}

// Quantisation of (slot, half) groups that are too heavy for the epilogue
// warps: after the gate items, by the consumer and epilogue warps together
// (warp index cw over kNCW + kEW warps), one ready count per half.
template <int QMAX>
__device__ __forceinline__ void deferred_quant_tasks(const LayerArgs& a, Smem& s, uint32_t* ctrl, int cw, int lane,
                                                     uint32_t& f) {
    const int nt = min(*static_cast<volatile int*>(&s.misc[5]), kMaxTasks);
    for (int t = 0; t < nt; ++t) {
        const int task = s.tasks[t], kk = task >> 1, hh = task & 1;
        const int nr2 = s.act_cnt[kk], roff2 = s.act_off[kk];
        for (int q = cw; q < nr2; q += kNCW + kEW) quant_middle_group<QMAX>(a, route_at(a, s, roff2 + q), hh, lane, f);
        named_barrier(kBarDotE, kDotEThreads);
        if (cw == 0 && lane == 0) red_release_add(ctrl + kCtrlReady + kk, 1u);
    }
}

// Slot-ordered combine (reduce_slots :176-185) of (tile, token) units
// cw + b*(kNCW+kEW), + G*(kNCW+kEW), ... once the tile's NA down items are counted.
__device__ __forceinline__ void combine_units(const LayerArgs& a, Smem& s, uint32_t* ctrl, int T, int R, int G, int b,
                                              int cw, int lane, int NA, uint32_t& f) {
    const float* route_out = ws_at<float>(a, a.L.route_out);
    const uint16_t* logit = a.shared_gate_weight ? a.logit_out : a.shared_logit;
    bool logit_ok = !(a.shared && a.shared_gate_weight);
    const volatile int* misc = s.misc;
    for (int u = b * (kNCW + kEW) + cw; u < T * kTiles; u += G * (kNCW + kEW)) {
        const int tile = u / T, t = u % T;
        if (misc[0]) break;
        if (!wait_counter(a.flags, s.misc, ctrl, ctrl + kCtrlColDone + tile, uint32_t(NA))) break;
        if (!logit_ok) {
            if (!wait_counter(a.flags, s.misc, ctrl, ctrl + kCtrlLogitDone, uint32_t(T))) break;
            logit_ok = true;
        }
        const int col = tile * 32 + lane;
        float sum = 0.f;
#pragma unroll
        for (int sl = 0; sl < kTop; ++sl) {
            const int r = t * kTop + sl;
            if (id_valid(s.ids[r])) sum = __fadd_rn(sum, __fmul_rn(__ldcg(route_out + size_t(r) * kH + col), s.wts[r]));
        }
        const uint16_t res = bf16_rne(sum);
        ws_at<float>(a, a.L.final_f32)[size_t(t) * kH + col] = sum;
        a.out[size_t(t) * kH + col] = res;
        if (!isfinite(sum) || (res & 0x7f80u) == 0x7f80u) f |= kFlagNonfiniteOutput;
        if (a.shared) {
            const float gate = bf16_to_f32(a.sigmoid_table[__ldcg(logit + t)]);
            const float sh = __fmul_rn(__ldcg(route_out + size_t(R + t) * kH + col), gate);
            a.shared_out[size_t(t) * kH + col] = bf16_rne(sh);
            if (!isfinite(sh)) f |= kFlagNonfiniteOutput;
        }
    }
}

// Epilogue warps of the throughput mode.  For every gate unit (an item's
// group terms for up to kTChunk routes, in one of two buffers) they sum the
// eight K-group terms of each route in ascending order, apply SiLU*up and
// store the middle row, while the consumer warps already compute the next
// unit; the buffer handshake is a pair of named barriers per buffer (the
// consumers arrive on "ready" and wait on "free", these warps the reverse),
// and the consumers never run more than two units ahead.  After an item
// they count it for its (slot, half) and quantise a completed half.
template <int QMAX>
__device__ __forceinline__ void epilogue_warps(const LayerArgs& a, Smem& s, uint32_t* ctrl, int T, int R, int G, int b,
                                               int warp, int lane, int NA, int gi0, int ng) {
    const int e = warp - kNCW;
    uint32_t f = 0;
    float* const middle = ws_at<float>(a, a.L.middle);
    const float* tb = s.tbuf;
    const volatile int* misc = s.misc;
    int u = 0;
    for (int item = 0; item < ng; ++item) {
        const int gi = gi0 + item, k = gi / 16, p = gi % 16, half = p / 8;
        const int nr = s.act_cnt[k], roff = s.act_off[k];
        const bool shared = s.act_e[k] == kE;
        const bool local_half = k * 16 + 8 * half >= gi0 && k * 16 + 8 * half + 8 <= gi0 + ng;
        const int nch = (nr + kTChunk - 1) / kTChunk;
        for (int c = 0; c < nch; ++c, ++u) {
            const int buf = u & 1;
            named_barrier(kBarTermsReady + buf, kDotEThreads);
            const int n = min(kTChunk, nr - c * kTChunk);
            if (!misc[0]) {
                for (int r = e; r < n; r += kEW) {
                    float gv = 0.f, uv = 0.f;
#pragma unroll
                    for (int g = 0; g < 8; ++g) {
                        gv = __fadd_rn(gv, tb[term_index(buf, g, 0, r, lane)]);
                        uv = __fadd_rn(uv, tb[term_index(buf, g, 1, r, lane)]);
                    }
                    float value;
                    if (shared) {
                        gv = bf16_round_f32(gv);
                        uv = bf16_round_f32(uv);
                        if (!isfinite(gv) || !isfinite(uv)) f |= kFlagNonfiniteProjection;
                        value = bf16_round_f32(__fmul_rn(a.silu_table[__float_as_uint(gv) >> 16], uv));
                    } else {
                        if (!isfinite(gv) || !isfinite(uv)) f |= kFlagNonfiniteProjection;
                        value = silu_mul(gv, uv);
                    }
                    if (!isfinite(value)) f |= kFlagNonfiniteMiddle;
                    middle[size_t(route_at(a, s, roff + c * kTChunk + r)) * kI + p * 32 + lane] = value;
                }
            }
            named_barrier_arrive(kBarTermsFree + buf, kDotEThreads);
        }
        // the item's middle columns are stored (both warps): count it, and
        // quantise its (slot, half) once all 8 items are in
        named_barrier(kBarE, kEW * 32);
        if (e == 0 && lane == 0) {
            int task = -1;
            if (local_half) {
                if (p % 8 == 7) task = 2 * k + half;
            } else if (atom_add_acq_rel(ctrl + kCtrlGateDone + 2 * k + half, 1u) == kGateTargetThr - 1) {
                task = 2 * k + half;
            }
            if (task >= 0 && nr > kHeavyTask) {
                const int t = atomicAdd(&s.misc[5], 1);
                if (t < kMaxTasks) s.tasks[t] = task;
                task = -1;
            }
            s.misc[10] = task;
        }
        named_barrier(kBarE, kEW * 32);
        const int task = misc[10];
        if (task >= 0 && !misc[0]) {
            const int kk = task >> 1, hh = task & 1;
            const int nr2 = s.act_cnt[kk], roff2 = s.act_off[kk];
            for (int q = e; q < nr2; q += kEW) quant_middle_group<QMAX>(a, route_at(a, s, roff2 + q), hh, lane, f);
            named_barrier(kBarE, kEW * 32);
            if (e == 0 && lane == 0) red_release_add(ctrl + kCtrlReady + kk, 1u);
        }
    }
    named_barrier(kBarDotE, kDotEThreads);  // every item counted, heavy halves posted
    deferred_quant_tasks<QMAX>(a, s, ctrl, warp, lane, f);
    combine_units(a, s, ctrl, T, R, G, b, warp, lane, NA, f);
    warp_flag_or(a.flags, f);
}

template <int QMAX>
__global__ void __launch_bounds__(kThreads, 1) decode_layer_kernel(const LayerArgs a, const int nst) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const Carve cv = carve(a.T, nst);
    Smem s;
    s.ring = smem_raw + cv.ring;
    s.full = reinterpret_cast<uint64_t*>(smem_raw + cv.full);
    s.empty = reinterpret_cast<uint64_t*>(smem_raw + cv.empty);
    s.last_st = reinterpret_cast<int*>(smem_raw + cv.last_st);
    s.xq = smem_raw + cv.xq;
    s.xs = reinterpret_cast<__half*>(smem_raw + cv.xs);
    s.xsum = reinterpret_cast<int*>(smem_raw + cv.xsum);
    s.ids = reinterpret_cast<int*>(smem_raw + cv.ids);
    s.wts = reinterpret_cast<float*>(smem_raw + cv.wts);
    // plan-only arrays live inside tbuf, which the items use only after the plan
    s.cnt = reinterpret_cast<int*>(smem_raw + cv.tbuf);
    s.off = s.cnt + (kE + 4);
    s.wpre = s.off + (kE + 4);
    s.xflag = reinterpret_cast<uint32_t*>(s.wpre + 2 * (kMaxSlots + 2));
    s.act_e = reinterpret_cast<int*>(smem_raw + cv.act_e);
    s.act_off = reinterpret_cast<int*>(smem_raw + cv.act_off);
    s.act_cnt = reinterpret_cast<int*>(smem_raw + cv.act_cnt);
    s.routes = reinterpret_cast<int*>(smem_raw + cv.routes);
    s.tbuf = reinterpret_cast<float*>(smem_raw + cv.tbuf);
    s.pbuf = reinterpret_cast<float*>(smem_raw + cv.pbuf);
    s.dscale = reinterpret_cast<__half*>(smem_raw + cv.dscale);
    s.dsum = reinterpret_cast<int*>(smem_raw + cv.dsum);
    s.tasks = reinterpret_cast<int*>(smem_raw + cv.tasks);

    s.misc = reinterpret_cast<int*>(smem_raw + cv.misc);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int T = a.T, R = T * kTop, G = gridDim.x, b = blockIdx.x;
    uint32_t* ctrl = ws_at<uint32_t>(a, a.L.ctrl);
    if (tid == 0) {
        DECODE_TRACE(0);
        DECODE_CLOCK(23);
    }

    // ---- routing (every CTA, identical) -----------------------------------
    if (tid == 0) {
        for (int i = 0; i < nst; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], 1);
            s.last_st[i] = -1;
        }
        fence_barrier_init();
        s.misc[0] = 0;
        s.misc[1] = 0x7fffffff;
        s.misc[4] = 0;  // stages issued so far (published by the producer)
        s.misc[5] = 0;  // middle-quantisation tasks posted
    }
    const bool small = R <= 32;  // T <= 4: one warp sorts the routes
    if (!small)
        for (int e = tid; e <= kE; e += kThreads) s.cnt[e] = 0;
    // router top-8 (from logits) or the caller's ids.  Up to 9 tokens: warp t
    // of every CTA routes token t.  More tokens: CTA t routes token t into
    // the workspace and every CTA reads the result back (one token per CTA
    // beats several tokens per warp).
    const bool spread_route = a.logits && T > kWarps;
    const int nroute_warps = a.logits && !spread_route ? min(T, kWarps) : 0;
    {
        uint32_t f = 0;
        if (spread_route) {
            if (b < T && warp == 0) {
                route_topk_warp(a.logits + size_t(b) * kE, lane, a.ids_out + b * kTop, a.weights_out + b * kTop, f);
                __syncwarp();
                if (lane == 0) red_release_add(ctrl + kCtrlRouteDone, 1u);
            }
        } else if (a.logits) {
            for (int t = warp; t < T; t += kWarps)
                route_topk_warp(a.logits + size_t(t) * kE, lane, s.ids + t * kTop, s.wts + t * kTop, f);
        } else {
            for (int r = tid; r < R; r += kThreads) {
                s.ids[r] = a.ids[r];
                s.wts[r] = a.weights[r];
            }
        }
        if (b == 0 || spread_route) warp_flag_or(a.flags, f);
    }
    // T > kRedundantX: token groups are quantised once, spread over the CTAs,
    // into the workspace, overlapping the routing; a warp holds at most one
    // group (T * 8 <= 256 < CTAs * 8), whose flags count once its token is
    // known to be live
    int xq_tok = -1;
    uint32_t xq_flags = 0;
    if (T > kRedundantX && warp < kNCW) {
        for (int q = b + G * warp; q < T * 8; q += G * kNCW) {
            const int t = q / 8, g = q % 8;
            const uint4 raw = *reinterpret_cast<const uint4*>(a.x + size_t(t) * kH + g * kG + lane * 8);
            xq_flags = wht_quant<QMAX>(
                __uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xffff0000u), __uint_as_float(raw.y << 16),
                __uint_as_float(raw.y & 0xffff0000u), __uint_as_float(raw.z << 16), __uint_as_float(raw.z & 0xffff0000u),
                __uint_as_float(raw.w << 16), __uint_as_float(raw.w & 0xffff0000u), lane,
                ws_at<uint2>(a, a.L.xq) + (size_t(t) * kH + g * kG) / 8, ws_at<__half>(a, a.L.xs) + t * 8 + g,
                ws_at<int32_t>(a, a.L.xsum) + t * 8 + g);
            xq_tok = t;
            __syncwarp();
            if (lane == 0) red_release_add(ctrl + kCtrlXDone, 1u);
        }
    }
    if (spread_route) {
        if (warp == 0) wait_counter(a.flags, s.misc, ctrl, ctrl + kCtrlRouteDone, uint32_t(T));
        __syncthreads();  // orders every warp after warp 0's acquire
        for (int r = tid; r < R; r += kThreads) {
            s.ids[r] = __ldcg(a.ids_out + r);
            s.wts[r] = __ldcg(a.weights_out + r);
        }
    }
    // T <= kRedundantX: the other warps quantise every token group meanwhile
    // (into shared memory; a dead token's codes are never read, and its flags
    // are dropped below once the ids are known)
    if (T <= kRedundantX && warp >= nroute_warps) {
        for (int q = warp - nroute_warps; q < T * 8; q += kWarps - nroute_warps) {
            const int t = q / 8, g = q % 8;
            const uint4 raw = *reinterpret_cast<const uint4*>(a.x + size_t(t) * kH + g * kG + lane * 8);
            uint32_t qf = wht_quant<QMAX>(
                __uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xffff0000u), __uint_as_float(raw.y << 16),
                __uint_as_float(raw.y & 0xffff0000u), __uint_as_float(raw.z << 16), __uint_as_float(raw.z & 0xffff0000u),
                __uint_as_float(raw.w << 16), __uint_as_float(raw.w & 0xffff0000u), lane,
                reinterpret_cast<uint2*>(s.xq + size_t(t) * kH + g * kG), s.xs + t * 8 + g, s.xsum + t * 8 + g);
            qf = __reduce_or_sync(0xffffffffu, qf);
            if (lane == 0) s.xflag[q] = qf;
        }
        DECODE_TRACE0(31);
    }
    __syncthreads();
    if (tid == 0) DECODE_TRACE(12);
    if (small) {
        // ---- plan for R <= 32 routes: warp 0 sorts (expert, route) keys -----
        if (warp == 0) {
            uint32_t f = 0;
            const int e = lane < R ? s.ids[lane] : -1;
            if (lane < R && !id_valid(e) && e != -1) f |= kFlagInvalidId;
            if (b == 0 && a.logits && lane < R) {
                a.ids_out[lane] = e;
                a.weights_out[lane] = s.wts[lane];
            }
            uint32_t key = lane < R && id_valid(e) ? (uint32_t(e) << 5) | uint32_t(lane) : 0xffffffffu;
            // bitonic sort, ascending over the 32 lanes
#pragma unroll 1
            for (int kk = 2; kk <= 32; kk <<= 1) {
#pragma unroll 1
                for (int j = kk >> 1; j > 0; j >>= 1) {
                    const uint32_t other = __shfl_xor_sync(0xffffffffu, key, j);
                    const bool keep_min = ((lane & kk) == 0) == ((lane & j) == 0);
                    key = keep_min ? min(key, other) : max(key, other);
                }
            }
            const bool v = key != 0xffffffffu;
            const int se = v ? int(key >> 5) : -1;
            const int prev = __shfl_up_sync(0xffffffffu, se, 1);
            const bool head = v && (lane == 0 || prev != se);
            const unsigned heads = __ballot_sync(0xffffffffu, head);
            const int nv = __popc(__ballot_sync(0xffffffffu, v));
            const int nact = __popc(heads);
            if (v) s.routes[lane] = int(key & 31u);
            if (head) {
                const int k = __popc(heads & ((1u << lane) - 1u));
                const unsigned later = heads & ~((2u << lane) - 1u);
                s.act_e[k] = se;
                s.act_off[k] = lane;
                s.act_cnt[k] = (later ? __ffs(later) - 1 : nv) - lane;
            }
            if (a.shared) {
                if (lane < T) s.routes[nv + lane] = R + lane;
                if (lane == 0) {
                    s.act_e[nact] = kE;
                    s.act_off[nact] = nv;
                    s.act_cnt[nact] = T;
                }
            }
            if (lane == 0) {
                s.misc[2] = nact;
                s.misc[3] = nact + (a.shared ? 1 : 0);
            }
            // flags of the token groups quantised during routing, live tokens only
            if (T <= kRedundantX && lane < T * 8) {
                const int t = lane / 8;
                bool live = a.shared_all_live;
                for (int sl = 0; sl < kTop; ++sl) live |= id_valid(s.ids[t * kTop + sl]);
                if (live) f |= s.xflag[lane];
            }
            if (b == 0) warp_flag_or(a.flags, f);
        }
    } else {
        // ---- plan for larger batches: histogram, scan, ordered placement ----
        {
            uint32_t f = 0;
            for (int r = tid; r < R; r += kThreads) {
                const int e = s.ids[r];
                if (id_valid(e)) atomicAdd(&s.cnt[e], 1);
                else if (e != -1) f |= kFlagInvalidId;
                if (b == 0 && a.logits && !spread_route) {
                    a.ids_out[r] = e;
                    a.weights_out[r] = s.wts[r];
                }
            }
            if (b == 0) warp_flag_or(a.flags, f);
        }
        __syncthreads();
        if (tid == 0) DECODE_TRACE(14);
        if (warp == 0) {
            // an expert with more than kSplit routes becomes several slots of
            // at most kSplit routes (its weights stream once per slot), so that
            // no item is much heavier than the others
            int c[8], tot = 0, nz = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                c[i] = s.cnt[8 * lane + i];
                tot += c[i];
                nz += (c[i] + kSplit - 1) / kSplit;
            }
            int it = tot, in = nz;
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                int ut = __shfl_up_sync(0xffffffffu, it, d), un = __shfl_up_sync(0xffffffffu, in, d);
                if (lane >= d) {
                    it += ut;
                    in += un;
                }
            }
            int run = it - tot, k = in - nz;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int e = 8 * lane + i;
                s.off[e] = run;
                s.cnt[e] = 0;  // from here on: placement cursor
                for (int q = 0; q < c[i]; q += kSplit, ++k) {
                    s.act_e[k] = e;
                    s.act_off[k] = run + q;
                    s.act_cnt[k] = min(kSplit, c[i] - q);
                }
                run += c[i];
            }
            const int nact = __shfl_sync(0xffffffffu, in, 31), total = __shfl_sync(0xffffffffu, it, 31);
            if (lane == 31) {
                int na = nact;
                if (a.shared)
                    for (int q = 0; q < T; q += kSplit, ++na) {
                        s.act_e[na] = kE;
                        s.act_off[na] = total + q;
                        s.act_cnt[na] = min(kSplit, T - q);
                    }
                s.misc[2] = nact;
                s.misc[3] = na;
            }
            __syncwarp();
            // routes of each expert in ascending route order (warp-wide match per 32 routes)
            for (int base = 0; base < R; base += 32) {
                const int r = base + lane;
                const int e = r < R ? s.ids[r] : -1;
                const bool valid = id_valid(e);
                const unsigned peers = __match_any_sync(0xffffffffu, valid ? e : -2 - lane);
                const int rank = __popc(peers & ((1u << lane) - 1u));
                if (valid) s.routes[checked(s.off[e] + s.cnt[e] + rank, R + T, a.flags)] = r;
                __syncwarp();
                if (valid && lane == 31 - __clz(peers)) s.cnt[e] += __popc(peers);
                __syncwarp();
            }
            if (a.shared)
                for (int t = lane; t < T; t += 32) s.routes[total + t] = R + t;
            // cost prefixes for the throughput-mode item ranges
            __syncwarp();
            const int NAp = s.misc[3];
            int run_g = 0, run_d = 0;
            for (int base = 0; base <= NAp; base += 32) {
                const int k = base + lane;
                const int nrk = k < NAp ? s.act_cnt[k] : 0;
                const int wg = k < NAp ? gate_cost(nrk) : 0, wd = k < NAp ? down_cost(nrk) : 0;
                int ig = 16 * wg, id = 64 * wd;
#pragma unroll
                for (int d = 1; d < 32; d <<= 1) {
                    const int ug = __shfl_up_sync(0xffffffffu, ig, d), ud = __shfl_up_sync(0xffffffffu, id, d);
                    if (lane >= d) {
                        ig += ug;
                        id += ud;
                    }
                }
                if (k <= NAp) {
                    s.wpre[k] = run_g + ig - 16 * wg;
                    s.wpre[kMaxSlots + 2 + k] = run_d + id - 64 * wd;
                }
                run_g += __shfl_sync(0xffffffffu, ig, 31);
                run_d += __shfl_sync(0xffffffffu, id, 31);
            }
            __syncwarp();
            if (lane < 4) {  // this CTA's item ranges, from the prefixes (read nowhere else)
                const int* W = lane < 2 ? s.wpre : s.wpre + kMaxSlots + 2;
                const int per = lane < 2 ? 16 : 64;
                s.misc[6 + lane] = range_start(W, NAp, per, b + (lane & 1), G);
            }
        }
    }
    __syncthreads();
    if (tid == 0) DECODE_TRACE(1);

    const int NA = s.misc[3];
    const int NGI = NA * 16, NDI = NA * 64;
    // latency mode (T <= 4): items round-robin over the CTAs; throughput mode:
    // contiguous cost-balanced ranges [gi0, gi0 + ng) and [dj0, dj0 + nd)
    const bool thr = T > kRedundantX;
    int ng, nd, gi0 = 0, dj0 = 0, jstart = 0;
    if (thr) {
        gi0 = s.misc[6];
        ng = s.misc[7] - gi0;
        dj0 = s.misc[8];
        nd = s.misc[9] - dj0;
    } else {
        ng = NGI > b ? (NGI - 1 - b) / G + 1 : 0;
        jstart = ((b - NGI) % G + G) % G;
        nd = NDI > jstart ? (NDI - 1 - jstart) / G + 1 : 0;
    }
    const int total_stages = 16 * ng + 2 * nd;
    if (tid == 0) {
        DECODE_VALUE(14, ng);
        DECODE_VALUE(13, nd);
        DECODE_VALUE(12, thr ? (s.act_cnt[gi0 / 16] | (s.act_cnt[min(dj0 / 64, NA - 1)] << 16)) : 0);
    }

    if (warp == kProd) {
        // ---- producer ------------------------------------------------------
        // Lanes issue a group of stages in parallel: the 16 stages of one gate
        // item, or the 8 stages of one batch of four down items.  Lane i waits
        // (bounded) until its slot's previous stage was released and issues
        // its stage at once, so the next item streams in while the current
        // one is computed; lane 0 publishes the issued count once the whole
        // group is out.  Stage st - nst was issued by an earlier group (groups
        // are at most 16 < nst stages) whose lane had waited for st - 2 nst,
        // so a slot's empty barrier is never more than one phase behind and
        // its parity is exact.  Every issued stage is recorded per slot for
        // the drain at exit.
        volatile int* misc = s.misc;
        int st0 = 0;
        while (st0 < total_stages) {
            if (st0 == 16 * ng && ng > 0) {
                // the down stages wait until this CTA's last gate stage has landed,
                // so that gate weights, needed first, get the HBM bandwidth first
                bool landed = true;
                if (lane == 0) {
                    const int last = st0 - 1;
                    const uint32_t parity = uint32_t(last / nst) & 1u;
                    const uint64_t t0 = now_ns();
                    while (!mbar_try_wait(&s.full[last % nst], parity)) {
                        if (misc[0] || now_ns() - t0 > kTimeoutNs) {
                            landed = false;
                            break;
                        }
                    }
                }
                if (!__shfl_sync(0xffffffffu, landed, 0)) {
                    if (lane == 0 && !misc[0]) give_up(a.flags, s.misc, ctrl, 2u, uint32_t(st0), uint32_t(st0 % nst), 1u);
                    break;
                }
            }
            const int gsz = st0 < 16 * ng ? 16 : 8;
            const int st = st0 + lane;
            const bool mine = lane < gsz && st < total_stages;
            const int slot = st % nst;
            bool ok = true;
            if (mine && st >= nst) {
                const uint32_t parity = uint32_t(st / nst - 1) & 1u;
                const uint64_t t0 = now_ns();
                while (!mbar_try_wait(&s.empty[slot], parity)) {
                    if (misc[0] || now_ns() - t0 > kTimeoutNs) {
                        ok = false;
                        break;
                    }
                }
            }
            if (mine && ok && !misc[0]) {
                int k, tile, g;
                bool gate;
                if (st < 16 * ng) {
                    const int item = st / 16, within = st % 16;
                    const int gi = thr ? gi0 + item : b + item * G;
                    k = gi / 16;
                    g = within / 2;
                    tile = gi % 16 + 16 * (within & 1);
                    gate = true;
                } else {
                    const int d = (st - 16 * ng) / 2;
                    const int dj = thr ? dj0 + d : jstart + d * G;
                    k = dj / 64;
                    tile = dj % 64;
                    g = (st - 16 * ng) % 2;
                    gate = false;
                }
                const int e = checked(s.act_e[k], kE + 1, a.flags);
                const uint32_t *codes, *meta;
                if (gate) {
                    const int groups = kH / kG;
                    codes = e == kE ? a.sgate_codes : a.gate_codes + size_t(e) * (2 * kI) * (kH / 8);
                    meta = e == kE ? a.sgate_meta : a.gate_meta + size_t(e) * (2 * kI) * groups;
                    codes += (size_t(tile) * groups + g) * 1024;
                    meta += (size_t(tile) * groups + g) * 32;
                } else {
                    const int groups = kI / kG;
                    codes = e == kE ? a.sdown_codes : a.down_codes + size_t(e) * kH * (kI / 8);
                    meta = e == kE ? a.sdown_meta : a.down_meta + size_t(e) * kH * groups;
                    codes += (size_t(tile) * groups + g) * 1024;
                    meta += (size_t(tile) * groups + g) * 32;
                }
                uint8_t* dst = s.ring + size_t(slot) * kStageBytes;
                mbar_arrive_expect_tx(&s.full[slot], kStageBytes);
                bulk_g2s(dst, codes, 4096, &s.full[slot]);
                bulk_g2s(dst + 4096, meta, 128, &s.full[slot]);
                s.last_st[slot] = st;
            }
            const bool all_ok = __all_sync(0xffffffffu, ok);
            const bool stop = __any_sync(0xffffffffu, misc[0] != 0);
            if (!all_ok || stop) {
                if (lane == 0 && !misc[0]) give_up(a.flags, s.misc, ctrl, 2u, uint32_t(st0), uint32_t(st0 % nst), 0u);
                break;
            }
            st0 = min(st0 + gsz, total_stages);
            __syncwarp();
            if (lane == 0) {
                // issued-count publication: a consumer only needs it to know that
                // the slot's previous phase completed (see wait_stage), which it
                // observed itself, so no fence is needed here
                misc[4] = st0;
                if (st0 <= 16) DECODE_TRACE(17);
            }
        }
        if (lane == 0) {
            atomicExch(&s.misc[1], st0);  // stages actually issued
            DECODE_TRACE(2);
        }
    } else if (NA == 0) {
        // every slot padded and no shared expert: the output is zero
        if (b == 0 && warp < kNCW)
            for (int i = tid; i < T * kH; i += kNCW * 32) {
                a.out[i] = 0;
                ws_at<float>(a, a.L.final_f32)[i] = 0.f;
            }
    } else if (warp >= kNCW) {
        // ---- epilogue warps (throughput mode) -------------------------------
        if (thr) epilogue_warps<QMAX>(a, s, ctrl, T, R, G, b, warp, lane, NA, gi0, ng);
    } else {
        // ---- consumers -----------------------------------------------------
        uint32_t f = 0;

        // shared-expert logits (fused routing): CTA G-1-t computes token t's
        if (a.shared_gate_weight && warp == kNCW - 1 && G - 1 - b < T) {
            const int t = G - 1 - b;
            const uint16_t v = shared_logit_warp(a.x + size_t(t) * kH, a.shared_gate_weight, lane);
            if (lane == 0) {
                a.logit_out[t] = v;
                red_release_add(ctrl + kCtrlLogitDone, 1u);
            }
        }

        // token activations: quantised during routing (T <= kRedundantX into
        // shared memory; otherwise into the workspace, copied in here)
        if (xq_tok >= 0) {
            bool live = a.shared_all_live;
            for (int sl = 0; sl < kTop; ++sl) live |= id_valid(s.ids[xq_tok * kTop + sl]);
            if (live) f |= xq_flags;
        }
        if (T > kRedundantX) {
            if (ng > 0) {
                if (warp == 0) wait_counter(a.flags, s.misc, ctrl, ctrl + kCtrlXDone, uint32_t(T * 8));
                named_barrier(kBarConsumers, kNCW * 32);  // orders every warp after warp 0's acquire
                const uint4* src = reinterpret_cast<const uint4*>(ws_at<uint8_t>(a, a.L.xq));
                uint4* dst = reinterpret_cast<uint4*>(s.xq);
                for (int i = tid; i < T * kH / 16; i += kNCW * 32) dst[i] = __ldcg(src + i);
                for (int i = tid; i < T * 8; i += kNCW * 32) {
                    s.xs[i] = __ldcg(ws_at<__half>(a, a.L.xs) + i);
                    s.xsum[i] = __ldcg(ws_at<int32_t>(a, a.L.xsum) + i);
                }
                named_barrier(kBarConsumers, kNCW * 32);
            }
        }
        if (tid == 0) DECODE_TRACE(3);

        // ---- gate items: all eight warps, warp w = K-group w -----------------
        bool alive = true;
        int tasks_done = 0;
        float* const tb = s.tbuf;
        float* const middle = ws_at<float>(a, a.L.middle);
        if (!thr) {
        for (int item = 0; item < ng; ++item) {
            const int gi = thr ? gi0 + item : b + item * G, k = gi / 16, p = gi % 16, half = p / 8;
            // a (slot, half) whose 8 items all lie in this CTA's range is
            // quantised here without counting across CTAs
            const bool local_half = thr && k * 16 + 8 * half >= gi0 && k * 16 + 8 * half + 8 <= gi0 + ng;
            const int nr = s.act_cnt[k], roff = s.act_off[k];
            const bool shared = s.act_e[k] == kE;
            const int stg = 16 * item + 2 * warp;  // gate stage; stg + 1 = up stage of the same group
            if (alive && !wait_stage(a.flags, s.misc, s.full, ctrl, stg, nst)) alive = false;
            if (alive && !wait_stage(a.flags, s.misc, s.full, ctrl, stg + 1, nst)) alive = false;
            if (tid == 0 && item == 0) DECODE_TRACE(4);
            if (item == 0) DECODE_TRACE0(18);
            if (item == 5) DECODE_TRACE0(25);
            const uint32_t* bg = reinterpret_cast<const uint32_t*>(s.ring + size_t(stg % nst) * kStageBytes);
            const uint32_t* bu = reinterpret_cast<const uint32_t*>(s.ring + size_t((stg + 1) % nst) * kStageBytes);
            const uint32_t mwg = alive ? bg[1024 + lane] : 0u, mwu = alive ? bu[1024 + lane] : 0u;
            const int nchunks = (nr + kChunk - 1) / kChunk;
            for (int c = 0; c < nchunks; ++c) {
                const int n = min(kChunk, nr - c * kChunk);
                if (alive) {
                    const uint4* act[kChunk];
                    float sa[kChunk];
                    int sm[kChunk];
#pragma unroll
                    for (int i = 0; i < kChunk; ++i) {
                        const int tok = checked(token_of(route_at(a, s, roff + c * kChunk + (i < n ? i : n - 1)), R), T, a.flags);
                        act[i] = reinterpret_cast<const uint4*>(s.xq + size_t(tok) * kH + warp * kG);
                        sa[i] = __half2float(s.xs[tok * 8 + warp]);
                        sm[i] = s.xsum[tok * 8 + warp];
                    }
                    int dg[kChunk], du[kChunk];
                    stage_dots2_n(n, bg, bu, act, lane, dg, du);
                    if (item == 0 && c == 0) DECODE_TRACE0(19);
                    if (item == 5 && c == 0) DECODE_TRACE0(26);
#pragma unroll
                    for (int i = 0; i < kChunk; ++i) {
                        if (i < n) {
                            tb[((warp * 2 + 0) * kChunk + i) * 32 + lane] = group_term(sa[i], dg[i], sm[i], mwg);
                            tb[((warp * 2 + 1) * kChunk + i) * 32 + lane] = group_term(sa[i], du[i], sm[i], mwu);
                        }
                    }
                    if (c == nchunks - 1) {
                        __syncwarp();
                        if (lane == 0) {
                            mbar_arrive(&s.empty[stg % nst]);
                            mbar_arrive(&s.empty[(stg + 1) % nst]);
                        }
                    }
                }
                named_barrier(kBarConsumers, kNCW * 32);
                if (item == 0 && c == 0) DECODE_TRACE0(20);
                if (item == 5 && c == 0) DECODE_TRACE0(27);
                // route c*8 + warp: ordered sum of the 8 group terms, SiLU * up
                const volatile int* misc = s.misc;
                if (warp < n && !misc[0]) {
                    float gv = 0.f, uv = 0.f;
#pragma unroll
                    for (int g = 0; g < 8; ++g) {
                        gv = __fadd_rn(gv, tb[((g * 2 + 0) * kChunk + warp) * 32 + lane]);
                        uv = __fadd_rn(uv, tb[((g * 2 + 1) * kChunk + warp) * 32 + lane]);
                    }
                    float value;
                    if (shared) {
                        gv = bf16_round_f32(gv);
                        uv = bf16_round_f32(uv);
                        if (!isfinite(gv) || !isfinite(uv)) f |= kFlagNonfiniteProjection;
                        value = bf16_round_f32(__fmul_rn(a.silu_table[__float_as_uint(gv) >> 16], uv));
                    } else {
                        if (!isfinite(gv) || !isfinite(uv)) f |= kFlagNonfiniteProjection;
                        value = silu_mul(gv, uv);
                    }
                    if (!isfinite(value)) f |= kFlagNonfiniteMiddle;
                    middle[size_t(route_at(a, s, roff + c * kChunk + warp)) * kI + p * 32 + lane] = value;
                }
                if (c + 1 < nchunks) named_barrier(kBarConsumers, kNCW * 32);  // tbuf is rewritten next
            }
            // this warp's share of the item is stored: count it; the warp that
            // completes the (slot, half) posts its quantisation to the CTA
            if (item == 0) DECODE_TRACE0(21);
            if (item == 5) DECODE_TRACE0(28);
            __syncwarp();
            if (local_half) {
                if (tid == 0 && p % 8 == 7) {
                    const int t = atomicAdd(&s.misc[5], 1);
                    if (t < kMaxTasks) s.tasks[t] = 2 * k + half;
                }
            } else if (lane == 0 && light_slot(T, nr)) {
                // light slot: no quantisation task to elect, nothing to wait for
                red_release_add(ctrl + kCtrlGateDone + 2 * k + half, 1u);
            } else if (lane == 0) {
                const uint32_t old = atom_add_acq_rel(ctrl + kCtrlGateDone + 2 * k + half, 1u);
                if (item == 0) DECODE_TRACE0(22);
                if (old == kGateTarget - 1) {
                    const int t = atomicAdd(&s.misc[5], 1);
                    if (t < kMaxTasks) s.tasks[t] = 2 * k + half;
                }
            }
            named_barrier(kBarConsumers, kNCW * 32);
            if (tid == 0 && item == 0) DECODE_TRACE(5);
            if (item == 4) DECODE_TRACE0(29);
            if (item == 5) DECODE_TRACE0(30);
            const int posted = min(*static_cast<volatile int*>(&s.misc[5]), kMaxTasks);
            // (the poster's acquiring counter update precedes the barrier above)
            for (; tasks_done < posted; ++tasks_done) {
                const int task = s.tasks[tasks_done], kk = task >> 1, hh = task & 1;
                const int nr2 = s.act_cnt[kk], roff2 = s.act_off[kk];
                for (int q = warp; q < nr2; q += kNCW) quant_middle_group<QMAX>(a, route_at(a, s, roff2 + q), hh, lane, f);
                __syncwarp();
                if (lane == 0) red_release_add(ctrl + kCtrlReady + kk, 1u);
                if (lane == 0 && warp == 0) DECODE_TRACE(6);
            }
        }
        } else {
            // throughput mode: units of up to kTChunk routes; the group terms
            // go to alternating buffers for the epilogue warps
            int u = 0;
            for (int item = 0; item < ng; ++item) {
                const int gi = gi0 + item, k = gi / 16;
                const int nr = s.act_cnt[k], roff = s.act_off[k];
                const int stg = 16 * item + 2 * warp;  // gate stage; stg + 1 = up stage of the same group
                if (alive && !wait_stage(a.flags, s.misc, s.full, ctrl, stg, nst)) alive = false;
                if (alive && !wait_stage(a.flags, s.misc, s.full, ctrl, stg + 1, nst)) alive = false;
                if (item == 5) DECODE_TRACE0(25);
                const uint32_t* bg = reinterpret_cast<const uint32_t*>(s.ring + size_t(stg % nst) * kStageBytes);
                const uint32_t* bu = reinterpret_cast<const uint32_t*>(s.ring + size_t((stg + 1) % nst) * kStageBytes);
                const uint32_t mwg = alive ? bg[1024 + lane] : 0u, mwu = alive ? bu[1024 + lane] : 0u;
                const int nch = (nr + kTChunk - 1) / kTChunk;
                for (int c = 0; c < nch; ++c, ++u) {
                    const int buf = u & 1;
                    if (u >= 2) named_barrier(kBarTermsFree + buf, kDotEThreads);  // unit u-2 consumed
                    const int n = min(kTChunk, nr - c * kTChunk);
                    if (alive) {
                        const uint4* act[kChunk];
                        float sa[kChunk];
                        int sm[kChunk];
#pragma unroll
                        for (int i = 0; i < kChunk; ++i) {
                            const int tok = checked(token_of(route_at(a, s, roff + c * kTChunk + (i < n ? i : n - 1)), R), T, a.flags);
                            act[i] = reinterpret_cast<const uint4*>(s.xq + size_t(tok) * kH + warp * kG);
                            sa[i] = __half2float(s.xs[tok * 8 + warp]);
                            sm[i] = s.xsum[tok * 8 + warp];
                        }
                        int dg[kChunk], du[kChunk];
                        stage_dots2_n(n, bg, bu, act, lane, dg, du);
                        if (item == 5 && c == 0) DECODE_TRACE0(26);
#pragma unroll
                        for (int i = 0; i < kTChunk; ++i) {
                            if (i < n) {
                                tb[term_index(buf, warp, 0, i, lane)] = group_term(sa[i], dg[i], sm[i], mwg);
                                tb[term_index(buf, warp, 1, i, lane)] = group_term(sa[i], du[i], sm[i], mwu);
                            }
                        }
                        if (c == nch - 1) {
                            __syncwarp();
                            if (lane == 0) {
                                mbar_arrive(&s.empty[stg % nst]);
                                mbar_arrive(&s.empty[(stg + 1) % nst]);
                            }
                        }
                    }
                    named_barrier_arrive(kBarTermsReady + buf, kDotEThreads);
                }
            }
            // the epilogue warps' last two buffer releases: tbuf is free after these
            for (int v = u >= 2 ? u - 2 : 0; v < u; ++v) named_barrier(kBarTermsFree + (v & 1), kDotEThreads);
            named_barrier(kBarDotE, kDotEThreads);  // every item counted, heavy halves posted
            deferred_quant_tasks<QMAX>(a, s, ctrl, warp, lane, f);
        }
        if (tid == 0) DECODE_TRACE(7);

        // ---- down items, latency mode: four at a time, warp pair q = item,
        // warp parity = K-group, slot-ordered combine by the tile's last item
        if (!thr) {
            const int pair = warp >> 1, g = warp & 1;
            uint8_t* dact = reinterpret_cast<uint8_t*>(s.tbuf) + size_t(warp) * kChunk * kG;
            __half* dsc = s.dscale + warp * kChunk;
            int* dsm = s.dsum + warp * kChunk;
            float* pb = s.pbuf + pair * kChunk * 32;
            float* const route_out = ws_at<float>(a, a.L.route_out);
            const int nbatch = (nd + 3) / 4;
            for (int j = 0; j < nbatch; ++j) {
                const int d = 4 * j + pair;
                if (d >= nd) continue;  // uniform within the pair
                const int dj = jstart + d * G, k = dj / 64, tile = dj % 64;
                const int nr = s.act_cnt[k], roff = s.act_off[k];
                const bool shared = s.act_e[k] == kE;
                // light slot: wait for this K-group's half of the middle rows and
                // quantise it here; heavy slot: wait for the finisher's ready count
                const bool selfq = light_slot(T, nr);
                bool ok = alive && wait_counter(a.flags, s.misc, ctrl,
                                                selfq ? ctrl + kCtrlGateDone + 2 * k + g : ctrl + kCtrlReady + k,
                                                selfq ? kGateTarget : kReadyTarget);
                if (lane == 0 && j == 0 && (warp == 0 || warp == 2)) DECODE_TRACE(warp == 0 ? 8 : 13);
                const int st = 16 * ng + 8 * j + warp;  // = 16 ng + 2 d + g
                if (ok && !wait_stage(a.flags, s.misc, s.full, ctrl, st, nst)) ok = false;
                if (j == 0) DECODE_TRACE0(26);
                if (!ok) alive = false;
                const uint32_t* blk = reinterpret_cast<const uint32_t*>(s.ring + size_t(st % nst) * kStageBytes);
                const uint32_t mw = ok ? blk[1024 + lane] : 0u;
                const int nchunks = (nr + kChunk - 1) / kChunk;
                float term[kChunk];
                for (int c = 0; c < nchunks; ++c) {
                    const int n = min(kChunk, nr - c * kChunk);
                    if (ok && selfq) {
                        // all loads first, then the transforms (n <= kSelfQuantMax, one chunk)
                        float4 v[kSelfQuantMax][2];
#pragma unroll
                        for (int i = 0; i < kSelfQuantMax; ++i)
                            if (i < n) load_middle(a, route_at(a, s, roff + i), g, lane, v[i][0], v[i][1]);
#pragma unroll
                        for (int i = 0; i < kSelfQuantMax; ++i)
                            if (i < n)
                                f |= quant_middle<QMAX>(v[i][0], v[i][1], lane, reinterpret_cast<uint2*>(dact + i * kG),
                                                        dsc + i, dsm + i);
                        if (j == 0) DECODE_TRACE0(25);
                    } else if (ok) {
                        for (int i = lane; i < n * 16; i += 32) {
                            const int ri = i / 16, part = i % 16;
                            const int route = route_at(a, s, roff + c * kChunk + ri);
                            reinterpret_cast<uint4*>(dact + ri * kG)[part] = __ldcg(
                                reinterpret_cast<const uint4*>(ws_at<uint8_t>(a, a.L.mq) + size_t(route) * kI + g * kG) +
                                part);
                        }
                        if (lane < n) {
                            const int route = route_at(a, s, roff + c * kChunk + lane);
                            dsc[lane] = __ldcg(ws_at<__half>(a, a.L.ms) + route * 2 + g);
                            dsm[lane] = __ldcg(ws_at<int32_t>(a, a.L.msum) + route * 2 + g);
                        }
                    }
                    if (ok) {
                        __syncwarp();
                        const uint4* act[kChunk];
#pragma unroll
                        for (int i = 0; i < kChunk; ++i)
                            act[i] = reinterpret_cast<const uint4*>(dact + (i < n ? i : n - 1) * kG);
                        int dot[kChunk];
                        stage_dots1_n(n, blk, act, lane, dot);
                        if (j == 0) DECODE_TRACE0(27);
#pragma unroll
                        for (int i = 0; i < kChunk; ++i)
                            term[i] = group_term(__half2float(dsc[i < n ? i : 0]), dot[i], dsm[i < n ? i : 0], mw);
                        if (g == 1) {
#pragma unroll
                            for (int i = 0; i < kChunk; ++i)
                                if (i < n) pb[i * 32 + lane] = term[i];
                        }
                        if (c == nchunks - 1) {
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&s.empty[st % nst]);
                        }
                        __syncwarp();
                    }
                    named_barrier(2 + pair, 64);
                    if (j == 0) DECODE_TRACE0(28);
                    const volatile int* misc = s.misc;
                    if (g == 0 && ok && !misc[0]) {
#pragma unroll
                        for (int i = 0; i < kChunk; ++i) {
                            if (i < n) {
                                float v = __fadd_rn(__fadd_rn(0.f, term[i]), pb[i * 32 + lane]);
                                if (shared) v = bf16_round_f32(v);
                                if (!isfinite(v)) f |= kFlagNonfiniteProjection;
                                route_out[size_t(route_at(a, s, roff + c * kChunk + i)) * kH + tile * 32 + lane] = v;
                            }
                        }
                    }
                    if (c + 1 < nchunks) named_barrier(2 + pair, 64);  // pbuf and activations are rewritten next
                }
                if (g == 1 || !ok) continue;
                __syncwarp();
                uint32_t old = 0;
                if (lane == 0) old = atom_add_acq_rel(ctrl + kCtrlColDone + tile, 1u);
                old = __shfl_sync(0xffffffffu, old, 0);
                __syncwarp();  // the combine's reads are ordered after lane 0's acquire
                if (lane == 0 && j == 0 && warp == 0) DECODE_TRACE(9);
                if (old != uint32_t(NA - 1)) continue;
                // last expert of this output tile: slot-ordered combine (reduce_slots :176-185)
                if (a.shared && a.shared_gate_weight &&
                    !wait_counter(a.flags, s.misc, ctrl, ctrl + kCtrlLogitDone, uint32_t(T)))
                    continue;
                const float* ro = route_out;
                float* fin = ws_at<float>(a, a.L.final_f32);
                const uint16_t* logit = a.shared_gate_weight ? a.logit_out : a.shared_logit;
                const int col = tile * 32 + lane;
                for (int t = 0; t < T; ++t) {
                    float sum = 0.f;
#pragma unroll
                    for (int sl = 0; sl < kTop; ++sl) {
                        const int r = t * kTop + sl;
                        if (id_valid(s.ids[r]))
                            sum = __fadd_rn(sum, __fmul_rn(__ldcg(ro + size_t(r) * kH + col), s.wts[r]));
                    }
                    const uint16_t res = bf16_rne(sum);
                    fin[size_t(t) * kH + col] = sum;
                    a.out[size_t(t) * kH + col] = res;
                    if (!isfinite(sum) || (res & 0x7f80u) == 0x7f80u) f |= kFlagNonfiniteOutput;
                    if (a.shared) {
                        const float gate = bf16_to_f32(a.sigmoid_table[__ldcg(logit + t)]);
                        const float sh = __fmul_rn(__ldcg(ro + size_t(R + t) * kH + col), gate);
                        a.shared_out[size_t(t) * kH + col] = bf16_rne(sh);
                        if (!isfinite(sh)) f |= kFlagNonfiniteOutput;
                    }
                }
                if (lane == 0) DECODE_TRACE(10);
            }
        } else {
            // ---- down items, throughput mode: per run of one slot's tiles,
            // the slot's middle activations (up to 32 routes) are loaded into
            // shared memory once; warp w takes tiles w, w+8, ... of the run,
            // both K-groups, and sums their terms in order itself
            uint8_t* const sact = reinterpret_cast<uint8_t*>(s.tbuf);  // [32 routes][512 B]
            float* const route_out = ws_at<float>(a, a.L.route_out);
            uint8_t* dact = reinterpret_cast<uint8_t*>(s.tbuf) + size_t(warp) * kChunk * kG;  // uncached runs
            for (int d0 = 0; d0 < nd;) {
                const int k = (dj0 + d0) / 64;
                const int d1 = min(nd, (k + 1) * 64 - dj0);  // end of this slot's run
                const int nr = s.act_cnt[k], roff = s.act_off[k];
                const bool shared = s.act_e[k] == kE;
                const bool cached = nr <= 32;
                if (warp == 0 && alive && !wait_counter(a.flags, s.misc, ctrl, ctrl + kCtrlReady + k, kReadyTargetThr))
                    alive = false;
                named_barrier(kBarConsumers, kNCW * 32);  // every warp after warp 0's acquire
                if (d0 == 0) DECODE_TRACE0(8);
                const volatile int* misc = s.misc;
                const bool ok_run = !misc[0];
                if (ok_run && cached) {
                    for (int i = tid; i < nr * 32; i += kNCW * 32) {
                        const int ri = i / 32, part = i % 32;
                        reinterpret_cast<uint4*>(sact + ri * kI)[part] = __ldcg(
                            reinterpret_cast<const uint4*>(ws_at<uint8_t>(a, a.L.mq) + size_t(route_at(a, s, roff + ri)) * kI) + part);
                    }
                    for (int i = tid; i < nr * 2; i += kNCW * 32) {
                        const int route = route_at(a, s, roff + i / 2);
                        s.dscale[i] = __ldcg(ws_at<__half>(a, a.L.ms) + route * 2 + i % 2);
                        s.dsum[i] = __ldcg(ws_at<int32_t>(a, a.L.msum) + route * 2 + i % 2);
                    }
                }
                named_barrier(kBarConsumers, kNCW * 32);
                bool run_ok = true;
                for (int dd = d0 + warp; dd < d1; dd += kNCW) {
                    const int tile = (dj0 + dd) % 64;
                    const int st0 = 16 * ng + 2 * dd;  // K-group 0; st0 + 1 = K-group 1
                    bool ok = ok_run && alive;
                    if (ok && !wait_stage(a.flags, s.misc, s.full, ctrl, st0, nst)) ok = false;
                    if (ok && !wait_stage(a.flags, s.misc, s.full, ctrl, st0 + 1, nst)) ok = false;
                    if (!ok) alive = false;
                    const uint32_t* blk[2] = {reinterpret_cast<const uint32_t*>(s.ring + size_t(st0 % nst) * kStageBytes),
                                              reinterpret_cast<const uint32_t*>(s.ring + size_t((st0 + 1) % nst) * kStageBytes)};
                    const uint32_t mw0 = ok ? blk[0][1024 + lane] : 0u, mw1 = ok ? blk[1][1024 + lane] : 0u;
                    for (int c = 0; ok && c * kChunk < nr; ++c) {
                        const int n = min(kChunk, nr - c * kChunk);
                        float term0[kChunk];
#pragma unroll 1
                        for (int g = 0; g < 2; ++g) {
                            const uint4* act[kChunk];
                            float sa[kChunk];
                            int sm[kChunk];
                            if (cached) {
#pragma unroll
                                for (int i = 0; i < kChunk; ++i) {
                                    const int ri = c * kChunk + (i < n ? i : n - 1);
                                    act[i] = reinterpret_cast<const uint4*>(sact + ri * kI + g * kG);
                                    sa[i] = __half2float(s.dscale[ri * 2 + g]);
                                    sm[i] = s.dsum[ri * 2 + g];
                                }
                            } else {
                                __syncwarp();  // earlier reads of dact are done
                                for (int i = lane; i < n * 16; i += 32) {
                                    const int ri = i / 16, part = i % 16;
                                    const int route = route_at(a, s, roff + c * kChunk + ri);
                                    reinterpret_cast<uint4*>(dact + ri * kG)[part] = __ldcg(
                                        reinterpret_cast<const uint4*>(ws_at<uint8_t>(a, a.L.mq) + size_t(route) * kI + g * kG) +
                                        part);
                                }
                                __syncwarp();
#pragma unroll
                                for (int i = 0; i < kChunk; ++i) {
                                    const int ri = i < n ? i : n - 1;
                                    const int route = route_at(a, s, roff + c * kChunk + ri);
                                    act[i] = reinterpret_cast<const uint4*>(dact + ri * kG);
                                    sa[i] = __half2float(__ldcg(ws_at<__half>(a, a.L.ms) + route * 2 + g));
                                    sm[i] = __ldcg(ws_at<int32_t>(a, a.L.msum) + route * 2 + g);
                                }
                            }
                            int dot[kChunk];
                            stage_dots1_n(n, blk[g], act, lane, dot);
                            if (g == 0) {
#pragma unroll
                                for (int i = 0; i < kChunk; ++i) term0[i] = group_term(sa[i], dot[i], sm[i], mw0);
                            } else if (!misc[0]) {
#pragma unroll
                                for (int i = 0; i < kChunk; ++i) {
                                    if (i < n) {
                                        float v = __fadd_rn(__fadd_rn(0.f, term0[i]), group_term(sa[i], dot[i], sm[i], mw1));
                                        if (shared) v = bf16_round_f32(v);
                                        if (!isfinite(v)) f |= kFlagNonfiniteProjection;
                                        route_out[size_t(route_at(a, s, roff + c * kChunk + i)) * kH + tile * 32 + lane] = v;
                                    }
                                }
                            }
                        }
                    }
                    if (ok) {
                        __syncwarp();
                        if (lane == 0) {
                            mbar_arrive(&s.empty[st0 % nst]);
                            mbar_arrive(&s.empty[(st0 + 1) % nst]);
                        }
                    }
                    run_ok = run_ok && ok;
                }
                // count this warp's tiles of the run: one fence for all of them
                if (run_ok && d0 + warp < d1) {
                    __syncwarp();
                    __threadfence();
                    for (int i = lane; d0 + warp + kNCW * i < d1; i += 32)
                        red_relaxed_add(ctrl + kCtrlColDone + (dj0 + d0 + warp + kNCW * i) % 64, 1u);
                }
                named_barrier(kBarConsumers, kNCW * 32);  // the run's activations are replaced next
                if (d0 == 0) DECODE_TRACE0(9);
                d0 = d1;
            }
            DECODE_TRACE0(16);
            combine_units(a, s, ctrl, T, R, G, b, warp, lane, NA, f);
            DECODE_TRACE0(10);
        }
        warp_flag_or(a.flags, f);
    }

    // ---- end: after an abort, let every issued copy land before the CTA exits
    __syncthreads();
    if (tid == 0) {
        DECODE_TRACE(11);
        DECODE_CLOCK(24);
        if (s.misc[0]) {
            const uint64_t t0 = now_ns();
            for (int slot = 0; slot < nst; ++slot) {
                const int last = s.last_st[slot];  // last stage issued into this slot
                if (last < 0) continue;
                const uint32_t parity = uint32_t(last / nst) & 1u;
                while (!mbar_try_wait(&s.full[slot], parity) && now_ns() - t0 < kTimeoutNs) {
                }
            }
        }
    }
}

__global__ void __launch_bounds__(256) ctrl_clear_kernel(uint32_t* ctrl, int words) {
    for (int i = threadIdx.x; i < words; i += blockDim.x) ctrl[i] = 0u;
}

struct DeviceConfig {
    int sms = 0;
    int max_smem = 0;
    bool attr_set[2] = {false, false};
};
DeviceConfig g_dev[64];

}  // namespace

#ifdef ORNITH_DECODE_TRACE
// Copies the phase timestamps of the last decode launch (kTraceCtas x kTraceSlots u64).
extern "C" __attribute__((visibility("default"))) int ornith_moe_b200_decode_trace(void* dst) {
    return int(cudaMemcpyFromSymbol(dst, g_decode_trace, sizeof(g_decode_trace)));
}
extern "C" __attribute__((visibility("default"))) int ornith_moe_b200_decode_trace_clear(void) {
    static unsigned long long zeros[kTraceCtas][kTraceSlots];
    return int(cudaMemcpyToSymbol(g_decode_trace, zeros, sizeof(zeros)));
}
#endif

bool decode_supported(int T) { return T >= 1 && T <= kDecodeMaxT; }

cudaError_t launch_decode(const LayerArgs& a, cudaStream_t stream) {
    if (a.T == 1) {  // the single-token kernel where the device fits it
        const cudaError_t s1 = launch_decode_single(a, stream);
        if (s1 != cudaErrorNotSupported) return s1;
    }
    int device = 0;
    cudaError_t st = cudaGetDevice(&device);
    if (st != cudaSuccess) return st;
    if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
    DeviceConfig& dc = g_dev[device];
    if (dc.sms == 0) {
        if ((st = cudaDeviceGetAttribute(&dc.sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess) return st;
        if ((st = cudaDeviceGetAttribute(&dc.max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, device)) != cudaSuccess)
            return st;
    }
    // one CTA receives at most ceil(257*16 / SMs) gate items, each posting at
    // most one quantisation task: the task list must hold that many
    if ((kE + 1) * 16 > dc.sms * kMaxTasks) return cudaErrorInvalidConfiguration;
    // ring depth: as many stages as fit next to the fixed carve, at most 48
    const Carve fixed = carve(a.T, 0);
    int nst = int((size_t(dc.max_smem) - fixed.total - 1024) / (kStageBytes + 16));
    nst = nst > 48 ? 48 : nst;
    if (nst < kMinStages) return cudaErrorInvalidConfiguration;
    const size_t smem = carve(a.T, nst).total;
    const int which = a.a8 ? 0 : 1;
    auto kernel = a.a8 ? decode_layer_kernel<127> : decode_layer_kernel<7>;
    if (!dc.attr_set[which]) {
        if ((st = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dc.max_smem)) != cudaSuccess)
            return st;
        dc.attr_set[which] = true;
    }
    // zero the counters with a one-CTA kernel: in a CUDA graph a kernel node
    // costs about a third of a memset node
    count_launches(1);
    ctrl_clear_kernel<<<1, 256, 0, stream>>>(ws_at<uint32_t>(a, a.L.ctrl), kCtrlClearWords);
    if ((st = cudaGetLastError()) != cudaSuccess) return st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(dc.sms);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    count_launches(1);
    return cudaLaunchKernelEx(&cfg, kernel, a, nst);
}

}  // namespace ornith
