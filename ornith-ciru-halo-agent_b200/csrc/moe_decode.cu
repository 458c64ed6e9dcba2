// Fused persistent routed-MoE layer for decode batches (T <= 32), sm_100a.
//
// One cooperative launch per layer, one CTA per SM.  The arithmetic is the
// reference's (kernels/routed_storage/routed_storage_n32_consumer.cpp:319-351);
// the schedule is B200-specific:
//
//  * every CTA builds the routing plan (expert slot counts, offsets, route
//    lists; slot 256 = shared expert) in shared memory from the 8T ids, so no
//    routing kernel or global scratch is needed;
//  * work items: gate item (expert slot, tile pair p) = gate tile p + up tile
//    p+16 over 8 K-groups (66 KB of packed weights); down item (slot, tile t)
//    over 2 K-groups (8.4 KB).  Items are dealt round-robin over CTAs, gate
//    items first;
//  * a producer warp streams each item's 4 KB (tile, group) weight blocks and
//    128 B metadata into a ring of shared-memory stages with cp.async.bulk
//    (no cluster multicast), all gate stages before any down stage, so HBM
//    streaming never waits on the compute dependencies below;
//  * consumer warp pairs run gate items (lane = output column, __dp4a integer
//    dots, the fixed fp32 group epilogue), exchange the up tile through shared
//    memory and write SiLU*up rows; the CTA that finishes an expert's 16th
//    gate item (global counter) quantises that expert's middle rows and
//    releases a ready flag;
//  * down items wait (bounded) on their expert's ready flag; the CTA that
//    finishes the last expert of an output tile performs the slot-ordered
//    combine of that tile.
// Every wait is bounded (about one second of %globaltimer), after which the
// kernel raises flag 64, lets in-flight copies land and returns.
#include "moe_layer.cuh"

namespace ornith {
namespace {

constexpr int kNCW = 8;                       // consumer warps
constexpr int kThreads = (kNCW + 1) * 32;     // + one producer warp
constexpr int kNP = kNCW / 2;                 // gate warp pairs
constexpr int kStageBytes = 4096 + 128;       // one (tile, group) block: codes + metadata
constexpr int kMaxR = 32;                     // routes per expert slot (T <= 32)
constexpr int kChunk = 8;                     // down-item activation chunk (routes)
constexpr uint64_t kTimeoutNs = 1000000000ull;
constexpr int kRedundantX = 4;                // T <= 4: every CTA quantises all tokens itself

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void named_barrier(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

struct Smem {
    uint8_t* ring;
    uint64_t* full;
    uint64_t* empty;
    uint8_t* xq;      // [T][2048] permuted int8
    float* xs;        // [T][8]
    int* xsum;        // [T][8]
    int* ids;         // [R]
    int* cnt;         // [E+1]
    int* off;         // [E+1]
    int* act_e;       // [E+1] expert of active slot k
    int* act_off;     // [E+1]
    int* act_cnt;     // [E+1]
    int* routes;      // [R+T]
    float* pairbuf;   // [kNP][kMaxR][32]
    uint8_t* dbuf;    // [kNCW][kChunk][512]
    float* dscale;    // [kNCW][kChunk][2]
    int* dsum;        // [kNCW][kChunk][2]
    int* misc;        // [0] abort, [1] final issued count, [2] nact, [3] NA, [4] issued so far
};

__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Byte offsets of the shared-memory carve for T tokens and nst ring stages.
struct Carve {
    size_t ring, full, empty, xq, xs, xsum, ids, cnt, off, act_e, act_off, act_cnt, routes, pairbuf, dbuf, dscale,
        dsum, misc, total;
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
    add(c.xq, size_t(T) * kH, 16);
    add(c.xs, size_t(T) * 8 * 4, 16);
    add(c.xsum, size_t(T) * 8 * 4, 16);
    add(c.ids, R * 4 + 4, 16);
    add(c.cnt, (kE + 1) * 4, 16);
    add(c.off, (kE + 1) * 4, 16);
    add(c.act_e, (kE + 1) * 4, 16);
    add(c.act_off, (kE + 1) * 4, 16);
    add(c.act_cnt, (kE + 1) * 4, 16);
    add(c.routes, (R + T) * 4 + 4, 16);
    add(c.pairbuf, size_t(kNP) * kMaxR * 32 * 4, 16);
    add(c.dbuf, size_t(kNCW) * kChunk * 512, 16);
    add(c.dscale, size_t(kNCW) * kChunk * 2 * 4, 16);
    add(c.dsum, size_t(kNCW) * kChunk * 2 * 4, 16);
    add(c.misc, 16 * 4, 16);
    c.total = align_up(cur, 128);
    return c;
}

__device__ __forceinline__ void warp_flag_or(uint32_t* flags, uint32_t f) {
    f = __reduce_or_sync(0xffffffffu, f);
    if (f && (threadIdx.x & 31) == 0) atomicOr(flags, f);
}

// Raise the abort state (CTA-local and global) and flag 64; the first CTA to
// give up records where (kCtrlGiveUp) for the caller's diagnosis.
__device__ __forceinline__ void give_up(const LayerArgs& a, Smem& s, uint32_t* ctrl, uint32_t tag, uint32_t x,
                                        uint32_t y, uint32_t observed) {
    atomicOr(a.flags, kFlagWaitTimeout);
    atomicExch(&s.misc[0], 1);
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
// Different warps consume different ring stages, so a warp can reach stage st
// before the slot's previous use (st - nst) has even landed.  An mbarrier
// parity wait cannot tell phases two apart, so the warp first waits until the
// producer has published that stage st was issued (misc[4] > st); from then
// on the slot's barrier is at most one phase behind and the parity is exact.
__device__ bool wait_stage(const LayerArgs& a, Smem& s, uint32_t* ctrl, int st, int nst) {
    const int slot = st % nst;
    const uint32_t parity = uint32_t(st / nst) & 1u;
    volatile int* misc = s.misc;
    uint64_t t0 = 0;
    for (int i = 0;; ++i) {
        if (misc[4] > st && mbar_try_wait(&s.full[slot], parity)) return true;
        if (misc[0] && st >= misc[1]) return false;
        if (i == 0) t0 = now_ns();
        else if ((i & 63) == 0 && now_ns() - t0 > kTimeoutNs) {
            give_up(a, s, ctrl, 1u, uint32_t(st), uint32_t(slot), uint32_t(misc[4]));
            // the copy, if it was issued, still lands: wait for it (bounded) before leaving
            if (st < misc[4]) {
                uint64_t t1 = now_ns();
                while (!mbar_try_wait(&s.full[slot], parity) && now_ns() - t1 < kTimeoutNs) {
                }
            }
            return false;
        }
    }
}

// Bounded wait on a global counter reaching `target` (lane 0 of the warp polls).
__device__ bool wait_counter(const LayerArgs& a, Smem& s, uint32_t* ctrl, const uint32_t* p, uint32_t target) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) {
        uint64_t t0 = now_ns();
        while (ld_acquire(p) < target) {
            volatile int* misc = s.misc;
            if (misc[0] || ld_acquire(ctrl + kCtrlAbort)) {
                ok = 0;
                break;
            }
            if (now_ns() - t0 > kTimeoutNs) {
                give_up(a, s, ctrl, 3u, uint32_t(p - ctrl), target, ld_acquire(p));
                ok = 0;
                break;
            }
            __nanosleep(64);
        }
    }
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__device__ __forceinline__ int token_of(int route, int R) { return route >= R ? route - R : route / kTop; }

// Exact integer dots of one (tile, group) stage for NRC routes; lane = output
// column.  Word j of the stage holds this column's codes for k = 8j..8j+7; the
// even and odd nibbles meet the permuted activation bytes in two __dp4a whose
// chains are kept apart for instruction-level parallelism (the integer sum is
// the same in any order).
template <int NRC>
__device__ __forceinline__ void stage_dots(const uint32_t* __restrict__ blk, const uint2* const (&act)[8], int lane,
                                           int (&dot)[8]) {
    int dl[NRC], dh[NRC];
#pragma unroll
    for (int i = 0; i < NRC; ++i) dl[i] = dh[i] = 0;
#pragma unroll 8
    for (int j = 0; j < 32; ++j) {
        const uint32_t w = blk[j * 32 + lane];
        const int lo = int(w & 0x0f0f0f0fu), hi = int((w >> 4) & 0x0f0f0f0fu);
#pragma unroll
        for (int i = 0; i < NRC; ++i) {
            const uint2 av = act[i][j];
            dl[i] = __dp4a(lo, int(av.x), dl[i]);
            dh[i] = __dp4a(hi, int(av.y), dh[i]);
        }
    }
#pragma unroll
    for (int i = 0; i < NRC; ++i) dot[i] = dl[i] + dh[i];
}
// n routes (1..8): act[i] for i >= n repeats a valid row and its dot is unused.
__device__ __forceinline__ void stage_dots_n(int n, const uint32_t* blk, const uint2* const (&act)[8], int lane,
                                             int (&dot)[8]) {
    if (n == 1) stage_dots<1>(blk, act, lane, dot);
    else if (n == 2) stage_dots<2>(blk, act, lane, dot);
    else if (n <= 4) stage_dots<4>(blk, act, lane, dot);
    else stage_dots<8>(blk, act, lane, dot);
}

// Transform + quantise one 256-group of one token into the given destination.
template <int QMAX>
__device__ void quant_token_group(const LayerArgs& a, int t, int g, int lane, uint2* q, __half* hs, float* fs,
                                  int32_t* sum, uint32_t& f, bool report) {
    bool live = a.shared_all_live;
    if (!live)
        for (int sl = 0; sl < kTop; ++sl) live |= id_valid(a.ids[t * kTop + sl]);
    float e[8];
    uint32_t lf = 0;
    if (live) {
        uint4 raw = *reinterpret_cast<const uint4*>(a.x + size_t(t) * kH + g * kG + lane * 8);
        uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            e[2 * i] = __uint_as_float(w4[i] << 16);
            e[2 * i + 1] = __uint_as_float(w4[i] & 0xffff0000u);
        }
#pragma unroll
        for (int s = 0; s < 8; ++s)
            if (!isfinite(e[s])) lf |= kFlagNonfiniteInput;
        wht128_halfwarp(e, lane);
#pragma unroll
        for (int s = 0; s < 8; ++s)
            if (!isfinite(e[s])) lf |= kFlagNonfiniteInput;
    } else {
#pragma unroll
        for (int s = 0; s < 8; ++s) e[s] = 0.f;
    }
    __half scale;
    int32_t gsum;
    uint32_t qf = 0;
    quantize_group_warp<QMAX>(e, lane, q, &scale, &gsum, qf);
    if (lane == 0) {
        if (hs) *hs = scale;
        if (fs) *fs = __half2float(scale);
        *sum = gsum;
    }
    if (live && report) f |= lf | qf;
}

template <int QMAX>
__global__ void __launch_bounds__(kThreads, 1) decode_layer_kernel(const LayerArgs a, const int nst) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const Carve cv = carve(a.T, nst);
    Smem s;
    s.ring = smem_raw + cv.ring;
    s.full = reinterpret_cast<uint64_t*>(smem_raw + cv.full);
    s.empty = reinterpret_cast<uint64_t*>(smem_raw + cv.empty);
    s.xq = smem_raw + cv.xq;
    s.xs = reinterpret_cast<float*>(smem_raw + cv.xs);
    s.xsum = reinterpret_cast<int*>(smem_raw + cv.xsum);
    s.ids = reinterpret_cast<int*>(smem_raw + cv.ids);
    s.cnt = reinterpret_cast<int*>(smem_raw + cv.cnt);
    s.off = reinterpret_cast<int*>(smem_raw + cv.off);
    s.act_e = reinterpret_cast<int*>(smem_raw + cv.act_e);
    s.act_off = reinterpret_cast<int*>(smem_raw + cv.act_off);
    s.act_cnt = reinterpret_cast<int*>(smem_raw + cv.act_cnt);
    s.routes = reinterpret_cast<int*>(smem_raw + cv.routes);
    s.pairbuf = reinterpret_cast<float*>(smem_raw + cv.pairbuf);
    s.dbuf = smem_raw + cv.dbuf;
    s.dscale = reinterpret_cast<float*>(smem_raw + cv.dscale);
    s.dsum = reinterpret_cast<int*>(smem_raw + cv.dsum);
    s.misc = reinterpret_cast<int*>(smem_raw + cv.misc);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int T = a.T, R = T * kTop, G = gridDim.x, b = blockIdx.x;
    uint32_t* ctrl = ws_at<uint32_t>(a, a.L.ctrl);

    // ---- routing plan (every CTA, identical) ------------------------------
    if (tid == 0) {
        for (int i = 0; i < nst; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], 1);
        }
        fence_barrier_init();
        s.misc[0] = 0;
        s.misc[1] = 0x7fffffff;
        s.misc[4] = 0;  // stages issued so far (published by the producer)
    }
    for (int e = tid; e <= kE; e += kThreads) s.cnt[e] = 0;
    for (int r = tid; r < R; r += kThreads) s.ids[r] = a.ids[r];
    __syncthreads();
    {
        uint32_t f = 0;
        for (int r = tid; r < R; r += kThreads) {
            const int e = s.ids[r];
            if (id_valid(e)) atomicAdd(&s.cnt[e], 1);
            else if (e != -1) f |= kFlagInvalidId;
        }
        if (b == 0) warp_flag_or(a.flags, f);
    }
    __syncthreads();
    if (warp == 0) {
        int c[8], tot = 0, nz = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            c[i] = s.cnt[8 * lane + i];
            tot += c[i];
            nz += c[i] > 0;
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
            if (c[i] > 0) {
                s.act_e[k] = e;
                s.act_off[k] = run;
                s.act_cnt[k] = c[i];
                ++k;
            }
            run += c[i];
        }
        if (lane == 31) {
            int nact = in;
            if (a.shared) {
                s.act_e[nact] = kE;
                s.act_off[nact] = it;
                s.act_cnt[nact] = T;
            }
            s.misc[2] = nact;
            s.misc[3] = nact + (a.shared ? 1 : 0);
        }
    }
    __syncthreads();
    for (int r = tid; r < R; r += kThreads) {
        const int e = s.ids[r];
        if (id_valid(e)) {
            int rank = 0;
            for (int q = 0; q < r; ++q) rank += s.ids[q] == e;
            s.routes[s.off[e] + rank] = r;
        }
    }
    if (a.shared) {
        const int base = s.act_off[s.misc[2]];
        for (int t = tid; t < T; t += kThreads) s.routes[base + t] = R + t;
    }
    __syncthreads();

    const int NA = s.misc[3];
    const int NGI = NA * 16, NDI = NA * 64;
    const int ng = NGI > b ? (NGI - 1 - b) / G + 1 : 0;
    const int jstart = ((b - NGI) % G + G) % G;
    const int nd = NDI > jstart ? (NDI - 1 - jstart) / G + 1 : 0;
    const int total_stages = 16 * ng + 2 * nd;

    if (warp == kNCW) {
        // ---- producer ------------------------------------------------------
        if (lane == 0) {
            int st = 0;
            for (; st < total_stages; ++st) {
                volatile int* misc = s.misc;
                if (misc[0]) break;
                const int slot = st % nst;
                if (st >= nst) {
                    const uint32_t parity = uint32_t(st / nst - 1) & 1u;
                    uint64_t t0 = now_ns();
                    bool ok = true;
                    while (!mbar_try_wait(&s.empty[slot], parity)) {
                        if (misc[0] || now_ns() - t0 > kTimeoutNs) {
                            ok = false;
                            break;
                        }
                    }
                    if (!ok) {
                        if (!misc[0]) give_up(a, s, ctrl, 2u, uint32_t(st), uint32_t(slot), 0u);
                        break;
                    }
                }
                int k, tile, g;
                bool gate;
                if (st < 16 * ng) {
                    const int item = st / 16, within = st % 16;
                    const int gi = b + item * G;
                    k = gi / 16;
                    g = within / 2;
                    tile = gi % 16 + 16 * (within & 1);
                    gate = true;
                } else {
                    const int d = (st - 16 * ng) / 2;
                    const int dj = jstart + d * G;
                    k = dj / 64;
                    tile = dj % 64;
                    g = (st - 16 * ng) % 2;
                    gate = false;
                }
                const int e = s.act_e[k];
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
                __threadfence_block();
                misc[4] = st + 1;
            }
            atomicExch(&s.misc[1], st);  // stages actually issued
        }
        return;
    }

    // ---- consumers: token activations ------------------------------------
    uint32_t f = 0;
    const bool report = b == 0;
    if (NA == 0) {
        // every slot padded and no shared expert: the output is zero
        if (b == 0)
            for (int i = tid; i < T * kH; i += kNCW * 32) {
                a.out[i] = 0;
                ws_at<float>(a, a.L.final_f32)[i] = 0.f;
            }
        return;
    }
    if (T <= kRedundantX) {
        for (int q = warp; q < T * 8; q += kNCW) {
            const int t = q / 8, g = q % 8;
            quant_token_group<QMAX>(a, t, g, lane, reinterpret_cast<uint2*>(s.xq + size_t(t) * kH + g * kG), nullptr,
                                    s.xs + t * 8 + g, s.xsum + t * 8 + g, f, report);
        }
        named_barrier(15, kNCW * 32);
    } else {
        for (int q = b + G * warp; q < T * 8; q += G * kNCW) {
            const int t = q / 8, g = q % 8;
            uint2* gq = ws_at<uint2>(a, a.L.xq) + (size_t(t) * kH + g * kG) / 8;
            quant_token_group<QMAX>(a, t, g, lane, gq, ws_at<__half>(a, a.L.xs) + t * 8 + g, nullptr,
                                    ws_at<int32_t>(a, a.L.xsum) + t * 8 + g, f, true);
            __syncwarp();
            if (lane == 0) {
                __threadfence();
                atomicAdd(ctrl + kCtrlXDone, 1u);
            }
        }
        if (ng > 0) {
            if (warp == 0) wait_counter(a, s, ctrl, ctrl + kCtrlXDone, uint32_t(T * 8));
            named_barrier(15, kNCW * 32);
            __threadfence();
            const uint4* src = reinterpret_cast<const uint4*>(ws_at<uint8_t>(a, a.L.xq));
            uint4* dst = reinterpret_cast<uint4*>(s.xq);
            for (int i = tid; i < T * kH / 16; i += kNCW * 32) dst[i] = __ldcg(src + i);
            for (int i = tid; i < T * 8; i += kNCW * 32) {
                s.xs[i] = __half2float(__ldcg(ws_at<__half>(a, a.L.xs) + i));
                s.xsum[i] = __ldcg(ws_at<int32_t>(a, a.L.xsum) + i);
            }
            named_barrier(15, kNCW * 32);
        }
    }

    float* const route_out_base = ws_at<float>(a, a.L.route_out);
    auto spill_row = [&](int route) { return route_out_base + size_t(route) * kH; };

    // ---- gate items (warp pairs) ------------------------------------------
    {
        const int pair = warp >> 1, role = warp & 1;
        float* xbuf = s.pairbuf + size_t(pair) * kMaxR * 32;
        for (int item = pair; item < ng; item += kNP) {
            const int gi = b + item * G, k = gi / 16, p = gi % 16;
            const int nr = s.act_cnt[k], roff = s.act_off[k];
            const bool shared = s.act_e[k] == kE;
            float acc[kMaxR];
#pragma unroll
            for (int r = 0; r < kMaxR; ++r) acc[r] = 0.f;
            bool alive = true;
            for (int g = 0; g < 8; ++g) {
                const int st = 16 * item + 2 * g + role;
                if (alive && !wait_stage(a, s, ctrl, st, nst)) alive = false;
                if (alive) {
                    const uint32_t* blk = reinterpret_cast<const uint32_t*>(s.ring + size_t(st % nst) * kStageBytes);
                    const uint32_t mw = blk[1024 + lane];
                    const int nchunks = (nr + 7) / 8;
                    for (int c = 0; c < nchunks; ++c) {
                        const int n = min(8, nr - c * 8);
                        const uint2* act[8];
                        float sa[8];
                        int sm[8], dot[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int ri = c * 8 + (i < n ? i : n - 1);
                            const int tok = token_of(s.routes[roff + ri], R);
                            act[i] = reinterpret_cast<const uint2*>(s.xq + size_t(tok) * kH + g * kG);
                            sa[i] = s.xs[tok * 8 + g];
                            sm[i] = s.xsum[tok * 8 + g];
                        }
                        stage_dots_n(n, blk, act, lane, dot);
                        if (c < kMaxR / 8) {
#pragma unroll
                            for (int cc = 0; cc < kMaxR / 8; ++cc) {
                                if (cc == c) {
#pragma unroll
                                    for (int i = 0; i < 8; ++i)
                                        if (c * 8 + i < nr)
                                            acc[cc * 8 + i] = __fadd_rn(acc[cc * 8 + i], group_term(sa[i], dot[i], sm[i], mw));
                                }
                            }
                        } else {
                            // routes beyond the register budget (duplicate expert ids in a
                            // token): accumulate in the route's route_out row, which is free
                            // until this expert's down items run
#pragma unroll
                            for (int i = 0; i < 8; ++i) {
                                if (c * 8 + i < nr) {
                                    float* ap = spill_row(s.routes[roff + c * 8 + i]) + role * kI + p * 32 + lane;
                                    const float prev = g == 0 ? 0.f : *ap;
                                    *ap = __fadd_rn(prev, group_term(sa[i], dot[i], sm[i], mw));
                                }
                            }
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&s.empty[st % nst]);
                }
            }
            // up tile -> partner; SiLU*up by the gate-tile warp
            if (role == 1) {
#pragma unroll
                for (int r = 0; r < kMaxR; ++r)
                    if (r < nr) xbuf[r * 32 + lane] = acc[r];
            }
            __threadfence_block();
            named_barrier(1 + pair, 64);
            if (role == 0 && alive) {
                float* middle = ws_at<float>(a, a.L.middle);
#pragma unroll
                for (int r = 0; r < kMaxR; ++r) {
                    if (r < nr) {
                        float gv = acc[r], uv = xbuf[r * 32 + lane], value;
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
                        middle[size_t(s.routes[roff + r]) * kI + p * 32 + lane] = value;
                    }
                }
                for (int r = kMaxR; r < nr; ++r) {
                    const float* row = spill_row(s.routes[roff + r]);
                    const float gv = row[p * 32 + lane], uv = row[kI + p * 32 + lane];
                    if (!isfinite(gv) || !isfinite(uv)) f |= kFlagNonfiniteProjection;
                    const float value = silu_mul(gv, uv);
                    if (!isfinite(value)) f |= kFlagNonfiniteMiddle;
                    middle[size_t(s.routes[roff + r]) * kI + p * 32 + lane] = value;
                }
            }
            named_barrier(1 + pair, 64);
            if (role == 0 && alive) {
                __syncwarp();
                uint32_t old = 0;
                if (lane == 0) {
                    __threadfence();
                    old = atomicAdd(ctrl + kCtrlGateDone + k, 1u);
                }
                old = __shfl_sync(0xffffffffu, old, 0);
                if (old == 15) {
                    // last gate item of this expert slot: quantise its middle rows
                    __threadfence();
                    const float* middle = ws_at<float>(a, a.L.middle);
                    for (int q = 0; q < nr * 2; ++q) {
                        const int route = s.routes[roff + q / 2], g = q % 2;
                        const float* src = middle + size_t(route) * kI + g * kG + lane * 8;
                        float4 v0 = ldcg4(src), v1 = ldcg4(src + 4);
                        float e[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            if (!isfinite(e[i])) f |= kFlagNonfiniteInput;
                        wht128_halfwarp(e, lane);
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            if (!isfinite(e[i])) f |= kFlagNonfiniteInput;
                        uint2* mq = ws_at<uint2>(a, a.L.mq) + (size_t(route) * kI + g * kG) / 8;
                        quantize_group_warp<QMAX>(e, lane, mq, ws_at<__half>(a, a.L.ms) + route * 2 + g,
                                                  ws_at<int32_t>(a, a.L.msum) + route * 2 + g, f);
                    }
                    __syncwarp();
                    if (lane == 0) {
                        __threadfence();
                        st_release(ctrl + kCtrlReady + k, 1u);
                    }
                }
            }
        }
    }

    // ---- down items ------------------------------------------------------
    {
        uint8_t* dbuf = s.dbuf + size_t(warp) * kChunk * 512;
        float* dsc = s.dscale + warp * kChunk * 2;
        int* dsm = s.dsum + warp * kChunk * 2;
        for (int item = warp; item < nd; item += kNCW) {
            const int dj = jstart + item * G, k = dj / 64, tile = dj % 64;
            const int nr = s.act_cnt[k], roff = s.act_off[k];
            const bool shared = s.act_e[k] == kE;
            bool alive = wait_counter(a, s, ctrl, ctrl + kCtrlReady + k, 1u);
            if (alive) __threadfence();
            float acc[kMaxR];
#pragma unroll
            for (int r = 0; r < kMaxR; ++r) acc[r] = 0.f;
            auto load_chunk = [&](int c) {
                const int n = min(kChunk, nr - c * kChunk);
                for (int i = lane; i < n * 32; i += 32) {
                    const int ri = i / 32, part = i % 32;
                    const int route = s.routes[roff + c * kChunk + ri];
                    reinterpret_cast<uint4*>(dbuf + ri * 512)[part] =
                        __ldcg(reinterpret_cast<const uint4*>(ws_at<uint8_t>(a, a.L.mq) + size_t(route) * kI) + part);
                }
                if (lane < n * 2) {
                    const int route = s.routes[roff + c * kChunk + lane / 2];
                    dsc[lane] = __half2float(__ldcg(ws_at<__half>(a, a.L.ms) + route * 2 + lane % 2));
                    dsm[lane] = __ldcg(ws_at<int32_t>(a, a.L.msum) + route * 2 + lane % 2);
                }
                __syncwarp();
            };
            const int nchunks = (nr + kChunk - 1) / kChunk;
            if (alive && nchunks == 1) load_chunk(0);
            for (int g = 0; g < 2; ++g) {
                const int st = 16 * ng + 2 * item + g;
                if (alive && !wait_stage(a, s, ctrl, st, nst)) alive = false;
                if (!alive) continue;
                const uint32_t* blk = reinterpret_cast<const uint32_t*>(s.ring + size_t(st % nst) * kStageBytes);
                const uint32_t mw = blk[1024 + lane];
                for (int c = 0; c < nchunks; ++c) {
                    if (nchunks > 1) {
                        __syncwarp();
                        load_chunk(c);
                    }
                    const int n = min(kChunk, nr - c * kChunk);
                    const uint2* act[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        act[i] = reinterpret_cast<const uint2*>(dbuf + (i < n ? i : n - 1) * 512 + g * kG);
                    int dot[8];
                    stage_dots_n(n, blk, act, lane, dot);
                    if (c < kMaxR / kChunk) {
#pragma unroll
                        for (int cc = 0; cc < kMaxR / kChunk; ++cc) {
                            if (cc == c) {
#pragma unroll
                                for (int i = 0; i < kChunk; ++i)
                                    if (c * kChunk + i < nr)
                                        acc[cc * kChunk + i] = __fadd_rn(
                                            acc[cc * kChunk + i], group_term(dsc[i * 2 + g], dot[i], dsm[i * 2 + g], mw));
                            }
                        }
                    } else {
                        // routes beyond the register budget: accumulate in route_out directly
#pragma unroll
                        for (int i = 0; i < kChunk; ++i) {
                            if (c * kChunk + i < nr) {
                                float* ap = spill_row(s.routes[roff + c * kChunk + i]) + tile * 32 + lane;
                                const float prev = g == 0 ? 0.f : *ap;
                                const float v = __fadd_rn(prev, group_term(dsc[i * 2 + g], dot[i], dsm[i * 2 + g], mw));
                                *ap = v;
                                if (g == 1 && !isfinite(v)) f |= kFlagNonfiniteProjection;
                            }
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&s.empty[st % nst]);
            }
            if (!alive) continue;
            float* route_out = ws_at<float>(a, a.L.route_out);
#pragma unroll
            for (int r = 0; r < kMaxR; ++r) {
                if (r < nr) {
                    float v = shared ? bf16_round_f32(acc[r]) : acc[r];
                    if (!isfinite(v)) f |= kFlagNonfiniteProjection;
                    route_out[size_t(s.routes[roff + r]) * kH + tile * 32 + lane] = v;
                }
            }
            __syncwarp();
            uint32_t old = 0;
            if (lane == 0) {
                __threadfence();
                old = atomicAdd(ctrl + kCtrlColDone + tile, 1u);
            }
            old = __shfl_sync(0xffffffffu, old, 0);
            if (old == uint32_t(NA - 1)) {
                // last expert of this output tile: slot-ordered combine (reduce_slots :176-185)
                __threadfence();
                const float* ro = ws_at<float>(a, a.L.route_out);
                float* fin = ws_at<float>(a, a.L.final_f32);
                const int c = tile * 32 + lane;
                for (int t = 0; t < T; ++t) {
                    float sum = 0.f;
#pragma unroll
                    for (int sl = 0; sl < kTop; ++sl) {
                        const int r = t * kTop + sl;
                        if (id_valid(s.ids[r])) sum = __fadd_rn(sum, __fmul_rn(__ldcg(ro + size_t(r) * kH + c), a.weights[r]));
                    }
                    const uint16_t res = bf16_rne(sum);
                    fin[size_t(t) * kH + c] = sum;
                    a.out[size_t(t) * kH + c] = res;
                    if (!isfinite(sum) || (res & 0x7f80u) == 0x7f80u) f |= kFlagNonfiniteOutput;
                    if (a.shared) {
                        const float gate = bf16_to_f32(a.sigmoid_table[a.shared_logit[t]]);
                        const float sh = __fmul_rn(__ldcg(ro + size_t(R + t) * kH + c), gate);
                        a.shared_out[size_t(t) * kH + c] = bf16_rne(sh);
                        if (!isfinite(sh)) f |= kFlagNonfiniteOutput;
                    }
                }
            }
        }
    }
    warp_flag_or(a.flags, f);
}

struct DeviceConfig {
    int sms = 0;
    int max_smem = 0;
    bool attr_set[2] = {false, false};
};
DeviceConfig g_dev[64];

}  // namespace

bool decode_supported(int T) { return T >= 1 && T <= kDecodeMaxT; }

cudaError_t launch_decode(const LayerArgs& a, cudaStream_t stream) {
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
    // ring depth: as many stages as fit next to the fixed carve, at most 48
    const Carve fixed = carve(a.T, 0);
    int nst = int((size_t(dc.max_smem) - fixed.total - 1024) / (kStageBytes + 16));
    nst = nst > 48 ? 48 : nst;
    if (nst < kNCW + 2) return cudaErrorInvalidConfiguration;
    const size_t smem = carve(a.T, nst).total;
    const int which = a.a8 ? 0 : 1;
    auto kernel = a.a8 ? decode_layer_kernel<127> : decode_layer_kernel<7>;
    if (!dc.attr_set[which]) {
        if ((st = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dc.max_smem)) != cudaSuccess)
            return st;
        dc.attr_set[which] = true;
    }
    if ((st = cudaMemsetAsync(a.ws + a.L.ctrl, 0, kCtrlClearWords * sizeof(uint32_t), stream)) != cudaSuccess)
        return st;
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
