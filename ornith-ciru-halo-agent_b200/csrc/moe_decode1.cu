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
// One cooperative launch of one CTA per SM (148 on B200), 9 warps:
//  * every CTA routes the token itself (top-8 of the logits, or the caller's
//    ids) and builds the same plan: slot 0 is the shared expert when present,
//    then the distinct routed experts in slot order (an expert named by
//    several slots is one plan slot whose routes share every value, since
//    they see the same token);
//  * gate item (slot k, tile pair p) -> CTA 16k + p: gate tile p and up tile
//    p + 16 over the 8 K-groups (66 KB), warp g takes K-group g; warp 0 sums
//    the eight group terms in order, applies SiLU*up and stores the slot's 32
//    middle columns, then raises the item's flag;
//  * output tile t (32 columns) -> CTA G-1-t, for every slot (the down
//    blocks of all slots, up to 76 KB): the CTA waits for every gate item's
//    flag, transforms and quantises each slot's middle row itself, computes
//    the tile's down projection of every slot and performs the slot-ordered
//    combine of the tile locally;
//  * the copy warp issues all of the CTA's weight blocks with cp.async.bulk
//    right after routing (the shared expert's, which need no routing, before
//    it), so at most one K-group's latency stands between the copies and the
//    compute.  No cluster multicast.
// Flags between CTAs carry a call number instead of being cleared: every CTA
// reads the last completed call's number from the workspace and uses the next
// one, and CTA 0 publishes it once every CTA has read it.  No separate clear
// launch is needed and stale words of earlier calls never match.
// Every wait is bounded (about one second of %globaltimer), after which the
// kernel raises flag 64, lets its issued copies land and returns.
#include <cstdlib>
#include <cstring>

#include "moe_layer.cuh"

namespace ornith {
namespace {

constexpr int kD1Warps = 9;                 // warps 0..7 compute, warp 8 routes and issues the copies
constexpr int kD1Threads = kD1Warps * 32;
constexpr int kD1Copier = 8;
constexpr int kD1Compute = 8 * 32;          // threads of the compute warps (named barrier 1)
constexpr int kBlkBytes = 4096 + 128;       // one (tile, 256-group) block: 32x32 code words + 32 metadata words
constexpr int kD1Slots = kTop + 1;          // eight routed experts and the shared expert
constexpr int kD1GateItems = kD1Slots * 16;
constexpr int kD1DownCtas = kH / 32;        // one per 32-column output tile
constexpr uint64_t kD1WaitNs = 1000000000ull;
static_assert(kD1GateItems <= 9 * 16, "gate flags fit their control words");

struct __align__(128) D1Smem {
    uint8_t gate[8][2][kBlkBytes];          // gate item: K-group g; [0] gate tile p, [1] up tile p + 16
    uint8_t down[kD1Slots][2][kBlkBytes];   // this CTA's output tile of every slot, K-groups 0 and 1
    uint8_t xq[kH];                         // the token's activations, permuted int8
    uint8_t mq[kD1Slots][2][kG];            // every slot's middle activations
    float terms[8][2][32];                  // gate item: group terms of gate and up
    float sout[kD1Slots][32];               // this tile's down projection of every slot
    uint64_t gbar[8];
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
    uint32_t issued;                        // bits 0..7: gate barriers issued, 8 + k: down barrier k issued
    int32_t abort;
    uint16_t logit;
};

__device__ __forceinline__ uint64_t d1_now() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void d1_barrier() { asm volatile("bar.sync 1, %0;" ::"r"(kD1Compute) : "memory"); }

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

__device__ __forceinline__ void copy_block(uint8_t* dst, const uint32_t* codes, const uint32_t* meta, uint64_t* bar) {
    bulk_g2s(dst, codes, 4096, bar);
    bulk_g2s(dst + 4096, meta, 128, bar);
}

// Gate item of expert e (kE: shared), tile pair p, K-group g (the calling lane).
__device__ __forceinline__ void issue_gate_group(const LayerArgs& a, D1Smem& S, int e, int p, int g) {
    const uint32_t* codes = e == kE ? a.sgate_codes : a.gate_codes + size_t(e) * (2 * kI) * (kH / 8);
    const uint32_t* meta = e == kE ? a.sgate_meta : a.gate_meta + size_t(e) * (2 * kI) * (kH / kG);
    mbar_arrive_expect_tx(&S.gbar[g], 2 * kBlkBytes);
    copy_block(S.gate[g][0], codes + size_t(p * 8 + g) * 1024, meta + size_t(p * 8 + g) * 32, &S.gbar[g]);
    copy_block(S.gate[g][1], codes + size_t((p + 16) * 8 + g) * 1024, meta + size_t((p + 16) * 8 + g) * 32, &S.gbar[g]);
}

// Down blocks of expert e for output tile `tile` into plan slot k.
__device__ __forceinline__ void issue_down_slot(const LayerArgs& a, D1Smem& S, int e, int k, int tile) {
    const uint32_t* codes = e == kE ? a.sdown_codes : a.down_codes + size_t(e) * kH * (kI / 8);
    const uint32_t* meta = e == kE ? a.sdown_meta : a.down_meta + size_t(e) * kH * (kI / kG);
    mbar_arrive_expect_tx(&S.dbar[k], 2 * kBlkBytes);
    copy_block(S.down[k][0], codes + size_t(tile * 2) * 1024, meta + size_t(tile * 2) * 32, &S.dbar[k]);
    copy_block(S.down[k][1], codes + size_t(tile * 2 + 1) * 1024, meta + size_t(tile * 2 + 1) * 32, &S.dbar[k]);
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

template <int QMAX>
__global__ void __launch_bounds__(kD1Threads, 1) decode_single_kernel(const LayerArgs a) {
    extern __shared__ __align__(128) uint8_t d1_raw[];
    D1Smem& S = *reinterpret_cast<D1Smem*>(d1_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int b = blockIdx.x, G = gridDim.x;
    uint32_t* ctrl = ws_at<uint32_t>(a, a.L.ctrl);
    const bool is_down = b >= G - kD1DownCtas;
    const int tile = G - 1 - b;  // output tile of a down CTA
    uint32_t f = 0;

    if (tid == 0) {
        for (int i = 0; i < 8; ++i) mbar_init(&S.gbar[i], 1);
        for (int i = 0; i < kD1Slots; ++i) mbar_init(&S.dbar[i], 1);
        fence_barrier_init();
        S.abort = 0;
        S.issued = 0;
        uint32_t tag = *reinterpret_cast<const volatile uint32_t*>(ctrl + kCtrlD1Epoch) + 1u;
        if (tag == 0u) tag = 1u;  // 0 never tags a call, so never-written words never match
        S.tag = tag;
        st_release(ctrl + kCtrlD1Seen + b, tag);  // after the read above: the epoch may advance
    }
    __syncthreads();

    if (warp == kD1Copier) {
        // the shared expert's blocks need no routing: issued first
        if (a.shared) {
            if (b < 16 && lane < 8) issue_gate_group(a, S, kE, b, lane);
            if (is_down && lane == 8) issue_down_slot(a, S, kE, 0, tile);
        }
        // router top-8 (from logits) or the caller's ids, then the plan
        uint32_t rf = 0;
        if (a.logits) {
            route_topk_warp(a.logits, lane, S.ids, S.wts, rf);
        } else if (lane < kTop) {
            S.ids[lane] = a.ids[lane];
            S.wts[lane] = a.weights[lane];
        }
        __syncwarp();
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
        if (lane == 0) {
            if (a.shared) S.act_e[0] = kE;
            S.nslot = base + __popc(heads);
        }
        if (b == 0) d1_flag_or(a.flags, rf);  // routing and id flags, once
    } else {
        // the token's 256-groups: warp g transforms and quantises group g
        const uint4 raw = *reinterpret_cast<const uint4*>(a.x + warp * kG + lane * 8);
        uint32_t qf = wht_quant<QMAX>(
            __uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xffff0000u), __uint_as_float(raw.y << 16),
            __uint_as_float(raw.y & 0xffff0000u), __uint_as_float(raw.z << 16), __uint_as_float(raw.z & 0xffff0000u),
            __uint_as_float(raw.w << 16), __uint_as_float(raw.w & 0xffff0000u), lane,
            reinterpret_cast<uint2*>(S.xq + warp * kG), S.xs + warp, S.xsum + warp);
        qf = __reduce_or_sync(0xffffffffu, qf);
        if (lane == 0) S.xflag[warp] = qf;
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
        // the routed experts' blocks of this CTA
        if (has_gate && !(a.shared && gk == 0) && lane < 8)
            issue_gate_group(a, S, checked(S.act_e[gk], kE + 1, a.flags), gp, lane);
        const int base = a.shared ? 1 : 0;
        if (is_down && lane >= 8 + base && lane < 8 + NA)
            issue_down_slot(a, S, checked(S.act_e[lane - 8], kE + 1, a.flags), lane - 8, tile);
        if (lane == 0) S.issued = (has_gate ? 0xffu : 0u) | (is_down ? ((1u << NA) - 1u) << 8 : 0u);
    } else if (NA == 0) {
        // every slot padded and no shared expert: the output is zero
        if (b == 0)
            for (int i = tid; i < kH; i += kD1Compute) {
                a.out[i] = 0;
                ws_at<float>(a, a.L.final_f32)[i] = 0.f;
            }
    } else {
        float* const middle = ws_at<float>(a, a.L.middle);
        // ---- gate item (slot gk, tile pair gp): warp g = K-group g ----------
        if (has_gate) {
            const int g = warp;
            if (d1_wait_copies(&S.gbar[g], &S.abort)) {
                const uint32_t* bg = reinterpret_cast<const uint32_t*>(S.gate[g][0]);
                const uint32_t* bu = reinterpret_cast<const uint32_t*>(S.gate[g][1]);
                const uint4* act = reinterpret_cast<const uint4*>(S.xq + g * kG);
                const int dg = block_dot(bg, act, lane), du = block_dot(bu, act, lane);
                const float sa = __half2float(S.xs[g]);
                const int sm = S.xsum[g];
                S.terms[g][0][lane] = group_term(sa, dg, sm, bg[1024 + lane]);
                S.terms[g][1][lane] = group_term(sa, du, sm, bu[1024 + lane]);
            } else if (lane == 0) {
                d1_give_up(S, a.flags);
            }
            d1_barrier();
            if (warp == 0 && !S.abort) {
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
                middle[size_t(gk) * kI + gp * 32 + lane] = value;
                __syncwarp();
                if (lane == 0) st_release(ctrl + kCtrlD1Gate + b, tag);  // the slot's 32 middle columns are out
            }
        }
        // ---- output tile: every slot's down projection, then the combine ----
        if (is_down) {
            if (a.shared && a.shared_gate_weight && warp == 7) {
                const uint16_t v = shared_logit_warp(a.x, a.shared_gate_weight, lane);
                if (lane == 0) {
                    S.logit = v;
                    if (tile == 0) a.logit_out[0] = v;
                }
            }
            if (warp == 0) {
                // every gate item's middle columns (bounded wait)
                const int n = NA * 16;
                const uint64_t t0 = d1_now();
                for (;;) {
                    bool mine = true;
                    for (int i = lane; i < n; i += 32) mine &= ld_acquire(ctrl + kCtrlD1Gate + i) == tag;
                    if (__all_sync(0xffffffffu, mine)) break;
                    const bool stop = __shfl_sync(0xffffffffu, int(S.abort != 0 || d1_now() - t0 > kD1WaitNs), 0);
                    if (stop) {
                        if (lane == 0) d1_give_up(S, a.flags);
                        break;
                    }
                    __nanosleep(64);
                }
            }
            d1_barrier();  // orders every warp's reads after warp 0's acquires
            const bool alive = !*reinterpret_cast<const volatile int32_t*>(&S.abort);
            if (alive) {
                // transform + quantise each slot's middle row (one 256-group per task)
                for (int j = warp; j < NA * 2; j += 8) {
                    const int k = j >> 1, g = j & 1;
                    const float4* src = reinterpret_cast<const float4*>(middle + size_t(k) * kI + g * kG + lane * 8);
                    const float4 v0 = __ldcg(src), v1 = __ldcg(src + 1);
                    f |= wht_quant<QMAX>(v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w, lane,
                                         reinterpret_cast<uint2*>(S.mq[k][g]), &S.ms[k][g], &S.msum[k][g]);
                }
            }
            d1_barrier();
            for (int k = warp; alive && k < NA; k += 8) {
                if (!d1_wait_copies(&S.dbar[k], &S.abort)) {
                    if (lane == 0) d1_give_up(S, a.flags);
                    break;
                }
                float v = 0.f;  // (0 + group 0 term) + group 1 term
#pragma unroll
                for (int g = 0; g < 2; ++g) {
                    const uint32_t* blk = reinterpret_cast<const uint32_t*>(S.down[k][g]);
                    const int dot = block_dot(blk, reinterpret_cast<const uint4*>(S.mq[k][g]), lane);
                    v = __fadd_rn(v, group_term(__half2float(S.ms[k][g]), dot, S.msum[k][g], blk[1024 + lane]));
                }
                if (S.act_e[k] == kE) v = bf16_round_f32(v);
                if (!isfinite(v)) f |= kFlagNonfiniteProjection;
                S.sout[k][lane] = v;
            }
            d1_barrier();
            if (!*reinterpret_cast<const volatile int32_t*>(&S.abort)) {
                const int col = tile * 32 + lane;
                float* const route_out = ws_at<float>(a, a.L.route_out);
                if (warp < kTop) {
                    const int k = S.slot_of[warp];
                    if (k >= 0) route_out[size_t(warp) * kH + col] = S.sout[k][lane];
                }
                if (warp == 0 && a.shared) route_out[size_t(kTop) * kH + col] = S.sout[0][lane];
                if (warp == 1) {
                    // slot-ordered combine of the token (reduce_slots :176-185)
                    float sum = 0.f;
#pragma unroll
                    for (int sl = 0; sl < kTop; ++sl)
                        if (id_valid(S.ids[sl])) sum = __fadd_rn(sum, __fmul_rn(S.sout[S.slot_of[sl]][lane], S.wts[sl]));
                    const uint16_t res = bf16_rne(sum);
                    ws_at<float>(a, a.L.final_f32)[col] = sum;
                    a.out[col] = res;
                    if (!isfinite(sum) || (res & 0x7f80u) == 0x7f80u) f |= kFlagNonfiniteOutput;
                    if (a.shared) {
                        const uint16_t lg = a.shared_gate_weight ? S.logit : a.shared_logit[0];
                        const float gate = bf16_to_f32(a.sigmoid_table[lg]);
                        const float sh = __fmul_rn(S.sout[0][lane], gate);
                        a.shared_out[col] = bf16_rne(sh);
                        if (!isfinite(sh)) f |= kFlagNonfiniteOutput;
                    }
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
        for (int i = 0; i < 8 + kD1Slots; ++i) {
            if (!(S.issued >> i & 1u)) continue;
            uint64_t* bar = i < 8 ? &S.gbar[i] : &S.dbar[i - 8];
            while (!mbar_try_wait(bar, 0) && d1_now() - t0 < kD1WaitNs) {
            }
        }
    }
}

struct D1Device {
    int sms = 0;
    int max_smem = 0;
    bool attr_set[2] = {false, false};
};
D1Device g_d1[64];

// ORNITH_MOE_B200_DECODE1=0 sends single-token calls to the multi-token
// kernel instead (the tests compare the two).
bool single_disabled() {
    const char* v = getenv("ORNITH_MOE_B200_DECODE1");
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
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    count_launches(1);
    return cudaLaunchKernelEx(&cfg, kernel, a);
}

}  // namespace ornith
