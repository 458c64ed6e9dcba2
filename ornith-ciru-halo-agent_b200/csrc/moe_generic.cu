// Multi-kernel routed-MoE layer for any batch (T <= 8192).
//
// Stage order follows the reference's launch sequence
// (kernels/routed_storage/routed_storage_n32_consumer.cpp:329-347):
//   routing plan -> token transform+quantise -> gate/up projection fused with
//   SiLU*up -> middle transform+quantise -> down projection -> slot combine.
// The projections are CUDA-core __dp4a kernels (one block per expert and
// output tile, weight words read with 128-byte coalesced loads); the
// tensor-core prefill path replaces them for large batches.
#include "moe_layer.cuh"

namespace ornith {

Workspace workspace_layout(int Tcap) {
    Workspace w{};
    size_t cursor = 0, t = size_t(Tcap), rows = t * (kTop + 1);
    auto add = [&](size_t& field, size_t bytes) {
        field = cursor;
        cursor = (cursor + bytes + 255) & ~size_t(255);
    };
    add(w.xq, t * kH);
    add(w.xs, t * (kH / kG) * 2);
    add(w.xsum, t * (kH / kG) * 4);
    add(w.middle, rows * kI * 4);
    add(w.mq, rows * kI);
    add(w.ms, rows * (kI / kG) * 2);
    add(w.msum, rows * (kI / kG) * 4);
    add(w.route_out, rows * kH * 4);
    add(w.final_f32, t * kH * 4);
    add(w.counts, (kE + 1) * 4);
    add(w.offsets, (kE + 2) * 4);
    add(w.routes, rows * 4);
    add(w.cursors, (kE + 1) * 4);
    add(w.active, (kE + 2) * 4);
    add(w.ctrl, kCtrlWords * 4);
    add(w.topk_w, t * kTop * 4);
    add(w.topk_ids, t * kTop * 4);
    add(w.logit, t * 2);
    add(w.xchg, size_t(kTop + 1) * kI * 8);
    add(w.xlogit, size_t(kD1LogitCopies) * kE * 8);
    if (Tcap > kDecodeMaxT) {
        const size_t mt = (rows + 127) / 128 + (kE + 1);
        add(w.rowpos, rows * 4);
        add(w.slot_tiles, (kE + 2) * 4);
        add(w.mtiles, mt * 16);
        add(w.n_mtiles, 16);
        add(w.pblock, size_t(2) * kPlanBlocks * (kE + 1) * 4);
        add(w.agate, mt * 8 * 32768);
        add(w.agate_sa, mt * 8 * 128 * 4);
        add(w.agate_sum, mt * 8 * 128 * 4);
        add(w.adown, mt * 2 * 32768);
        add(w.adown_sa, mt * 2 * 128 * 4);
        add(w.adown_sum, mt * 2 * 128 * 4);
    }
    w.bytes = cursor;
    return w;
}

namespace {

__device__ __forceinline__ void flag_or(uint32_t* flags, uint32_t f) {
    // warp-aggregated sticky OR
    f = __reduce_or_sync(0xffffffffu, f);
    if (f && (threadIdx.x & 31) == 0) atomicOr(flags, f);
}

// Routing plan: counts per expert slot (slot E = shared expert, T rows),
// exclusive offsets, and the route list grouped by expert slot.  Routes of
// one expert may appear in any order: every route's output is independent.
// routed_storage_n32_prefill.h:19-42 (histogram, scan, scatter).
__global__ __launch_bounds__(1024) void plan_kernel(LayerArgs a) {
    __shared__ int counts[kE + 1];
    __shared__ int offsets[kE + 2];
    const int R = a.T * kTop;
    for (int e = threadIdx.x; e <= kE; e += blockDim.x) counts[e] = 0;
    __syncthreads();
    uint32_t f = 0;
    for (int r = threadIdx.x; r < R; r += blockDim.x) {
        int e = a.ids[r];
        if (id_valid(e)) atomicAdd(&counts[e], 1);
        else if (e != -1) f |= kFlagInvalidId;
    }
    flag_or(a.flags, f);
    __syncthreads();
    if (threadIdx.x == 0) {
        counts[kE] = a.shared ? a.T : 0;
        int total = 0;
        for (int e = 0; e <= kE; ++e) {
            offsets[e] = total;
            total += counts[e];
        }
        offsets[kE + 1] = total;
    }
    __syncthreads();
    int32_t* g_counts = ws_at<int32_t>(a, a.L.counts);
    int32_t* g_offsets = ws_at<int32_t>(a, a.L.offsets);
    int32_t* g_cursors = ws_at<int32_t>(a, a.L.cursors);
    int32_t* g_routes = ws_at<int32_t>(a, a.L.routes);
    for (int e = threadIdx.x; e <= kE; e += blockDim.x) {
        g_counts[e] = counts[e];
        g_offsets[e] = offsets[e];
        g_cursors[e] = 0;
    }
    if (threadIdx.x == 0) g_offsets[kE + 1] = offsets[kE + 1];
    __syncthreads();
    for (int r = threadIdx.x; r < R; r += blockDim.x) {
        int e = a.ids[r];
        if (id_valid(e)) {
            int slot = atomicAdd(reinterpret_cast<int*>(&counts[e]), -1) - 1;  // descending fill
            g_routes[checked(offsets[e] + slot, R + a.T, a.flags)] = r;
        }
    }
    if (a.shared)
        for (int t = threadIdx.x; t < a.T; t += blockDim.x) g_routes[offsets[kE] + t] = R + t;
}

// Token transform + quantise: one warp per (token, 256-group).
// transform<true> (:22-43) + quantize (:44-76); rows whose ids are all invalid
// are zero and unchecked unless every row is live (shared-slot semantics).
template <int QMAX>
__global__ __launch_bounds__(256) void quant_tokens_kernel(LayerArgs a) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int groups = kH / kG;
    if (warp >= a.T * groups) return;
    const int t = warp / groups, g = warp % groups;
    bool live = a.shared_all_live;
    if (!live)
        for (int s = 0; s < kTop; ++s) live |= id_valid(a.ids[t * kTop + s]);
    float e[8];
    uint32_t f = 0;
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
            if (!isfinite(e[s])) f |= kFlagNonfiniteInput;
        wht128_halfwarp(e, lane);
#pragma unroll
        for (int s = 0; s < 8; ++s)
            if (!isfinite(e[s])) f |= kFlagNonfiniteInput;
    } else {
#pragma unroll
        for (int s = 0; s < 8; ++s) e[s] = 0.f;
    }
    uint32_t qf = 0;
    uint2* q = ws_at<uint2>(a, a.L.xq) + (size_t(t) * kH + g * kG) / 8;
    quantize_group_warp<QMAX>(e, lane, q, ws_at<__half>(a, a.L.xs) + t * groups + g,
                              ws_at<int32_t>(a, a.L.xsum) + t * groups + g, qf);
    if (live) f |= qf;
    flag_or(a.flags, f);
}

// Gate/up projection fused with SiLU*up for one expert slot and one pair of
// 32-column tiles (gate tile p, up tile p+16).  Lane = column.  Per route and
// group: exact integer dot, then the reference epilogue in ascending group
// order (:138-159).  Shared-slot rows round gate/up to bf16, take SiLU from the
// table and round the product to bf16 (:225-228, :246-250).
__global__ __launch_bounds__(256) void gate_kernel(LayerArgs a) {
    const int p = blockIdx.x, slot = blockIdx.y;
    const int32_t* counts = ws_at<int32_t>(a, a.L.counts);
    const int32_t* offsets = ws_at<int32_t>(a, a.L.offsets);
    const int nr = counts[slot];
    if (nr == 0) return;
    const bool shared = slot == kE;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int groups = kH / kG;
    const uint32_t* codes = shared ? a.sgate_codes : a.gate_codes + size_t(slot) * (2 * kI) * (kH / 8);
    const uint32_t* meta = shared ? a.sgate_meta : a.gate_meta + size_t(slot) * (2 * kI) * groups;
    const int32_t* routes = ws_at<int32_t>(a, a.L.routes) + offsets[slot];
    const int R = a.T * kTop;
    const uint2* xq = ws_at<uint2>(a, a.L.xq);
    const __half* xs = ws_at<__half>(a, a.L.xs);
    const int32_t* xsum = ws_at<int32_t>(a, a.L.xsum);
    float* middle = ws_at<float>(a, a.L.middle);
    uint32_t f = 0;
    for (int i = warp; i < nr; i += nwarps) {
        const int route = checked(routes[i], R + a.T, a.flags);
        const int token = checked(route >= R ? route - R : route / kTop, a.T, a.flags);
        float acc[2] = {0.f, 0.f};
        for (int g = 0; g < groups; ++g) {
            const uint2* act = xq + (size_t(token) * kH + g * kG) / 8;
            const float sa = __half2float(xs[token * groups + g]);
            const int sum = xsum[token * groups + g];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int tile = p + 16 * h;
                const uint32_t* blk = codes + ((size_t(tile) * groups + g) * 32) * 32;
                int dot = 0;
#pragma unroll 8
                for (int j = 0; j < 32; ++j) dot = dot8(blk[j * 32 + lane], act[j], dot);
                uint32_t m = meta[(size_t(tile) * groups + g) * 32 + lane];
                acc[h] = __fadd_rn(acc[h], group_term(sa, dot, sum, m));
            }
        }
        float gv = acc[0], uv = acc[1], value;
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
        middle[size_t(route) * kI + p * 32 + lane] = value;
    }
    flag_or(a.flags, f);
}

// Middle transform + quantise: one warp per (row, 256-group) of the
// [R+T, 512] SiLU*up buffer (transform<false> + quantize, :344-345).
template <int QMAX>
__global__ __launch_bounds__(256) void quant_middle_kernel(LayerArgs a) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int R = a.T * kTop, rows = R + (a.shared ? a.T : 0), groups = kI / kG;
    if (warp >= rows * groups) return;
    const int row = warp / groups, g = warp % groups;
    if (row < R && !id_valid(a.ids[row])) return;
    const float4* src = reinterpret_cast<const float4*>(ws_at<float>(a, a.L.middle) + size_t(row) * kI + g * kG + lane * 8);
    float4 v0 = src[0], v1 = src[1];
    float e[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    uint32_t f = 0;
#pragma unroll
    for (int s = 0; s < 8; ++s)
        if (!isfinite(e[s])) f |= kFlagNonfiniteInput;
    wht128_halfwarp(e, lane);
#pragma unroll
    for (int s = 0; s < 8; ++s)
        if (!isfinite(e[s])) f |= kFlagNonfiniteInput;
    uint2* q = ws_at<uint2>(a, a.L.mq) + (size_t(row) * kI + g * kG) / 8;
    quantize_group_warp<QMAX>(e, lane, q, ws_at<__half>(a, a.L.ms) + row * groups + g,
                              ws_at<int32_t>(a, a.L.msum) + row * groups + g, f);
    flag_or(a.flags, f);
}

// Down projection for one expert slot and one 32-column output tile.
__global__ __launch_bounds__(256) void down_kernel(LayerArgs a) {
    const int tile = blockIdx.x, slot = blockIdx.y;
    const int32_t* counts = ws_at<int32_t>(a, a.L.counts);
    const int32_t* offsets = ws_at<int32_t>(a, a.L.offsets);
    const int nr = counts[slot];
    if (nr == 0) return;
    const bool shared = slot == kE;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int groups = kI / kG;
    const uint32_t* codes = shared ? a.sdown_codes : a.down_codes + size_t(slot) * kH * (kI / 8);
    const uint32_t* meta = shared ? a.sdown_meta : a.down_meta + size_t(slot) * kH * groups;
    const int32_t* routes = ws_at<int32_t>(a, a.L.routes) + offsets[slot];
    const uint2* mq = ws_at<uint2>(a, a.L.mq);
    const __half* ms = ws_at<__half>(a, a.L.ms);
    const int32_t* msum = ws_at<int32_t>(a, a.L.msum);
    float* route_out = ws_at<float>(a, a.L.route_out);
    uint32_t f = 0;
    for (int i = warp; i < nr; i += nwarps) {
        const int route = checked(routes[i], a.T * (kTop + 1), a.flags);
        float acc = 0.f;
        for (int g = 0; g < groups; ++g) {
            const uint2* act = mq + (size_t(route) * kI + g * kG) / 8;
            const uint32_t* blk = codes + ((size_t(tile) * groups + g) * 32) * 32;
            int dot = 0;
#pragma unroll 8
            for (int j = 0; j < 32; ++j) dot = dot8(blk[j * 32 + lane], act[j], dot);
            uint32_t m = meta[(size_t(tile) * groups + g) * 32 + lane];
            acc = __fadd_rn(acc, group_term(__half2float(ms[route * groups + g]), dot, msum[route * groups + g], m));
        }
        if (shared) acc = bf16_round_f32(acc);
        if (!isfinite(acc)) f |= kFlagNonfiniteProjection;
        route_out[size_t(route) * kH + tile * 32 + lane] = acc;
    }
    flag_or(a.flags, f);
}

// Slot-ordered weighted combine (reduce_slots :176-185, reduce_slots_shared :296-306).
// One CTA per token, eight columns per thread: every slot's row is read as
// one contiguous 8 KB burst (two float4 per thread, streamed past L1/L2).
// BY_POSITION: the rows of route_out are in slot-position order (the
// tensor-core path) and rowpos maps a route to its row.
template <bool BY_POSITION>
__global__ __launch_bounds__(256) void combine_kernel(LayerArgs a) {
    const int t = blockIdx.x, c = threadIdx.x * 8;
    const float* route_out = ws_at<float>(a, a.L.route_out);
    const int32_t* rowpos = BY_POSITION ? ws_at<int32_t>(a, a.L.rowpos) : nullptr;
    auto row_ptr = [&](int r) {
        const int row = BY_POSITION ? checked(rowpos[r], a.T * (kTop + 1), a.flags) : r;
        return reinterpret_cast<const float4*>(route_out + size_t(row) * kH + c);
    };
    uint32_t f = 0;
    float sum[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) sum[j] = 0.f;
#pragma unroll
    for (int s = 0; s < kTop; ++s) {
        const int r = t * kTop + s;
        if (!id_valid(a.ids[r])) continue;
        const float w = a.weights[r];
        const float4* src = row_ptr(r);
        const float4 v0 = __ldcs(src), v1 = __ldcs(src + 1);
        const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) sum[j] = __fadd_rn(sum[j], __fmul_rn(v[j], w));
    }
    const size_t index = size_t(t) * kH + c;
    uint32_t packed[4];
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
        const uint16_t lo = bf16_rne(sum[j]), hi = bf16_rne(sum[j + 1]);
        if (!isfinite(sum[j]) || (lo & 0x7f80u) == 0x7f80u) f |= kFlagNonfiniteOutput;
        if (!isfinite(sum[j + 1]) || (hi & 0x7f80u) == 0x7f80u) f |= kFlagNonfiniteOutput;
        packed[j / 2] = uint32_t(lo) | (uint32_t(hi) << 16);
    }
    float4* fin = reinterpret_cast<float4*>(ws_at<float>(a, a.L.final_f32) + index);
    fin[0] = make_float4(sum[0], sum[1], sum[2], sum[3]);
    fin[1] = make_float4(sum[4], sum[5], sum[6], sum[7]);
    *reinterpret_cast<uint4*>(a.out + index) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    if (a.shared) {
        const float gate = bf16_to_f32(a.sigmoid_table[a.shared_logit[t]]);
        const float4* src = row_ptr(a.T * kTop + t);
        const float4 v0 = __ldcs(src), v1 = __ldcs(src + 1);
        const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        uint32_t sp[4];
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
            const float s0 = __fmul_rn(v[j], gate), s1 = __fmul_rn(v[j + 1], gate);
            if (!isfinite(s0) || !isfinite(s1)) f |= kFlagNonfiniteOutput;
            sp[j / 2] = uint32_t(bf16_rne(s0)) | (uint32_t(bf16_rne(s1)) << 16);
        }
        *reinterpret_cast<uint4*>(a.shared_out + index) = make_uint4(sp[0], sp[1], sp[2], sp[3]);
    }
    flag_or(a.flags, f);
}

#define ORNITH_CHECK_LAUNCH()                       \
    do {                                            \
        cudaError_t s_ = cudaGetLastError();        \
        if (s_ != cudaSuccess) return s_;           \
    } while (0)

}  // namespace

cudaError_t launch_generic(const LayerArgs& a, cudaStream_t stream) {
    count_launches(5);
    const int R = a.T * kTop;
    const int rows = R + (a.shared ? a.T : 0);
    plan_kernel<<<1, 1024, 0, stream>>>(a);
    ORNITH_CHECK_LAUNCH();
    const int tok_warps = a.T * (kH / kG);
    if (a.a8) quant_tokens_kernel<127><<<(tok_warps + 7) / 8, 256, 0, stream>>>(a);
    else quant_tokens_kernel<7><<<(tok_warps + 7) / 8, 256, 0, stream>>>(a);
    ORNITH_CHECK_LAUNCH();
    gate_kernel<<<dim3(16, kE + 1), 256, 0, stream>>>(a);
    ORNITH_CHECK_LAUNCH();
    const int mid_warps = rows * (kI / kG);
    if (a.a8) quant_middle_kernel<127><<<(mid_warps + 7) / 8, 256, 0, stream>>>(a);
    else quant_middle_kernel<7><<<(mid_warps + 7) / 8, 256, 0, stream>>>(a);
    ORNITH_CHECK_LAUNCH();
    down_kernel<<<dim3(kH / 32, kE + 1), 256, 0, stream>>>(a);
    ORNITH_CHECK_LAUNCH();
    return launch_combine(a, stream);
}

cudaError_t launch_quant_tokens(const LayerArgs& a, cudaStream_t stream) {
    count_launches(1);
    const int tok_warps = a.T * (kH / kG);
    if (a.a8) quant_tokens_kernel<127><<<(tok_warps + 7) / 8, 256, 0, stream>>>(a);
    else quant_tokens_kernel<7><<<(tok_warps + 7) / 8, 256, 0, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_combine(const LayerArgs& a, cudaStream_t stream, bool by_position) {
    count_launches(1);
    if (by_position) combine_kernel<true><<<a.T, 256, 0, stream>>>(a);
    else combine_kernel<false><<<a.T, 256, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace ornith
