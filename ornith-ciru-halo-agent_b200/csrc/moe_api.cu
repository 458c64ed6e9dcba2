// C-ABI entry points of libornith_moe_b200.so (declared in include/ornith_moe_b200.h).
//
// Argument validation and return codes mirror the reference's routed library
// (kernels/routed_storage/routed_storage_n32_consumer.cpp:309-401): bad
// Tcap/T/bytes or null pointers give cudaErrorInvalidValue, T == 0 succeeds
// without touching any pointer, launch errors are returned as CUDA errors.
// Alignment is checked as the dense library does (dense_g256_consumer.cpp:256-262).
#include <stdint.h>

#include <atomic>
#include <cstdlib>
#include <cstring>

#include "../../include/ornith_moe_b200.h"
#include "moe_layer.cuh"
#include "nvtx_range.h"

using namespace ornith;

namespace ornith {
static std::atomic<unsigned long long> g_launches{0};
void count_launches(int n) { g_launches.fetch_add(static_cast<unsigned long long>(n), std::memory_order_relaxed); }
static bool generic_forced() {
    const char* path = getenv("ORNITH_MOE_B200_PATH");
    return path && strcmp(path, "generic") == 0;
}
bool rows_by_position(int T) { return !generic_forced() && T > kDecodeMaxT; }
}  // namespace ornith

namespace {

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Top-8 routing, one warp per token (see ornith_moe_b200_route_topk).
// Lane l holds logits l, l+32, ..., l+224; each of 8 rounds takes the warp-wide
// maximum among the finite, unselected logits, lower index first on ties.
__global__ __launch_bounds__(256) void route_topk_kernel(const float* logits, int T, float* weights,
                                                         int32_t* ids, uint32_t* flags) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= T) return;
    uint32_t f = 0;
    route_topk_warp(logits + size_t(warp) * kE, lane, ids + size_t(warp) * kTop, weights + size_t(warp) * kTop, f);
    f = __reduce_or_sync(0xffffffffu, f);
    if (f && lane == 0) atomicOr(flags, f);
}

// Shared-expert gate logit bf16(sum_k x[t,k]*w[k]) with fp32 products and sums:
// lane partial sums over k = lane + 32i (i ascending), then an xor tree.
__global__ __launch_bounds__(256) void shared_logit_kernel(const uint16_t* x, const uint16_t* w, int T, uint16_t* logit) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= T) return;
    const uint16_t v = shared_logit_warp(x + size_t(warp) * kH, w, lane);
    if (lane == 0) logit[warp] = v;
}

// combine_rows_kernel with the per-slot rows gathered: row_index[8t+s] is the
// row of slot s of token t in `rows` (n rows).
__global__ __launch_bounds__(256) void combine_gathered_kernel(const float* rows, int n, const int32_t* row_index,
                                                               const float* weights, const int32_t* ids, int T,
                                                               uint16_t* out, uint32_t* flags) {
    const size_t index = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    uint32_t f = 0;
    if (index < size_t(T) * kH) {
        const int t = int(index / kH), c = int(index % kH);
        float sum = 0.f;
#pragma unroll
        for (int s = 0; s < kTop; ++s) {
            const int r = t * kTop + s;
            const int id = ids[r];
            if (id >= kE || id < -1) f |= kFlagInvalidId;  // -1 is padding
            if (!id_valid(id)) continue;
            const int row = row_index[r];
            if (row < 0 || row >= n) {
                f |= kFlagInvalidId;
                continue;
            }
            sum = __fadd_rn(sum, __fmul_rn(rows[size_t(row) * kH + c], weights[r]));
        }
        const uint16_t res = bf16_rne(sum);
        out[index] = res;
        if (!isfinite(sum) || (res & 0x7f80u) == 0x7f80u) f |= kFlagNonfiniteOutput;
    }
    f = __reduce_or_sync(0xffffffffu, f);
    if (f && (threadIdx.x & 31) == 0) atomicOr(flags, f);
}

// Copies route rows out of route_out (through rowpos on the tensor-core
// path).  One CTA per row, 256 threads x 8 floats.
__global__ __launch_bounds__(256) void gather_route_rows_kernel(const float* route_out, const int32_t* rowpos,
                                                                const int32_t* route_index, int R, int rows,
                                                                float* dst, uint32_t* flags) {
    const int i = blockIdx.x;
    const int r = route_index[i];
    int row = -1;
    if (r >= 0 && r < R) row = rowpos ? rowpos[r] : r;
    float4* d = reinterpret_cast<float4*>(dst + size_t(i) * kH) + threadIdx.x * 2;
    if (row < 0 || row >= rows) {
        d[0] = d[1] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (threadIdx.x == 0) atomicOr(flags, kFlagInvalidId);
        return;
    }
    const float4* src = reinterpret_cast<const float4*>(route_out + size_t(row) * kH) + threadIdx.x * 2;
    d[0] = __ldcs(src);
    d[1] = __ldcs(src + 1);
}

// Route-ordered copy of route_out: CTA p copies the row at position p (the
// route routes[p] on the tensor-core path, route p otherwise) to rows[route].
__global__ __launch_bounds__(256) void scatter_route_rows_kernel(const float* route_out, const int32_t* routes,
                                                                 const int32_t* n_positions, int R, float* dst) {
    const int p = blockIdx.x;
    int r = p;
    if (routes) {
        if (p >= *n_positions) return;
        r = routes[p];
    }
    if (r < 0 || r >= R) return;  // the shared expert's rows
    const float4* src = reinterpret_cast<const float4*>(route_out + size_t(p) * kH) + threadIdx.x * 2;
    float4* d = reinterpret_cast<float4*>(dst + size_t(r) * kH) + threadIdx.x * 2;
    d[0] = __ldcs(src);
    d[1] = __ldcs(src + 1);
}

// Router logits (iu4_correctness/gates_projection.py:17-25):
// logits[t][e] = sum_k f32(x[t][k]) * f32(W[e][k]), fp32.  One warp per expert
// keeps its 2048 weights in registers (64 per lane: k = 256 j + 8 lane + i)
// and walks the CTA's tokens; per token a lane accumulates its 64 products
// with FMA in k order, then an xor tree (16, 8, 4, 2, 1) adds the lanes.  The
// reference's Triton reduction order is unspecified, so the logits agree to
// rounding (relative 1e-5), not bit for bit.
constexpr int kRouterTokens = 64;  // tokens per CTA
__global__ __launch_bounds__(256) void router_logits_kernel(const uint16_t* x, const uint16_t* w, int T,
                                                            float* logits) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e = blockIdx.x * 8 + warp;
    const int t0 = blockIdx.y * kRouterTokens, t1 = min(T, t0 + kRouterTokens);
    uint4 wr[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) wr[j] = __ldg(reinterpret_cast<const uint4*>(w + size_t(e) * kH + j * 256 + lane * 8));
    for (int t = t0; t < t1; ++t) {
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint4 xr = __ldg(reinterpret_cast<const uint4*>(x + size_t(t) * kH + j * 256 + lane * 8));
            const uint32_t xv[4] = {xr.x, xr.y, xr.z, xr.w}, wv[4] = {wr[j].x, wr[j].y, wr[j].z, wr[j].w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                acc = __fmaf_rn(__uint_as_float(xv[i] << 16), __uint_as_float(wv[i] << 16), acc);
                acc = __fmaf_rn(__uint_as_float(xv[i] & 0xffff0000u), __uint_as_float(wv[i] & 0xffff0000u), acc);
            }
        }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, d));
        if (lane == 0) logits[size_t(t) * kE + e] = acc;
    }
}

// N16 -> N32 bank repack (method.py:142-147).  One thread per destination word.
__global__ void repack_codes_kernel(const uint32_t* src, uint32_t* dst, int E, int N, int groups) {
    const size_t total = size_t(E) * (N / 32) * groups * 32 * 32;
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
        size_t rem = i;
        const int col = int(rem % 32); rem /= 32;
        const int j = int(rem % 32); rem /= 32;
        const int g = int(rem % groups); rem /= groups;
        const int t2 = int(rem % (N / 32)); rem /= (N / 32);
        const size_t e = rem;
        const int half = col / 16, l = col % 16;
        dst[i] = src[((((e * (N / 16) + 2 * t2 + half) * groups + g) * 32 + j) * 16) + l];
    }
}
__global__ void repack_meta_kernel(const uint32_t* src, uint32_t* dst, int E, int N, int groups) {
    const size_t total = size_t(E) * (N / 32) * groups * 32;
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
        size_t rem = i;
        const int col = int(rem % 32); rem /= 32;
        const int g = int(rem % groups); rem /= groups;
        const int t2 = int(rem % (N / 32)); rem /= (N / 32);
        const size_t e = rem;
        const int half = col / 16, l = col % 16;
        dst[i] = src[(((e * (N / 16) + 2 * t2 + half) * groups + g) * 16) + l];
    }
}

// Slot-ordered combine from explicit per-route rows (the expert-parallel home
// rank's final step): out[t,c] = bf16(sum over valid slots s, in slot order,
// of route_out[8t+s][c] * w[t,s]), starting from +0 (reduce_slots :176-185).
__global__ __launch_bounds__(256) void combine_rows_kernel(const float* route_out, const float* weights,
                                                           const int32_t* ids, int T, uint16_t* out, uint32_t* flags) {
    const size_t index = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    uint32_t f = 0;
    if (index < size_t(T) * kH) {
        const int t = int(index / kH), c = int(index % kH);
        float sum = 0.f;
#pragma unroll
        for (int s = 0; s < kTop; ++s) {
            const int r = t * kTop + s;
            if (id_valid(ids[r])) sum = __fadd_rn(sum, __fmul_rn(route_out[size_t(r) * kH + c], weights[r]));
        }
        const uint16_t res = bf16_rne(sum);
        out[index] = res;
        if (!isfinite(sum) || (res & 0x7f80u) == 0x7f80u) f |= kFlagNonfiniteOutput;
    }
    f = __reduce_or_sync(0xffffffffu, f);
    if (f && (threadIdx.x & 31) == 0) atomicOr(flags, f);
}

void fill_layout(int Tcap, OrnithRoutedDirectLayout* out) {
    const Workspace w = workspace_layout(Tcap);
    OrnithRoutedDirectLayout l;
    l.workspace_bytes = w.bytes;
    l.gate_x = SIZE_MAX;
    l.gate_low = w.xq;
    l.gate_high = SIZE_MAX;
    l.gate_scales = w.xs;
    l.gate_sums = w.xsum;
    l.gate_y = SIZE_MAX;
    l.middle = w.middle;
    l.down_x = SIZE_MAX;
    l.down_low = w.mq;
    l.down_high = SIZE_MAX;
    l.down_scales = w.ms;
    l.down_sums = w.msum;
    l.route_out = w.route_out;
    l.final_f32 = w.final_f32;
    *out = l;
}

// Path selection: the fused persistent kernel for decode batches, the
// multi-kernel path otherwise.  ORNITH_MOE_B200_PATH=generic forces the
// multi-kernel path (used by the tests to check both paths).
bool force_generic() { return generic_forced(); }

// The fused decode kernel serves the call (it also routes from logits itself).
bool uses_decode(int T) { return !force_generic() && decode_supported(T); }

cudaError_t run_layer(const LayerArgs& a, cudaStream_t stream) {
    if (uses_decode(a.T)) {
        NvtxRange r("ornith.layer.decode");
        return launch_decode(a, stream);
    }
    if (rows_by_position(a.T)) {
        NvtxRange r("ornith.layer.prefill");
        return launch_prefill(a, stream);
    }
    NvtxRange r("ornith.layer.generic");
    return launch_generic(a, stream);
}

cudaError_t routed_launch(int act_bits, const void* input, const void* weights, const void* ids,
                          const void* gate_codes, const void* gate_meta, const void* down_codes,
                          const void* down_meta, void* workspace, size_t bytes, void* output, void* flags,
                          int T, int Tcap, cudaStream_t stream) {
    if (Tcap < 0 || Tcap > kTcapMax || T < 0 || T > Tcap) return cudaErrorInvalidValue;
    const Workspace w = workspace_layout(Tcap);
    if (bytes < w.bytes) return cudaErrorInvalidValue;
    if (!T) return cudaSuccess;
    if (!input || !weights || !ids || !gate_codes || !gate_meta || !down_codes || !down_meta || !workspace ||
        !output || !flags)
        return cudaErrorInvalidValue;
    if (!aligned(input, 16) || !aligned(output, 16) || !aligned(gate_codes, 16) || !aligned(gate_meta, 16) ||
        !aligned(down_codes, 16) || !aligned(down_meta, 16) || !aligned(workspace, 256) || !aligned(weights, 4) ||
        !aligned(ids, 4) || !aligned(flags, 4))
        return cudaErrorInvalidValue;
    LayerArgs a{};
    a.x = static_cast<const uint16_t*>(input);
    a.weights = static_cast<const float*>(weights);
    a.ids = static_cast<const int32_t*>(ids);
    a.gate_codes = static_cast<const uint32_t*>(gate_codes);
    a.gate_meta = static_cast<const uint32_t*>(gate_meta);
    a.down_codes = static_cast<const uint32_t*>(down_codes);
    a.down_meta = static_cast<const uint32_t*>(down_meta);
    a.out = static_cast<uint16_t*>(output);
    a.flags = static_cast<uint32_t*>(flags);
    a.ws = static_cast<uint8_t*>(workspace);
    a.L = w;
    a.T = T;
    a.a8 = act_bits == 8;
    return run_layer(a, stream);
}

cudaError_t layer_from_logits(const void* input, const void* logits, const void* router_weight,
                              const void* gate_codes, const void* gate_meta, const void* down_codes,
                              const void* down_meta, const void* shared_gate_codes, const void* shared_gate_meta,
                              const void* shared_down_codes, const void* shared_down_meta,
                              const void* shared_gate_weight, const void* shared_silu, const void* shared_sigmoid,
                              void* workspace, size_t bytes, void* output, void* shared_output, void* flags, int T,
                              int Tcap, int act_bits, cudaStream_t stream);

}  // namespace

extern "C" {

cudaError_t ornith_routed_direct_get_layout(int Tcap, OrnithRoutedDirectLayout* out) {
    if (!out || Tcap < 0 || Tcap > kTcapMax) return cudaErrorInvalidValue;
    fill_layout(Tcap, out);
    return cudaSuccess;
}

cudaError_t ornith_routed_direct_launch(const void* input, const void* weights, const void* ids, const void* gate_codes,
                                        const void* gate_meta, const void* down_codes, const void* down_meta,
                                        void* workspace, size_t bytes, void* output, void* flags, int T, int Tcap,
                                        cudaStream_t stream) {
    return routed_launch(8, input, weights, ids, gate_codes, gate_meta, down_codes, down_meta, workspace, bytes,
                         output, flags, T, Tcap, stream);
}

cudaError_t ornith_routed_direct_launch_a4(const void* input, const void* weights, const void* ids,
                                           const void* gate_codes, const void* gate_meta, const void* down_codes,
                                           const void* down_meta, void* workspace, size_t bytes, void* output,
                                           void* flags, int T, int Tcap, cudaStream_t stream) {
    return routed_launch(4, input, weights, ids, gate_codes, gate_meta, down_codes, down_meta, workspace, bytes,
                         output, flags, T, Tcap, stream);
}

cudaError_t ornith_routed_direct_launch_a4_prefill(const void* input, const void* weights, const void* ids,
                                                   const void* gate_codes, const void* gate_meta,
                                                   const void* down_codes, const void* down_meta, void* workspace,
                                                   size_t bytes, void* output, void* flags, int T, int Tcap,
                                                   cudaStream_t stream) {
    return routed_launch(T > 64 ? 4 : 8, input, weights, ids, gate_codes, gate_meta, down_codes, down_meta,
                         workspace, bytes, output, flags, T, Tcap, stream);
}

int ornith_routed_storage_n32(void) { return 32; }
int ornith_routed_prefill_output_tile(void) { return 32; }

cudaError_t ornith_routed_shared_get_layout(int Tcap, OrnithRoutedDirectLayout* out) {
    if (!out || Tcap < 0 || Tcap > 16) return cudaErrorInvalidValue;
    fill_layout(Tcap, out);
    return cudaSuccess;
}

cudaError_t ornith_routed_direct_launch_shared_tables(
    const void* input, const void* weights, const void* ids, const void* gate_codes, const void* gate_meta,
    const void* down_codes, const void* down_meta, const void* shared_gate_codes, const void* shared_gate_meta,
    const void* shared_down_codes, const void* shared_down_meta, const void* shared_logit, const void* shared_silu,
    const void* shared_sigmoid, void* workspace, size_t bytes, void* output, void* shared_output, void* flags, int T,
    int Tcap, cudaStream_t stream) {
    if (Tcap < 0 || Tcap > 16 || T < 0 || T > Tcap) return cudaErrorInvalidValue;
    const Workspace w = workspace_layout(Tcap);
    if (bytes < w.bytes) return cudaErrorInvalidValue;
    if (!T) return cudaSuccess;
    if (!input || !weights || !ids || !gate_codes || !gate_meta || !down_codes || !down_meta || !shared_gate_codes ||
        !shared_gate_meta || !shared_down_codes || !shared_down_meta || !shared_logit || !shared_silu ||
        !shared_sigmoid || !workspace || !output || !shared_output || !flags)
        return cudaErrorInvalidValue;
    if (!aligned(input, 16) || !aligned(output, 16) || !aligned(shared_output, 16) || !aligned(gate_codes, 16) ||
        !aligned(gate_meta, 16) || !aligned(down_codes, 16) || !aligned(down_meta, 16) ||
        !aligned(shared_gate_codes, 16) || !aligned(shared_gate_meta, 16) || !aligned(shared_down_codes, 16) ||
        !aligned(shared_down_meta, 16) || !aligned(workspace, 256) || !aligned(weights, 4) || !aligned(ids, 4) ||
        !aligned(flags, 4) || !aligned(shared_silu, 4) || !aligned(shared_logit, 2) || !aligned(shared_sigmoid, 2))
        return cudaErrorInvalidValue;
    LayerArgs a{};
    a.x = static_cast<const uint16_t*>(input);
    a.weights = static_cast<const float*>(weights);
    a.ids = static_cast<const int32_t*>(ids);
    a.gate_codes = static_cast<const uint32_t*>(gate_codes);
    a.gate_meta = static_cast<const uint32_t*>(gate_meta);
    a.down_codes = static_cast<const uint32_t*>(down_codes);
    a.down_meta = static_cast<const uint32_t*>(down_meta);
    a.sgate_codes = static_cast<const uint32_t*>(shared_gate_codes);
    a.sgate_meta = static_cast<const uint32_t*>(shared_gate_meta);
    a.sdown_codes = static_cast<const uint32_t*>(shared_down_codes);
    a.sdown_meta = static_cast<const uint32_t*>(shared_down_meta);
    a.shared_logit = static_cast<const uint16_t*>(shared_logit);
    a.silu_table = static_cast<const float*>(shared_silu);
    a.sigmoid_table = static_cast<const uint16_t*>(shared_sigmoid);
    a.out = static_cast<uint16_t*>(output);
    a.shared_out = static_cast<uint16_t*>(shared_output);
    a.flags = static_cast<uint32_t*>(flags);
    a.ws = static_cast<uint8_t*>(workspace);
    a.L = w;
    a.T = T;
    a.a8 = 1;
    a.shared = 1;
    a.shared_all_live = 1;
    return run_layer(a, stream);
}

uint32_t ornith_moe_b200_abi_version(void) { return 1; }

unsigned long long ornith_moe_b200_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

cudaError_t ornith_moe_b200_route_topk(const void* logits, int T, void* weights, void* ids, void* flags,
                                       cudaStream_t stream) {
    if (T < 0 || T > kTcapMax) return cudaErrorInvalidValue;
    if (!T) return cudaSuccess;
    if (!logits || !weights || !ids || !flags || !aligned(logits, 4) || !aligned(weights, 4) || !aligned(ids, 4) ||
        !aligned(flags, 4))
        return cudaErrorInvalidValue;
    count_launches(1);
    route_topk_kernel<<<(T + 7) / 8, 256, 0, stream>>>(static_cast<const float*>(logits), T,
                                                        static_cast<float*>(weights), static_cast<int32_t*>(ids),
                                                        static_cast<uint32_t*>(flags));
    return cudaGetLastError();
}

cudaError_t ornith_moe_b200_combine(const void* route_out_f32, const void* weights, const void* ids, int T,
                                    void* output, void* flags, cudaStream_t stream) {
    if (T < 0 || T > kTcapMax) return cudaErrorInvalidValue;
    if (!T) return cudaSuccess;
    if (!route_out_f32 || !weights || !ids || !output || !flags || !aligned(route_out_f32, 4) ||
        !aligned(weights, 4) || !aligned(ids, 4) || !aligned(output, 2) || !aligned(flags, 4))
        return cudaErrorInvalidValue;
    count_launches(1);
    combine_rows_kernel<<<(T * kH + 255) / 256, 256, 0, stream>>>(
        static_cast<const float*>(route_out_f32), static_cast<const float*>(weights), static_cast<const int32_t*>(ids),
        T, static_cast<uint16_t*>(output), static_cast<uint32_t*>(flags));
    return cudaGetLastError();
}

cudaError_t ornith_moe_b200_combine_gathered(const void* rows_f32, int n_rows, const void* row_index_i32,
                                             const void* weights, const void* ids, int T, void* output, void* flags,
                                             cudaStream_t stream) {
    if (T < 0 || T > kTcapMax || n_rows < 0) return cudaErrorInvalidValue;
    if (!T) return cudaSuccess;
    if ((!rows_f32 && n_rows) || !row_index_i32 || !weights || !ids || !output || !flags ||
        !aligned(rows_f32, 4) || !aligned(row_index_i32, 4) || !aligned(weights, 4) || !aligned(ids, 4) ||
        !aligned(output, 2) || !aligned(flags, 4))
        return cudaErrorInvalidValue;
    count_launches(1);
    combine_gathered_kernel<<<(T * kH + 255) / 256, 256, 0, stream>>>(
        static_cast<const float*>(rows_f32), n_rows, static_cast<const int32_t*>(row_index_i32),
        static_cast<const float*>(weights), static_cast<const int32_t*>(ids), T, static_cast<uint16_t*>(output),
        static_cast<uint32_t*>(flags));
    return cudaGetLastError();
}

cudaError_t ornith_moe_b200_gather_route_rows(const void* workspace, size_t bytes, int T, int Tcap,
                                             const void* route_index_i32, int n, void* rows_f32, void* flags,
                                             cudaStream_t stream) {
    if (Tcap < 0 || Tcap > kTcapMax || T < 0 || T > Tcap || n < 0) return cudaErrorInvalidValue;
    const Workspace w = workspace_layout(Tcap);
    if (bytes < w.bytes) return cudaErrorInvalidValue;
    if (!n) return cudaSuccess;
    if (!workspace || !route_index_i32 || !rows_f32 || !flags || !aligned(workspace, 256) ||
        !aligned(route_index_i32, 4) || !aligned(rows_f32, 16) || !aligned(flags, 4))
        return cudaErrorInvalidValue;
    const uint8_t* ws = static_cast<const uint8_t*>(workspace);
    const int32_t* rowpos = rows_by_position(T) ? reinterpret_cast<const int32_t*>(ws + w.rowpos) : nullptr;
    count_launches(1);
    gather_route_rows_kernel<<<n, 256, 0, stream>>>(reinterpret_cast<const float*>(ws + w.route_out), rowpos,
                                                    static_cast<const int32_t*>(route_index_i32), T * kTop,
                                                    T * (kTop + 1), static_cast<float*>(rows_f32),
                                                    static_cast<uint32_t*>(flags));
    return cudaGetLastError();
}

cudaError_t ornith_moe_b200_scatter_route_rows(const void* workspace, size_t bytes, int T, int Tcap, void* rows_f32,
                                              cudaStream_t stream) {
    if (Tcap < 0 || Tcap > kTcapMax || T < 0 || T > Tcap) return cudaErrorInvalidValue;
    const Workspace w = workspace_layout(Tcap);
    if (bytes < w.bytes) return cudaErrorInvalidValue;
    if (!T) return cudaSuccess;
    if (!workspace || !rows_f32 || !aligned(workspace, 256) || !aligned(rows_f32, 16)) return cudaErrorInvalidValue;
    const uint8_t* ws = static_cast<const uint8_t*>(workspace);
    const bool by_position = rows_by_position(T);
    count_launches(1);
    // positions: routed rows first, the shared expert's rows (if any) last
    scatter_route_rows_kernel<<<T * (kTop + (by_position ? 1 : 0)), 256, 0, stream>>>(
        reinterpret_cast<const float*>(ws + w.route_out),
        by_position ? reinterpret_cast<const int32_t*>(ws + w.routes) : nullptr,
        by_position ? reinterpret_cast<const int32_t*>(ws + w.offsets) + kE + 1 : nullptr, T * kTop,
        static_cast<float*>(rows_f32));
    return cudaGetLastError();
}

cudaError_t ornith_moe_b200_router_logits(const void* input, const void* router_weight, int T, void* logits,
                                         cudaStream_t stream) {
    if (T < 0 || T > kTcapMax) return cudaErrorInvalidValue;
    if (!T) return cudaSuccess;
    if (!input || !router_weight || !logits || !aligned(input, 16) || !aligned(router_weight, 16) ||
        !aligned(logits, 4))
        return cudaErrorInvalidValue;
    count_launches(1);
    router_logits_kernel<<<dim3(kE / 8, (T + kRouterTokens - 1) / kRouterTokens), 256, 0, stream>>>(
        static_cast<const uint16_t*>(input), static_cast<const uint16_t*>(router_weight), T, static_cast<float*>(logits));
    return cudaGetLastError();
}

cudaError_t ornith_moe_b200_launch_from_hidden(
    const void* input, const void* router_weight, void* logits, const void* gate_codes, const void* gate_meta,
    const void* down_codes, const void* down_meta, const void* shared_gate_codes, const void* shared_gate_meta,
    const void* shared_down_codes, const void* shared_down_meta, const void* shared_gate_weight,
    const void* shared_silu, const void* shared_sigmoid, void* workspace, size_t bytes, void* output,
    void* shared_output, void* flags, int T, int Tcap, int act_bits, cudaStream_t stream) {
    if (Tcap < 0 || Tcap > kTcapMax || T < 0 || T > Tcap) return cudaErrorInvalidValue;
    // one token on the fused decode path: the single-token kernel computes the
    // router logits itself (one launch per layer); it refuses devices it does
    // not fit, and the separate router launch runs then
    if (T == 1 && uses_decode(T)) {
        if (!router_weight || !aligned(router_weight, 16)) return cudaErrorInvalidValue;
        const cudaError_t st =
            layer_from_logits(input, logits, router_weight, gate_codes, gate_meta, down_codes, down_meta,
                              shared_gate_codes, shared_gate_meta, shared_down_codes, shared_down_meta,
                              shared_gate_weight, shared_silu, shared_sigmoid, workspace, bytes, output,
                              shared_output, flags, T, Tcap, act_bits, stream);
        if (st != cudaErrorNotSupported) return st;
    }
    cudaError_t st = ornith_moe_b200_router_logits(input, router_weight, T, logits, stream);
    if (st != cudaSuccess) return st;
    return ornith_moe_b200_launch_from_logits(input, logits, gate_codes, gate_meta, down_codes, down_meta,
                                              shared_gate_codes, shared_gate_meta, shared_down_codes,
                                              shared_down_meta, shared_gate_weight, shared_silu, shared_sigmoid,
                                              workspace, bytes, output, shared_output, flags, T, Tcap, act_bits,
                                              stream);
}

cudaError_t ornith_moe_b200_get_layout(int Tcap, size_t* workspace_bytes) {
    if (!workspace_bytes || Tcap < 0 || Tcap > kTcapMax) return cudaErrorInvalidValue;
    *workspace_bytes = workspace_layout(Tcap).bytes;
    return cudaSuccess;
}

cudaError_t ornith_moe_b200_launch_from_logits(
    const void* input, const void* logits, const void* gate_codes, const void* gate_meta, const void* down_codes,
    const void* down_meta, const void* shared_gate_codes, const void* shared_gate_meta, const void* shared_down_codes,
    const void* shared_down_meta, const void* shared_gate_weight, const void* shared_silu, const void* shared_sigmoid,
    void* workspace, size_t bytes, void* output, void* shared_output, void* flags, int T, int Tcap, int act_bits,
    cudaStream_t stream) {
    return layer_from_logits(input, logits, nullptr, gate_codes, gate_meta, down_codes, down_meta, shared_gate_codes,
                             shared_gate_meta, shared_down_codes, shared_down_meta, shared_gate_weight, shared_silu,
                             shared_sigmoid, workspace, bytes, output, shared_output, flags, T, Tcap, act_bits,
                             stream);
}

}  // extern "C"

namespace {

// The routed layer from router logits.  With router_weight (the from-hidden
// entry at T = 1 on the fused decode path) the single-token kernel writes the
// logits into `logits` itself, or the call returns cudaErrorNotSupported
// having launched nothing.
cudaError_t layer_from_logits(const void* input, const void* logits, const void* router_weight,
                              const void* gate_codes, const void* gate_meta, const void* down_codes,
                              const void* down_meta, const void* shared_gate_codes, const void* shared_gate_meta,
                              const void* shared_down_codes, const void* shared_down_meta,
                              const void* shared_gate_weight, const void* shared_silu, const void* shared_sigmoid,
                              void* workspace, size_t bytes, void* output, void* shared_output, void* flags, int T,
                              int Tcap, int act_bits, cudaStream_t stream) {
    if (Tcap < 0 || Tcap > kTcapMax || T < 0 || T > Tcap) return cudaErrorInvalidValue;
    if (act_bits != 0 && act_bits != 4 && act_bits != 8) return cudaErrorInvalidValue;
    const Workspace w = workspace_layout(Tcap);
    if (bytes < w.bytes) return cudaErrorInvalidValue;
    const bool shared = shared_gate_codes || shared_gate_meta || shared_down_codes || shared_down_meta;
    if (!T) return cudaSuccess;
    if (!input || !logits || !gate_codes || !gate_meta || !down_codes || !down_meta || !workspace || !output || !flags)
        return cudaErrorInvalidValue;
    if (shared && (!shared_gate_codes || !shared_gate_meta || !shared_down_codes || !shared_down_meta ||
                   !shared_gate_weight || !shared_silu || !shared_sigmoid || !shared_output))
        return cudaErrorInvalidValue;
    const int bits = act_bits == 0 ? (T > 64 ? 4 : 8) : act_bits;
    if (shared && (bits != 8 || T > 64)) return cudaErrorInvalidValue;
    if (!aligned(input, 16) || !aligned(output, 16) || !aligned(gate_codes, 16) || !aligned(gate_meta, 16) ||
        !aligned(down_codes, 16) || !aligned(down_meta, 16) || !aligned(workspace, 256) || !aligned(logits, 4) ||
        !aligned(flags, 4))
        return cudaErrorInvalidValue;
    if (shared && (!aligned(shared_output, 16) || !aligned(shared_gate_codes, 16) || !aligned(shared_gate_meta, 16) ||
                   !aligned(shared_down_codes, 16) || !aligned(shared_down_meta, 16) ||
                   !aligned(shared_gate_weight, 2) || !aligned(shared_silu, 4) || !aligned(shared_sigmoid, 2)))
        return cudaErrorInvalidValue;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    float* tw = reinterpret_cast<float*>(ws + w.topk_w);
    int32_t* tid = reinterpret_cast<int32_t*>(ws + w.topk_ids);
    uint16_t* logit = reinterpret_cast<uint16_t*>(ws + w.logit);
    // decode batches: the fused kernel routes and computes the shared logits
    // itself (one launch per layer); otherwise two small kernels run first
    const bool fused = uses_decode(T);
    if (router_weight && (!fused || T != 1)) return cudaErrorNotSupported;
    cudaError_t s = cudaSuccess;
    if (!fused) {
        count_launches(1);
        route_topk_kernel<<<(T + 7) / 8, 256, 0, stream>>>(static_cast<const float*>(logits), T, tw, tid,
                                                            static_cast<uint32_t*>(flags));
        s = cudaGetLastError();
        if (s != cudaSuccess) return s;
    }
    LayerArgs a{};
    if (fused) {
        a.logits = static_cast<const float*>(logits);
        a.ids_out = tid;
        a.weights_out = tw;
    }
    if (router_weight) {
        a.router_weight = static_cast<const uint16_t*>(router_weight);
        a.logits_out = static_cast<float*>(const_cast<void*>(logits));
    }
    a.x = static_cast<const uint16_t*>(input);
    a.weights = tw;
    a.ids = tid;
    a.gate_codes = static_cast<const uint32_t*>(gate_codes);
    a.gate_meta = static_cast<const uint32_t*>(gate_meta);
    a.down_codes = static_cast<const uint32_t*>(down_codes);
    a.down_meta = static_cast<const uint32_t*>(down_meta);
    a.out = static_cast<uint16_t*>(output);
    a.flags = static_cast<uint32_t*>(flags);
    a.ws = ws;
    a.L = w;
    a.T = T;
    a.a8 = bits == 8;
    if (shared) {
        if (fused) {
            a.shared_gate_weight = static_cast<const uint16_t*>(shared_gate_weight);
            a.logit_out = logit;
        } else {
            count_launches(1);
            shared_logit_kernel<<<(T + 7) / 8, 256, 0, stream>>>(
                a.x, static_cast<const uint16_t*>(shared_gate_weight), T, logit);
            s = cudaGetLastError();
            if (s != cudaSuccess) return s;
        }
        a.sgate_codes = static_cast<const uint32_t*>(shared_gate_codes);
        a.sgate_meta = static_cast<const uint32_t*>(shared_gate_meta);
        a.sdown_codes = static_cast<const uint32_t*>(shared_down_codes);
        a.sdown_meta = static_cast<const uint32_t*>(shared_down_meta);
        a.shared_logit = logit;
        a.silu_table = static_cast<const float*>(shared_silu);
        a.sigmoid_table = static_cast<const uint16_t*>(shared_sigmoid);
        a.shared_out = static_cast<uint16_t*>(shared_output);
        a.shared = 1;
        a.shared_all_live = 1;
    }
    if (router_weight) return launch_decode_single(a, stream);
    return run_layer(a, stream);
}

}  // namespace

extern "C" {

cudaError_t ornith_moe_b200_repack_n16_to_n32(const void* codes_n16, const void* meta_n16, void* codes_n32,
                                              void* meta_n32, int experts, int N, int K, cudaStream_t stream) {
    if (experts <= 0 || N <= 0 || N % 32 || K <= 0 || K % kG) return cudaErrorInvalidValue;
    if (!codes_n16 || !meta_n16 || !codes_n32 || !meta_n32 || !aligned(codes_n16, 4) || !aligned(meta_n16, 4) ||
        !aligned(codes_n32, 4) || !aligned(meta_n32, 4))
        return cudaErrorInvalidValue;
    const size_t code_bytes = size_t(experts) * N * K / 2, meta_bytes = size_t(experts) * N * (K / kG) * 4;
    auto overlap = [](const void* a, size_t na, const void* b, size_t nb) {
        uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
        return x < y + nb && y < x + na;
    };
    if (overlap(codes_n16, code_bytes, codes_n32, code_bytes) || overlap(meta_n16, meta_bytes, meta_n32, meta_bytes) ||
        overlap(codes_n32, code_bytes, meta_n32, meta_bytes))
        return cudaErrorInvalidValue;
    const int groups = K / kG;
    count_launches(2);
    repack_codes_kernel<<<1184, 256, 0, stream>>>(static_cast<const uint32_t*>(codes_n16),
                                                  static_cast<uint32_t*>(codes_n32), experts, N, groups);
    cudaError_t s = cudaGetLastError();
    if (s != cudaSuccess) return s;
    repack_meta_kernel<<<296, 256, 0, stream>>>(static_cast<const uint32_t*>(meta_n16), static_cast<uint32_t*>(meta_n32),
                                                experts, N, groups);
    return cudaGetLastError();
}

}  // extern "C"
