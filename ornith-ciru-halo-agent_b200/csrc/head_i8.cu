// W8 LM head of Ornith (vocabulary 248,320 x hidden 2048): the largest weight
// stream of a decode step after the MoE layers (508 MB of int8 codes).
//
// Restates the reference's head library (kernels/head/head_i8_tile_api.h:21-41,
// head_i8_tile_consumer.cpp) behind the same C ABI: per row, bf16 -> fp32, a
// 128-point Hadamard per 128-group, A8 quantisation per 128-group, exact int32
// dots of signed int8 codes, then over the 16 groups in ascending order
// value = value + w_scale*(sa*float(dot)) (no offset, no FMA), bf16 RNE.
// The reference's compact, WMMA and 64-row shared-memory jobs all compute
// this sequence; one kernel serves the three geometries bit for bit.
//
// B200 layout of the work:
//   head_quant_kernel     one warp per (row, pair of 128-groups): each half
//                         warp transforms and quantises one group in
//                         registers; activations stay in the reference's
//                         word format (four signed bytes, lowest k first);
//   head_project_kernel   one CTA per 32 vocabulary columns with every row of
//                         the call (M <= 64): warp w streams the 2 KB code
//                         blocks of groups w and w+8 of its two 16-column
//                         tiles once (64-byte rows, coalesced), dots them
//                         with __dp4a against each row's broadcast activation
//                         words and leaves one fp32 term per (group, row,
//                         column) in shared memory; after one barrier the
//                         terms are summed in group order.  Every weight byte
//                         is read once per call, so at decode sizes the
//                         kernel is bound by HBM.
#include <stdint.h>

#include <atomic>
#include <climits>

#include "../../include/ornith_moe_b200.h"
#include "abi_check.h"
#include "moe_common.cuh"
#include "nvtx_range.h"

namespace ornith {
void count_launches(int n);

namespace head {

constexpr int kK = 2048, kGroups = 16, kMaxM = 64, kWarps = 8;  // 16 groups of 128
constexpr uint32_t kNonfiniteTransform = 1, kInvalidActivation = 2, kNonfiniteProjection = 4,
                   kNonfiniteBf16 = 8;  // head_i8_tile_api.h:16-21

bool shape_ok(int N) { return N == 256 || N == 1024 || N == 4096 || N == 65536 || N == 248320; }
size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

// Layout (head_i8_tile_api.h:13-15): `activation_words` UINT32[Mcap,512] in the
// reference's format, `activation_scales` fp16 [Mcap,16], `projection` the
// fp32 diagnostic [Mcap,N]; `transformed` has no counterpart here (SIZE_MAX).
OrnithHeadI8Layout layout(int Mcap, int N) {
    OrnithHeadI8Layout l{};
    size_t cursor = 0, m = size_t(Mcap);
    auto add = [&](size_t& field, size_t bytes) {
        field = cursor;
        cursor = align256(cursor + bytes);
    };
    l.transformed = SIZE_MAX;
    add(l.activation_words, m * kK);
    add(l.activation_scales, m * kGroups * 2);
    add(l.projection, m * size_t(N) * 4);
    l.workspace_bytes = cursor;
    return l;
}

__device__ __forceinline__ void flag_or(uint32_t* flags, uint32_t f) {
    f = __reduce_or_sync(0xffffffffu, f);
    if (f && (threadIdx.x & 31) == 0) atomicOr(flags, f);
}

// transform (:30-43) and encode_a8 (:44-71): lane l holds elements 8l..8l+7
// of a 256-element span, so half warp h owns 128-group 2p+h.
__global__ __launch_bounds__(256) void head_quant_kernel(const uint16_t* x, int M, uint32_t* words,
                                                         __half* scales, uint32_t* flags) {
    const int warp = int((size_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (warp >= M * (kK / 256)) return;  // whole warps leave together
    const int r = warp / (kK / 256), span = warp % (kK / 256);
    const size_t at = size_t(r) * kK + size_t(span) * 256;
    const uint4 raw = *reinterpret_cast<const uint4*>(x + at + lane * 8);
    const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
    float e[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        e[2 * i] = __uint_as_float(w4[i] << 16);
        e[2 * i + 1] = __uint_as_float(w4[i] & 0xffff0000u);
    }
    uint32_t f = 0;
#pragma unroll
    for (int s = 0; s < 8; ++s)
        if (!isfinite(e[s])) f |= kNonfiniteTransform;
    wht128_halfwarp(e, lane);
    float v[8], absmax = 0.f;
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        if (!isfinite(e[s])) f |= kNonfiniteTransform | kInvalidActivation;
        v[s] = isfinite(e[s]) ? e[s] : 0.f;
        absmax = fmaxf(absmax, fabsf(v[s]));
    }
    // maximum over the half warp (xor distances below 16 stay inside it)
#pragma unroll
    for (int d = 8; d > 0; d >>= 1) absmax = fmaxf(absmax, __shfl_xor_sync(0xffffffffu, absmax, d));
    const float rawscale = __fdiv_rn(absmax, 127.f);
    const bool valid = isfinite(rawscale) && rawscale <= 65504.f;
    if (!valid) f |= kInvalidActivation;
    const bool zero = absmax == 0.f || !valid;
    const __half scale = __float2half_rn(zero ? 1.f : fmaxf(rawscale, 0x1p-14f));
    const float sf = __half2float(scale);
    uint32_t packed[2] = {0u, 0u};
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        int q = zero ? 0 : __float2int_rn(__fdiv_rn(v[s], sf));
        q = q < -127 ? -127 : (q > 127 ? 127 : q);
        packed[s >> 2] |= (uint32_t(q) & 255u) << (8 * (s & 3));
    }
    *reinterpret_cast<uint2*>(words + at / 4 + lane * 2) = make_uint2(packed[0], packed[1]);
    if ((lane & 15) == 0) scales[size_t(r) * kGroups + span * 2 + (lane >> 4)] = scale;
    flag_or(flags, f);
}

// Column n = 32*blockIdx.x + lane; its word kw of group g sits at
// ((n/16*(K/16) + 8g + j/4)*4 + j%4)*16 + n%16 with j = kw - 32g
// (tile_word, :19-21): per (16-column tile, group) one contiguous 2 KB block.
template <bool DOTS>
__global__ __launch_bounds__(256) void head_project_kernel(const uint32_t* codes, const __half* wscales,
                                                           const uint32_t* words, const __half* ascales, int M,
                                                           int N, float* diag, uint16_t* out, int32_t* dots,
                                                           uint32_t* flags) {
    extern __shared__ float terms[];  // [kGroups][M][32]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int n = blockIdx.x * 32 + lane;
    const size_t tile = size_t(n >> 4);
    const int c = n & 15;
#pragma unroll 1
    for (int g = warp; g < kGroups; g += kWarps) {
        uint32_t w[32];
        const uint32_t* blk = codes + (tile * (kK / 16) + 8 * g) * 64 + c;
#pragma unroll
        for (int j = 0; j < 32; ++j) w[j] = __ldcs(blk + j * 16);
        const float sw = __half2float(wscales[size_t(n) * kGroups + g]);
#pragma unroll 1
        for (int m = 0; m < M; ++m) {
            const uint4* act = reinterpret_cast<const uint4*>(words + size_t(m) * (kK / 4) + 32 * g);
            int dot = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint4 a = __ldg(act + j);
                dot = __dp4a(int(w[4 * j]), int(a.x), dot);
                dot = __dp4a(int(w[4 * j + 1]), int(a.y), dot);
                dot = __dp4a(int(w[4 * j + 2]), int(a.z), dot);
                dot = __dp4a(int(w[4 * j + 3]), int(a.w), dot);
            }
            if (DOTS) dots[(size_t(m) * N + n) * kGroups + g] = dot;
            const float sa = __half2float(ascales[size_t(m) * kGroups + g]);
            terms[(g * M + m) * 32 + lane] = __fmul_rn(sw, __fmul_rn(sa, float(dot)));
        }
    }
    __syncthreads();
    uint32_t f = 0;
    for (int m = warp; m < M; m += kWarps) {
        float v = 0.f;
#pragma unroll
        for (int g = 0; g < kGroups; ++g) v = __fadd_rn(v, terms[(g * M + m) * 32 + lane]);
        if (!isfinite(v)) f |= kNonfiniteProjection;
        const uint16_t b = bf16_rne(v);
        if ((b & 0x7f80u) == 0x7f80u) f |= kNonfiniteBf16;
        const size_t idx = size_t(m) * N + n;
        diag[idx] = v;
        out[idx] = b;
    }
    flag_or(flags, f);
}

std::atomic<bool> g_smem_attr[2][64];

}  // namespace head
}  // namespace ornith

using namespace ornith;

extern "C" uint32_t ornith_head_i8_tile_abi_version(void) { return 1; }

extern "C" cudaError_t ornith_head_i8_tile_get_layout(int Mcap, int N, OrnithHeadI8Layout* out) {
    if (!out || Mcap < 0 || Mcap > head::kMaxM || !head::shape_ok(N)) return cudaErrorInvalidValue;
    *out = head::layout(Mcap, N);
    return cudaSuccess;
}

extern "C" cudaError_t ornith_head_i8_tile_launch(const void* input, const void* weights, const void* scales,
                                                  void* workspace, size_t workspace_bytes, void* output,
                                                  void* group_dots, size_t group_dots_bytes, void* flags, int M,
                                                  int Mcap, int N, int geometry, cudaStream_t stream) {
    using namespace head;
    OrnithHeadI8Layout l{};
    // argument contract of head_i8_tile_consumer.cpp:251-269
    if (ornith_head_i8_tile_get_layout(Mcap, N, &l) != cudaSuccess || M < 0 || M > Mcap || geometry < 0 ||
        geometry > 2)
        return cudaErrorInvalidValue;
    if ((group_dots == nullptr) != (group_dots_bytes == 0) ||
        (group_dots && group_dots_bytes < size_t(M) * N * kGroups * 4))
        return cudaErrorInvalidValue;
    if (M == 0) return cudaSuccess;
    if (workspace_bytes < l.workspace_bytes) return cudaErrorInvalidValue;
    const void* const ptr[7] = {input, weights, scales, workspace, output, group_dots, flags};
    const size_t size[7] = {size_t(M) * kK * 2, size_t(N) * kK, size_t(N) * kGroups * 2, workspace_bytes,
                            size_t(M) * N * 2, group_dots_bytes, 4};
    const uintptr_t align[7] = {16, 4, 2, 256, 2, 4, 4};
    if (!buffers_ok(ptr, size, align, 3, 5)) return cudaErrorInvalidValue;  // group_dots may be null
    NvtxRange range("ornith.head");
    auto* ws = static_cast<uint8_t*>(workspace);
    auto* fl = static_cast<uint32_t*>(flags);
    auto* words = reinterpret_cast<uint32_t*>(ws + l.activation_words);
    auto* ascales = reinterpret_cast<__half*>(ws + l.activation_scales);
    count_launches(1);
    const int warps = M * (kK / 256);
    head_quant_kernel<<<(warps + 7) / 8, 256, 0, stream>>>(static_cast<const uint16_t*>(input), M, words, ascales,
                                                           fl);
    cudaError_t st = cudaGetLastError();
    if (st != cudaSuccess) return st;
    const size_t smem = size_t(kGroups) * M * 32 * sizeof(float);
    const bool with_dots = group_dots != nullptr;
    auto kernel = with_dots ? head_project_kernel<true> : head_project_kernel<false>;
    if (smem > 48 * 1024) {
        int device = 0;
        if ((st = cudaGetDevice(&device)) != cudaSuccess) return st;
        if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
        std::atomic<bool>& done = g_smem_attr[with_dots][device];
        if (!done.load(std::memory_order_acquire)) {
            st = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      int(size_t(kGroups) * kMaxM * 32 * sizeof(float)));
            if (st != cudaSuccess) return st;
            done.store(true, std::memory_order_release);
        }
    }
    count_launches(1);
    kernel<<<N / 32, kWarps * 32, smem, stream>>>(static_cast<const uint32_t*>(weights),
                                                  static_cast<const __half*>(scales), words, ascales, M, N,
                                                  reinterpret_cast<float*>(ws + l.projection),
                                                  static_cast<uint16_t*>(output),
                                                  static_cast<int32_t*>(group_dots), fl);
    return cudaGetLastError();
}

extern "C" int ornith_head_i8_tile_shortlist(void) { return 1; }
