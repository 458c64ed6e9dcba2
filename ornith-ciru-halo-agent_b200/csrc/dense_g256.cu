// Dense G256 projections for Ornith's dense layers (QKVZ, output and MLP
// projections: N <= 12288 columns, K <= 8192, or the 248,320-column head).
//
// Restates the reference's dense library (kernels/dense_n32/, contract in
// dense_g256_api.h:20-44) behind the same C ABI:
//   * A8 projection out[M,N] = bf16(x . W^T): per row, bf16 -> fp32, a
//     128-point Hadamard per 128-block, A8 quantisation per 256-group, then
//     per column and ascending group value += w_scale*(sa*dot) +
//     w_offset*(sa*sum) (dense_g256_consumer.cpp:80-142, :250-358);
//   * the bf16 prefill preparation: bf16(H128(x)) and the dequantised bf16
//     weight matrix, which the caller multiplies with a bf16 GEMM
//     (dense_g256_consumer.cpp:192-247, native.py:138-149).
// The reference computes the A8 projection with WMMA iu4 jobs of 16 rows x 16
// columns or one-row compact jobs; every form reduces to the same integer dots
// and the same fp32 sequence, so one B200 kernel serves all three geometries.
//
// B200 layout of the work:
//   dense_quant_kernel     one warp per (row, 256-group): Hadamard in
//                          registers and shuffles, A8 quantisation into int8
//                          rows (the permuted [even | odd] byte order that
//                          dot8 expects), fp16 scales and int32 sums;
//   dense_project_kernel   one CTA per 32 output columns and 16 rows; warp w
//                          streams the weight words of groups w, w+8, ... for
//                          its 32 columns once (coalesced 64/128-byte rows of
//                          the N16/N32 tiles), dots them against every row of
//                          the block (activations are warp-uniform broadcast
//                          loads) and leaves one fp32 term per (group, row,
//                          column) in shared memory; after one barrier the
//                          terms are summed in ascending group order.  At
//                          decode sizes (M <= 16) every weight byte is read
//                          once and the kernel is bound by HBM;
//   dense_fused_kernel     decode rows (M <= 4): the quantisation of the
//                          projection kernel's own groups inside it, so one
//                          launch per call;
//   dense_transform_bf16_kernel, dense_dequant_bf16_kernel
//                          the prefill preparation (one warp per row group;
//                          one CTA per 16-column tile and group, transposed
//                          through shared memory so that both the code reads
//                          and the bf16 row writes are whole lines).
#include <stdint.h>

#include <atomic>
#include <climits>
#include <cstring>

#include "../../include/ornith_moe_b200.h"
#include "abi_check.h"
#include "moe_common.cuh"
#include "nvtx_range.h"

namespace ornith {
void count_launches(int n);

namespace dense {

constexpr int kMaxM = 8192, kMaxN = 12288, kHeadN = 248320, kMaxK = 8192;
constexpr int kN32Rows = 16;   // rows of the N32 entry (dense_g256_consumer.cpp:380)
constexpr int kRowBlock = 16;  // rows per projection CTA
constexpr int kWarps = 8;      // warps per projection CTA

// Dense flag bits (dense_g256_api.h:14-19).
constexpr uint32_t kNonfiniteTransform = 1, kInvalidActivation = 2, kNonfiniteProjection = 4,
                   kNonfiniteBf16 = 8;
static_assert(kNonfiniteTransform == kFlagNonfiniteInput && kInvalidActivation == kFlagInvalidActivation,
              "quantize_group_warp raises the dense bits 1 and 2");

bool shape_ok(int N, int K) {
    return N > 0 && (N <= kMaxN || N == kHeadN) && N % 16 == 0 && K > 0 && K <= kMaxK && K % kG == 0;
}
size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

// This library's workspace inside the reference's layout struct: `low` holds
// the int8 activations [Mcap,K] (one byte per element in place of the
// reference's two nibble planes), `scales` fp16 [Mcap,K/256], `sums` int32
// [Mcap,K/256], `projection` the fp32 diagnostic [Mcap,N]; `transformed` and
// `high` have no counterpart and hold SIZE_MAX (the reference's own marker for
// an absent field, dense_g256_consumer.cpp:19).
OrnithDenseG256Layout layout(int Mcap, int N, int K) {
    OrnithDenseG256Layout l{};
    size_t cursor = 0, m = size_t(Mcap);
    auto add = [&](size_t& field, size_t bytes) {
        field = cursor;
        cursor = align256(cursor + bytes);
    };
    l.transformed = SIZE_MAX;
    l.high = SIZE_MAX;
    add(l.low, m * K);
    add(l.scales, m * (K / kG) * 2);
    add(l.sums, m * (K / kG) * 4);
    add(l.projection, m * N * 4);
    l.workspace_bytes = cursor;
    return l;
}

__device__ __forceinline__ void flag_or(uint32_t* flags, uint32_t f) {
    f = __reduce_or_sync(0xffffffffu, f);
    if (f && (threadIdx.x & 31) == 0) atomicOr(flags, f);
}

// Eight bf16 of one lane (elements 8*lane .. 8*lane+7 of a 256-group) to fp32,
// then the Hadamard of the lane's 128-block; flag 1 on a non-finite input or
// result (transform, dense_g256_consumer.cpp:27-39).
__device__ __forceinline__ uint32_t load_transform(const uint16_t* src, int lane, float (&e)[8]) {
    const uint4 raw = *reinterpret_cast<const uint4*>(src + lane * 8);
    const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
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
#pragma unroll
    for (int s = 0; s < 8; ++s)
        if (!isfinite(e[s])) f |= kNonfiniteTransform;
    return f;
}

// Hadamard + A8 quantisation, one warp per (row, group) (quantize,
// dense_g256_consumer.cpp:41-73; transform_quantize_a8 :276-323).
__global__ __launch_bounds__(256) void dense_quant_kernel(const uint16_t* x, int M, int K, uint8_t* q,
                                                          __half* scales, int32_t* sums, uint32_t* flags) {
    const int warp = int((size_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    const int groups = K / kG;
    if (warp >= M * groups) return;  // whole warps leave together
    const int r = warp / groups, g = warp % groups;
    const size_t at = size_t(r) * K + size_t(g) * kG;
    float e[8];
    uint32_t f = load_transform(x + at, lane, e);
    quantize_group_warp<127>(e, lane, reinterpret_cast<uint2*>(q + at), scales + size_t(r) * groups + g,
                             sums + size_t(r) * groups + g, f);
    flag_or(flags, f);
}

// A8 projection of rows [m0, m0+16) against 32 columns.  W = columns per tile
// of the weight storage: 16 for the reference's N16 banks
// (codes U32[N/16][K/256][32][16], metadata [N/16][K/256][16]) and 32 for the
// N32 shadow (dense_n32.py:30-31).  Lanes past N (N a multiple of 16 only)
// load nothing and store nothing.
template <int W>
__global__ __launch_bounds__(256, 1) void dense_project_kernel(const uint32_t* codes, const uint32_t* meta,
                                                            const uint8_t* q, const __half* scales,
                                                            const int32_t* sums, int M, int N, int K,
                                                            float* diag, uint16_t* out, uint32_t* flags) {
    extern __shared__ float terms[];  // [groups][kRowBlock][32]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int groups = K / kG;
    const int n = blockIdx.x * 32 + lane;
    const bool live = n < N;
    const int m0 = blockIdx.y * kRowBlock, rows = min(kRowBlock, M - m0);
    const size_t tile_groups = size_t(n / W) * groups;
    const int c = n % W;
    // with one row block every weight word is used once: stream it past the
    // caches; with several, the other row blocks re-read it from L2
    const bool once = gridDim.y == 1;
    for (int g = warp; g < groups; g += kWarps) {
        uint32_t w[32];
        const uint32_t* blk = codes + (tile_groups + g) * 32 * W + c;
        const uint32_t* mp = meta + (tile_groups + g) * W + c;
        if (once) {
#pragma unroll
            for (int j = 0; j < 32; ++j) w[j] = live ? __ldcs(blk + j * W) : 0u;
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) w[j] = live ? __ldg(blk + j * W) : 0u;
        }
        const uint32_t mt = live ? __ldg(mp) : 0u;
        // the even and odd nibbles of each word as bytes, once per group
        // instead of once per row (dot8's masks); the dots are the same.
        // Measured on a B200 at 16 rows: 0.94 ms per 40-bank step against
        // 1.06 ms with the masks inside the row loop.
        uint32_t wlo[32], whi[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            wlo[j] = w[j] & 0x0f0f0f0fu;
            whi[j] = (w[j] >> 4) & 0x0f0f0f0fu;
        }
        for (int m = 0; m < rows; ++m) {
            const size_t row = size_t(m0 + m);
            const uint4* act = reinterpret_cast<const uint4*>(q + row * K + size_t(g) * kG);
            int dot = 0;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const uint4 a = __ldg(act + j);
                dot = __dp4a(int(wlo[2 * j]), int(a.x), dot);
                dot = __dp4a(int(whi[2 * j]), int(a.y), dot);
                dot = __dp4a(int(wlo[2 * j + 1]), int(a.z), dot);
                dot = __dp4a(int(whi[2 * j + 1]), int(a.w), dot);
            }
            const float sa = __half2float(scales[row * groups + g]);
            terms[(g * kRowBlock + m) * 32 + lane] = group_term(sa, dot, sums[row * groups + g], mt);
        }
    }
    __syncthreads();
    uint32_t f = 0;
    for (int m = warp; m < rows; m += kWarps) {
        float v = 0.f;
        for (int g = 0; g < groups; ++g) v = __fadd_rn(v, terms[(g * kRowBlock + m) * 32 + lane]);
        if (live) {
            // store(), dense_g256_consumer.cpp:74-79
            if (!isfinite(v)) f |= kNonfiniteProjection;
            const uint16_t b = bf16_rne(v);
            if ((b & 0x7f80u) == 0x7f80u) f |= kNonfiniteBf16;
            const size_t idx = size_t(m0 + m) * N + n;
            diag[idx] = v;
            out[idx] = b;
        }
    }
    flag_or(flags, f);
}

// Decode rows (M <= 4, the reference's compact crossover, geometry 2): the
// quantisation runs inside the projection, one launch per call.  Warp w first
// issues the weight loads of its group, then transforms and quantises that
// group of every row into its own shared-memory slot (each CTA repeats this
// for the groups it needs, a few hundred instructions per warp, hidden
// behind the weight stream), and dots from there.  Every CTA computes the
// same activations, so the flags it raises are those of the two-kernel path.
// The activation fields of the workspace are not written on this path.
constexpr int kFusedRows = 4;
template <int W>
__global__ __launch_bounds__(256, 3) void dense_fused_kernel(const uint16_t* x, const uint32_t* codes,
                                                          const uint32_t* meta, int M, int N, int K, float* diag,
                                                          uint16_t* out, uint32_t* flags) {
    extern __shared__ float terms[];  // [groups][kFusedRows][32]
    __shared__ __align__(16) uint8_t act[kWarps][kFusedRows][kG];
    __shared__ __half asc[kWarps][kFusedRows];
    __shared__ int32_t asum[kWarps][kFusedRows];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int groups = K / kG;
    const int n = blockIdx.x * 32 + lane;
    const bool live = n < N;
    const size_t tile_groups = size_t(n / W) * groups;
    const int c = n % W;
    uint32_t f = 0;
    for (int g = warp; g < groups; g += kWarps) {
        uint32_t w[32];
        const uint32_t* blk = codes + (tile_groups + g) * 32 * W + c;
#pragma unroll
        for (int j = 0; j < 32; ++j) w[j] = live ? __ldcs(blk + j * W) : 0u;
        const uint32_t mt = live ? __ldg(meta + (tile_groups + g) * W + c) : 0u;
        for (int m = 0; m < M; ++m) {
            float e[8];
            uint32_t qf = load_transform(x + size_t(m) * K + size_t(g) * kG, lane, e);
            quantize_group_warp<127>(e, lane, reinterpret_cast<uint2*>(act[warp][m]), &asc[warp][m],
                                     &asum[warp][m], qf);
            f |= qf;
        }
        __syncwarp();
        for (int m = 0; m < M; ++m) {
            const uint4* a4 = reinterpret_cast<const uint4*>(act[warp][m]);
            int dot = 0;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const uint4 a = a4[j];
                dot = dot8(w[2 * j], make_uint2(a.x, a.y), dot);
                dot = dot8(w[2 * j + 1], make_uint2(a.z, a.w), dot);
            }
            terms[(g * kFusedRows + m) * 32 + lane] =
                group_term(__half2float(asc[warp][m]), dot, asum[warp][m], mt);
        }
        __syncwarp();  // the slot is rewritten for the warp's next group
    }
    __syncthreads();
    for (int m = warp; m < M; m += kWarps) {
        float v = 0.f;
        for (int g = 0; g < groups; ++g) v = __fadd_rn(v, terms[(g * kFusedRows + m) * 32 + lane]);
        if (live) {
            if (!isfinite(v)) f |= kNonfiniteProjection;
            const uint16_t b = bf16_rne(v);
            if ((b & 0x7f80u) == 0x7f80u) f |= kNonfiniteBf16;
            const size_t idx = size_t(m) * N + n;
            diag[idx] = v;
            out[idx] = b;
        }
    }
    flag_or(flags, f);
}

// bf16(H128(x)), one warp per (row, 256-group) (transform_bf16,
// dense_g256_consumer.cpp:192-205): flag 1 on a non-finite input or fp32
// result, flag 8 on a bf16 whose exponent is all ones.
__global__ __launch_bounds__(256) void dense_transform_bf16_kernel(const uint16_t* x, int M, int K, uint16_t* xt,
                                                                   uint32_t* flags) {
    const int warp = int((size_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    const int groups = K / kG;
    if (warp >= M * groups) return;
    const size_t at = size_t(warp / groups) * K + size_t(warp % groups) * kG;
    float e[8];
    uint32_t f = load_transform(x + at, lane, e);
    uint32_t packed[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint16_t lo = bf16_rne(e[2 * i]), hi = bf16_rne(e[2 * i + 1]);
        if ((lo & 0x7f80u) == 0x7f80u || (hi & 0x7f80u) == 0x7f80u) f |= kNonfiniteBf16;
        packed[i] = uint32_t(lo) | (uint32_t(hi) << 16);
    }
    *reinterpret_cast<uint4*>(xt + at + lane * 8) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    flag_or(flags, f);
}

// Dequantised bf16 weights w[N,K] = bf16(scale*code + offset) (fp32 product,
// then sum; dequantize_bf16, dense_g256_consumer.cpp:209-230), one CTA per
// (16-column tile, group): the tile's 2 KB of codes are read as whole lines,
// decoded into a padded shared image [16 columns][256 k] and written as 16
// rows of 512 contiguous bytes.  Flag 8 on a bf16 whose exponent is all ones.
constexpr int kDequantPitch = kG * 2 + 16;  // bytes per column row of the shared image (padded)
__global__ __launch_bounds__(256) void dense_dequant_bf16_kernel(const uint32_t* codes, const uint32_t* meta,
                                                                 int K, uint16_t* w, uint32_t* flags) {
    __shared__ __align__(16) uint8_t image[16 * kDequantPitch];
    const int groups = K / kG;
    const int tile = blockIdx.x / groups, g = blockIdx.x % groups;
    const uint32_t* blk = codes + (size_t(tile) * groups + g) * 32 * 16;
    const uint32_t* mb = meta + (size_t(tile) * groups + g) * 16;
    uint32_t f = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int i = threadIdx.x + 256 * h;  // word j = i / 16 of column c = i % 16
        const int j = i >> 4, c = i & 15;
        const uint32_t code = __ldcs(blk + i);
        const uint32_t mt = __ldg(mb + c);
        const float scale = __half2float(__ushort_as_half(uint16_t(mt & 0xffffu)));
        const float offset = __half2float(__ushort_as_half(uint16_t(mt >> 16)));
        uint32_t packed[4];
#pragma unroll
        for (int d = 0; d < 8; d += 2) {
            const uint16_t lo = bf16_rne(__fadd_rn(__fmul_rn(scale, float((code >> (4 * d)) & 15u)), offset));
            const uint16_t hi = bf16_rne(__fadd_rn(__fmul_rn(scale, float((code >> (4 * d + 4)) & 15u)), offset));
            if ((lo & 0x7f80u) == 0x7f80u || (hi & 0x7f80u) == 0x7f80u) f |= kNonfiniteBf16;
            packed[d / 2] = uint32_t(lo) | (uint32_t(hi) << 16);
        }
        *reinterpret_cast<uint4*>(image + c * kDequantPitch + j * 16) =
            make_uint4(packed[0], packed[1], packed[2], packed[3]);
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int chunk = threadIdx.x + 256 * h;  // 16-byte chunk p of column row c
        const int c = chunk >> 5, p = chunk & 31;
        const uint4 v = *reinterpret_cast<const uint4*>(image + c * kDequantPitch + p * 16);
        *reinterpret_cast<uint4*>(w + size_t(tile * 16 + c) * K + size_t(g) * kG + p * 8) = v;
    }
    flag_or(flags, f);
}

std::atomic<bool> g_smem_attr[2][64];

template <int W>
cudaError_t project(const uint32_t* codes, const uint32_t* meta, uint8_t* ws, const OrnithDenseG256Layout& l,
                    uint16_t* out, uint32_t* flags, int M, int N, int K, cudaStream_t stream) {
    const size_t smem = size_t(K / kG) * kRowBlock * 32 * sizeof(float);
    if (smem > 48 * 1024) {
        int device = 0;
        cudaError_t st = cudaGetDevice(&device);
        if (st != cudaSuccess) return st;
        if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
        std::atomic<bool>& done = g_smem_attr[W == 32][device];
        if (!done.load(std::memory_order_acquire)) {
            st = cudaFuncSetAttribute(dense_project_kernel<W>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      int(kMaxK / kG) * kRowBlock * 32 * int(sizeof(float)));
            if (st != cudaSuccess) return st;
            done.store(true, std::memory_order_release);
        }
    }
    count_launches(1);
    const dim3 grid((N + 31) / 32, (M + kRowBlock - 1) / kRowBlock);
    dense_project_kernel<W><<<grid, kWarps * 32, smem, stream>>>(
        codes, meta, ws + l.low, reinterpret_cast<const __half*>(ws + l.scales),
        reinterpret_cast<const int32_t*>(ws + l.sums), M, N, K, reinterpret_cast<float*>(ws + l.projection), out,
        flags);
    return cudaGetLastError();
}

template <int W>
cudaError_t project_fused(const uint16_t* x, const uint32_t* codes, const uint32_t* meta, uint8_t* ws,
                          const OrnithDenseG256Layout& l, uint16_t* out, uint32_t* flags, int M, int N, int K,
                          cudaStream_t stream) {
    count_launches(1);
    const size_t smem = size_t(K / kG) * kFusedRows * 32 * sizeof(float);
    dense_fused_kernel<W><<<(N + 31) / 32, kWarps * 32, smem, stream>>>(
        x, codes, meta, M, N, K, reinterpret_cast<float*>(ws + l.projection), out, flags);
    return cudaGetLastError();
}

cudaError_t quantize(const uint16_t* x, uint8_t* ws, const OrnithDenseG256Layout& l, uint32_t* flags, int M, int K,
                     cudaStream_t stream) {
    count_launches(1);
    const size_t warps = size_t(M) * (K / kG);
    dense_quant_kernel<<<unsigned((warps + 7) / 8), 256, 0, stream>>>(
        x, M, K, ws + l.low, reinterpret_cast<__half*>(ws + l.scales), reinterpret_cast<int32_t*>(ws + l.sums),
        flags);
    return cudaGetLastError();
}

}  // namespace dense
}  // namespace ornith

using namespace ornith;

extern "C" uint32_t ornith_dense_g256_abi_version(void) { return 1; }

extern "C" cudaError_t ornith_dense_g256_get_layout(int Mcap, int N, int K, int bits, OrnithDenseG256Layout* out) {
    if (!out || Mcap < 0 || Mcap > dense::kMaxM || !dense::shape_ok(N, K) || bits != 8) return cudaErrorInvalidValue;
    *out = dense::layout(Mcap, N, K);
    return cudaSuccess;
}

extern "C" cudaError_t ornith_dense_g256_launch(const void* input, const void* codes, const void* metadata,
                                                void* workspace, size_t bytes, void* output, void* flags, int M,
                                                int Mcap, int N, int K, int bits, int transform, int geometry,
                                                cudaStream_t stream) {
    OrnithDenseG256Layout l{};
    if (ornith_dense_g256_get_layout(Mcap, N, K, bits, &l) != cudaSuccess || M < 0 || M > Mcap ||
        transform != 128 || geometry < 0 || geometry > 2)
        return cudaErrorInvalidValue;
    if (M == 0) return cudaSuccess;
    if (bytes < l.workspace_bytes) return cudaErrorInvalidValue;
    const void* const ptr[6] = {input, codes, metadata, workspace, output, flags};
    const size_t size[6] = {size_t(M) * K * 2, size_t(N) * K / 2, size_t(N) * (K / kG) * 4, bytes,
                            size_t(M) * N * 2, 4};
    const uintptr_t align[6] = {16, 4, 4, 256, 2, 4};
    if (!buffers_ok(ptr, size, align, 3)) return cudaErrorInvalidValue;
    NvtxRange range("ornith.dense.a8");
    auto* ws = static_cast<uint8_t*>(workspace);
    auto* fl = static_cast<uint32_t*>(flags);
    if (M <= dense::kFusedRows)
        return dense::project_fused<16>(static_cast<const uint16_t*>(input), static_cast<const uint32_t*>(codes),
                                        static_cast<const uint32_t*>(metadata), ws, l,
                                        static_cast<uint16_t*>(output), fl, M, N, K, stream);
    cudaError_t st = dense::quantize(static_cast<const uint16_t*>(input), ws, l, fl, M, K, stream);
    if (st != cudaSuccess) return st;
    return dense::project<16>(static_cast<const uint32_t*>(codes), static_cast<const uint32_t*>(metadata), ws, l,
                              static_cast<uint16_t*>(output), fl, M, N, K, stream);
}

extern "C" cudaError_t ornith_dense_g256_launch_n32(const void* input, const void* codes, const void* metadata,
                                                    void* workspace, size_t bytes, void* output, void* flags, int M,
                                                    int Mcap, int N, int K, int bits, int transform, int geometry,
                                                    cudaStream_t stream) {
    OrnithDenseG256Layout l{};
    // dense_g256_consumer.cpp:363-364: 1 <= M <= 16, M <= Mcap, N % 32 == 0, geometry 2
    if (M < 1 || M > dense::kN32Rows || M > Mcap || N % 32 || transform != 128 || geometry != 2 ||
        ornith_dense_g256_get_layout(Mcap, N, K, bits, &l) != cudaSuccess || bytes < l.workspace_bytes)
        return cudaErrorInvalidValue;
    const void* const ptr[6] = {input, codes, metadata, workspace, output, flags};
    const size_t size[6] = {size_t(M) * K * 2, size_t(N) * K / 2, size_t(N) * (K / kG) * 4, bytes,
                            size_t(M) * N * 2, 4};
    const uintptr_t align[6] = {16, 4, 4, 256, 2, 4};
    if (!buffers_ok(ptr, size, align, 3)) return cudaErrorInvalidValue;
    NvtxRange range("ornith.dense.a8_n32");
    auto* ws = static_cast<uint8_t*>(workspace);
    auto* fl = static_cast<uint32_t*>(flags);
    if (M <= dense::kFusedRows)
        return dense::project_fused<32>(static_cast<const uint16_t*>(input), static_cast<const uint32_t*>(codes),
                                        static_cast<const uint32_t*>(metadata), ws, l,
                                        static_cast<uint16_t*>(output), fl, M, N, K, stream);
    cudaError_t st = dense::quantize(static_cast<const uint16_t*>(input), ws, l, fl, M, K, stream);
    if (st != cudaSuccess) return st;
    return dense::project<32>(static_cast<const uint32_t*>(codes), static_cast<const uint32_t*>(metadata), ws, l,
                              static_cast<uint16_t*>(output), fl, M, N, K, stream);
}

extern "C" int ornith_dense_g256_n32_rows(void) { return dense::kN32Rows; }

extern "C" cudaError_t ornith_dense_g256_prepare_bf16(const void* input, const void* codes, const void* metadata,
                                                      void* transformed, void* weights, void* flags, int M, int N,
                                                      int K, cudaStream_t stream) {
    if (M < 0 || M > dense::kMaxM || !dense::shape_ok(N, K)) return cudaErrorInvalidValue;
    if (M == 0) return cudaSuccess;
    const void* const ptr[6] = {input, codes, metadata, transformed, weights, flags};
    const size_t size[6] = {size_t(M) * K * 2, size_t(N) * K / 2, size_t(N) * (K / kG) * 4, size_t(M) * K * 2,
                            size_t(N) * K * 2, 4};
    const uintptr_t align[6] = {16, 16, 4, 16, 16, 4};
    if (!buffers_ok(ptr, size, align, 3)) return cudaErrorInvalidValue;
    NvtxRange range("ornith.dense.prepare_bf16");
    auto* fl = static_cast<uint32_t*>(flags);
    count_launches(2);
    const size_t warps = size_t(M) * (K / kG);
    dense::dense_transform_bf16_kernel<<<unsigned((warps + 7) / 8), 256, 0, stream>>>(
        static_cast<const uint16_t*>(input), M, K, static_cast<uint16_t*>(transformed), fl);
    cudaError_t st = cudaGetLastError();
    if (st != cudaSuccess) return st;
    dense::dense_dequant_bf16_kernel<<<unsigned((N / 16) * (K / kG)), 256, 0, stream>>>(
        static_cast<const uint32_t*>(codes), static_cast<const uint32_t*>(metadata), K,
        static_cast<uint16_t*>(weights), fl);
    return cudaGetLastError();
}
