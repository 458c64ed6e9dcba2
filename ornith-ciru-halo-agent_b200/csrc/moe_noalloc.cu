// Routed-MoE launch for callers that cannot allocate device memory.
//
// Some callers of this library have no way to obtain device memory for the
// workspace that ornith_routed_direct_launch needs: kernel-library plugins
// inside frameworks that own every device allocation and hand a plugin only its
// input and output tensors, embedders whose allocator is not reachable from the
// code that issues the launch, and code paths that must not call cudaMalloc
// (for instance while another component is capturing the stream).
// ornith_routed_direct_launch_noalloc serves them: the caller passes inputs and
// outputs only, and the scratch lives in a file-scope __device__ array of a
// fixed 1 MiB in this library, enough for up to 8 tokens per call.
//
// What a caller must know:
//   * every GPU that loads the library holds this 1 MiB array until the
//     process exits;
//   * every call on a device shares the one array and it keeps the previous
//     call's contents; the counters that must start at zero are cleared by
//     each launch itself (a clearing kernel on the caller's stream) and nothing
//     else is assumed to be zero;
//   * two calls whose work can overlap on the GPU (different streams without
//     ordering between them, or different host threads) race on the array, so
//     callers must order them, for example on one stream;
//   * the first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (once per device, with that device current), so
//     that first call should come before any stream capture;
//   * that address is kept for the life of the process: calls after
//     cudaDeviceReset, or after the device's primary context was destroyed and
//     made again, are not supported.
// The arithmetic is that of ornith_routed_direct_launch (A8) through the
// fused decode kernel, which this entry always runs (the environment setting
// that forces the multi-kernel path, and the NVTX layer range, belong to the
// workspace entry only); only the place of the scratch differs.
#include <mutex>

#include "../../include/ornith_moe_b200.h"
#include "moe_layer.cuh"

namespace ornith {
namespace {

constexpr int kNoAllocMaxT = 8;
constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;

// Host code may only use this name to look up the device address below: as
// a host expression it is a stand-in, not a pointer a kernel can use.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[64] = {};

// Device address of the scratch array on the current device (looked up once).
cudaError_t noalloc_scratch(void** out) {
    int device = 0;
    cudaError_t st = cudaGetDevice(&device);
    if (st != cudaSuccess) return st;
    if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (!g_noalloc_ptr[device]) {
        void* p = nullptr;
        st = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (st != cudaSuccess) return st;
        g_noalloc_ptr[device] = p;
    }
    *out = g_noalloc_ptr[device];
    return cudaSuccess;
}

bool aligned_to(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace
}  // namespace ornith

using namespace ornith;

extern "C" cudaError_t ornith_routed_direct_launch_noalloc(const void* input, const void* weights, const void* ids,
                                                           const void* gate_codes, const void* gate_meta,
                                                           const void* down_codes, const void* down_meta,
                                                           void* output, void* flags, int T, cudaStream_t stream) {
    // more tokens than the fixed scratch holds: refuse rather than overrun it
    if (T < 0 || T > kNoAllocMaxT) return cudaErrorInvalidValue;
    if (!T) return cudaSuccess;
    if (!input || !weights || !ids || !gate_codes || !gate_meta || !down_codes || !down_meta || !output || !flags)
        return cudaErrorInvalidValue;
    if (!aligned_to(input, 16) || !aligned_to(output, 16) || !aligned_to(gate_codes, 16) ||
        !aligned_to(gate_meta, 16) || !aligned_to(down_codes, 16) || !aligned_to(down_meta, 16) ||
        !aligned_to(weights, 4) || !aligned_to(ids, 4) || !aligned_to(flags, 4))
        return cudaErrorInvalidValue;
    const Workspace w = workspace_layout(kNoAllocMaxT);
    if (w.bytes > kNoAllocScratchBytes) return cudaErrorInvalidConfiguration;
    void* scratch = nullptr;
    cudaError_t st = noalloc_scratch(&scratch);
    if (st != cudaSuccess) return st;
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
    a.ws = static_cast<uint8_t*>(scratch);
    a.L = w;
    a.T = T;
    a.a8 = 1;
    return launch_decode(a, stream);
}
