// Expert-parallel exchanges over NVLink peer memory (declared in
// include/ornith_moe_b200.h).  Dispatch: the home rank stores each token row
// it sends (bf16, 4 KB) and its local ids straight into the expert rank's
// receive buffer.  Return: the expert rank gathers the fp32 down projections
// of the (token, slot) rows it computed and stores each one straight into its
// home rank's receive buffer.  Each direction then raises a flag in the
// receiving ranks' flag arrays, and the receiver waits for the flags of the
// other ranks (bounded) before it reads its buffer.  This replaces the
// gathers and the NCCL all_to_alls of the compact exchange with one kernel
// per direction and side.
//
// Receive buffers are plain device allocations shared by CUDA IPC handles.
// Only ordinary stores reach peer memory: no TMA, no bulk copies, no
// multicast.  The launcher checks every destination range against the
// buffer's capacity on the host before the launch, and the kernel checks each
// row again, so no store can leave a peer's buffer.  Every wait has a time
// limit (flag 64 when it runs out).
//
// Flag arrays.  Every receiving rank has one array per direction of 2*world
// uint32 words: the call numbers (epochs) that each sender raised, then one
// status word per sender.  A sender stores its own timeout bit (flag 64: one
// of its bounded waits gave up) into its status word before it publishes the
// epoch, and the receiver's wait ORs that bit into its own flags after it has
// seen the epoch.  A rank that went on with stale rows after a wait ran out
// therefore makes every rank it sends to report flag 64 as well, instead of
// handing over wrong rows under clean flags.
//
// Wait limit.  The waits on other ranks give up after a limit that is a
// library setting (ornith_moe_b200_set_peer_wait_limit_ns, 1 s by default),
// read when the wait is launched (a captured graph keeps the value it was
// captured with).
//
// Ordering.  Each thread fences at system scope after its stores, the CTA
// meets at a barrier and counts itself done on a device counter; the last CTA
// fences again and publishes `epoch` into slot `me` of every other rank's
// flag array with a system-scope release store.  The home rank's wait reads
// the flags with system-scope acquire loads; its combine is the next kernel
// on the same stream.  A receive buffer is written again only after the next
// layer call's count exchange, which every rank enters after its combine was
// issued on its stream, so a block is never overwritten while it is read.
#include <stdint.h>

#include <atomic>
#include <cstring>

#include "../../include/ornith_moe_b200.h"
#include "moe_layer.cuh"
#include "nvtx_range.h"

namespace ornith {
namespace {

constexpr int kP2PMaxWorld = 8;
constexpr uint64_t kP2PDefaultWaitNs = 1000000000ull;
constexpr uint64_t kP2PMinWaitNs = 1000ull;            // 1 us
constexpr uint64_t kP2PMaxWaitNs = 60000000000ull;     // 60 s
std::atomic<uint64_t> g_peer_wait_ns{kP2PDefaultWaitNs};

struct ReturnArgs {
    const float* route_out;
    const int32_t* rowpos;  // route -> row of route_out on the tensor-core path, else null
    const int32_t* route_index;
    int R, rows, n;
    int seg[kP2PMaxWorld + 1];         // rows [seg[h], seg[h+1]) of route_index go home to rank h
    float* dst[kP2PMaxWorld];          // receive rows of each home rank (this rank's own buffer for h == me)
    long long off[kP2PMaxWorld];       // first row of this rank's block in home h's buffer
    long long cap;                     // rows of every receive buffer
    uint32_t* sig[kP2PMaxWorld];       // flag array of each home rank
    int world, me;
    uint32_t epoch;
    uint32_t* counter;                 // CTAs done; zero between calls
    uint32_t* flags;
};

bool p2p_aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

__device__ __forceinline__ uint64_t p2p_now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Last CTA of a sending kernel: for every other rank h, this rank's timeout
// bit into its status word of h's array, then the epoch (release, system
// scope, so the status store is visible before the epoch is).
__device__ __forceinline__ void publish_epoch(uint32_t* const* sig, int world, int me, uint32_t epoch,
                                              const uint32_t* flags) {
    const uint32_t status = flags ? (*reinterpret_cast<const volatile uint32_t*>(flags) & kFlagWaitTimeout) : 0u;
    for (int h = 0; h < world; ++h) {
        if (h == me) continue;
        asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(sig[h] + world + me), "r"(status) : "memory");
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(sig[h] + me), "r"(epoch) : "memory");
    }
}

__global__ __launch_bounds__(256) void ep_return_p2p_kernel(const ReturnArgs a) {
    uint32_t f = 0;
    for (int i = blockIdx.x; i < a.n; i += gridDim.x) {
        int h = 0;
#pragma unroll
        for (int k = 1; k < kP2PMaxWorld; ++k)
            if (k < a.world && i >= a.seg[k]) h = k;
        const long long drow = a.off[h] + (i - a.seg[h]);
        if (drow < 0 || drow >= a.cap) {  // never true after the launcher's checks
            f |= kFlagInvalidId;
            continue;
        }
        float4* d = reinterpret_cast<float4*>(a.dst[h] + size_t(drow) * kH) + threadIdx.x * 2;
        const int r = a.route_index[i];
        int row = -1;
        if (r >= 0 && r < a.R) row = a.rowpos ? a.rowpos[r] : r;
        if (row < 0 || row >= a.rows) {
            d[0] = d[1] = make_float4(0.f, 0.f, 0.f, 0.f);
            f |= kFlagInvalidId;
            continue;
        }
        const float4* src = reinterpret_cast<const float4*>(a.route_out + size_t(row) * kH) + threadIdx.x * 2;
        const float4 v0 = __ldcs(src), v1 = __ldcs(src + 1);
        d[0] = v0;
        d[1] = v1;
    }
    if (f && threadIdx.x == 0) atomicOr(a.flags, f);
    __threadfence_system();  // this thread's stores, before the CTA counts itself done
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t done = atomicAdd(a.counter, 1u);
        if (done == gridDim.x - 1) {  // the last CTA: every row of this call is stored
            __threadfence_system();
            publish_epoch(a.sig, a.world, a.me, a.epoch, a.flags);
            *a.counter = 0u;  // ready for the next call on this stream
        }
    }
}

struct DispatchArgs {
    const uint16_t* x;                 // bf16 token rows [T][2048] of this (home) rank
    const long long* token_index;      // plan: token of sent row i
    const int32_t* local_ids;          // plan: [n][8] ids in the destination's numbering
    int T, n;
    int seg[kP2PMaxWorld + 1];         // sent rows [seg[d], seg[d+1]) go to expert rank d
    uint16_t* dst_x[kP2PMaxWorld];     // token rows of each expert rank's receive buffer
    int32_t* dst_ids[kP2PMaxWorld];    // local ids of each expert rank's receive buffer
    long long off[kP2PMaxWorld];       // first row of this rank's block at expert rank d
    long long cap;                     // rows of every token receive buffer
    uint32_t* sig[kP2PMaxWorld];       // dispatch flag array of each expert rank
    int world, me;
    uint32_t epoch;
    uint32_t* counter;
    uint32_t* flags;
};

// Home side of the dispatch: sent row i (token token_index[i], the local ids
// of plan row i) is stored at row off[d] + i - seg[d] of expert rank d.
// 256 threads copy one 4 KB token row (one 16-byte store each) and threads
// 0..1 the 32 bytes of ids.  Completion is published as in the return.
__global__ __launch_bounds__(256) void ep_dispatch_p2p_kernel(const DispatchArgs a) {
    uint32_t f = 0;
    for (int i = blockIdx.x; i < a.n; i += gridDim.x) {
        int d = 0;
#pragma unroll
        for (int k = 1; k < kP2PMaxWorld; ++k)
            if (k < a.world && i >= a.seg[k]) d = k;
        const long long drow = a.off[d] + (i - a.seg[d]);
        const long long t = a.token_index[i];
        if (drow < 0 || drow >= a.cap || t < 0 || t >= a.T) {  // never true after the launcher's checks
            f |= kFlagInvalidId;
            continue;
        }
        const uint4* src = reinterpret_cast<const uint4*>(a.x + size_t(t) * kH);
        uint4* dx = reinterpret_cast<uint4*>(a.dst_x[d] + size_t(drow) * kH);
        dx[threadIdx.x] = __ldg(src + threadIdx.x);
        if (threadIdx.x < 2) {
            const uint4* si = reinterpret_cast<const uint4*>(a.local_ids + size_t(i) * kTop);
            uint4* di = reinterpret_cast<uint4*>(a.dst_ids[d] + size_t(drow) * kTop);
            di[threadIdx.x] = __ldg(si + threadIdx.x);
        }
    }
    if (f && threadIdx.x == 0) atomicOr(a.flags, f);
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t done = atomicAdd(a.counter, 1u);
        if (done == gridDim.x - 1) {
            __threadfence_system();
            publish_epoch(a.sig, a.world, a.me, a.epoch, a.flags);
            *a.counter = 0u;
        }
    }
}

// ---- fixed-size exchange (every rank the same T tokens; graph-capturable) ----
// Each rank's receive buffers come in two sets, chosen by the parity of the
// call; the call number lives in device memory (`epoch`: the dispatch kernel
// of call k reads k - 1 and its last CTA stores k), so no host value changes
// between calls.  A rank writes into a peer's set k % 2 only after it has
// seen the peer's dispatch flags of call k - 1, i.e. after the peer finished
// every kernel of call k - 2, the last reader of that set.
struct FixedArgs {
    const uint16_t* x;                 // this rank's token rows [T][2048]
    const int32_t* local_ids;          // [world][T][8]: ids of this rank's tokens in rank d's numbering
    const float* local_w;              // [world][T][8]: their weights (rank-partial combine), or null
    int T, world, me;
    uint16_t* dst_x[2][kP2PMaxWorld];  // per set: token rows [world][T][2048] of rank d
    int32_t* dst_ids[2][kP2PMaxWorld]; // per set: ids [world][T][8] of rank d
    float* dst_w[2][kP2PMaxWorld];     // per set: weights [world][T][8] of rank d (with local_w)
    uint32_t* sig[kP2PMaxWorld];       // dispatch flag array of each rank
    uint32_t* epoch;                   // this rank's call counter
    uint32_t* counter;
    const uint32_t* flags;             // this rank's flags (its timeout bit travels with the epoch)
};

// Dispatch: block `me` of every rank's token buffer receives this rank's T
// rows, and its ids buffer the ids in that rank's numbering.  Item i is
// (rank d = i / T, token t = i % T).
__global__ __launch_bounds__(256) void ep_fixed_dispatch_kernel(const FixedArgs a) {
    const uint32_t call = *a.epoch + 1u;   // stored by the last CTA only, after every CTA read it
    const int set = int(call & 1u);
    for (int i = blockIdx.x; i < a.T * a.world; i += gridDim.x) {
        const int d = i / a.T, t = i % a.T;
        const size_t row = size_t(a.me) * a.T + t;
        reinterpret_cast<uint4*>(a.dst_x[set][d] + row * kH)[threadIdx.x] =
            __ldg(reinterpret_cast<const uint4*>(a.x + size_t(t) * kH) + threadIdx.x);
        if (threadIdx.x < 2)
            reinterpret_cast<uint4*>(a.dst_ids[set][d] + row * kTop)[threadIdx.x] =
                __ldg(reinterpret_cast<const uint4*>(a.local_ids + (size_t(d) * a.T + t) * kTop) + threadIdx.x);
        else if (threadIdx.x < 4 && a.local_w)
            reinterpret_cast<uint4*>(a.dst_w[set][d] + row * kTop)[threadIdx.x - 2] =
                __ldg(reinterpret_cast<const uint4*>(a.local_w + (size_t(d) * a.T + t) * kTop) + threadIdx.x - 2);
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(a.counter, 1u) == gridDim.x - 1) {
        __threadfence_system();
        publish_epoch(a.sig, a.world, a.me, call, a.flags);
        *a.counter = 0u;
        *a.epoch = call;
    }
}

struct FixedReturnArgs {
    const float* route_out;
    const int32_t* rowpos;             // route -> row of route_out on the tensor-core path, else null
    const int32_t* ids;                // [world * T][8] the local ids the layer call used
    int T, world, me;
    float* dst_rows[2][kP2PMaxWorld];  // per set: result rows [T * 8][2048] of home rank h
    uint32_t* sig[kP2PMaxWorld];       // return flag array of each rank
    const uint32_t* epoch;
    uint32_t* counter;
    uint32_t* flags;
};

// Return: received row r = h * T + t computed the slots s whose local id is
// valid here; each goes to row t * 8 + s of home h's result buffer (every
// slot has one owner, so the rows of different ranks never collide).
__global__ __launch_bounds__(256) void ep_fixed_return_kernel(const FixedReturnArgs a) {
    const uint32_t call = *a.epoch;
    const int set = int(call & 1u);
    const int R = a.T * a.world * kTop;
    uint32_t f = 0;
    for (int i = blockIdx.x; i < R; i += gridDim.x) {
        if (a.ids[i] < 0) continue;   // padding, or a slot another rank owns
        const int r = i / kTop, s = i % kTop, h = r / a.T, t = r % a.T;
        const int row = a.rowpos ? a.rowpos[i] : i;
        float4* d = reinterpret_cast<float4*>(a.dst_rows[set][h] + (size_t(t) * kTop + s) * kH) + threadIdx.x * 2;
        if (row < 0 || row >= R + a.T * a.world) {
            d[0] = d[1] = make_float4(0.f, 0.f, 0.f, 0.f);
            f |= kFlagInvalidId;
            continue;
        }
        const float4* src = reinterpret_cast<const float4*>(a.route_out + size_t(row) * kH) + threadIdx.x * 2;
        const float4 v0 = __ldcs(src), v1 = __ldcs(src + 1);
        d[0] = v0;
        d[1] = v1;
    }
    if (f && threadIdx.x == 0) atomicOr(a.flags, f);
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(a.counter, 1u) == gridDim.x - 1) {
        __threadfence_system();
        publish_epoch(a.sig, a.world, a.me, call, a.flags);
        *a.counter = 0u;
    }
}

struct FixedPartialArgs {
    const float* partial;              // the layer call's fp32 sums [world * T][2048] (final_f32)
    const int32_t* ids;                // [world * T][8] the local ids the layer call used
    int T, world, me;
    float* dst_part[2][kP2PMaxWorld];  // per set: partial rows [world][T][2048] of home rank h
    uint32_t* sig[kP2PMaxWorld];       // return flag array of each rank
    const uint32_t* epoch;
    uint32_t* counter;
    uint32_t* flags;
};

// Rank-partial return: received row r = h * T + t, if any of its slots has a
// valid local id here, goes to row me * T + t of home h's partial buffer (its
// sum over this rank's slots); rows with no slot here are not sent (the home
// rank reads only the rows of ranks that own one of the token's slots).
__global__ __launch_bounds__(256) void ep_fixed_return_partial_kernel(const FixedPartialArgs a) {
    const uint32_t call = *a.epoch;
    const int set = int(call & 1u);
    for (int r = blockIdx.x; r < a.T * a.world; r += gridDim.x) {
        const int4 i0 = __ldg(reinterpret_cast<const int4*>(a.ids + size_t(r) * kTop));
        const int4 i1 = __ldg(reinterpret_cast<const int4*>(a.ids + size_t(r) * kTop) + 1);
        const int top = max(max(max(i0.x, i0.y), max(i0.z, i0.w)), max(max(i1.x, i1.y), max(i1.z, i1.w)));
        if (top < 0) continue;  // no slot of this token here
        const int h = r / a.T, t = r % a.T;
        const float4* src = reinterpret_cast<const float4*>(a.partial + size_t(r) * kH) + threadIdx.x * 2;
        float4* d = reinterpret_cast<float4*>(a.dst_part[set][h] + (size_t(a.me) * a.T + t) * kH) + threadIdx.x * 2;
        const float4 v0 = __ldcs(src), v1 = __ldcs(src + 1);
        d[0] = v0;
        d[1] = v1;
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(a.counter, 1u) == gridDim.x - 1) {
        __threadfence_system();
        publish_epoch(a.sig, a.world, a.me, call, a.flags);
        *a.counter = 0u;
    }
}

// Lane d waits until rank d's epoch in this rank's array reaches `epoch`
// (wrap-around safe), for at most limit_ns of %globaltimer; then ORs rank d's
// timeout bit (its status word) into this rank's flags.  A wait that runs out
// raises flag 64 and returns.
__device__ __forceinline__ void wait_peer_epoch(const uint32_t* sig, int world, int d, uint32_t epoch,
                                                uint64_t limit_ns, uint32_t* flags) {
    const uint64_t t0 = p2p_now_ns();
    for (;;) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(sig + d) : "memory");
        if (int32_t(v - epoch) >= 0) break;
        if (p2p_now_ns() - t0 > limit_ns) {
            atomicOr(flags, uint32_t(kFlagWaitTimeout));
            return;
        }
        __nanosleep(200);
    }
    uint32_t status;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(status) : "l"(sig + world + d) : "memory");
    if (status & kFlagWaitTimeout) atomicOr(flags, uint32_t(kFlagWaitTimeout));
}

// Waits as ep_wait_signals_kernel does, for the call number in device memory.
__global__ __launch_bounds__(32) void ep_wait_epoch_kernel(const uint32_t* sig, int world, int me,
                                                           const uint32_t* epoch, uint64_t limit_ns,
                                                           uint32_t* flags) {
    const int d = threadIdx.x;
    if (d >= world || d == me) return;
    wait_peer_epoch(sig, world, d, *epoch, limit_ns, flags);
}

__global__ __launch_bounds__(32) void ep_wait_signals_kernel(const uint32_t* sig, int world, int me, uint32_t epoch,
                                                             uint64_t limit_ns, uint32_t* flags) {
    const int d = threadIdx.x;
    if (d >= world || d == me) return;
    wait_peer_epoch(sig, world, d, epoch, limit_ns, flags);
}

}  // namespace
}  // namespace ornith

using namespace ornith;

extern "C" cudaError_t ornith_moe_b200_ep_buffer_alloc(size_t bytes, void** ptr) {
    if (!ptr || !bytes) return cudaErrorInvalidValue;
    *ptr = nullptr;
    void* p = nullptr;
    cudaError_t st = cudaMalloc(&p, bytes);
    if (st != cudaSuccess) return st;
    if ((st = cudaMemset(p, 0, bytes)) != cudaSuccess) {
        cudaFree(p);
        return st;
    }
    *ptr = p;
    return cudaSuccess;
}

extern "C" cudaError_t ornith_moe_b200_ep_buffer_free(void* ptr) { return ptr ? cudaFree(ptr) : cudaSuccess; }

extern "C" cudaError_t ornith_moe_b200_ep_ipc_handle(const void* base, void* handle_out) {
    if (!base || !handle_out) return cudaErrorInvalidValue;
    cudaIpcMemHandle_t h;
    const cudaError_t st = cudaIpcGetMemHandle(&h, const_cast<void*>(base));
    if (st == cudaSuccess) memcpy(handle_out, &h, sizeof(h));
    return st;
}

extern "C" cudaError_t ornith_moe_b200_ep_ipc_open(const void* handle, void** ptr) {
    if (!handle || !ptr) return cudaErrorInvalidValue;
    *ptr = nullptr;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
}

extern "C" cudaError_t ornith_moe_b200_ep_ipc_close(void* ptr) {
    return ptr ? cudaIpcCloseMemHandle(ptr) : cudaSuccess;
}

extern "C" cudaError_t ornith_moe_b200_ep_return_p2p(const void* workspace, size_t bytes, int T, int Tcap,
                                                     const void* route_index_i32, int n, const int32_t* seg,
                                                     void* const* dst_rows, const int64_t* dst_offset,
                                                     int64_t dst_capacity_rows, void* const* signals, int world,
                                                     int me, uint32_t epoch, void* counter_u32, void* flags,
                                                     cudaStream_t stream) {
    if (Tcap < 0 || Tcap > kTcapMax || T < 0 || T > Tcap || n < 0 || world < 1 || world > kP2PMaxWorld || me < 0 ||
        me >= world || dst_capacity_rows < 0)
        return cudaErrorInvalidValue;
    const Workspace w = workspace_layout(Tcap);
    if (bytes < w.bytes) return cudaErrorInvalidValue;
    if (!workspace || (n && !route_index_i32) || !seg || !dst_rows || !dst_offset || !signals || !counter_u32 ||
        !flags || !p2p_aligned(workspace, 256) || !p2p_aligned(route_index_i32, 4) || !p2p_aligned(counter_u32, 4) ||
        !p2p_aligned(flags, 4))
        return cudaErrorInvalidValue;
    ReturnArgs a{};
    if (seg[0] != 0 || seg[world] != n) return cudaErrorInvalidValue;
    for (int h = 0; h < world; ++h) {
        const int rows_h = seg[h + 1] - seg[h];
        // every destination range inside its buffer, checked before any store is issued
        if (rows_h < 0 || dst_offset[h] < 0 || dst_offset[h] + rows_h > dst_capacity_rows) return cudaErrorInvalidValue;
        if ((rows_h && !dst_rows[h]) || !p2p_aligned(dst_rows[h], 16)) return cudaErrorInvalidValue;
        if (h != me && (!signals[h] || !p2p_aligned(signals[h], 4))) return cudaErrorInvalidValue;
        a.seg[h] = seg[h];
        a.dst[h] = static_cast<float*>(dst_rows[h]);
        a.off[h] = dst_offset[h];
        a.sig[h] = static_cast<uint32_t*>(signals[h]);
    }
    a.seg[world] = n;
    const uint8_t* ws = static_cast<const uint8_t*>(workspace);
    a.route_out = reinterpret_cast<const float*>(ws + w.route_out);
    a.rowpos = rows_by_position(T) ? reinterpret_cast<const int32_t*>(ws + w.rowpos) : nullptr;
    a.route_index = static_cast<const int32_t*>(route_index_i32);
    a.R = T * kTop;
    a.rows = T * (kTop + 1);
    a.n = n;
    a.cap = dst_capacity_rows;
    a.world = world;
    a.me = me;
    a.epoch = epoch;
    a.counter = static_cast<uint32_t*>(counter_u32);
    a.flags = static_cast<uint32_t*>(flags);
    NvtxRange range("ornith.ep.return_p2p");
    int device = 0, sms = 0;
    cudaError_t st = cudaGetDevice(&device);
    if (st != cudaSuccess) return st;
    if ((st = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess) return st;
    // at least one CTA: with no rows the call still raises the flags
    const int grid = n < 2 * sms ? (n > 0 ? n : 1) : 2 * sms;
    count_launches(1);
    ep_return_p2p_kernel<<<grid, 256, 0, stream>>>(a);
    return cudaGetLastError();
}

extern "C" cudaError_t ornith_moe_b200_ep_dispatch_p2p(const void* x_bf16, int T, const void* token_index_i64,
                                                       const void* local_ids_i32, int n, const int32_t* seg,
                                                       void* const* dst_x, void* const* dst_ids,
                                                       const int64_t* dst_offset, int64_t dst_capacity_rows,
                                                       void* const* signals, int world, int me, uint32_t epoch,
                                                       void* counter_u32, void* flags, cudaStream_t stream) {
    if (T < 0 || T > kTcapMax || n < 0 || n > T * world || world < 1 || world > kP2PMaxWorld || me < 0 ||
        me >= world || dst_capacity_rows < 0)
        return cudaErrorInvalidValue;
    if ((n && (!x_bf16 || !token_index_i64 || !local_ids_i32)) || !seg || !dst_x || !dst_ids || !dst_offset ||
        !signals || !counter_u32 || !flags || !p2p_aligned(x_bf16, 16) || !p2p_aligned(token_index_i64, 8) ||
        !p2p_aligned(local_ids_i32, 16) || !p2p_aligned(counter_u32, 4) || !p2p_aligned(flags, 4))
        return cudaErrorInvalidValue;
    DispatchArgs a{};
    if (seg[0] != 0 || seg[world] != n) return cudaErrorInvalidValue;
    for (int d = 0; d < world; ++d) {
        const int rows_d = seg[d + 1] - seg[d];
        if (rows_d < 0 || dst_offset[d] < 0 || dst_offset[d] + rows_d > dst_capacity_rows) return cudaErrorInvalidValue;
        if ((rows_d && (!dst_x[d] || !dst_ids[d])) || !p2p_aligned(dst_x[d], 16) || !p2p_aligned(dst_ids[d], 16))
            return cudaErrorInvalidValue;
        if (d != me && (!signals[d] || !p2p_aligned(signals[d], 4))) return cudaErrorInvalidValue;
        a.seg[d] = seg[d];
        a.dst_x[d] = static_cast<uint16_t*>(dst_x[d]);
        a.dst_ids[d] = static_cast<int32_t*>(dst_ids[d]);
        a.off[d] = dst_offset[d];
        a.sig[d] = static_cast<uint32_t*>(signals[d]);
    }
    a.seg[world] = n;
    a.x = static_cast<const uint16_t*>(x_bf16);
    a.token_index = static_cast<const long long*>(token_index_i64);
    a.local_ids = static_cast<const int32_t*>(local_ids_i32);
    a.T = T;
    a.n = n;
    a.cap = dst_capacity_rows;
    a.world = world;
    a.me = me;
    a.epoch = epoch;
    a.counter = static_cast<uint32_t*>(counter_u32);
    a.flags = static_cast<uint32_t*>(flags);
    NvtxRange range("ornith.ep.dispatch_p2p");
    int device = 0, sms = 0;
    cudaError_t st = cudaGetDevice(&device);
    if (st != cudaSuccess) return st;
    if ((st = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess) return st;
    const int grid = n < 2 * sms ? (n > 0 ? n : 1) : 2 * sms;
    count_launches(1);
    ep_dispatch_p2p_kernel<<<grid, 256, 0, stream>>>(a);
    return cudaGetLastError();
}

namespace {
cudaError_t fixed_dispatch(const void* x_bf16, const void* local_ids_i32, const void* local_w_f32, int T,
                           void* const* dst_x, void* const* dst_ids, void* const* dst_w, int64_t dst_capacity_rows,
                           void* const* signals, int world, int me, void* epoch_u32, void* counter_u32,
                           const void* flags_u32, cudaStream_t stream) {
    if (local_w_f32 && (!dst_w || !p2p_aligned(local_w_f32, 16))) return cudaErrorInvalidValue;
    if (T < 1 || T > kTcapMax || world < 1 || world > kP2PMaxWorld || me < 0 || me >= world || !x_bf16 ||
        !local_ids_i32 || !dst_x || !dst_ids || !signals || !epoch_u32 || !counter_u32 || !flags_u32 ||
        !p2p_aligned(x_bf16, 16) || !p2p_aligned(local_ids_i32, 16) || !p2p_aligned(epoch_u32, 4) ||
        !p2p_aligned(counter_u32, 4) || !p2p_aligned(flags_u32, 4) || size_t(T) * world > size_t(kTcapMax))
        return cudaErrorInvalidValue;
    // every set of every rank's token buffer holds the world*T rows this exchange writes
    if (dst_capacity_rows < int64_t(T) * world) return cudaErrorInvalidValue;
    FixedArgs a{};
    for (int set = 0; set < 2; ++set)
        for (int d = 0; d < world; ++d) {
            void* px = dst_x[set * world + d];
            void* pi = dst_ids[set * world + d];
            if (!px || !pi || !p2p_aligned(px, 16) || !p2p_aligned(pi, 16)) return cudaErrorInvalidValue;
            a.dst_x[set][d] = static_cast<uint16_t*>(px);
            a.dst_ids[set][d] = static_cast<int32_t*>(pi);
            if (local_w_f32) {
                void* pw = dst_w[set * world + d];
                if (!pw || !p2p_aligned(pw, 16)) return cudaErrorInvalidValue;
                a.dst_w[set][d] = static_cast<float*>(pw);
            }
        }
    a.local_w = static_cast<const float*>(local_w_f32);
    for (int d = 0; d < world; ++d) {
        if (d != me && (!signals[d] || !p2p_aligned(signals[d], 4))) return cudaErrorInvalidValue;
        a.sig[d] = static_cast<uint32_t*>(signals[d]);
    }
    a.x = static_cast<const uint16_t*>(x_bf16);
    a.local_ids = static_cast<const int32_t*>(local_ids_i32);
    a.T = T;
    a.world = world;
    a.me = me;
    a.epoch = static_cast<uint32_t*>(epoch_u32);
    a.counter = static_cast<uint32_t*>(counter_u32);
    a.flags = static_cast<const uint32_t*>(flags_u32);
    NvtxRange range("ornith.ep.fixed_dispatch");
    int device = 0, sms = 0;
    cudaError_t st = cudaGetDevice(&device);
    if (st != cudaSuccess) return st;
    if ((st = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess) return st;
    const int items = T * world;
    count_launches(1);
    ep_fixed_dispatch_kernel<<<items < 2 * sms ? items : 2 * sms, 256, 0, stream>>>(a);
    return cudaGetLastError();
}
}  // namespace

extern "C" cudaError_t ornith_moe_b200_ep_fixed_dispatch(const void* x_bf16, const void* local_ids_i32, int T,
                                                         void* const* dst_x, void* const* dst_ids,
                                                         int64_t dst_capacity_rows, void* const* signals, int world,
                                                         int me, void* epoch_u32, void* counter_u32,
                                                         const void* flags_u32, cudaStream_t stream) {
    return fixed_dispatch(x_bf16, local_ids_i32, nullptr, T, dst_x, dst_ids, nullptr, dst_capacity_rows, signals,
                          world, me, epoch_u32, counter_u32, flags_u32, stream);
}

extern "C" cudaError_t ornith_moe_b200_ep_fixed_dispatch_weights(
    const void* x_bf16, const void* local_ids_i32, const void* local_w_f32, int T, void* const* dst_x,
    void* const* dst_ids, void* const* dst_w, int64_t dst_capacity_rows, void* const* signals, int world, int me,
    void* epoch_u32, void* counter_u32, const void* flags_u32, cudaStream_t stream) {
    if (!local_w_f32) return cudaErrorInvalidValue;
    return fixed_dispatch(x_bf16, local_ids_i32, local_w_f32, T, dst_x, dst_ids, dst_w, dst_capacity_rows, signals,
                          world, me, epoch_u32, counter_u32, flags_u32, stream);
}

extern "C" cudaError_t ornith_moe_b200_ep_fixed_return_partial(const void* workspace, size_t bytes, int T,
                                                               int Tcap, const void* ids_i32, void* const* dst_part,
                                                               int64_t dst_capacity_rows, void* const* signals,
                                                               int world, int me, const void* epoch_u32,
                                                               void* counter_u32, void* flags, cudaStream_t stream) {
    // T: tokens per rank; the layer call ran on world * T rows with capacity Tcap
    if (T < 1 || world < 1 || world > kP2PMaxWorld || me < 0 || me >= world || Tcap < 0 || Tcap > kTcapMax ||
        T * world > Tcap)
        return cudaErrorInvalidValue;
    // every set of every home rank's partial buffer holds world*T rows
    if (dst_capacity_rows < int64_t(T) * world) return cudaErrorInvalidValue;
    const Workspace w = workspace_layout(Tcap);
    if (bytes < w.bytes || !workspace || !ids_i32 || !dst_part || !signals || !epoch_u32 || !counter_u32 ||
        !flags || !p2p_aligned(workspace, 256) || !p2p_aligned(ids_i32, 16) || !p2p_aligned(epoch_u32, 4) ||
        !p2p_aligned(counter_u32, 4) || !p2p_aligned(flags, 4))
        return cudaErrorInvalidValue;
    FixedPartialArgs a{};
    for (int set = 0; set < 2; ++set)
        for (int h = 0; h < world; ++h) {
            void* p = dst_part[set * world + h];
            if (!p || !p2p_aligned(p, 16)) return cudaErrorInvalidValue;
            a.dst_part[set][h] = static_cast<float*>(p);
        }
    for (int h = 0; h < world; ++h) {
        if (h != me && (!signals[h] || !p2p_aligned(signals[h], 4))) return cudaErrorInvalidValue;
        a.sig[h] = static_cast<uint32_t*>(signals[h]);
    }
    a.partial = reinterpret_cast<const float*>(static_cast<const uint8_t*>(workspace) + w.final_f32);
    a.ids = static_cast<const int32_t*>(ids_i32);
    a.T = T;
    a.world = world;
    a.me = me;
    a.epoch = static_cast<const uint32_t*>(epoch_u32);
    a.counter = static_cast<uint32_t*>(counter_u32);
    a.flags = static_cast<uint32_t*>(flags);
    NvtxRange range("ornith.ep.fixed_return_partial");
    int device = 0, sms = 0;
    cudaError_t st = cudaGetDevice(&device);
    if (st != cudaSuccess) return st;
    if ((st = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess) return st;
    const int items = T * world;
    count_launches(1);
    ep_fixed_return_partial_kernel<<<items < 2 * sms ? items : 2 * sms, 256, 0, stream>>>(a);
    return cudaGetLastError();
}

extern "C" cudaError_t ornith_moe_b200_ep_fixed_return(const void* workspace, size_t bytes, int T, int Tcap,
                                                       const void* ids_i32, void* const* dst_rows,
                                                       int64_t dst_capacity_rows, void* const* signals, int world,
                                                       int me, const void* epoch_u32, void* counter_u32, void* flags,
                                                       cudaStream_t stream) {
    // T: tokens per rank; the layer call ran on world * T rows with capacity Tcap
    if (T < 1 || world < 1 || world > kP2PMaxWorld || me < 0 || me >= world || Tcap < 0 || Tcap > kTcapMax ||
        T * world > Tcap)
        return cudaErrorInvalidValue;
    // every set of every home rank's result buffer holds the T*8 slot rows
    if (dst_capacity_rows < int64_t(T) * kTop) return cudaErrorInvalidValue;
    const Workspace w = workspace_layout(Tcap);
    if (bytes < w.bytes || !workspace || !ids_i32 || !dst_rows || !signals || !epoch_u32 || !counter_u32 ||
        !flags || !p2p_aligned(workspace, 256) || !p2p_aligned(ids_i32, 4) || !p2p_aligned(epoch_u32, 4) ||
        !p2p_aligned(counter_u32, 4) || !p2p_aligned(flags, 4))
        return cudaErrorInvalidValue;
    FixedReturnArgs a{};
    for (int set = 0; set < 2; ++set)
        for (int h = 0; h < world; ++h) {
            void* p = dst_rows[set * world + h];
            if (!p || !p2p_aligned(p, 16)) return cudaErrorInvalidValue;
            a.dst_rows[set][h] = static_cast<float*>(p);
        }
    for (int h = 0; h < world; ++h) {
        if (h != me && (!signals[h] || !p2p_aligned(signals[h], 4))) return cudaErrorInvalidValue;
        a.sig[h] = static_cast<uint32_t*>(signals[h]);
    }
    const int rows_in = T * world;
    const uint8_t* ws = static_cast<const uint8_t*>(workspace);
    a.route_out = reinterpret_cast<const float*>(ws + w.route_out);
    a.rowpos = rows_by_position(rows_in) ? reinterpret_cast<const int32_t*>(ws + w.rowpos) : nullptr;
    a.ids = static_cast<const int32_t*>(ids_i32);
    a.T = T;
    a.world = world;
    a.me = me;
    a.epoch = static_cast<const uint32_t*>(epoch_u32);
    a.counter = static_cast<uint32_t*>(counter_u32);
    a.flags = static_cast<uint32_t*>(flags);
    NvtxRange range("ornith.ep.fixed_return");
    int device = 0, sms = 0;
    cudaError_t st = cudaGetDevice(&device);
    if (st != cudaSuccess) return st;
    if ((st = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess) return st;
    const int items = rows_in * kTop;
    count_launches(1);
    ep_fixed_return_kernel<<<items < 2 * sms ? items : 2 * sms, 256, 0, stream>>>(a);
    return cudaGetLastError();
}

extern "C" cudaError_t ornith_moe_b200_ep_wait_epoch(const void* signals_u32, int world, int me,
                                                     const void* epoch_u32, void* flags, cudaStream_t stream) {
    if (world < 1 || world > kP2PMaxWorld || me < 0 || me >= world || !signals_u32 || !epoch_u32 || !flags ||
        !p2p_aligned(signals_u32, 4) || !p2p_aligned(epoch_u32, 4) || !p2p_aligned(flags, 4))
        return cudaErrorInvalidValue;
    if (world == 1) return cudaSuccess;
    NvtxRange range("ornith.ep.wait");
    count_launches(1);
    ep_wait_epoch_kernel<<<1, 32, 0, stream>>>(static_cast<const uint32_t*>(signals_u32), world, me,
                                               static_cast<const uint32_t*>(epoch_u32), g_peer_wait_ns.load(),
                                               static_cast<uint32_t*>(flags));
    return cudaGetLastError();
}

extern "C" cudaError_t ornith_moe_b200_ep_wait_signals(const void* signals_u32, int world, int me, uint32_t epoch,
                                                       void* flags, cudaStream_t stream) {
    if (world < 1 || world > kP2PMaxWorld || me < 0 || me >= world || !signals_u32 || !flags ||
        !p2p_aligned(signals_u32, 4) || !p2p_aligned(flags, 4))
        return cudaErrorInvalidValue;
    if (world == 1) return cudaSuccess;
    NvtxRange range("ornith.ep.wait");
    count_launches(1);
    ep_wait_signals_kernel<<<1, 32, 0, stream>>>(static_cast<const uint32_t*>(signals_u32), world, me, epoch,
                                                 g_peer_wait_ns.load(), static_cast<uint32_t*>(flags));
    return cudaGetLastError();
}

extern "C" cudaError_t ornith_moe_b200_set_peer_wait_limit_ns(uint64_t limit_ns) {
    if (limit_ns < kP2PMinWaitNs || limit_ns > kP2PMaxWaitNs) return cudaErrorInvalidValue;
    g_peer_wait_ns.store(limit_ns);
    return cudaSuccess;
}

extern "C" uint64_t ornith_moe_b200_peer_wait_limit_ns(void) { return g_peer_wait_ns.load(); }
