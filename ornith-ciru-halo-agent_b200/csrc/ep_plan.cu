// Dispatch plan of one expert-parallel layer call, built on the device
// (ornith_moe_b200_ep_plan, declared in include/ornith_moe_b200.h).
//
// For the rank's T tokens and a placement (owning rank and bank index of each
// of the 256 experts) one CTA produces everything the exchange needs:
//   counts      int64 [world][2]  (tokens sent to d, (token, slot) rows d returns)
//   token_index int64 [n]         sent rows grouped by destination, tokens ascending
//   dest        int64 [n]         destination of each sent row
//   local_ids   int32 [n][8]      ids in the destination's bank numbering, -1 for
//                                 slots owned elsewhere, padding or invalid
//   slot_mask   uint8 [n][8]      1 where the destination owns the slot
//   row_index   int32 [T][8]      row of (t, s) among the returned rows, which
//                                 arrive destination by destination in the order
//                                 of the sent rows, slots ascending; -1 where no
//                                 rank owns the slot
// with n = sum of the tokens sent.  The buffers hold the largest n, T * world
// rows; only the first n are written.  Ids outside 0..255 (and -1 padding)
// belong to no rank.  The outputs equal those of the torch form of the plan
// in the Python module ornith_b200.ep (_owner_mask, _plan_from_mask,
// route_row_index) bit for bit.
//
// Thread i owns the contiguous tokens [i*c, (i+1)*c), c = ceil(T/1024) <= 8.
// A first pass counts, per destination, the tokens each thread sends and the
// slots they carry; two block-wide exclusive scans (warp shuffles, then the 32
// warp totals) give each thread its first position and first returned row per
// destination; a second pass writes its rows in token order.
#include <stdint.h>

#include "../../include/ornith_moe_b200.h"
#include "moe_layer.cuh"
#include "nvtx_range.h"

namespace ornith {
namespace {

constexpr int kPlanThreads = 1024;
constexpr int kPlanMaxWorld = 8;
constexpr int kPlanValues = 2 * kPlanMaxWorld;  // per destination: tokens sent, slots returned

bool plan_aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Owners of the eight slots of token t (-1: no rank) and the mask of destinations.
__device__ __forceinline__ uint32_t token_owners(const int32_t* ids, int t, const int* owner, int world, int (&own)[8],
                                                 int (&id)[8]) {
    uint32_t mask = 0;
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        id[s] = ids[size_t(t) * 8 + s];
        const bool valid = id[s] >= 0 && id[s] < 256;
        const int d = owner[valid ? id[s] : 0];  // every index in range
        own[s] = (valid && d >= 0 && d < world) ? d : -1;
        if (own[s] >= 0) mask |= 1u << own[s];
    }
    return mask;
}

__global__ __launch_bounds__(kPlanThreads) void ep_plan_kernel(const int32_t* ids, int T, const int32_t* owner_table,
                                                               const int32_t* local_table, int world,
                                                               long long* counts, long long* token_index,
                                                               long long* dest, int32_t* local_ids, uint8_t* slot_mask,
                                                               int32_t* row_index) {
    __shared__ int owner[256], local[256];
    __shared__ int warp_part[32][kPlanValues];  // warp totals, then exclusive warp offsets
    __shared__ int totals[kPlanValues];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int e = tid; e < 256; e += kPlanThreads) {
        owner[e] = owner_table[e];
        local[e] = local_table[e];
    }
    __syncthreads();
    const int chunk = (T + kPlanThreads - 1) / kPlanThreads;
    const int t0 = min(T, tid * chunk), t1 = min(T, t0 + chunk);

    // pass 1: this thread's tokens sent and slots returned, per destination
    int mine[kPlanValues];
#pragma unroll
    for (int v = 0; v < kPlanValues; ++v) mine[v] = 0;
    for (int t = t0; t < t1; ++t) {
        int own[8], id[8];
        const uint32_t mask = token_owners(ids, t, owner, world, own, id);
#pragma unroll
        for (int d = 0; d < kPlanMaxWorld; ++d) {
            mine[d] += int((mask >> d) & 1u);
            int n = 0;
#pragma unroll
            for (int s = 0; s < 8; ++s) n += own[s] == d;
            mine[kPlanMaxWorld + d] += n;
        }
    }

    // block-wide exclusive scans of the 16 values (thread order = token order)
    int before[kPlanValues];
#pragma unroll
    for (int v = 0; v < kPlanValues; ++v) {
        int x = mine[v];
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, off);
            if (lane >= off) x += y;
        }
        before[v] = x - mine[v];  // exclusive within the warp
        if (lane == 31) warp_part[warp][v] = x;
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
        for (int v = 0; v < kPlanValues; ++v) {
            const int w = warp_part[lane][v];
            int x = w;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, x, off);
                if (lane >= off) x += y;
            }
            warp_part[lane][v] = x - w;
            if (lane == 31) totals[v] = x;
        }
    }
    __syncthreads();

    // first position and first returned row of this thread, per destination
    int pos[kPlanMaxWorld], row[kPlanMaxWorld];
    int tok_base = 0, row_base = 0;
#pragma unroll
    for (int d = 0; d < kPlanMaxWorld; ++d) {
        pos[d] = tok_base + warp_part[warp][d] + before[d];
        row[d] = row_base + warp_part[warp][kPlanMaxWorld + d] + before[kPlanMaxWorld + d];
        tok_base += totals[d];
        row_base += totals[kPlanMaxWorld + d];
    }
    if (tid < world) {
        counts[2 * tid] = totals[tid];
        counts[2 * tid + 1] = totals[kPlanMaxWorld + tid];
    }

    // pass 2: the rows, in token order
    for (int t = t0; t < t1; ++t) {
        int own[8], id[8];
        const uint32_t mask = token_owners(ids, t, owner, world, own, id);
        int ri[8];
#pragma unroll
        for (int s = 0; s < 8; ++s) ri[s] = -1;
#pragma unroll
        for (int d = 0; d < kPlanMaxWorld; ++d) {
            if (!((mask >> d) & 1u)) continue;
            const int p = pos[d]++;
            token_index[p] = t;
            dest[p] = d;
#pragma unroll
            for (int s = 0; s < 8; ++s) {
                const bool here = own[s] == d;  // implies 0 <= id[s] < 256
                const int lid = local[here ? id[s] : 0];
                local_ids[size_t(p) * 8 + s] = here ? lid : -1;
                slot_mask[size_t(p) * 8 + s] = here ? 1 : 0;
                if (here) ri[s] = row[d]++;
            }
        }
#pragma unroll
        for (int s = 0; s < 8; ++s) row_index[size_t(t) * 8 + s] = ri[s];
    }
}

}  // namespace
}  // namespace ornith

using namespace ornith;

extern "C" cudaError_t ornith_moe_b200_ep_plan(const void* ids_i32, int T, const void* owner_i32,
                                               const void* local_i32, int world, void* counts_i64,
                                               void* token_index_i64, void* dest_i64, void* local_ids_i32,
                                               void* slot_mask_u8, void* row_index_i32, cudaStream_t stream) {
    if (T < 0 || T > kTcapMax || world < 1 || world > kPlanMaxWorld) return cudaErrorInvalidValue;
    if (!owner_i32 || !local_i32 || !counts_i64 || !plan_aligned(owner_i32, 4) || !plan_aligned(local_i32, 4) ||
        !plan_aligned(counts_i64, 8))
        return cudaErrorInvalidValue;
    if (T && (!ids_i32 || !token_index_i64 || !dest_i64 || !local_ids_i32 || !slot_mask_u8 || !row_index_i32 ||
              !plan_aligned(ids_i32, 4) || !plan_aligned(token_index_i64, 8) || !plan_aligned(dest_i64, 8) ||
              !plan_aligned(local_ids_i32, 4) || !plan_aligned(row_index_i32, 4)))
        return cudaErrorInvalidValue;
    NvtxRange range("ornith.ep.plan");
    count_launches(1);
    // T == 0 still launches: the counts are written (zeros); no other buffer is touched
    ep_plan_kernel<<<1, kPlanThreads, 0, stream>>>(
        static_cast<const int32_t*>(ids_i32), T, static_cast<const int32_t*>(owner_i32),
        static_cast<const int32_t*>(local_i32), world, static_cast<long long*>(counts_i64),
        static_cast<long long*>(token_index_i64), static_cast<long long*>(dest_i64),
        static_cast<int32_t*>(local_ids_i32), static_cast<uint8_t*>(slot_mask_u8),
        static_cast<int32_t*>(row_index_i32));
    return cudaGetLastError();
}
