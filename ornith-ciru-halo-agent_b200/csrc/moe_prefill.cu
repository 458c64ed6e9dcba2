// Tensor-core prefill path of the routed-MoE layer (T > 32), sm_100a.
//
// Same arithmetic as the reference's grouped path
// (kernels/routed_storage/routed_storage_n32_prefill.h:43-165): per 256-group
// exact integer dots, then the fixed fp32 epilogue in ascending group order.
// B200 schedule:
//
//   prefill_count/scan/place_kernel  routing plan (slot counts/offsets/route
//                         lists, the inverse map route -> position) and the
//                         list of 128-route M-tiles per expert slot;
//   quant_tokens_kernel   Hadamard + quantise each token group once (xq);
//   pack_gather_kernel    copy each M-tile's token rows into the no-swizzle
//                         K-major core-matrix layout tcgen05 reads;
//   mma_kernel<8, gate>   gate/up grouped GEMM: tcgen05.mma.kind::i8
//                         (s8 activations x u8 codes -> s32 in TMEM),
//                         M=128 x N=256 (128 gate + 128 matching up columns),
//                         fused SiLU*up epilogue -> fp32 middle rows;
//   pack_middle_kernel    Hadamard + quantise the middle rows into down M-tiles;
//   mma_kernel<2, down>   down grouped GEMM, N=256 output columns -> route_out;
//   combine               slot-ordered weighted sum (shared with the
//                         multi-kernel path), reading rows through rowpos.
// middle and route_out rows are in slot-position order: the 128 rows of an
// M-tile are one contiguous block, so the epilogue's row stores stay inside
// it instead of scattering over the whole buffer (one TLB reach per tile).
//
// mma_kernel roles (24 warps, one CTA per SM, persistent over tiles):
//   warp 0      producer: cp.async.bulk of the activation half-tile (16 KB),
//               the packed u4 codes (8 x 2 KB) and per-group metadata;
//   warp 1      TMEM allocator and single-thread MMA issuer;
//   warps 2-5   converters: u4 codes -> u8 core matrices in shared memory;
//   warps 6-7   idle (they complete the second setup warpgroup);
//   warps 8-23  four epilogue warpgroups (64 TMEM columns each), which take
//               the registers the setup warpgroups give up (setmaxnreg).
// K advances in half-groups of 128 through a 3-stage ring.  The int32
// accumulator of a 256-group is double buffered in TMEM (2 x 256 columns); the
// group's first MMA overwrites it, so no epilogue store re-initialises it.  The
// epilogue adds the bits of 1.5*2^23 as an integer: the cell then reads as the
// float 1.5*2^23 + dot exactly (|dot| < 2^22), and float(dot) is one
// subtraction (re-initialising the cells to those bits with TMEM stores
// instead held 16 registers per thread and was 6% slower).
// Activations use the dp4a byte order [q0 q2 q4 q6 | q1 q3 q5 q7] per 8-block,
// so unpacking a packed code word is two masks, with no byte shuffles.
// No TMA or bulk load uses cluster multicast.  Every wait is bounded.
#include "moe_layer.cuh"
#include "nvtx_range.h"

namespace ornith {
namespace {

constexpr int kMT = 128;                  // routes per M-tile
constexpr int kNT = 256;                  // B rows (output columns) per tile
constexpr int kStages = 3;
constexpr int kABytes = kMT * 128;        // activation half-tile (K = 128)
constexpr int kBpBytes = kNT * 128 / 2;   // packed codes half-tile
constexpr int kBuBytes = kNT * 128;       // unpacked codes half-tile
constexpr int kStageBytes = kABytes + kBpBytes + kBuBytes;
constexpr int kMetaBytes = kNT * 4 + kMT * 4 + kMT * 4;  // B meta, A scale, A sum
constexpr int kEpiWarps = 16;
// fp32 column scales then offsets of one epilogue warp's 64 columns, one copy per warp
constexpr int kMetaFWarpFloats = 2 * 64;
constexpr int kMetaFBytes = kEpiWarps * kMetaFWarpFloats * 4;
constexpr int kMetaSlots = 4;  // metadata ring: the producer runs up to 4 groups ahead of the epilogue
constexpr int kWarps = 24;
constexpr int kThreads = kWarps * 32;
constexpr int kEpiFirst = 8;    // epilogue warps 8..23 (warpgroups 2..5)
// Converter warps 2..5, one per scheduler.  Dealing the conversion over warps
// 2..7 instead was measured slower on a B200 (46.3 against 45.8 ms per
// 40-layer prefill-8192 step), so the converters are not latency-bound.
constexpr int kConvWarps = 4;
// Register split (setmaxnreg, per warpgroup): the two setup warpgroups drop to
// kRegsSetup, the four epilogue warpgroups rise to kRegsEpi.  The sum must not
// exceed what the CTA was launched with (kThreads x kRegsLaunch), which the
// launcher checks against the compiled count before the first launch.
constexpr int kRegsSetup = 48, kRegsEpi = 96, kRegsLaunch = 80;
static_assert(2 * 128 * kRegsSetup + 4 * 128 * kRegsEpi <= kThreads * kRegsLaunch, "register split");
constexpr uint32_t kMagic = 0x4B400000u;  // 1.5 * 2^23
constexpr float kMagicF = 12582912.0f;
constexpr uint64_t kTimeoutNs = 1000000000ull;
constexpr uint32_t kSuspendNs = 20000;  // longest suspension of one wait attempt

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Per-role timestamps of a few CTAs (clock64), compiled in only with
// -DORNITH_PREFILL_TRACE; the default build has none.
#ifdef ORNITH_PREFILL_TRACE
constexpr int kPTraceCtas = 4, kPTraceKinds = 12, kPTraceLen = 256;
__device__ unsigned long long g_prefill_trace[2][kPTraceCtas][kPTraceKinds][kPTraceLen];
#define PREFILL_TRACE(kind, idx)                                                                         \
    ((blockIdx.x % 37 == 0 && blockIdx.x / 37 < kPTraceCtas && (idx) < kPTraceLen)                      \
         ? void(g_prefill_trace[GATE ? 0 : 1][blockIdx.x / 37][kind][idx] = clock64())                  \
         : void(0))
// spin iterations of the bounded waits, per warp (kind 11)
#define PREFILL_SPINS(n)                                                                                 \
    ((blockIdx.x % 37 == 0 && blockIdx.x / 37 < kPTraceCtas)                                           \
         ? void(atomicAdd(&g_prefill_trace[0][blockIdx.x / 37][11][threadIdx.x >> 5], (unsigned long long)(n))) \
         : void(0))
#else
#define PREFILL_TRACE(kind, idx) ((void)0)
#define PREFILL_SPINS(n) ((void)0)
#endif

// ---- tcgen05 wrappers ----------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// K-major, no-swizzle shared-memory matrix descriptor (sm_100 format, version 1):
// core matrices of 8 rows x 16 bytes, LBO = byte stride between the two
// K-adjacent core matrices, SBO = byte stride between 8-row groups.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return uint64_t((addr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
           (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46);
}
// Instruction descriptor, kind::i8: D s32, A s8 (signed), B u8 (unsigned),
// both K-major, N = 256, M = 128.
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (0u << 10) | (uint32_t(kNT >> 3) << 17) | (uint32_t(kMT >> 4) << 24);

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t enable_d) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(enable_d)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }


// Named barrier that also ANDs a predicate across the participating threads,
// so that every thread takes the same exit decision (no thread is ever left
// waiting at a barrier the others skipped).
__device__ __forceinline__ bool named_and(int id, int threads, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(uint32_t(pred)), "r"(id), "r"(threads)
        : "memory");
    return r != 0;
}

// Bounded mbarrier wait; returns false (and raises the abort state) on timeout.
__device__ bool bwait(uint64_t* bar, uint32_t parity, volatile int* abort, uint32_t* flags) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = now_ns();
    unsigned spins = 0;
    while (!mbar_try_wait_suspend(bar, parity, kSuspendNs)) {
        ++spins;
        if (*abort) return false;
        if (now_ns() - t0 > kTimeoutNs) {
            atomicOr(flags, kFlagWaitTimeout);
            *abort = 1;
            return false;
        }
    }
    if ((threadIdx.x & 31) == 0) PREFILL_SPINS(spins + 1);
    return true;
}
// Drain wait used on the abort path: lets an issued copy land (bounded).
__device__ void drain_wait(uint64_t* bar, uint32_t parity) {
    const uint64_t t0 = now_ns();
    while (!mbar_try_wait(bar, parity) && now_ns() - t0 < kTimeoutNs) {
    }
}

// 8 x 8 transpose of float4 chunks inside each group of eight lanes: chunk r
// of lane 8a + j ends in chunk j of lane 8a + r.  Three butterfly stages; at
// stage d every chunk whose index differs from the lane in bit d trades
// places with the partner lane's chunk of index r ^ d.
__device__ __forceinline__ void transpose8(float4 (&c)[8], int lane) {
#pragma unroll
    for (int d = 1; d < 8; d <<= 1) {
        const bool hi = (lane & d) != 0;
#pragma unroll
        for (int r0 = 0; r0 < 8; ++r0) {
            if (r0 & d) continue;
            const int r1 = r0 | d;
            const float4 send = hi ? c[r0] : c[r1];
            float4 recv;
            recv.x = __shfl_xor_sync(0xffffffffu, send.x, d);
            recv.y = __shfl_xor_sync(0xffffffffu, send.y, d);
            recv.z = __shfl_xor_sync(0xffffffffu, send.z, d);
            recv.w = __shfl_xor_sync(0xffffffffu, send.w, d);
            if (hi) c[r0] = recv;
            else c[r1] = recv;
        }
    }
}

struct MmaArgs {
    const uint8_t* atiles;   // [MT][KG][32768] activation tiles
    const float* asa;        // [MT][KG][128] activation scales
    const int32_t* asum;     // [MT][KG][128] activation sums
    const int4* mtiles;      // {slot, first position, rows, 0}
    const int32_t* n_mtiles;
    const uint32_t* codes;   // routed bank
    const uint32_t* meta;
    const uint32_t* scodes;  // shared bank
    const uint32_t* smeta;
    float* out;              // gate: middle [positions][512]; down: route_out [positions][2048]
    const float* silu_table;
    uint32_t* flags;
    int rows;                // positions of the plan (8T routes + T shared rows), for debug checks
};

template <int KG, bool GATE>
__global__ void __launch_bounds__(kThreads, 1) mma_kernel(const MmaArgs p) {
    constexpr int NUPT = GATE ? 4 : 8;  // N-tiles per M-tile
    constexpr int K = KG * kG;
    constexpr int BANK_N = GATE ? 2 * kI : kH;
    constexpr size_t BANK_CODES = size_t(BANK_N) * K / 8;
    constexpr size_t BANK_META = size_t(BANK_N) * KG;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* stages = smem;
    uint8_t* metabuf = smem + kStages * kStageBytes;  // [kMetaSlots][kMetaBytes]
    float* metaf = reinterpret_cast<float*>(metabuf + kMetaSlots * kMetaBytes);  // [epilogue warp][scales 64 | offsets 64]
    uint64_t* bars = reinterpret_cast<uint64_t*>(metabuf + kMetaSlots * kMetaBytes + kMetaFBytes);
    uint64_t* full = bars;                       // [kStages] producer -> converters
    uint64_t* conv = bars + kStages;             // [kStages] converters -> MMA
    uint64_t* empty = bars + 2 * kStages;        // [kStages] MMA -> producer
    uint64_t* meta_full = bars + 3 * kStages;    // [kMetaSlots]
    uint64_t* meta_empty = meta_full + kMetaSlots;  // [kMetaSlots]
    uint64_t* acc_full = meta_empty + kMetaSlots;   // [2]
    uint64_t* acc_empty = acc_full + 2;          // [2]
    uint64_t* drain = acc_empty + 2;             // [1] final MMA completion
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&conv[i], kConvWarps);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < kMetaSlots; ++i) {
            mbar_init(&meta_full[i], 1);
            mbar_init(&meta_empty[i], kEpiWarps);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], kEpiWarps);
        }
        mbar_init(drain, 1);
        *abort = 0;
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int n_units = *p.n_mtiles * NUPT;
    if (tid == 0) PREFILL_TRACE(9, 0);

    auto unit_bank = [&](int unit, const uint32_t*& codes, const uint32_t*& meta) {
        const int4 mt = p.mtiles[unit / NUPT];
        const int e = checked(mt.x, kE + 1, p.flags);  // the slot's expert selects the bank
        const bool shared = e == kE;
        codes = shared ? p.scodes : p.codes + size_t(e) * BANK_CODES;
        meta = shared ? p.smeta : p.meta + size_t(e) * BANK_META;
    };
    // 32-column bank tile feeding B-tile rows 32i..32i+31 of N-tile nt
    auto n32_of = [&](int nt, int i) { return GATE ? (i < 4 ? 4 * nt + i : 16 + 4 * nt + (i - 4)) : 8 * nt + i; };

    if (warp < kEpiFirst) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsSetup));
        if (warp == 0) {
            // ---------------- producer ----------------
            if (lane == 0) {
                int issued = 0, metas = 0;
                for (int unit = blockIdx.x; unit < n_units && !*abort; unit += gridDim.x) {
                    const uint32_t *codes, *meta;
                    unit_bank(unit, codes, meta);
                    const int nt = unit % NUPT, tile = unit / NUPT;
                    for (int g = 0; g < KG && !*abort; ++g) {
                        if (!(metas < kMetaSlots || bwait(&meta_empty[metas % kMetaSlots],
                                                          uint32_t(metas / kMetaSlots - 1) & 1u, abort, p.flags)))
                            break;
                        {
                            const int mb = metas % kMetaSlots;
                            uint8_t* m = metabuf + mb * kMetaBytes;
                            mbar_arrive_expect_tx(&meta_full[mb], kMetaBytes);
                            for (int i = 0; i < 8; ++i)
                                bulk_g2s(m + i * 128, meta + (size_t(n32_of(nt, i)) * KG + g) * 32, 128, &meta_full[mb]);
                            bulk_g2s(m + kNT * 4, p.asa + (size_t(tile) * KG + g) * kMT, kMT * 4, &meta_full[mb]);
                            bulk_g2s(m + kNT * 4 + kMT * 4, p.asum + (size_t(tile) * KG + g) * kMT, kMT * 4, &meta_full[mb]);
                            PREFILL_TRACE(0, metas);
                            ++metas;
                        }
                        for (int h = 0; h < 2; ++h) {
                            const int s = issued % kStages;
                            if (issued >= kStages &&
                                !bwait(&empty[s], uint32_t(issued / kStages - 1) & 1u, abort, p.flags))
                                break;
                            uint8_t* sA = stages + size_t(s) * kStageBytes;
                            uint8_t* sBp = sA + kABytes;
                            mbar_arrive_expect_tx(&full[s], kABytes + kBpBytes);
                            bulk_g2s(sA, p.atiles + (size_t(tile) * KG + g) * 32768 + h * kABytes, kABytes, &full[s]);
                            for (int i = 0; i < 8; ++i)
                                bulk_g2s(sBp + i * 2048, codes + (size_t(n32_of(nt, i)) * KG + g) * 1024 + h * 512, 2048,
                                         &full[s]);
                            PREFILL_TRACE(1, issued);
                            ++issued;
                        }
                    }
                }
                if (*abort) {
                    // every issued copy lands before the CTA can leave
                    for (int k = issued - kStages; k < issued; ++k)
                        if (k >= 0) drain_wait(&full[k % kStages], uint32_t(k / kStages) & 1u);
                    for (int k = metas - kMetaSlots; k < metas; ++k)
                        if (k >= 0) drain_wait(&meta_full[k % kMetaSlots], uint32_t(k / kMetaSlots) & 1u);
                }
            }
        } else if (warp == 1) {
            // ---------------- MMA issuer ----------------
            if (lane == 0) {
                int st = 0, gg = 0;
                bool any = false;
                for (int unit = blockIdx.x; unit < n_units && !*abort; unit += gridDim.x) {
                    for (int g = 0; g < KG && !*abort; ++g, ++gg) {
                        const int b = gg & 1;
                        if (!bwait(&acc_empty[b], uint32_t(gg / 2) & 1u, abort, p.flags)) break;
                        tc_fence_after();
                        PREFILL_TRACE(4, gg);
                        const uint32_t d = tmem + uint32_t(b * kNT);
                        for (int h = 0; h < 2; ++h, ++st) {
                            const int s = st % kStages;
                            if (!bwait(&conv[s], uint32_t(st / kStages) & 1u, abort, p.flags)) break;
                            tc_fence_after();
                            PREFILL_TRACE(5, st);
                            const uint32_t aaddr = smem_addr(stages + size_t(s) * kStageBytes);
                            const uint32_t baddr = aaddr + kABytes + kBpBytes;
#pragma unroll
                            for (int kk = 0; kk < 4; ++kk)
                                mma_i8(d, smem_desc(aaddr + kk * 2 * 2048, 2048, 128),
                                       smem_desc(baddr + kk * 2 * 4096, 4096, 128), (h | kk) != 0 ? 1u : 0u);
                            mma_commit(&empty[s]);
                            any = true;
                        }
                        mma_commit(&acc_full[b]);
                    }
                }
                if (any) {
                    // every MMA issued has finished reading shared memory before the CTA leaves
                    mma_commit(drain);
                    drain_wait(drain, 0);
                }
            }
        } else if (warp < 2 + kConvWarps) {
            // ---------------- converters ----------------
            const int cw = warp - 2;  // converter warp 0..kConvWarps-1
            int st = 0;
            for (int unit = blockIdx.x; unit < n_units && !*abort; unit += gridDim.x) {
                for (int g = 0; g < KG && !*abort; ++g) {
                    for (int h = 0; h < 2; ++h, ++st) {
                        const int s = st % kStages;
                        if (!bwait(&full[s], uint32_t(st / kStages) & 1u, abort, p.flags)) break;
                        if (warp == 2 && lane == 0) PREFILL_TRACE(2, st);
                        // Work item (i, q, c): 32-column tile i (8), word pair q (8),
                        // column c = lane; converter warp cw takes the pairs
                        // q = cw + 4*qq.  Packed word j of column c of tile i is
                        // bp[512 i + 32 j + c]; column n = 32 i + c of the K-major
                        // core-matrix layout takes pair q at byte
                        // 4096 q + 128 (n >> 3) + 16 (n & 7).  Every offset below
                        // is a compile-time constant from two per-thread bases.
                        const uint32_t* bp = reinterpret_cast<const uint32_t*>(stages + size_t(s) * kStageBytes + kABytes) +
                                             lane + 64 * cw;
                        uint8_t* bu = stages + size_t(s) * kStageBytes + kABytes + kBpBytes + cw * 4096 + (lane >> 3) * 128 +
                                      (lane & 7) * 16;
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            uint32_t w[4];
#pragma unroll
                            for (int qq = 0; qq < 2; ++qq) {
                                w[2 * qq] = bp[i * 512 + qq * 256];
                                w[2 * qq + 1] = bp[i * 512 + qq * 256 + 32];
                            }
#pragma unroll
                            for (int qq = 0; qq < 2; ++qq)
                                *reinterpret_cast<uint4*>(bu + qq * 16384 + i * 512) =
                                    make_uint4(w[2 * qq] & 0x0f0f0f0fu, (w[2 * qq] >> 4) & 0x0f0f0f0fu,
                                               w[2 * qq + 1] & 0x0f0f0f0fu, (w[2 * qq + 1] >> 4) & 0x0f0f0f0fu);
                        }
                        fence_proxy_async();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&conv[s]);
                        if (warp == 2 && lane == 0) PREFILL_TRACE(3, st);
                    }
                }
            }
        }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsEpi));
        // ---------------- epilogue ----------------
        const int ew = warp - kEpiFirst;         // 0..15
        const int wg = ew >> 2;                  // column quarter
        const int row = 32 * (warp & 3) + lane;  // TMEM lane = tile row
        const uint32_t lane_base = uint32_t(32 * (warp & 3)) << 16;
        // column offsets (within a 256-column accumulator) owned by this warpgroup
        const int c0 = GATE ? 32 * wg : 64 * wg;
        const int c1 = GATE ? kMT + 32 * wg : 64 * wg + 32;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&acc_empty[0]);
            mbar_arrive(&acc_empty[1]);
        }
        uint32_t f = 0;
        int gg = 0;
        int un = 0;  // units done (trace index)
        float* const wmeta = metaf + ew * kMetaFWarpFloats;  // this warp's converted column metadata
        // The only barrier of the epilogue warps is the vote at each unit's
        // start (named_and), which every warp reaches once per unit: a warp
        // whose wait fails skips the rest of its unit, and the next vote ends
        // the loop for all of them (the failed wait has raised the abort state).
        for (int unit = blockIdx.x; unit < n_units; unit += gridDim.x) {
            if (!named_and(1, kEpiWarps * 32, !*abort)) break;
            const int4 mt = p.mtiles[unit / NUPT];
            const int nt = unit % NUPT;
            // 64 accumulators as 32 packed pairs (columns 2i, 2i + 1): the
            // per-group sequence runs on f32x2 arithmetic, two IEEE
            // round-to-nearest results per instruction, each the scalar one
            float2 acc2[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) acc2[i] = make_float2(0.f, 0.f);
            auto acc = [&](int i) -> float { return (i & 1) ? acc2[i >> 1].y : acc2[i >> 1].x; };
            bool ok = true;
            for (int g = 0; g < KG; ++g, ++gg) {
                const int b = gg & 1;
                const int ms = gg % kMetaSlots;
                const uint8_t* mslot = metabuf + ms * kMetaBytes;
                if (!ok || !bwait(&meta_full[ms], uint32_t(gg / kMetaSlots) & 1u, abort, p.flags)) {
                    ok = false;  // the unit's remaining groups are skipped; the next vote ends the loop
                    continue;
                }
                // this warp's 64 columns of the group's metadata, in its own copy
                // (the previous group's reads of it ended at that group's __syncwarp)
                {
                    const uint32_t m0 = reinterpret_cast<const uint32_t*>(mslot)[c0 + lane];
                    const uint32_t m1 = reinterpret_cast<const uint32_t*>(mslot)[c1 + lane];
                    wmeta[lane] = __half2float(__ushort_as_half(uint16_t(m0 & 0xffffu)));
                    wmeta[32 + lane] = __half2float(__ushort_as_half(uint16_t(m1 & 0xffffu)));
                    wmeta[64 + lane] = __half2float(__ushort_as_half(uint16_t(m0 >> 16)));
                    wmeta[96 + lane] = __half2float(__ushort_as_half(uint16_t(m1 >> 16)));
                    __syncwarp();
                }
                if (ew == 0 && lane == 0) PREFILL_TRACE(6, gg);
                if (!bwait(&acc_full[b], uint32_t(gg / 2) & 1u, abort, p.flags)) {
                    ok = false;
                    continue;
                }
                tc_fence_after();
                if (ew == 0 && lane == 0) PREFILL_TRACE(7, gg);
                const float* swf = wmeta;       // local column j: c0 + j (j < 32), c1 + j - 32
                const float* offf = wmeta + 64;
                const float sa = reinterpret_cast<const float*>(mslot + kNT * 4)[row];
                const int ssumi = reinterpret_cast<const int32_t*>(mslot + kNT * 4 + kMT * 4)[row];
                const float ssum = __fmul_rn(sa, float(ssumi));
                const float2 sa2 = make_float2(sa, sa), ssum2 = make_float2(ssum, ssum);
                const float2 nmagic2 = make_float2(-kMagicF, -kMagicF);
                const uint32_t base = tmem + lane_base + uint32_t(b * kNT);
#pragma unroll
                for (int part = 0; part < 4; ++part) {
                    const int col = (part < 2 ? c0 : c1) + 16 * (part & 1);
                    const int lcol = 16 * part;  // the same columns in the warp's metadata copy
                    uint32_t r[16];
                    tmem_ld16(base + col, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float4 sw4 = *reinterpret_cast<const float4*>(swf + lcol + 4 * q);
                        const float4 of4 = *reinterpret_cast<const float4*>(offf + lcol + 4 * q);
#pragma unroll
                        for (int hp = 0; hp < 2; ++hp) {
                            const int i = 4 * q + 2 * hp;
                            const float2 sw2 = hp ? make_float2(sw4.z, sw4.w) : make_float2(sw4.x, sw4.y);
                            const float2 of2 = hp ? make_float2(of4.z, of4.w) : make_float2(of4.x, of4.y);
                            // fd = dot exactly ((r + bits of 1.5*2^23) - 1.5*2^23), then sw*(sa*fd) + of*ssum:
                            // packed products, scalar sums of products.  A packed
                            // sum with a packed product among its operands was
                            // found contracted into a fused multiply-add on sm_100a
                            // despite .rn and -fmad=false, changing the rounding.
                            const float2 fd2 = __fadd2_rn(
                                make_float2(__uint_as_float(r[i] + kMagic), __uint_as_float(r[i + 1] + kMagic)), nmagic2);
                            const float2 p1 = __fmul2_rn(sw2, __fmul2_rn(sa2, fd2));
                            const float2 p2 = __fmul2_rn(of2, ssum2);
                            const float2 term2 = make_float2(__fadd_rn(p1.x, p2.x), __fadd_rn(p1.y, p2.y));
                            float2& a2 = acc2[(part * 16 + i) >> 1];
                            a2 = __fadd2_rn(a2, term2);
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&acc_empty[b]);
                    mbar_arrive(&meta_empty[ms]);
                }
                if (ew == 0 && lane == 0) PREFILL_TRACE(8, gg);
            }
            if (!ok) continue;  // the next unit's vote ends the loop
            if (ew == 0 && lane == 0) PREFILL_TRACE(9, 2 + 4 * un);
            // Unit results, written as whole 128-byte lines: the eight float4
            // chunks of a lane are transposed across its group of eight lanes,
            // so that store m of lane 8a + j writes chunk j of tile row
            // rbase + m.  Flags count only the tile's real rows.
            const bool valid = row < mt.z;
            const bool shared = mt.x == kE;
            const int rbase = 32 * (warp & 3) + 8 * (lane >> 3), jc = lane & 7;
            float4 c[8];
            if (GATE) {
                if (shared) {
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        float v[4];
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float gv = bf16_round_f32(acc(4 * k + j)), uv = bf16_round_f32(acc(32 + 4 * k + j));
                            if (valid && (!isfinite(gv) || !isfinite(uv))) f |= kFlagNonfiniteProjection;
                            v[j] = bf16_round_f32(__fmul_rn(p.silu_table[__float_as_uint(gv) >> 16], uv));
                            if (valid && !isfinite(v[j])) f |= kFlagNonfiniteMiddle;
                        }
                        c[k] = make_float4(v[0], v[1], v[2], v[3]);
                    }
                } else {
                    // silu_mul in batches of 4: the four quotients are
                    // independent straight-line chains and interleave (batches of
                    // 8 ran slower: more registers live beside the 64
                    // accumulators); the rare ones the fast form cannot confirm
                    // take the general form, behind a warp vote so that the common
                    // case never issues it.  Rows past the tile's end hold stale
                    // sums: they take g = 1 so that they never reach the slow
                    // division
#pragma unroll
                    for (int i = 0; i < 32; i += 4) {
                        float gs[4], q[4], v[4];
                        bool ok[4];
#pragma unroll
                        for (int j = 0; j < 4; ++j) gs[j] = valid ? acc(i + j) : 1.f;
#pragma unroll
                        for (int j = 0; j < 4; ++j) q[j] = silu_quotient_fast(gs[j], ok[j]);
                        bool all_ok = true;
#pragma unroll
                        for (int j = 0; j < 4; ++j) all_ok &= ok[j];
                        if (!__all_sync(0xffffffffu, all_ok)) {
#pragma unroll 1
                            for (int j = 0; j < 4; ++j)
                                if (!ok[j]) q[j] = __fdiv_rn(gs[j], __fadd_rn(1.f, portable_exp(-gs[j])));
                        }
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float gv = acc(i + j), uv = acc(32 + i + j);
                            if (valid && (!isfinite(gv) || !isfinite(uv))) f |= kFlagNonfiniteProjection;
                            v[j] = __fmul_rn(q[j], uv);
                            if (valid && !isfinite(v[j])) f |= kFlagNonfiniteMiddle;
                        }
                        c[i / 4] = make_float4(v[0], v[1], v[2], v[3]);
                    }
                }
                if (ew == 0 && lane == 0) PREFILL_TRACE(9, 3 + 4 * un);
                transpose8(c, lane);
                if (ew == 0 && lane == 0) PREFILL_TRACE(9, 4 + 4 * un);
                float* dst = p.out + size_t(checked_range(mt.y, mt.z, p.rows, p.flags) + rbase) * kI + kMT * nt +
                             32 * wg + 4 * jc;
#pragma unroll
                for (int m = 0; m < 8; ++m)
                    if (rbase + m < mt.z) *reinterpret_cast<float4*>(dst + size_t(m) * kI) = c[m];
            } else {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        float v[4];
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            v[j] = shared ? bf16_round_f32(acc(32 * h + 4 * k + j)) : acc(32 * h + 4 * k + j);
                            if (valid && !isfinite(v[j])) f |= kFlagNonfiniteProjection;
                        }
                        c[k] = make_float4(v[0], v[1], v[2], v[3]);
                    }
                    if (ew == 0 && lane == 0 && h == 0) PREFILL_TRACE(9, 3 + 4 * un);
                    transpose8(c, lane);
                    if (ew == 0 && lane == 0 && h == 0) PREFILL_TRACE(9, 4 + 4 * un);
                    float* dst = p.out + size_t(checked_range(mt.y, mt.z, p.rows, p.flags) + rbase) * kH + kNT * nt +
                                 64 * wg + 32 * h + 4 * jc;
#pragma unroll
                    for (int m = 0; m < 8; ++m)
                        if (rbase + m < mt.z) *reinterpret_cast<float4*>(dst + size_t(m) * kH) = c[m];
                }
            }
            if (ew == 0 && lane == 0) PREFILL_TRACE(9, 5 + 4 * un);
            if (lane == 0) PREFILL_TRACE(10, 16 * un + ew);
            ++un;
        }
        if (ew == 0 && lane == 0) PREFILL_TRACE(9, 1);
        f = __reduce_or_sync(0xffffffffu, f);
        if (f && lane == 0) atomicOr(p.flags, f);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 512);
}

// Routing plan for the tensor-core path, in three launches over blocks of
// routes: per-block expert counts; one CTA turning them into slot offsets,
// per-block bases and the list of 128-route M-tiles per slot (slot 256 = the
// shared expert, rows R..R+T-1); placement of every route at
// offset + block base + rank within the block.  Routes of one slot may appear
// in any order (every route's row is computed independently); rowpos is the
// inverse map.
__device__ __forceinline__ int plan_chunk(int R, int nblk) { return (R + nblk - 1) / nblk; }

__global__ __launch_bounds__(256) void prefill_count_kernel(LayerArgs a, int nblk) {
    __shared__ int hist[kE + 1];
    for (int e = threadIdx.x; e <= kE; e += blockDim.x) hist[e] = 0;
    __syncthreads();
    const int R = a.T * kTop, chunk = plan_chunk(R, nblk);
    const int r0 = blockIdx.x * chunk, r1 = min(R, r0 + chunk);
    uint32_t f = 0;
    for (int r = r0 + threadIdx.x; r < r1; r += blockDim.x) {
        const int e = a.ids[r];
        if (id_valid(e)) atomicAdd(&hist[e], 1);
        else if (e != -1) f |= kFlagInvalidId;
    }
    f = __reduce_or_sync(0xffffffffu, f);
    if (f && (threadIdx.x & 31) == 0) atomicOr(a.flags, f);
    __syncthreads();
    // expert-major [E + 1][kPlanBlocks], so that the scan reads each expert's
    // block counts as one contiguous run
    int* bc = ws_at<int32_t>(a, a.L.pblock) + blockIdx.x;
    for (int e = threadIdx.x; e <= kE; e += blockDim.x) bc[size_t(e) * kPlanBlocks] = hist[e];
}

__global__ __launch_bounds__(1024) void prefill_scan_kernel(LayerArgs a, int nblk) {
    __shared__ int warp_tot[32][2];
    __shared__ int total[kE];
    const int e = threadIdx.x, lane = e & 31, w = e >> 5;
    const int* bc = ws_at<int32_t>(a, a.L.pblock);
    int* bb = ws_at<int32_t>(a, a.L.pblock) + size_t(kPlanBlocks) * (kE + 1);
    // Per-block bases inside each expert's run: warp w takes experts w, w+32,
    // ...; lane l holds the counts of blocks 8l..8l+7 (all loaded before use),
    // a serial prefix over those and a warp scan over the lanes.
    static_assert(kPlanBlocks == 256, "eight blocks per lane");
    for (int ex = w; ex < kE; ex += 32) {
        int v[8], run = 0;
        {
            // blocks 8l..8l+7 of expert ex: two 16-byte loads (entries past
            // nblk were not written by this call and count as zero)
            const int4* src = reinterpret_cast<const int4*>(bc + size_t(ex) * kPlanBlocks + 8 * lane);
            const int4 lo = src[0], hi = src[1];
            const int raw[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = 8 * lane + k < nblk ? raw[k] : 0;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int c0 = run;
            run += v[k];
            v[k] = c0;
        }
        int incl = run;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, incl, d);
            if (lane >= d) incl += u;
        }
        const int base = incl - run;
        // expert-major as well: each lane's eight bases are one 32-byte run
        // (entries past nblk are written too and never read)
        int4* dst = reinterpret_cast<int4*>(bb + size_t(ex) * kPlanBlocks + 8 * lane);
        dst[0] = make_int4(base + v[0], base + v[1], base + v[2], base + v[3]);
        dst[1] = make_int4(base + v[4], base + v[5], base + v[6], base + v[7]);
        if (lane == 31) total[ex] = incl;
    }
    __syncthreads();
    int c = 0;
    if (e < kE) c = total[e];
    else if (e == kE) c = a.shared ? a.T : 0;
    const int t = e <= kE ? (c + kMT - 1) / kMT : 0;
    // exclusive scans of counts and tile counts over the 257 slots
    int ic = c, it = t;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int uc = __shfl_up_sync(0xffffffffu, ic, d), ut = __shfl_up_sync(0xffffffffu, it, d);
        if (lane >= d) {
            ic += uc;
            it += ut;
        }
    }
    if (lane == 31) {
        warp_tot[w][0] = ic;
        warp_tot[w][1] = it;
    }
    __syncthreads();
    if (w == 0) {
        int vc = warp_tot[lane][0], vt = warp_tot[lane][1];
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int uc = __shfl_up_sync(0xffffffffu, vc, d), ut = __shfl_up_sync(0xffffffffu, vt, d);
            if (lane >= d) {
                vc += uc;
                vt += ut;
            }
        }
        warp_tot[lane][0] = vc;  // inclusive over warps
        warp_tot[lane][1] = vt;
    }
    __syncthreads();
    const int before_c = (w ? warp_tot[w - 1][0] : 0) + ic - c;
    const int before_t = (w ? warp_tot[w - 1][1] : 0) + it - t;
    int32_t* g_offsets = ws_at<int32_t>(a, a.L.offsets);
    int32_t* g_tiles = ws_at<int32_t>(a, a.L.slot_tiles);
    int4* mtiles = ws_at<int4>(a, a.L.mtiles);
    if (e <= kE) {
        g_offsets[e] = before_c;
        g_tiles[e] = before_t;
        for (int m = 0; m * kMT < c; ++m) mtiles[before_t + m] = make_int4(e, before_c + m * kMT, min(kMT, c - m * kMT), 0);
        if (e == kE) {
            g_offsets[kE + 1] = before_c + c;
            g_tiles[kE + 1] = before_t + t;
            *ws_at<int32_t>(a, a.L.n_mtiles) = before_t + t;
        }
    }
}

__global__ __launch_bounds__(256) void prefill_place_kernel(LayerArgs a, int nblk) {
    __shared__ int base[kE + 1];
    const int R = a.T * kTop, chunk = plan_chunk(R, nblk);
    const int r0 = blockIdx.x * chunk, r1 = min(R, r0 + chunk);
    const int32_t* g_offsets = ws_at<int32_t>(a, a.L.offsets);
    const int* bb = ws_at<int32_t>(a, a.L.pblock) + size_t(kPlanBlocks) * (kE + 1) + blockIdx.x;
    for (int e = threadIdx.x; e < kE; e += blockDim.x) base[e] = g_offsets[e] + bb[size_t(e) * kPlanBlocks];
    __syncthreads();
    int32_t* routes = ws_at<int32_t>(a, a.L.routes);
    int32_t* rowpos = ws_at<int32_t>(a, a.L.rowpos);
    for (int r = r0 + threadIdx.x; r < r1; r += blockDim.x) {
        const int e = a.ids[r];
        if (id_valid(e)) {
            const int pos = checked(atomicAdd(&base[e], 1), R + a.T, a.flags);
            routes[pos] = r;
            rowpos[r] = pos;
        }
    }
    if (a.shared && blockIdx.x == 0) {
        const int sh = g_offsets[kE];
        for (int t = threadIdx.x; t < a.T; t += blockDim.x) {
            routes[sh + t] = R + t;
            rowpos[R + t] = sh + t;
        }
    }
}

// Shared-memory image of one 32 KB activation tile group: the K-major
// core-matrix layout [chunk 16][row 128][16 bytes] with the row rotated by
// the chunk, so that the 16 chunks of one row (written together) and
// consecutive rows of one chunk (read together) both spread over all banks.
__device__ __forceinline__ uint32_t tile_slot(int chunk, int row) {
    return uint32_t(chunk) * 2048u + uint32_t((row + chunk) & (kMT - 1)) * 16u;
}
// Copies the shared-memory tile image to its global tile in whole lines.
__device__ __forceinline__ void store_tile(const uint8_t* img, uint8_t* dst) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int idx = k * 256 + threadIdx.x;  // chunk * 128 + row
        reinterpret_cast<uint4*>(dst)[idx] = *reinterpret_cast<const uint4*>(img + tile_slot(idx >> 7, idx & 127));
    }
}

// Gate activation tiles from the quantised tokens (xq, xs, xsum, written once
// per token by the token quantisation kernel): one CTA per (M-tile, 256-group)
// reads its 128 token rows whole (16 threads x 16 bytes per row), rearranges
// them in shared memory and writes the 32 KB tile in whole lines.  Rows past
// the tile's end are zero.
__global__ __launch_bounds__(256) void pack_gather_kernel(LayerArgs a) {
    __shared__ __align__(16) uint8_t img[32768];
    const int tile = blockIdx.x >> 3, g = blockIdx.x & 7;
    if (tile >= *ws_at<int32_t>(a, a.L.n_mtiles)) return;
    const int4 mt = ws_at<int4>(a, a.L.mtiles)[tile];
    const int R = a.T * kTop;
    const int32_t* routes = ws_at<int32_t>(a, a.L.routes) + checked_range(mt.y, mt.z, a.T * (kTop + 1), a.flags);
    const uint8_t* xq = ws_at<uint8_t>(a, a.L.xq) + g * kG;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int idx = k * 256 + threadIdx.x;  // row * 16 + chunk
        const int row = idx >> 4, chunk = idx & 15;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (row < mt.z) {
            const int route = routes[row];
            const int t = checked(route >= R ? route - R : route / kTop, a.T, a.flags);
            v = __ldcg(reinterpret_cast<const uint4*>(xq + size_t(t) * kH) + chunk);
        }
        *reinterpret_cast<uint4*>(img + tile_slot(chunk, row)) = v;
    }
    if (threadIdx.x < kMT) {
        const int row = threadIdx.x;
        float sa = 0.f;
        int32_t sum = 0;
        if (row < mt.z) {
            const int route = routes[row];
            const int t = checked(route >= R ? route - R : route / kTop, a.T, a.flags);
            sa = __half2float(ws_at<__half>(a, a.L.xs)[t * (kH / kG) + g]);
            sum = ws_at<int32_t>(a, a.L.xsum)[t * (kH / kG) + g];
        }
        ws_at<float>(a, a.L.agate_sa)[(size_t(tile) * 8 + g) * kMT + row] = sa;
        ws_at<int32_t>(a, a.L.agate_sum)[(size_t(tile) * 8 + g) * kMT + row] = sum;
    }
    __syncthreads();
    store_tile(img, ws_at<uint8_t>(a, a.L.agate) + (size_t(tile) * 8 + g) * 32768);
}

// Middle Hadamard + quantise into the down activation tiles: one CTA per
// eight consecutive rows of an (M-tile, 256-group), one warp per row (read
// whole from the slot-ordered middle buffer).  The eight quantised rows meet
// in shared memory and leave as 16 whole 128-byte lines (one per K-chunk).
// Rows past the tile's end are zero.
template <int QMAX>
__global__ __launch_bounds__(256) void pack_middle_kernel(LayerArgs a) {
    __shared__ __align__(16) uint2 img[16][8][2];  // [chunk][row][half]
    __shared__ uint2 qbuf[8][32];
    __shared__ __half sbuf[8];
    __shared__ int32_t mbuf[8];
    const int tile = blockIdx.x >> 5, g = (blockIdx.x >> 4) & 1, r0 = (blockIdx.x & 15) * 8;
    if (tile >= *ws_at<int32_t>(a, a.L.n_mtiles)) return;
    const int4 mt = ws_at<int4>(a, a.L.mtiles)[tile];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, row = r0 + warp;
    float* tsa = ws_at<float>(a, a.L.adown_sa) + (size_t(tile) * 2 + g) * kMT;
    int32_t* tsum = ws_at<int32_t>(a, a.L.adown_sum) + (size_t(tile) * 2 + g) * kMT;
    uint32_t f = 0;
    if (row < mt.z) {
        const float4* src =
            reinterpret_cast<const float4*>(ws_at<float>(a, a.L.middle) +
                                            size_t(checked(mt.y + row, a.T * (kTop + 1), a.flags)) * kI + g * kG +
                                            lane * 8);
        const float4 v0 = __ldcs(src), v1 = __ldcs(src + 1);
        float e[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
        for (int s = 0; s < 8; ++s)
            if (!isfinite(e[s])) f |= kFlagNonfiniteInput;
        wht128_halfwarp(e, lane);
#pragma unroll
        for (int s = 0; s < 8; ++s)
            if (!isfinite(e[s])) f |= kFlagNonfiniteInput;
        quantize_group_warp<QMAX>(e, lane, qbuf[warp], &sbuf[warp], &mbuf[warp], f);
        __syncwarp();
        img[lane >> 1][warp][lane & 1] = qbuf[warp][lane];
        if (lane == 0) {
            tsa[row] = __half2float(sbuf[warp]);
            tsum[row] = mbuf[warp];
        }
    } else {
        img[lane >> 1][warp][lane & 1] = make_uint2(0u, 0u);
        if (lane == 0) {
            tsa[row] = 0.f;
            tsum[row] = 0;
        }
    }
    f = __reduce_or_sync(0xffffffffu, f);
    if (f && lane == 0) atomicOr(a.flags, f);
    __syncthreads();
    if (threadIdx.x < 128) {
        const int chunk = threadIdx.x >> 3, ri = threadIdx.x & 7;
        uint8_t* dst = ws_at<uint8_t>(a, a.L.adown) + (size_t(tile) * 2 + g) * 32768 + chunk * 2048 + (r0 + ri) * 16;
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(&img[chunk][ri][0]);
    }
}

constexpr size_t kMmaSmem = size_t(kStages) * kStageBytes + kMetaSlots * kMetaBytes + kMetaFBytes + 64 * 8 + 64;

struct DeviceState {
    int sms = 0;
    bool attr = false;
};
DeviceState g_state[64];

}  // namespace

#ifdef ORNITH_PREFILL_TRACE
// Copies the role timestamps of the last gate and down launches.
extern "C" __attribute__((visibility("default"))) int ornith_moe_b200_prefill_trace(void* dst) {
    return int(cudaMemcpyFromSymbol(dst, g_prefill_trace, sizeof(g_prefill_trace)));
}
#endif

cudaError_t launch_prefill(const LayerArgs& a, cudaStream_t stream) {
    int device = 0;
    cudaError_t st = cudaGetDevice(&device);
    if (st != cudaSuccess) return st;
    if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
    DeviceState& ds = g_state[device];
    if (!ds.sms && (st = cudaDeviceGetAttribute(&ds.sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess)
        return st;
    auto gate = mma_kernel<8, true>;
    auto down = mma_kernel<2, false>;
    if (!ds.attr) {
        if ((st = cudaFuncSetAttribute(gate, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kMmaSmem))) != cudaSuccess)
            return st;
        if ((st = cudaFuncSetAttribute(down, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kMmaSmem))) != cudaSuccess)
            return st;
        // setmaxnreg.inc waits for registers the CTA does not have if the
        // kernel was compiled with fewer launch registers than the split assumes
        for (const void* k : {reinterpret_cast<const void*>(gate), reinterpret_cast<const void*>(down)}) {
            cudaFuncAttributes fa;
            if ((st = cudaFuncGetAttributes(&fa, k)) != cudaSuccess) return st;
            if (fa.numRegs < kRegsLaunch || fa.maxThreadsPerBlock < kThreads) return cudaErrorInvalidConfiguration;
        }
        ds.attr = true;
    }
    const int T = a.T, R = T * kTop, rows = R + (a.shared ? T : 0);
    const int nblk = min(kPlanBlocks, max(1, (R + 255) / 256));
    count_launches(7);  // plan x3, gather, gate, middle, down; quantisation and combine count their own
    {
        NvtxRange r("ornith.prefill.plan");
        prefill_count_kernel<<<nblk, 256, 0, stream>>>(a, nblk);
        prefill_scan_kernel<<<1, 1024, 0, stream>>>(a, nblk);
        prefill_place_kernel<<<nblk, 256, 0, stream>>>(a, nblk);
        if ((st = cudaGetLastError()) != cudaSuccess) return st;
    }
    // upper bound of M-tiles (the kernels read the device-side count)
    const int max_tiles = (rows + kMT - 1) / kMT + (kE + 1);
    {
        NvtxRange r("ornith.prefill.pack_tokens");
        if ((st = launch_quant_tokens(a, stream)) != cudaSuccess) return st;
        pack_gather_kernel<<<max_tiles * 8, 256, 0, stream>>>(a);
        if ((st = cudaGetLastError()) != cudaSuccess) return st;
    }
    MmaArgs g{};
    g.atiles = ws_at<uint8_t>(a, a.L.agate);
    g.asa = ws_at<float>(a, a.L.agate_sa);
    g.asum = ws_at<int32_t>(a, a.L.agate_sum);
    g.mtiles = ws_at<int4>(a, a.L.mtiles);
    g.n_mtiles = ws_at<int32_t>(a, a.L.n_mtiles);
    g.codes = a.gate_codes;
    g.meta = a.gate_meta;
    g.scodes = a.sgate_codes;
    g.smeta = a.sgate_meta;
    g.out = ws_at<float>(a, a.L.middle);
    g.silu_table = a.silu_table;
    g.flags = a.flags;
    g.rows = T * (kTop + 1);
    {
        NvtxRange r("ornith.prefill.gate_up");
        gate<<<min(ds.sms, max_tiles * 4), kThreads, kMmaSmem, stream>>>(g);
        if ((st = cudaGetLastError()) != cudaSuccess) return st;
    }
    {
        NvtxRange r("ornith.prefill.pack_middle");
        if (a.a8) pack_middle_kernel<127><<<max_tiles * 32, 256, 0, stream>>>(a);
        else pack_middle_kernel<7><<<max_tiles * 32, 256, 0, stream>>>(a);
        if ((st = cudaGetLastError()) != cudaSuccess) return st;
    }
    MmaArgs d = g;
    d.atiles = ws_at<uint8_t>(a, a.L.adown);
    d.asa = ws_at<float>(a, a.L.adown_sa);
    d.asum = ws_at<int32_t>(a, a.L.adown_sum);
    d.codes = a.down_codes;
    d.meta = a.down_meta;
    d.scodes = a.sdown_codes;
    d.smeta = a.sdown_meta;
    d.out = ws_at<float>(a, a.L.route_out);
    {
        NvtxRange r("ornith.prefill.down");
        down<<<min(ds.sms, max_tiles * 8), kThreads, kMmaSmem, stream>>>(d);
        if ((st = cudaGetLastError()) != cudaSuccess) return st;
    }
    NvtxRange r("ornith.prefill.combine");
    return launch_combine(a, stream, true);
}

}  // namespace ornith
