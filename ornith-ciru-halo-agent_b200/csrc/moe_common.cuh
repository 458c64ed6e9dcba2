// Shared device helpers of the B200 routed-MoE layer (sm_100a).
//
// The arithmetic here restates, operation for operation, the fixed-order
// integer/fp32 pipeline of the reference's routed library
// (kernels/routed_storage/routed_storage_n32_consumer.cpp of
// ciru-ai/ornith-ciru-halo-agent) so that results are bit-identical:
//   * bf16 round-to-nearest-even                     (:17-21)
//   * 128-point Walsh-Hadamard butterfly x 0x3db504f3 (:22-43)
//   * per-256-group A8/A4 activation quantisation      (:44-76)
//   * per-group projection epilogue                    (:152-158)
//   * SiLU with the reference's portable exp           (:168-175, portable_exp.h:6-25)
// The library is compiled with -fmad=false so no fp32 step is contracted.
//
// Data layout choices that are B200-specific (not the reference's):
//   * activations are int8 (one byte per element, 2048 B per token row), with
//     each 8-element block stored as [q0 q2 q4 q6 | q1 q3 q5 q7] so that the
//     even and odd nibbles of one packed weight word, masked to bytes, meet
//     their activations in two __dp4a instructions;
//   * one warp quantises one 256-group: lane l owns elements 8l..8l+7, the
//     Hadamard steps 1,2,4 stay in registers and steps 8..64 are xor shuffles.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ornith {

constexpr int kE = 256, kTop = 8, kH = 2048, kI = 512, kG = 256;
constexpr int kTcapMax = 8192;
constexpr float kInvSqrt128 = 0x1.6a09e6p-4f;  // 0x3db504f3

// Sticky error bits (routed_storage_n32_consumer.cpp:33,51,58,86,115,174,183).
enum : uint32_t {
    kFlagNonfiniteInput = 1,
    kFlagInvalidActivation = 2,
    kFlagInvalidId = 4,
    kFlagNonfiniteProjection = 8,
    kFlagNonfiniteMiddle = 16,
    kFlagNonfiniteOutput = 32,
    kFlagWaitTimeout = 64,  // a bounded device wait gave up; results are incomplete
    kFlagDebugBounds = 128, // debug builds: a data-dependent index was out of range (access redirected)
};

// Debug builds (-DORNITH_DEBUG_BOUNDS=1) pass the data-dependent indices of
// the hot kernels (plan positions, route and token numbers read back from
// plans, expert slots that select a bank) through checked(): an index outside
// [0, limit) raises flag 128 and is replaced by 0, so the access stays inside
// its buffer and nothing traps.  It stands in for a device sanitizer, which
// the shared GPUs do not offer.  In the default build checked() is the index.
#ifndef ORNITH_DEBUG_BOUNDS
#define ORNITH_DEBUG_BOUNDS 0
#endif
__device__ __forceinline__ int checked(int idx, int limit, uint32_t* flags) {
#if ORNITH_DEBUG_BOUNDS
    if (idx < 0 || idx >= limit) {
        atomicOr(flags, uint32_t(kFlagDebugBounds));
        return 0;
    }
#endif
    (void)limit;
    (void)flags;
    return idx;
}
// The same for the rows [first, first + count) of a tile, which must lie in
// [0, limit); an out-of-range tile is moved to row 0 (count <= limit on every
// path that uses it).
__device__ __forceinline__ int checked_range(int first, int count, int limit, uint32_t* flags) {
#if ORNITH_DEBUG_BOUNDS
    if (first < 0 || count < 0 || first + count > limit) {
        atomicOr(flags, uint32_t(kFlagDebugBounds));
        return 0;
    }
#endif
    (void)count;
    (void)limit;
    (void)flags;
    return first;
}

__device__ __forceinline__ uint16_t bf16_rne(float value) {
    uint32_t bits = __float_as_uint(value);
    if ((bits & 0x7fffffffu) > 0x7f800000u) return uint16_t((bits >> 16) | 0x40u);
    return uint16_t((bits + 0x7fffu + ((bits >> 16) & 1u)) >> 16);
}
__device__ __forceinline__ float bf16_to_f32(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }
__device__ __forceinline__ float bf16_round_f32(float v) { return bf16_to_f32(bf16_rne(v)); }

// The reference's deterministic exponential (portable_exp.h:6-25): Cody-Waite
// reduction n = rint(x*log2 e), two-part ln2, degree-8 Taylor in Horner form
// evaluated without FMA, then ldexp.  Written without branches so that many
// independent evaluations interleave: the same steps run on x clamped into
// [-104, 89] and the special cases (NaN, x <= -104 -> 0, x >= 89 -> inf) are
// selected at the end.  ldexp(p, n) is two power-of-two scalings: p lies in
// [0.7, 1.42] and n in [-150, 128], so p * 2^(n>>1) is exact (normal) and the
// second product rounds once, which is the correctly rounded p * 2^n that
// ldexpf returns.
__device__ __forceinline__ float portable_exp(float x) {
    const float xc = fminf(fmaxf(x, -104.f), 89.f);
    const float n_float = rintf(__fmul_rn(xc, 0x1.715476p+0f));
    const int n = static_cast<int>(n_float);
    const float high = __fmul_rn(n_float, 0x1.62e400p-1f);
    const float low = __fmul_rn(n_float, 0x1.7f7d1cp-20f);
    const float r = __fsub_rn(__fsub_rn(xc, high), low);
    float p = 0x1.a01a02p-16f;
    p = __fadd_rn(__fmul_rn(p, r), 0x1.a01a02p-13f);
    p = __fadd_rn(__fmul_rn(p, r), 0x1.6c16c2p-10f);
    p = __fadd_rn(__fmul_rn(p, r), 0x1.111112p-7f);
    p = __fadd_rn(__fmul_rn(p, r), 0x1.555556p-5f);
    p = __fadd_rn(__fmul_rn(p, r), 0x1.555556p-3f);
    p = __fadd_rn(__fmul_rn(p, r), 0x1p-1f);
    p = __fadd_rn(__fmul_rn(p, r), 0x1p+0f);
    p = __fadd_rn(__fmul_rn(p, r), 0x1p+0f);
    const int n1 = n >> 1, n2 = n - n1;
    float res = __fmul_rn(__fmul_rn(p, __int_as_float((n1 + 127) << 23)), __int_as_float((n2 + 127) << 23));
    res = x >= 89.f ? __int_as_float(0x7f800000) : res;
    res = x <= -104.f ? 0.f : res;
    return isnan(x) ? x : res;
}

// g / d rounded to nearest even, for the SiLU denominator d = 1 + exp(-g) >= 1,
// without a call on the common path.  Markstein's FMA-based method (P. W.
// Markstein, IBM J. Res. Dev. 34(1), 1990): one Newton step on the hardware
// reciprocal estimate, q0 = g*y, one FMA correction q1 = q0 + (g - d*q0)*y.
// q1 is then checked exactly: r1 = g - d*q1 is exact by FMA when q1 is within
// one ulp, and q1 is the correctly rounded quotient iff |r1| < d*ulp(q1)/2
// when q1 is not a power of two (both neighbours one ulp away).  *ok is false
// where that check cannot confirm q1 (powers of two, tiny non-zero quotients,
// d >= 2^24, |g| >= 2^64, non-finite operands); the caller then divides with
// __fdiv_rn.  Checked against __fdiv_rn for every fp32 g with
// d = 1 + portable_exp(-g).
__device__ __forceinline__ float div_rn_ge1(float g, float d, bool& ok) {
    float y0;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y0) : "f"(d));
    const float e = __fmaf_rn(-d, y0, 1.f);
    const float y1 = __fmaf_rn(y0, e, y0);
    const float q0 = __fmul_rn(g, y1);
    const float r0 = __fmaf_rn(-d, q0, g);
    const float q1 = __fmaf_rn(r0, y1, q0);
    const float r1 = __fmaf_rn(-d, q1, g);
    const uint32_t qb = __float_as_uint(q1);
    const float half_ulp = __uint_as_float((qb & 0x7f800000u) - (24u << 23));
    ok = d < 16777216.f && fabsf(g) < 0x1p64f && fabsf(q1) >= 0x1p-100f && (qb & 0x7fffffu) != 0u &&
         fabsf(r1) < __fmul_rn(d, half_ulp);
    // a zero dividend gives itself (its sign kept) for every finite d >= 1
    const bool zero = g == 0.f && d < 16777216.f;
    ok = ok || zero;
    return zero ? g : q1;
}

// The SiLU quotient g / (1 + portable_exp(-g)) for |g| < 80, the common case,
// in about half the instructions of the general form: the exponent argument is
// inside portable_exp's range, so its range selects drop out and ldexp is one
// exact product (n in [-116, 116], p * 2^n normal); the division is
// div_rn_ge1.  *ok is false outside |g| < 80 or where div_rn_ge1 cannot confirm
// the quotient; the caller then uses the general form.  Checked against the
// general form on the GPU for every fp32 g.
__device__ __forceinline__ float silu_quotient_fast(float g, bool& ok) {
    const float x = -g;
    // rint(t) for |t| < 2^22 as (t + 1.5*2^23) - 1.5*2^23 (the addition rounds
    // to the nearest even integer), and n from the sum's low mantissa bits:
    // both on the FMA and integer pipes instead of the conversion unit
    const float shifted = __fadd_rn(__fmul_rn(x, 0x1.715476p+0f), 12582912.f);
    const float n_float = __fsub_rn(shifted, 12582912.f);
    const int n = __float_as_int(shifted) - 0x4B400000;
    const float high = __fmul_rn(n_float, 0x1.62e400p-1f);
    const float low = __fmul_rn(n_float, 0x1.7f7d1cp-20f);
    const float r = __fsub_rn(__fsub_rn(x, high), low);
    float p = 0x1.a01a02p-16f;
    p = __fadd_rn(__fmul_rn(p, r), 0x1.a01a02p-13f);
    p = __fadd_rn(__fmul_rn(p, r), 0x1.6c16c2p-10f);
    p = __fadd_rn(__fmul_rn(p, r), 0x1.111112p-7f);
    p = __fadd_rn(__fmul_rn(p, r), 0x1.555556p-5f);
    p = __fadd_rn(__fmul_rn(p, r), 0x1.555556p-3f);
    p = __fadd_rn(__fmul_rn(p, r), 0x1p-1f);
    p = __fadd_rn(__fmul_rn(p, r), 0x1p+0f);
    p = __fadd_rn(__fmul_rn(p, r), 0x1p+0f);
    const float e = __fmul_rn(p, __int_as_float((n + 127) << 23));
    const float d = __fadd_rn(1.f, e);
    bool dok;
    const float q = div_rn_ge1(g, d, dok);
    ok = dok && fabsf(g) < 80.f;
    return q;
}

// Routed SiLU*up (middle_kernel): (g / (1 + exp(-g))) * up, IEEE division.
__device__ __forceinline__ float silu_mul(float g, float up) {
    float denominator = __fadd_rn(1.f, portable_exp(-g));
    return __fmul_rn(__fdiv_rn(g, denominator), up);
}

// One projection epilogue step for a 256-group:
// value + (w_scale*(sa*dot) + w_offset*(sa*sum)).
__device__ __forceinline__ float group_term(float sa, int dot, int sum, uint32_t meta) {
    float scaled_dot = __fmul_rn(sa, float(dot));
    float scaled_sum = __fmul_rn(sa, float(sum));
    float w_scale = __half2float(__ushort_as_half(uint16_t(meta & 0xffffu)));
    float w_offset = __half2float(__ushort_as_half(uint16_t(meta >> 16)));
    return __fadd_rn(__fmul_rn(w_scale, scaled_dot), __fmul_rn(w_offset, scaled_sum));
}

// In-register 128-point Hadamard over a half-warp: lane l (0..15 within its
// half) holds elements 8l..8l+7 of one 128-block.  Stage order and operand
// order are those of the reference's shared-memory butterfly.
__device__ __forceinline__ void wht128_halfwarp(float (&e)[8], int lane) {
#pragma unroll
    for (int step = 1; step < 8; step *= 2) {
        float n[8];
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            int lo = s & ~step;
            n[s] = (s & step) ? __fsub_rn(e[lo], e[lo + step]) : __fadd_rn(e[lo], e[lo + step]);
        }
#pragma unroll
        for (int s = 0; s < 8; ++s) e[s] = n[s];
    }
    // across lanes: the upper lane of each pair computes other - e, the IEEE
    // sum (-e) + other, and the lower one e + other.  fma(sign, e, other) with
    // sign = -1 or +1 is that sum in one instruction: the product is exact and
    // the single rounding is the addition's, signed zeros included.
#pragma unroll
    for (int lstep = 1; lstep < 16; lstep *= 2) {
        const float sign = (lane & lstep) != 0 ? -1.f : 1.f;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            const float other = __shfl_xor_sync(0xffffffffu, e[s], lstep);
            e[s] = __fmaf_rn(sign, e[s], other);
        }
    }
#pragma unroll
    for (int s = 0; s < 8; ++s) e[s] = __fmul_rn(e[s], kInvSqrt128);
}

// Quantise one 256-group held by a warp (8 elements per lane, already
// Hadamard-transformed).  Writes the permuted int8 words for lane l's 8
// elements (word pair index l), and returns scale/sum through lane 0.
// routed_storage_n32_consumer.cpp:44-76.
template <int QMAX>
__device__ __forceinline__ void quantize_group_warp(const float (&t)[8], int lane, uint2* q_out,
                                                    __half* scale_out, int32_t* sum_out, uint32_t& flags) {
    float v[8], absmax = 0.f;
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        bool finite = isfinite(t[s]);
        if (!finite) flags |= kFlagInvalidActivation;
        v[s] = finite ? t[s] : 0.f;
        absmax = fmaxf(absmax, fabsf(v[s]));
    }
    // non-negative floats order like their bit patterns: one warp max reduction
    absmax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(absmax)));
    float raw = __fdiv_rn(absmax, float(QMAX));
    bool valid = isfinite(raw) && raw <= 65504.f;
    if (!valid) flags |= kFlagInvalidActivation;
    const bool zero = absmax == 0.f || !valid;
    __half scale = __float2half_rn(zero ? 1.f : fmaxf(raw, 0x1p-14f));
    float sf = __half2float(scale);
    // q = rint(RN(v / sf)) exactly, mostly without a division: with
    // r = RN(1/sf) and y = RN(v*r), |y - v/sf| <= 2^-16 and
    // |RN(v/sf) - v/sf| <= 2^-18 because |v/sf| < 128 (sf is absmax/QMAX
    // rounded to fp16, or 2^-14 above it).  So y and RN(v/sf) round to the
    // same integer unless y lies within 2^-15 of a half-integer; only then is
    // the quotient computed with the IEEE division.
    // The reference clamps q to [-QMAX, QMAX]; no clamp is needed here: sf is
    // absmax / QMAX rounded to fp16 (relative error <= 2^-11) or 2^-14 above
    // it, so |v / sf| <= QMAX * (1 + 2^-11) + 2^-16 < QMAX + 1/2 and every
    // quotient rounds to at most QMAX in magnitude.
    const float rcp = __fdiv_rn(1.f, sf);
    int q[8], sum = 0;
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        int qi = 0;
        if (!zero) {
            const float y = __fmul_rn(v[s], rcp);
            const float k = rintf(y);
            qi = __fsub_rn(0.5f, fabsf(__fsub_rn(y, k))) > 0x1p-15f ? int(k) : __float2int_rn(__fdiv_rn(v[s], sf));
        }
        q[s] = qi;
        sum += qi;
    }
    // low bytes of q0 q2 q4 q6 and of q1 q3 q5 q7, three byte permutes each
    const uint32_t even = __byte_perm(__byte_perm(uint32_t(q[0]), uint32_t(q[2]), 0x0040),
                                      __byte_perm(uint32_t(q[4]), uint32_t(q[6]), 0x0040), 0x5410);
    const uint32_t odd = __byte_perm(__byte_perm(uint32_t(q[1]), uint32_t(q[3]), 0x0040),
                                     __byte_perm(uint32_t(q[5]), uint32_t(q[7]), 0x0040), 0x5410);
    q_out[lane] = make_uint2(even, odd);
    sum = int(__reduce_add_sync(0xffffffffu, uint32_t(sum)));
    if (lane == 0) {
        *scale_out = scale;
        *sum_out = sum;
    }
}

// Hadamard + quantise one 256-group held by the warp (lane l: elements
// 8l..8l+7, as scalars so that nothing goes through local memory).  Writes
// the permuted int8 codes to q and, from lane 0, the scale and code sum;
// returns the flags (non-finite values before or after the transform, invalid
// scale).  Out of line: every activation group of the layer goes through
// this one copy.
template <int QMAX>
__device__ __noinline__ uint32_t wht_quant(float e0, float e1, float e2, float e3, float e4, float e5, float e6,
                                           float e7, int lane, uint2* q, __half* scale, int32_t* sum) {
    float e[8] = {e0, e1, e2, e3, e4, e5, e6, e7};
    uint32_t f = 0;
    // A non-finite input makes every output of its 128-block non-finite (each
    // output is a signed sum of all 128 inputs), and the lane holds outputs of
    // its own block, so testing the outputs alone raises the same flag as
    // testing inputs and outputs.
    wht128_halfwarp(e, lane);
#pragma unroll
    for (int i = 0; i < 8; ++i)
        if (!isfinite(e[i])) f |= kFlagNonfiniteInput;
    quantize_group_warp<QMAX>(e, lane, q, scale, sum, f);
    return f;
}

// Counter updates between CTAs.  red_release_add publishes the caller's
// earlier writes (and, after a warp or CTA barrier, those of the threads it
// synchronised with) without waiting for the update to land;
// atom_add_acq_rel also returns the previous value and acquires what earlier
// releasers published.
__device__ __forceinline__ void red_release_add(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_relaxed_add(uint32_t* p, uint32_t v) {
    asm volatile("red.relaxed.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t atom_add_acq_rel(uint32_t* p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Integer dot of one packed weight word (8 u4 codes, k = 8j+d at bits 4d) with
// its 8 activations in the permuted [even | odd] int8 layout.
__device__ __forceinline__ int dot8(uint32_t w, uint2 a, int acc) {
    int lo = int(w & 0x0f0f0f0fu);
    int hi = int((w >> 4) & 0x0f0f0f0fu);
    acc = __dp4a(lo, int(a.x), acc);
    return __dp4a(hi, int(a.y), acc);
}

__device__ __forceinline__ bool id_valid(int id) { return id >= 0 && id < kE; }

// ---------------------------------------------------------------------------
// PTX wrappers: mbarriers and bulk (non-tensor) global->shared copies.
// No cluster multicast anywhere in this library.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
// try_wait that may suspend the thread for up to hint_ns until the phase
// completes (instead of returning at once), so waiting warps stop taking issue
// slots from the working ones.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bulk copy global -> this CTA's shared memory, completing on `bar`.
// dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release(uint32_t* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded waits: every spin in this library gives up after about a second,
// raises kFlagWaitTimeout and lets the kernel wind down.
constexpr uint32_t kSpinLimit = 1u << 23;

}  // namespace ornith
