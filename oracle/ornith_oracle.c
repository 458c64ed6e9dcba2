/*
 * CPU oracle for the Ornith routed mixture-of-experts layer.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * product in ornith-ciru-halo-agent_b200/csrc and the timed CPU baseline of
 * bench.py.  Nothing in the product path links, loads or calls it.
 *
 * It restates, in plain C, the arithmetic of the reference's production
 * routed library (ciru-ai/ornith-ciru-halo-agent):
 *   kernels/routed_storage/routed_storage_n32_consumer.cpp   (stage order :319-351)
 *   kernels/routed_storage/routed_storage_n32_prefill.h      (grouped jobs, same
 *                                                             per-group sequence)
 *   kernels/routed_storage/portable_exp.h                    (exp)
 *   kernels/dense_n32/dense_g256_api.h:32-38                 (prose arithmetic contract)
 * Every function cites the lines it follows.  Parity is pinned twice: against
 * the reference's own HIP source compiled for the CPU with a SIMT shim
 * (oracle/build_ref.py -> oracle/_ref/), and against the committed golden
 * vectors in tests/golden/ (SiLU/sigmoid tables with the reference's sha256,
 * and routed outputs produced by that compiled reference).
 *
 * Build: gcc -O2 -ffp-contract=off -fopenmp (see oracle/Makefile).  Without
 * -ffp-contract=off the fixed fp32 order below would be fused into FMAs.
 *
 * Shapes are fixed by the reference: E=256 experts, top-8, H=2048, I=512,
 * quantisation group G=256, Hadamard block 128.
 *
 * Weight banks use the reference's N32 storage:
 *   codes u32 [E][N/32][K/256][32 words][32 columns], word j of group g for
 *         column n holds k = 256g + 8j + d in bits 4d..4d+3 (u4 code 0..15);
 *   meta  u32 [E][N/32][K/256][32 columns] = fp16 scale (low half) |
 *         fp16 offset (high half); weight = scale*code + offset.
 * Activations are int8 per element with one fp16 scale and one int32 sum per
 * 256-group (the reference packs them as nibble planes; the integer dot is the
 * same).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_E 256
#define ORC_TOP 8
#define ORC_H 2048
#define ORC_I 512
#define ORC_G 256

enum {
    ORC_FLAG_NONFINITE_INPUT = 1,   /* transform input or output not finite */
    ORC_FLAG_INVALID_ACT = 2,       /* activation quantisation invalid */
    ORC_FLAG_INVALID_ID = 4,        /* expert id outside [-1, E) */
    ORC_FLAG_NONFINITE_PROJ = 8,    /* projection output not finite */
    ORC_FLAG_NONFINITE_MIDDLE = 16, /* SiLU*up not finite */
    ORC_FLAG_NONFINITE_OUT = 32     /* combined output not finite / bf16 overflow */
};

static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* bf16 round-to-nearest-even, NaN quieted.  routed_storage_n32_consumer.cpp:17-21 */
uint16_t orc_bf16_rne(float value) {
    uint32_t bits = f2u(value);
    if ((bits & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((bits >> 16) | 0x40u);
    return (uint16_t)((bits + 0x7fffu + ((bits >> 16) & 1u)) >> 16);
}
float orc_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

/* IEEE binary16 -> binary32 (exact). */
float orc_half_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    if (e == 0) {
        float f = (float)m * 0x1p-24f;
        return sign ? -f : f;
    }
    if (e == 31) return u2f(sign | 0x7f800000u | (m << 13));
    return u2f(sign | ((e + 112u) << 23) | (m << 13));
}

/* IEEE binary32 -> binary16, round to nearest even (the semantics of
 * __float2half_rn used at routed_storage_n32_consumer.cpp:59). */
uint16_t orc_f32_to_half_rne(float f) {
    uint32_t x = f2u(f), sign = (x >> 16) & 0x8000u, ax = x & 0x7fffffffu;
    if (ax > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 -> inf */
    if (ax < 0x38800000u) {                                   /* below 2^-14 */
        if (ax < 0x33000000u) return (uint16_t)sign;          /* below 2^-25 -> 0 */
        uint32_t mant = (ax & 0x7fffffu) | 0x800000u;
        int e = (int)(ax >> 23) - 127;                        /* -25 .. -15 */
        int shift = -(e + 1);                                  /* 14 .. 24 */
        uint32_t q = mant >> shift, rem = mant & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t h = ((((ax >> 23) - 112u) << 10) | ((ax & 0x7fffffu) >> 13));
    uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

/* Deterministic fp32 exponential of the reference: Cody-Waite reduction with
 * n = rint(x*log2 e), two-part ln2, degree-8 Taylor polynomial in Horner form
 * (no FMA), ldexp.  kernels/routed_storage/portable_exp.h:6-25 */
float orc_portable_exp(float x) {
    if (isnan(x)) return x;
    if (x <= -104.f) return 0.f;
    if (x >= 89.f) return INFINITY;
    const float n_float = nearbyintf(x * 0x1.715476p+0f);
    const int n = (int)n_float;
    const float high = n_float * 0x1.62e400p-1f;
    const float low = n_float * 0x1.7f7d1cp-20f;
    const float reduced_high = x - high;
    const float r = reduced_high - low;
    float p = 0x1.a01a02p-16f;
    p = p * r + 0x1.a01a02p-13f;
    p = p * r + 0x1.6c16c2p-10f;
    p = p * r + 0x1.111112p-7f;
    p = p * r + 0x1.555556p-5f;
    p = p * r + 0x1.555556p-3f;
    p = p * r + 0x1p-1f;
    p = p * r + 0x1p+0f;
    p = p * r + 0x1p+0f;
    return ldexpf(p, n);
}

/* SiLU of the routed middle: g / (1 + exp(-g)), IEEE division.
 * routed_storage_n32_consumer.cpp:173 */
float orc_silu(float g) { return g / (1.f + orc_portable_exp(-g)); }

/* One 128-point Walsh-Hadamard butterfly, stage order step = 1,2,...,64,
 * element `lane` of stage s = src[lo] +/- src[lo+step] with lo = lane & ~step,
 * then times 0x3db504f3 (1/sqrt(128) rounded to fp32).
 * routed_storage_n32_consumer.cpp:34-41 */
void orc_wht128(const float* in, float* out) {
    float a[128], b[128];
    memcpy(a, in, sizeof a);
    float *src = a, *dst = b;
    for (int step = 1; step < 128; step *= 2) {
        for (int lane = 0; lane < 128; ++lane) {
            int lo = lane & ~step;
            dst[lane] = (lane & step) ? src[lo] - src[lo + step] : src[lo] + src[lo + step];
        }
        float* t = src; src = dst; dst = t;
    }
    for (int lane = 0; lane < 128; ++lane) out[lane] = src[lane] * 0x1.6a09e6p-4f;
}

static int id_valid(int32_t id) { return id >= 0 && id < ORC_E; }

/* transform<BF16=true> over token rows: bf16 -> fp32, H128 per 128-block.
 * A row whose eight ids are all invalid becomes zeros without flag checks
 * (routed_storage_n32_consumer.cpp:22-43).  ids == NULL keeps every row live,
 * which is fused_transform_quantize<0> (:237-239, the shared-slot variant). */
void orc_transform_tokens(const uint16_t* x, const int32_t* ids, int T, float* y, uint32_t* flags) {
    uint32_t f = 0;
#pragma omp parallel for reduction(| : f) schedule(static)
    for (int t = 0; t < T; ++t) {
        int live = 1;
        if (ids) {
            live = 0;
            for (int s = 0; s < ORC_TOP; ++s) live |= id_valid(ids[t * ORC_TOP + s]);
        }
        float* row = y + (size_t)t * ORC_H;
        if (!live) { memset(row, 0, ORC_H * sizeof(float)); continue; }
        for (int b = 0; b < ORC_H / 128; ++b) {
            float in[128];
            for (int l = 0; l < 128; ++l) {
                in[l] = orc_bf16_to_f32(x[(size_t)t * ORC_H + b * 128 + l]);
                if (!isfinite(in[l])) f |= ORC_FLAG_NONFINITE_INPUT;
            }
            orc_wht128(in, row + b * 128);
            for (int l = 0; l < 128; ++l) if (!isfinite(row[b * 128 + l])) f |= ORC_FLAG_NONFINITE_INPUT;
        }
    }
    *flags |= f;
}

/* transform<BF16=false> over fp32 rows of length K (routed_storage_n32_consumer.cpp:22-43). */
void orc_transform_rows(const float* x, int rows, int K, float* y, uint32_t* flags) {
    uint32_t f = 0;
#pragma omp parallel for reduction(| : f) schedule(static)
    for (int r = 0; r < rows; ++r) {
        for (int b = 0; b < K / 128; ++b) {
            const float* in = x + (size_t)r * K + b * 128;
            float* out = y + (size_t)r * K + b * 128;
            for (int l = 0; l < 128; ++l) if (!isfinite(in[l])) f |= ORC_FLAG_NONFINITE_INPUT;
            orc_wht128(in, out);
            for (int l = 0; l < 128; ++l) if (!isfinite(out[l])) f |= ORC_FLAG_NONFINITE_INPUT;
        }
    }
    *flags |= f;
}

/* Quantise one 256-group (routed_storage_n32_consumer.cpp:44-76):
 * non-finite -> 0 (flag 2); absmax; raw = absmax/qmax (IEEE division);
 * valid = finite(raw) && raw <= 65504; scale = fp16_rne(absmax==0||!valid ? 1
 * : max(raw, 2^-14)); q = rint(v/scale) (ties to even) clamped to +-qmax, 0 for
 * zero or invalid groups; sum = sum of q.  qmax = 127 (A8) or 7 (A4). */
void orc_quantize_group(const float* v, int a8, int8_t* q, uint16_t* scale_out, int32_t* sum_out, uint32_t* flags) {
    float vals[ORC_G], absmax = 0.f;
    for (int i = 0; i < ORC_G; ++i) {
        int finite = isfinite(v[i]);
        if (!finite) *flags |= ORC_FLAG_INVALID_ACT;
        vals[i] = finite ? v[i] : 0.f;
        absmax = fmaxf(absmax, fabsf(vals[i]));
    }
    const int qmax = a8 ? 127 : 7;
    float raw = absmax / (float)qmax;
    int valid = isfinite(raw) && raw <= 65504.f;
    if (!valid) *flags |= ORC_FLAG_INVALID_ACT;
    uint16_t scale = orc_f32_to_half_rne(absmax == 0.f || !valid ? 1.f : fmaxf(raw, 0x1p-14f));
    float sf = orc_half_to_f32(scale);
    int32_t sum = 0;
    for (int i = 0; i < ORC_G; ++i) {
        int qi = (absmax == 0.f || !valid) ? 0 : (int)nearbyintf(vals[i] / sf);
        qi = qi < -qmax ? -qmax : (qi > qmax ? qmax : qi);
        q[i] = (int8_t)qi;
        sum += qi;
    }
    *scale_out = scale;
    *sum_out = sum;
}

void orc_quantize_rows(const float* y, int rows, int K, int a8, int8_t* q, uint16_t* scales, int32_t* sums, uint32_t* flags) {
    uint32_t f = 0;
    const int groups = K / ORC_G;
#pragma omp parallel for reduction(| : f) schedule(static)
    for (int r = 0; r < rows; ++r) {
        uint32_t lf = 0;
        for (int g = 0; g < groups; ++g) {
            size_t at = (size_t)r * K + (size_t)g * ORC_G;
            orc_quantize_group(y + at, a8, q + at, scales + (size_t)r * groups + g, sums + (size_t)r * groups + g, &lf);
        }
        f |= lf;
    }
    *flags |= f;
}

/* Projection of routes that share one expert bank (N32 storage).
 * For every route i (activation row rows[i], output row dst[i]) and column n,
 * over groups g ascending:
 *   dot = sum_k code[n,k]*q[k] (exact integer), sa = fp16 activation scale,
 *   scaled_dot = sa*dot; scaled_sum = sa*sum_q; product = w_scale*scaled_dot;
 *   correction = w_offset*scaled_sum; value = value + (product + correction).
 * Shared rows are rounded to bf16 (shared MLP output contract).
 * routed_storage_n32_consumer.cpp:124-161 (direct), :187-230 (shared slot);
 * routed_storage_n32_prefill.h:43-149 computes the same per-group sequence. */
static void project_bank(int N, int K, const uint32_t* codes_e, const uint32_t* meta_e,
                         const int* rows, const int* dst, int nr,
                         const int8_t* q, const uint16_t* scales, const int32_t* sums,
                         float* out, int bf16_round, uint32_t* flags) {
    const int groups = K / ORC_G;
    int8_t* wt = (int8_t*)malloc(32 * ORC_G);
    float* acc = (float*)malloc(sizeof(float) * (size_t)nr * 32);
    for (int nt = 0; nt < N / 32; ++nt) {
        for (size_t i = 0; i < (size_t)nr * 32; ++i) acc[i] = 0.f;
        for (int g = 0; g < groups; ++g) {
            const uint32_t* blk = codes_e + ((size_t)nt * groups + g) * 32 * 32;
            for (int j = 0; j < 32; ++j)
                for (int c = 0; c < 32; ++c) {
                    uint32_t w = blk[j * 32 + c];
                    for (int d = 0; d < 8; ++d) wt[c * ORC_G + j * 8 + d] = (int8_t)((w >> (4 * d)) & 15u);
                }
            const uint32_t* mb = meta_e + ((size_t)nt * groups + g) * 32;
            for (int i = 0; i < nr; ++i) {
                const int8_t* qa = q + (size_t)rows[i] * K + (size_t)g * ORC_G;
                float sa = orc_half_to_f32(scales[(size_t)rows[i] * groups + g]);
                float scaled_sum = sa * (float)sums[(size_t)rows[i] * groups + g];
                for (int c = 0; c < 32; ++c) {
                    const int8_t* wc = wt + c * ORC_G;
                    int32_t dot = 0;
                    for (int k = 0; k < ORC_G; ++k) dot += (int32_t)wc[k] * (int32_t)qa[k];
                    float sw = orc_half_to_f32((uint16_t)(mb[c] & 0xffffu));
                    float off = orc_half_to_f32((uint16_t)(mb[c] >> 16));
                    float scaled_dot = sa * (float)dot;
                    float product = sw * scaled_dot, correction = off * scaled_sum;
                    acc[(size_t)i * 32 + c] = acc[(size_t)i * 32 + c] + (product + correction);
                }
            }
        }
        for (int i = 0; i < nr; ++i)
            for (int c = 0; c < 32; ++c) {
                float v = acc[(size_t)i * 32 + c];
                if (bf16_round) v = orc_bf16_to_f32(orc_bf16_rne(v));
                out[(size_t)dst[i] * N + nt * 32 + c] = v;
                if (!isfinite(v)) *flags |= ORC_FLAG_NONFINITE_PROJ;
            }
    }
    free(wt);
    free(acc);
}

/* Routed projection for R routes: route r uses expert ids[r]; its activation
 * row is r/8 (gate/up, `row = Gate ? route/Top : route`) or r (down).
 * Invalid ids give a zero output row; ids outside [-1, E) set flag 4.
 * routed_storage_n32_consumer.cpp:130-135, :89 */
void orc_project_routed(int N, int K, int gate, const int32_t* ids, int R,
                        const uint32_t* codes, const uint32_t* meta,
                        const int8_t* q, const uint16_t* scales, const int32_t* sums,
                        float* out, uint32_t* flags) {
    const size_t bank_codes = (size_t)N * K / 8, bank_meta = (size_t)N * (K / ORC_G);
    int* count = (int*)calloc(ORC_E + 1, sizeof(int));
    int* start = (int*)calloc(ORC_E + 1, sizeof(int));
    int* order = (int*)malloc(sizeof(int) * (size_t)(R > 0 ? R : 1));
    uint32_t f = 0;
    for (int r = 0; r < R; ++r) {
        int e = ids[r];
        if (id_valid(e)) count[e]++;
        else {
            if (e != -1) f |= ORC_FLAG_INVALID_ID;
            for (int n = 0; n < N; ++n) out[(size_t)r * N + n] = 0.f;
        }
    }
    for (int e = 0, acc = 0; e < ORC_E; ++e) { start[e] = acc; acc += count[e]; }
    {
        int* fill = (int*)calloc(ORC_E, sizeof(int));
        for (int r = 0; r < R; ++r) if (id_valid(ids[r])) order[start[ids[r]] + fill[ids[r]]++] = r;
        free(fill);
    }
#pragma omp parallel for reduction(| : f) schedule(dynamic, 1)
    for (int e = 0; e < ORC_E; ++e) {
        if (!count[e]) continue;
        int* rows = (int*)malloc(sizeof(int) * count[e]);
        for (int i = 0; i < count[e]; ++i) rows[i] = gate ? order[start[e] + i] / ORC_TOP : order[start[e] + i];
        uint32_t lf = 0;
        project_bank(N, K, codes + (size_t)e * bank_codes, meta + (size_t)e * bank_meta,
                     rows, order + start[e], count[e], q, scales, sums, out, 0, &lf);
        f |= lf;
        free(rows);
    }
    *flags |= f;
    free(count); free(start); free(order);
}

/* Shared expert bank applied to `rows` activation rows; output rows
 * dst_offset..dst_offset+rows-1, rounded to bf16 (:225-228). */
void orc_project_shared(int N, int K, int rows, const uint32_t* codes, const uint32_t* meta,
                        const int8_t* q, const uint16_t* scales, const int32_t* sums,
                        float* out, int dst_offset, uint32_t* flags) {
    if (rows <= 0) return;
    int nthreads = 1;
#ifdef _OPENMP
    nthreads = omp_get_max_threads();
#endif
    int chunk = (rows + nthreads - 1) / nthreads;
    uint32_t f = 0;
#pragma omp parallel for reduction(| : f) schedule(static, 1)
    for (int c0 = 0; c0 < rows; c0 += chunk) {
        int n = rows - c0 < chunk ? rows - c0 : chunk;
        int* src = (int*)malloc(sizeof(int) * n);
        int* dst = (int*)malloc(sizeof(int) * n);
        for (int i = 0; i < n; ++i) { src[i] = c0 + i; dst[i] = dst_offset + c0 + i; }
        uint32_t lf = 0;
        project_bank(N, K, codes, meta, src, dst, n, q, scales, sums, out, 1, &lf);
        f |= lf;
        free(src); free(dst);
    }
    *flags |= f;
}

/* SiLU*up of the routed middle (middle_kernel, routed_storage_n32_consumer.cpp:168-175):
 * m[r,c] = (g/(1+exp(-g)))*up with g = gate_y[r,c], up = gate_y[r,512+c];
 * invalid routes give zeros. */
void orc_middle(const float* gate_y, const int32_t* ids, int R, float* middle, uint32_t* flags) {
    uint32_t f = 0;
#pragma omp parallel for reduction(| : f) schedule(static)
    for (int r = 0; r < R; ++r) {
        for (int c = 0; c < ORC_I; ++c) {
            if (!id_valid(ids[r])) { middle[(size_t)r * ORC_I + c] = 0.f; continue; }
            float g = gate_y[(size_t)r * 2 * ORC_I + c], up = gate_y[(size_t)r * 2 * ORC_I + ORC_I + c];
            float result = orc_silu(g) * up;
            middle[(size_t)r * ORC_I + c] = result;
            if (!isfinite(result)) f |= ORC_FLAG_NONFINITE_MIDDLE;
        }
    }
    *flags |= f;
}

/* Shared-slot middle (fused_transform_quantize<1>, :240-252): SiLU from the
 * 65,536-entry table indexed by the bf16 bits of g, times up, rounded to bf16. */
void orc_middle_shared(const float* gate_y, int rows, const float* silu_table, float* middle, uint32_t* flags) {
    for (int r = 0; r < rows; ++r)
        for (int c = 0; c < ORC_I; ++c) {
            float g = gate_y[(size_t)r * 2 * ORC_I + c], up = gate_y[(size_t)r * 2 * ORC_I + ORC_I + c];
            float silu = silu_table[f2u(g) >> 16];
            float value = orc_bf16_to_f32(orc_bf16_rne(silu * up));
            if (!isfinite(value)) *flags |= ORC_FLAG_NONFINITE_MIDDLE;
            middle[(size_t)r * ORC_I + c] = value;
        }
}

/* Weighted slot-ordered combine (reduce_slots, :176-185):
 * sum = +0; for slot 0..7 with a valid id: sum = sum + route_out*w;
 * out = bf16_rne(sum); flag 32 if sum is not finite or rounds to bf16 inf/nan. */
void orc_combine(const float* route_out, const float* weights, const int32_t* ids, int T,
                 float* out_f32, uint16_t* out, uint32_t* flags) {
    uint32_t f = 0;
#pragma omp parallel for reduction(| : f) schedule(static)
    for (int t = 0; t < T; ++t)
        for (int c = 0; c < ORC_H; ++c) {
            float sum = 0.f;
            for (int s = 0; s < ORC_TOP; ++s) {
                size_t r = (size_t)t * ORC_TOP + s;
                if (id_valid(ids[r])) { float product = route_out[r * ORC_H + c] * weights[r]; sum = sum + product; }
            }
            uint16_t result = orc_bf16_rne(sum);
            if (out_f32) out_f32[(size_t)t * ORC_H + c] = sum;
            out[(size_t)t * ORC_H + c] = result;
            if (!isfinite(sum) || (result & 0x7f80u) == 0x7f80u) f |= ORC_FLAG_NONFINITE_OUT;
        }
    *flags |= f;
}

/* Full routed layer (ornith_routed_direct_launch{,_a4}), stage order of
 * routed_storage_n32_consumer.cpp:337-347: transform, quantize, gate/up
 * projection, SiLU*up, transform, quantize, down projection, combine.
 * a8 = 1 for A8 activations, 0 for A4.  out_f32 may be NULL. */
int orc_routed_layer(const uint16_t* x, const float* weights, const int32_t* ids, int T,
                     const uint32_t* gate_codes, const uint32_t* gate_meta,
                     const uint32_t* down_codes, const uint32_t* down_meta,
                     int a8, uint16_t* out, float* out_f32, uint32_t* flags) {
    if (T <= 0) return 0;
    const size_t R = (size_t)T * ORC_TOP;
    float* gx = (float*)malloc(sizeof(float) * (size_t)T * ORC_H);
    int8_t* gq = (int8_t*)malloc((size_t)T * ORC_H);
    uint16_t* gs = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * (ORC_H / ORC_G));
    int32_t* gsum = (int32_t*)malloc(sizeof(int32_t) * (size_t)T * (ORC_H / ORC_G));
    float* gy = (float*)malloc(sizeof(float) * R * 2 * ORC_I);
    float* mid = (float*)malloc(sizeof(float) * R * ORC_I);
    float* dx = (float*)malloc(sizeof(float) * R * ORC_I);
    int8_t* dq = (int8_t*)malloc(R * ORC_I);
    uint16_t* ds = (uint16_t*)malloc(sizeof(uint16_t) * R * (ORC_I / ORC_G));
    int32_t* dsum = (int32_t*)malloc(sizeof(int32_t) * R * (ORC_I / ORC_G));
    float* ro = (float*)malloc(sizeof(float) * R * ORC_H);
    if (!gx || !gq || !gs || !gsum || !gy || !mid || !dx || !dq || !ds || !dsum || !ro) return -1;
    orc_transform_tokens(x, ids, T, gx, flags);
    orc_quantize_rows(gx, T, ORC_H, a8, gq, gs, gsum, flags);
    orc_project_routed(2 * ORC_I, ORC_H, 1, ids, (int)R, gate_codes, gate_meta, gq, gs, gsum, gy, flags);
    orc_middle(gy, ids, (int)R, mid, flags);
    orc_transform_rows(mid, (int)R, ORC_I, dx, flags);
    orc_quantize_rows(dx, (int)R, ORC_I, a8, dq, ds, dsum, flags);
    orc_project_routed(ORC_H, ORC_I, 0, ids, (int)R, down_codes, down_meta, dq, ds, dsum, ro, flags);
    orc_combine(ro, weights, ids, T, out_f32, out, flags);
    free(gx); free(gq); free(gs); free(gsum); free(gy); free(mid); free(dx); free(dq); free(ds); free(dsum); free(ro);
    return 0;
}

/* Routed layer with the shared expert fused as a ninth slot
 * (ornith_routed_direct_launch_shared_tables, routed_storage_n32_consumer.cpp:385-401):
 * every row live for the input transform, A8 throughout, shared gate/up and
 * down outputs rounded to bf16, shared SiLU from silu_table[bf16 bits],
 * shared output = bf16(down * bf16_to_f32(sigmoid_table[logit bits])), written
 * separately (:296-306).  logit is bf16 [T]. */
int orc_routed_layer_shared(const uint16_t* x, const float* weights, const int32_t* ids, int T,
                            const uint32_t* gate_codes, const uint32_t* gate_meta,
                            const uint32_t* down_codes, const uint32_t* down_meta,
                            const uint32_t* sgate_codes, const uint32_t* sgate_meta,
                            const uint32_t* sdown_codes, const uint32_t* sdown_meta,
                            const uint16_t* logit, const float* silu_table, const uint16_t* sigmoid_table,
                            uint16_t* out, uint16_t* shared_out, float* out_f32, uint32_t* flags) {
    if (T <= 0) return 0;
    const size_t R = (size_t)T * ORC_TOP, RS = R + (size_t)T;
    float* gx = (float*)malloc(sizeof(float) * (size_t)T * ORC_H);
    int8_t* gq = (int8_t*)malloc((size_t)T * ORC_H);
    uint16_t* gs = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * (ORC_H / ORC_G));
    int32_t* gsum = (int32_t*)malloc(sizeof(int32_t) * (size_t)T * (ORC_H / ORC_G));
    float* gy = (float*)malloc(sizeof(float) * RS * 2 * ORC_I);
    float* mid = (float*)malloc(sizeof(float) * RS * ORC_I);
    float* dx = (float*)malloc(sizeof(float) * RS * ORC_I);
    int8_t* dq = (int8_t*)malloc(RS * ORC_I);
    uint16_t* ds = (uint16_t*)malloc(sizeof(uint16_t) * RS * (ORC_I / ORC_G));
    int32_t* dsum = (int32_t*)malloc(sizeof(int32_t) * RS * (ORC_I / ORC_G));
    float* ro = (float*)malloc(sizeof(float) * RS * ORC_H);
    if (!gx || !gq || !gs || !gsum || !gy || !mid || !dx || !dq || !ds || !dsum || !ro) return -1;
    orc_transform_tokens(x, NULL, T, gx, flags);
    orc_quantize_rows(gx, T, ORC_H, 1, gq, gs, gsum, flags);
    orc_project_routed(2 * ORC_I, ORC_H, 1, ids, (int)R, gate_codes, gate_meta, gq, gs, gsum, gy, flags);
    orc_project_shared(2 * ORC_I, ORC_H, T, sgate_codes, sgate_meta, gq, gs, gsum, gy, (int)R, flags);
    orc_middle(gy, ids, (int)R, mid, flags);
    orc_middle_shared(gy + R * 2 * ORC_I, T, silu_table, mid + R * ORC_I, flags);
    orc_transform_rows(mid, (int)RS, ORC_I, dx, flags);
    orc_quantize_rows(dx, (int)RS, ORC_I, 1, dq, ds, dsum, flags);
    orc_project_routed(ORC_H, ORC_I, 0, ids, (int)R, down_codes, down_meta, dq, ds, dsum, ro, flags);
    /* shared down rows R..R+T-1 read activation rows R..R+T-1 */
    {
        int nthreads = 1;
#ifdef _OPENMP
        nthreads = omp_get_max_threads();
#endif
        int chunk = (T + nthreads - 1) / nthreads;
        uint32_t f = 0;
#pragma omp parallel for reduction(| : f) schedule(static, 1)
        for (int c0 = 0; c0 < T; c0 += chunk) {
            int n = T - c0 < chunk ? T - c0 : chunk;
            int* src = (int*)malloc(sizeof(int) * n);
            for (int i = 0; i < n; ++i) src[i] = (int)R + c0 + i;
            uint32_t lf = 0;
            project_bank(ORC_H, ORC_I, sdown_codes, sdown_meta, src, src, n, dq, ds, dsum, ro, 1, &lf);
            f |= lf;
            free(src);
        }
        *flags |= f;
    }
    orc_combine(ro, weights, ids, T, out_f32, out, flags);
    {
        uint32_t f = 0;
        for (int t = 0; t < T; ++t) {
            float gate = orc_bf16_to_f32(sigmoid_table[logit[t]]);
            for (int c = 0; c < ORC_H; ++c) {
                float shared = ro[(R + (size_t)t) * ORC_H + c] * gate;
                shared_out[(size_t)t * ORC_H + c] = orc_bf16_rne(shared);
                if (!isfinite(shared)) f |= ORC_FLAG_NONFINITE_OUT;
            }
        }
        *flags |= f;
    }
    free(gx); free(gq); free(gs); free(gsum); free(gy); free(mid); free(dx); free(dq); free(ds); free(dsum); free(ro);
    return 0;
}

/* Router top-8 with renormalised softmax weights.
 * Semantics of vLLM's fused_topk with renormalize=True as restated on the CPU
 * (vllm/model_executor/layers/fused_moe/cpu_fused_moe.py:145-150): take the
 * eight largest logits, weights = softmax over those eight.  Slot order is
 * descending logit with the lower expert index first on ties (the order of
 * vLLM's GPU topk_softmax).  The exponential is the reference's portable exp so
 * that host and device agree bit for bit:
 *   m = l[slot 0]; e_s = exp_p(l_s - m); S = ((e_0 + e_1) + ...) + e_7;
 *   w_s = e_s / S (IEEE division).
 * Non-finite logits never win selection; a row with fewer than eight finite
 * logits pads the remaining slots with id -1 and weight 0. */
void orc_route_topk(const float* logits, int T, float* weights, int32_t* ids) {
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t) {
        const float* l = logits + (size_t)t * ORC_E;
        unsigned char taken[ORC_E];
        memset(taken, 0, sizeof taken);
        int sel[ORC_TOP];
        for (int s = 0; s < ORC_TOP; ++s) {
            int best = -1;
            for (int e = 0; e < ORC_E; ++e) {
                if (taken[e] || !isfinite(l[e])) continue;
                if (best < 0 || l[e] > l[best]) best = e;
            }
            sel[s] = best;
            if (best >= 0) taken[best] = 1;
        }
        float ex[ORC_TOP], sum = 0.f;
        float m = sel[0] >= 0 ? l[sel[0]] : 0.f;
        for (int s = 0; s < ORC_TOP; ++s) {
            ex[s] = sel[s] >= 0 ? orc_portable_exp(l[sel[s]] - m) : 0.f;
            sum = sum + ex[s];
        }
        for (int s = 0; s < ORC_TOP; ++s) {
            ids[(size_t)t * ORC_TOP + s] = sel[s];
            weights[(size_t)t * ORC_TOP + s] = sel[s] >= 0 ? ex[s] / sum : 0.f;
        }
    }
}

/* Router logits (a1 of the reference, iu4_correctness/gates_projection.py:17-25):
 * logits[t,e] = sum_k f32(x[t,k]) * f32(W[e,k]).  The reference's Triton
 * reduction order is unspecified; this restatement accumulates in double and
 * rounds once, which the parity tests treat as a tolerance-level reference. */
void orc_router_logits(const uint16_t* x, const uint16_t* w, int T, float* logits) {
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t)
        for (int e = 0; e < ORC_E; ++e) {
            double acc = 0.0;
            for (int k = 0; k < ORC_H; ++k)
                acc += (double)orc_bf16_to_f32(x[(size_t)t * ORC_H + k]) * (double)orc_bf16_to_f32(w[(size_t)e * ORC_H + k]);
            logits[(size_t)t * ORC_E + e] = (float)acc;
        }
}

/* Dequantised fp32 evaluation with no activation quantisation (reported only:
 * it measures the quantisation error of the reference's format, it is not the
 * parity target).  Weight = scale*code + offset (dense_g256_consumer.cpp:219),
 * applied in the Hadamard basis of the activations. */
void orc_fp32_reference_layer(const uint16_t* x, const float* weights, const int32_t* ids, int T,
                              const uint32_t* gate_codes, const uint32_t* gate_meta,
                              const uint32_t* down_codes, const uint32_t* down_meta, float* out) {
    const size_t gc = (size_t)2 * ORC_I * ORC_H / 8, gm = (size_t)2 * ORC_I * (ORC_H / ORC_G);
    const size_t dc = (size_t)ORC_H * ORC_I / 8, dm = (size_t)ORC_H * (ORC_I / ORC_G);
    uint32_t dummy = 0;
    float* gx = (float*)malloc(sizeof(float) * (size_t)T * ORC_H);
    orc_transform_tokens(x, ids, T, gx, &dummy);
#pragma omp parallel for schedule(dynamic, 1)
    for (int t = 0; t < T; ++t) {
        float acc_out[ORC_H];
        for (int c = 0; c < ORC_H; ++c) acc_out[c] = 0.f;
        for (int s = 0; s < ORC_TOP; ++s) {
            int e = ids[(size_t)t * ORC_TOP + s];
            if (!id_valid(e)) continue;
            float gu[2 * ORC_I], mid[ORC_I], mx[ORC_I];
            for (int n = 0; n < 2 * ORC_I; ++n) {
                double a = 0.0;
                for (int k = 0; k < ORC_H; ++k) {
                    int g = k / ORC_G, j = (k % ORC_G) / 8, d = k % 8;
                    uint32_t w = gate_codes[e * gc + (((size_t)(n / 32) * (ORC_H / ORC_G) + g) * 32 + j) * 32 + (n & 31)];
                    uint32_t mt = gate_meta[e * gm + ((size_t)(n / 32) * (ORC_H / ORC_G) + g) * 32 + (n & 31)];
                    float wv = orc_half_to_f32((uint16_t)(mt & 0xffff)) * (float)((w >> (4 * d)) & 15u) + orc_half_to_f32((uint16_t)(mt >> 16));
                    a += (double)wv * gx[(size_t)t * ORC_H + k];
                }
                gu[n] = (float)a;
            }
            for (int c = 0; c < ORC_I; ++c) mid[c] = orc_silu(gu[c]) * gu[ORC_I + c];
            for (int b = 0; b < ORC_I / 128; ++b) orc_wht128(mid + b * 128, mx + b * 128);
            for (int n = 0; n < ORC_H; ++n) {
                double a = 0.0;
                for (int k = 0; k < ORC_I; ++k) {
                    int g = k / ORC_G, j = (k % ORC_G) / 8, d = k % 8;
                    uint32_t w = down_codes[e * dc + (((size_t)(n / 32) * (ORC_I / ORC_G) + g) * 32 + j) * 32 + (n & 31)];
                    uint32_t mt = down_meta[e * dm + ((size_t)(n / 32) * (ORC_I / ORC_G) + g) * 32 + (n & 31)];
                    float wv = orc_half_to_f32((uint16_t)(mt & 0xffff)) * (float)((w >> (4 * d)) & 15u) + orc_half_to_f32((uint16_t)(mt >> 16));
                    a += (double)wv * mx[k];
                }
                acc_out[n] += (float)a * weights[(size_t)t * ORC_TOP + s];
            }
        }
        for (int c = 0; c < ORC_H; ++c) out[(size_t)t * ORC_H + c] = acc_out[c];
    }
    free(gx);
}

/* N16 checkpoint bank -> N32 storage, the one-time repack of
 * plugin-site/ornith_g256/method.py:142-147: codes [E,N/16,Gr,32,16] ->
 * [E,N/32,Gr,32,32] with column c of an N32 tile = 16*half + lane16;
 * metadata [E,N/16,Gr,16] -> [E,N/32,Gr,32]. */
void orc_repack_n16_to_n32(const uint32_t* codes16, const uint32_t* meta16, int E, int N, int K,
                           uint32_t* codes32, uint32_t* meta32) {
    const int nt = N / 16, groups = K / ORC_G;
    for (int e = 0; e < E; ++e)
        for (int t2 = 0; t2 < nt / 2; ++t2)
            for (int g = 0; g < groups; ++g) {
                for (int j = 0; j < 32; ++j)
                    for (int half = 0; half < 2; ++half)
                        for (int l = 0; l < 16; ++l)
                            codes32[((((size_t)e * (nt / 2) + t2) * groups + g) * 32 + j) * 32 + half * 16 + l] =
                                codes16[((((size_t)e * nt + 2 * t2 + half) * groups + g) * 32 + j) * 16 + l];
                for (int half = 0; half < 2; ++half)
                    for (int l = 0; l < 16; ++l)
                        meta32[(((size_t)e * (nt / 2) + t2) * groups + g) * 32 + half * 16 + l] =
                            meta16[(((size_t)e * nt + 2 * t2 + half) * groups + g) * 16 + l];
            }
}

/* ------------------------------------------------------------------------
 * Dense G256 projection (the reference's dense-layer library,
 * kernels/dense_n32/dense_g256_api.h:20-38 and dense_g256_consumer.cpp).
 * Dense flag bits (dense_g256_api.h:14-19): 1 non-finite transform input or
 * output, 2 invalid activation, 4 non-finite projection, 8 non-finite bf16. */
enum { ORC_DENSE_NONFINITE_BF16 = 8, ORC_DENSE_NONFINITE_PROJ = 4 };

/* Column n, group g, word j of a dense bank stored `width` columns per tile
 * (16: codes U32[N/16][K/256][32][16], dense_g256_api.h:27; 32: the N32 shadow
 * U32[N/32][K/256][32][32], dense_n32.py:30-31). */
static size_t dense_code_at(int width, int groups, int n, int g, int j) {
    return (((size_t)(n / width) * groups + g) * 32 + j) * width + (n % width);
}
static size_t dense_meta_at(int width, int groups, int n, int g) {
    return ((size_t)(n / width) * groups + g) * width + (n % width);
}

/* store() of dense_g256_consumer.cpp:74-79: flag 4 for a non-finite fp32
 * value, bf16 RNE, flag 8 when the bf16 exponent is all ones. */
static uint16_t dense_store(float v, uint32_t* f) {
    if (!isfinite(v)) *f |= ORC_DENSE_NONFINITE_PROJ;
    uint16_t r = orc_bf16_rne(v);
    if ((r & 0x7f80u) == 0x7f80u) *f |= ORC_DENSE_NONFINITE_BF16;
    return r;
}

/* A8 dense projection out[M,N] = bf16(x[M,K] . W[N,K]^T) in the reference's
 * arithmetic: per row, bf16 -> fp32, H128 per 128-block (flag 1 on non-finite
 * input or output, transform :27-39), A8 quantisation per 256-group (quantize
 * :41-73, flag 2), then per column over ascending groups
 *   value = value + (w_scale*(sa*dot) + w_offset*(sa*sum))
 * (compact_projection :116-142, wmma_projection :80-115, compact_projection_n32
 * :250-272, compact_projection_n32_rows :325-358 all compute this sequence),
 * stored through dense_store.  diag (may be NULL) receives the fp32 values. */
void orc_dense_project(const uint16_t* x, int M, int N, int K, int width,
                       const uint32_t* codes, const uint32_t* meta,
                       uint16_t* out, float* diag, uint32_t* flags) {
    const int groups = K / ORC_G;
    float* y = (float*)malloc(sizeof(float) * (size_t)M * K);
    int8_t* q = (int8_t*)malloc((size_t)M * K);
    uint16_t* sc = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)M * groups);
    int32_t* sums = (int32_t*)malloc(sizeof(int32_t) * (size_t)M * groups);
    uint32_t f = 0;
    for (int r = 0; r < M; ++r)
        for (int b = 0; b < K / 128; ++b) {
            float in[128];
            for (int l = 0; l < 128; ++l) {
                in[l] = orc_bf16_to_f32(x[(size_t)r * K + b * 128 + l]);
                if (!isfinite(in[l])) f |= ORC_FLAG_NONFINITE_INPUT;
            }
            float* o = y + (size_t)r * K + b * 128;
            orc_wht128(in, o);
            for (int l = 0; l < 128; ++l) if (!isfinite(o[l])) f |= ORC_FLAG_NONFINITE_INPUT;
        }
    orc_quantize_rows(y, M, K, 1, q, sc, sums, &f);
#pragma omp parallel for reduction(| : f) schedule(static)
    for (int n = 0; n < N; ++n) {
        int8_t wc[ORC_G];
        float* acc = (float*)calloc((size_t)M, sizeof(float));
        for (int g = 0; g < groups; ++g) {
            for (int j = 0; j < 32; ++j) {
                uint32_t w = codes[dense_code_at(width, groups, n, g, j)];
                for (int d = 0; d < 8; ++d) wc[j * 8 + d] = (int8_t)((w >> (4 * d)) & 15u);
            }
            uint32_t mt = meta[dense_meta_at(width, groups, n, g)];
            float sw = orc_half_to_f32((uint16_t)(mt & 0xffffu)), off = orc_half_to_f32((uint16_t)(mt >> 16));
            for (int r = 0; r < M; ++r) {
                const int8_t* qa = q + (size_t)r * K + (size_t)g * ORC_G;
                int32_t dot = 0;
                for (int k = 0; k < ORC_G; ++k) dot += (int32_t)wc[k] * (int32_t)qa[k];
                float sa = orc_half_to_f32(sc[(size_t)r * groups + g]);
                float scaled_dot = sa * (float)dot, scaled_sum = sa * (float)sums[(size_t)r * groups + g];
                float product = sw * scaled_dot, correction = off * scaled_sum;
                acc[r] = acc[r] + (product + correction);
            }
        }
        for (int r = 0; r < M; ++r) {
            uint32_t lf = 0;
            out[(size_t)r * N + n] = dense_store(acc[r], &lf);
            if (diag) diag[(size_t)r * N + n] = acc[r];
            f |= lf;
        }
        free(acc);
    }
    *flags |= f;
    free(y);
    free(q);
    free(sc);
    free(sums);
}

/* Prefill preparation (ornith_dense_g256_prepare_bf16, dense_g256_consumer.cpp
 * :192-247): xt[M,K] = bf16(H128(x)) with flag 1 on non-finite input/output
 * and flag 8 on a bf16 with all-ones exponent; w[N,K] = bf16(scale*code +
 * offset) from the N16 bank (fp32 product, then sum), flag 8 likewise. */
void orc_dense_prepare_bf16(const uint16_t* x, int M, int N, int K,
                            const uint32_t* codes16, const uint32_t* meta16,
                            uint16_t* xt, uint16_t* w, uint32_t* flags) {
    const int groups = K / ORC_G;
    uint32_t f = 0;
    for (int r = 0; r < M; ++r)
        for (int b = 0; b < K / 128; ++b) {
            float in[128], o[128];
            for (int l = 0; l < 128; ++l) {
                in[l] = orc_bf16_to_f32(x[(size_t)r * K + b * 128 + l]);
                if (!isfinite(in[l])) f |= ORC_FLAG_NONFINITE_INPUT;
            }
            orc_wht128(in, o);
            for (int l = 0; l < 128; ++l) {
                if (!isfinite(o[l])) f |= ORC_FLAG_NONFINITE_INPUT;
                uint16_t h = orc_bf16_rne(o[l]);
                if ((h & 0x7f80u) == 0x7f80u) f |= ORC_DENSE_NONFINITE_BF16;
                xt[(size_t)r * K + b * 128 + l] = h;
            }
        }
#pragma omp parallel for reduction(| : f) schedule(static)
    for (int n = 0; n < N; ++n)
        for (int g = 0; g < groups; ++g) {
            uint32_t mt = meta16[dense_meta_at(16, groups, n, g)];
            float sw = orc_half_to_f32((uint16_t)(mt & 0xffffu)), off = orc_half_to_f32((uint16_t)(mt >> 16));
            for (int j = 0; j < 32; ++j) {
                uint32_t code = codes16[dense_code_at(16, groups, n, g, j)];
                for (int d = 0; d < 8; ++d) {
                    float v = sw * (float)((code >> (4 * d)) & 15u) + off;
                    uint16_t h = orc_bf16_rne(v);
                    if ((h & 0x7f80u) == 0x7f80u) f |= ORC_DENSE_NONFINITE_BF16;
                    w[(size_t)n * K + (size_t)g * ORC_G + j * 8 + d] = h;
                }
            }
        }
    *flags |= f;
}

/* ------------------------------------------------------------------------
 * W8 LM head (kernels/head/head_i8_tile_api.h:21-41, head_i8_tile_consumer.cpp).
 * K = 2048 in 16 groups of 128.  Weights: signed int8 codes in words
 * UINT32[N/16][K/16][4][16] (word kw = k/4 of column n at
 * ((n/16*(K/16) + kw/4)*4 + kw%4)*16 + n%16, byte k%4 = bits 8(k%4)..),
 * fp16 scales [N][16], no offset.  Per row: H128 per group (flag 1), A8 per
 * 128-group (quantisation as the routed path, over 128 elements, flag 2),
 * exact int32 group dots, then over groups g = 0..15
 *   value = value + w_scale[n][g]*(sa[g]*float(dot))
 * (compact_projection :87-116 and the WMMA forms compute this sequence),
 * stored through dense_store (flags 4 and 8).  group_dots (may be NULL)
 * receives the raw dots [M][N][16]. */
void orc_head_project(const uint16_t* x, int M, int N, const uint32_t* words, const uint16_t* scales,
                      uint16_t* out, float* diag, int32_t* group_dots, uint32_t* flags) {
    enum { HK = 2048, HG = 128, HGROUPS = 16 };
    int8_t* q = (int8_t*)malloc((size_t)M * HK);
    float* sa = (float*)malloc(sizeof(float) * (size_t)M * HGROUPS);
    uint32_t f = 0;
    for (int r = 0; r < M; ++r)
        for (int g = 0; g < HGROUPS; ++g) {
            float in[HG], t[HG], v[HG], absmax = 0.f;
            for (int l = 0; l < HG; ++l) {
                in[l] = orc_bf16_to_f32(x[(size_t)r * HK + g * HG + l]);
                if (!isfinite(in[l])) f |= ORC_FLAG_NONFINITE_INPUT;
            }
            orc_wht128(in, t);
            for (int l = 0; l < HG; ++l) {
                if (!isfinite(t[l])) f |= ORC_FLAG_NONFINITE_INPUT;
                int finite = isfinite(t[l]);
                if (!finite) f |= ORC_FLAG_INVALID_ACT;
                v[l] = finite ? t[l] : 0.f;
                absmax = fmaxf(absmax, fabsf(v[l]));
            }
            float raw = absmax / 127.f;
            int valid = isfinite(raw) && raw <= 65504.f;
            if (!valid) f |= ORC_FLAG_INVALID_ACT;
            uint16_t scale = orc_f32_to_half_rne(absmax == 0.f || !valid ? 1.f : fmaxf(raw, 0x1p-14f));
            float sf = orc_half_to_f32(scale);
            for (int l = 0; l < HG; ++l) {
                int qi = (absmax == 0.f || !valid) ? 0 : (int)nearbyintf(v[l] / sf);
                q[(size_t)r * HK + g * HG + l] = (int8_t)(qi < -127 ? -127 : (qi > 127 ? 127 : qi));
            }
            sa[(size_t)r * HGROUPS + g] = sf;
        }
#pragma omp parallel for reduction(| : f) schedule(static)
    for (int n = 0; n < N; ++n) {
        int8_t wc[HK];
        for (int k = 0; k < HK; k += 4) {
            int kw = k / 4;
            uint32_t w = words[(((size_t)(n / 16) * (HK / 16) + kw / 4) * 4 + kw % 4) * 16 + n % 16];
            for (int b = 0; b < 4; ++b) wc[k + b] = (int8_t)((w >> (8 * b)) & 255u);
        }
        for (int r = 0; r < M; ++r) {
            float value = 0.f;
            for (int g = 0; g < HGROUPS; ++g) {
                int32_t dot = 0;
                for (int l = 0; l < HG; ++l) dot += (int32_t)wc[g * HG + l] * (int32_t)q[(size_t)r * HK + g * HG + l];
                if (group_dots) group_dots[((size_t)r * N + n) * HGROUPS + g] = dot;
                float scaled = sa[(size_t)r * HGROUPS + g] * (float)dot;
                float term = orc_half_to_f32(scales[(size_t)n * HGROUPS + g]) * scaled;
                value = value + term;
            }
            uint32_t lf = 0;
            out[(size_t)r * N + n] = dense_store(value, &lf);
            if (diag) diag[(size_t)r * N + n] = value;
            f |= lf;
        }
    }
    *flags |= f;
    free(q);
    free(sa);
}

int orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}
