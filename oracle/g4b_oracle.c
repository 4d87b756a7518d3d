/*
 * g4b_oracle.c -- CPU restatement of the gemma4-adreno quantized-weight hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library and the timed CPU baseline in bench.py.  Nothing in the product
 * (the g4b package or its CUDA library) links, imports or calls it.
 *
 * Each function restates one reference routine, in the reference's own
 * arithmetic order, and cites the file:line it follows (paths are relative to
 * the reference project root):
 *
 *   orc_quant_i4        src/vk_engine.py:126-131   int4 block quantisation + nibble packing
 *   orc_e4m3_encode     src/vk_engine.py:136       torch float8_e4m3fn cast (round-to-nearest-even)
 *   orc_e4m3_decode     vk/gemv_fp8.comp:14-18     the shader's e4m3 decode
 *   orc_fp8_scales      src/vk_engine.py:133-137   per-tensor power-of-two lift + e4m3 scales
 *   orc_split           src/vk_engine.py:143-148   split-K heuristic
 *   orc_w8a8_weights    src/vk_engine.py:152-157   folded int8 weights + f16 column scales
 *   orc_gemv            vk/gemv.comp:11-33, vk/gemv_fp8.comp:20-40
 *   orc_reduce          vk/reduce.comp:8-12
 *   orc_dequant_f16     vk/coopgemm_i4h.comp:19-25 (the shared-memory dequant tile)
 *   orc_gemm_i4         vk/coopgemm_i4h.comp:13-35 with an f32 accumulator (vk/coopgemm_i4f.comp:16-32)
 *   orc_cast_i8         vk/cast_i8.comp:11-19
 *   orc_gemm_w8a8       vk/coopgemm_w8a8.comp:18-37
 *   orc_w4a8_requant    vk/coopgemm_w4a8.comp:28-34
 *   orc_gemm_w4a8       vk/coopgemm_w4a8.comp:21-50
 *   orc_rmsnorm         vk/rmsnorm.comp:8-12
 *   orc_normadd         vk/normadd.comp:8-12
 *   orc_gelumul         vk/gelumul.comp:7-8
 *   orc_attn_prepkv     vk/prepkv.comp:14-31
 *   orc_attn_decode     vk/attn.comp:15-55
 *   orc_attn_prefill_prepkv  vk/pre_prepkv.comp:15-30
 *   orc_attn_prefill    vk/pre_attn.comp:16-53
 *
 * Choices the GLSL leaves to the implementation, fixed here and stated once:
 *   - round(): round-half-to-even (roundEven), the same as numpy's np.round used
 *     by the reference's host quantiser and benchmarks.
 *   - no multiply-add contraction (built with -ffp-contract=off): every GLSL
 *     '*' and '+' is one correctly rounded f32 operation.
 *   - 1.0/s and amax/127.0 are correctly rounded f32 divisions.
 *   - inversesqrt(v) is 1.0f / sqrtf(v), both correctly rounded (GLSL allows
 *     2 ULP); tanh is the C library's tanhf.
 *
 * Parity pinning: the packing functions are pinned bit-for-bit against golden
 * vectors produced by running the reference's own quant() (tests/golden/).  The
 * shader restatements cannot be pinned against the shaders (no Vulkan stack on
 * these machines); they are pinned against the reference benchmarks' seeded
 * cosine checks (benchmarks/vk_gemv.py:56-65,143; benchmarks/coopgemm_i4.py:42-52;
 * benchmarks/coopgemm_w4a8.py:74-110; benchmarks/coopgemm_i8.py:41-44,80).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_BLK 32

/* ---------------------------------------------------------------- f16 helpers */
/* IEEE binary16 <-> binary32, round-to-nearest-even, with subnormals.  Written
 * out rather than relying on the compiler's _Float16 so the oracle does not
 * depend on F16C availability. */
static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

float orc_f16_to_f32(uint16_t h) {
    uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31, m = h & 1023;
    if (e == 0) {
        if (m == 0) return u2f(s);
        /* subnormal: m * 2^-24, exact in f32 */
        float v = (float)m * 5.9604644775390625e-08f;
        return s ? -v : v;
    }
    if (e == 31) return u2f(s | 0x7f800000u | (m << 13));
    return u2f(s | ((e + 112) << 23) | (m << 13));
}

uint16_t orc_f32_to_f16(float f) {
    uint32_t u = f2u(f);
    uint32_t s = (u >> 16) & 0x8000u;
    uint32_t a = u & 0x7fffffffu;
    if (a >= 0x7f800000u) return (uint16_t)(s | 0x7c00u | (a > 0x7f800000u ? 0x200u : 0));
    if (a >= 0x477ff000u) return (uint16_t)(s | 0x7c00u);   /* rounds to >= 65520 -> inf */
    if (a < 0x38800000u) {                                     /* below 2^-14: subnormal or zero */
        if (a < 0x33000000u) return (uint16_t)s;              /* < 2^-25 -> 0 (2^-25 ties to 0) */
        uint32_t e = a >> 23, m = (a & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126 - e;                              /* 14..24 */
        uint32_t q = m >> shift, rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) q++;
        return (uint16_t)(s | q);
    }
    uint32_t e = (a >> 23) - 112, m = a & 0x7fffffu;
    uint32_t q = (e << 10) | (m >> 13), rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) q++;
    return (uint16_t)(s | q);
}

/* ------------------------------------------------------------- e4m3 helpers */
/* vk/gemv_fp8.comp:14-18: sign, 4-bit exponent (bias 7), 3-bit mantissa.
 * exponent 0 -> m * 2^-9 ; otherwise (1 + m/8) * 2^(e-7).  No NaN case. */
float orc_e4m3_decode(uint8_t b) {
    uint32_t s = (b >> 7) & 1u, ex = (b >> 3) & 15u, m = b & 7u;
    float v = (ex == 0u) ? (float)m * (1.0f / 512.0f) : (1.0f + (float)m * 0.125f) * ldexpf(1.0f, (int)ex - 7);
    return s ? -v : v;
}

/* float8_e4m3fn encode with round-to-nearest-even, as torch's cast does for
 * finite inputs of magnitude <= 448 (the reference clips to [0, 448] first,
 * src/vk_engine.py:135).  Larger magnitudes saturate to 448 here. */
uint8_t orc_e4m3_encode(float f) {
    uint32_t u = f2u(f);
    uint8_t sign = (uint8_t)((u >> 24) & 0x80u);
    float a = fabsf(f);
    if (!(a == a)) return (uint8_t)(sign | 0x7f);
    if (a >= 464.0f) return (uint8_t)(sign | 0x7e);             /* 448 is the largest finite */
    if (a < ldexpf(1.0f, -6)) {                                 /* subnormal band: multiples of 2^-9 */
        float q = a * 512.0f;                                   /* exact */
        float r = nearbyintf(q);                                /* RNE (default rounding mode) */
        return (uint8_t)(sign | (uint8_t)r);                    /* r == 8 encodes 2^-6 (exp 1, m 0) */
    }
    int e; float fr = frexpf(a, &e);                            /* a = fr * 2^e, fr in [0.5, 1) */
    int E = e - 1;                                              /* a = 1.xxx * 2^E, E in [-6, 8] */
    float mant = ldexpf(a, -E) - 1.0f;                          /* [0, 1), exact */
    float q = nearbyintf(mant * 8.0f);                          /* RNE to 3 bits */
    if (q >= 8.0f) { q = 0.0f; E += 1; }
    if (E > 8 || (E == 8 && q > 6.0f)) return (uint8_t)(sign | 0x7e);
    (void)fr;
    return (uint8_t)(sign | (uint8_t)((E + 7) << 3) | (uint8_t)q);
}

/* ------------------------------------------------------------------ packing */
/* src/vk_engine.py:126-131.  W is [N, K] row-major f32.
 * sc_out  : [N, nblk] f32 block scales (max(absmax/7, 1e-8))
 * q_out   : [N, K] nibbles (clip(rint(W/sc) + 8, 0, 15)), may be NULL
 * wp      : [K, N/8] u32, nibble j of word (k, g) = column 8g + j
 * sc16    : [nblk, N] f16 bits (the transposed scales) */
void orc_quant_i4(const float* W, int N, int K, float* sc_out, uint8_t* q_out,
                  uint32_t* wp, uint16_t* sc16) {
    int nblk = K / ORC_BLK;
    memset(wp, 0, sizeof(uint32_t) * (size_t)K * (N / 8));
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; n++) {
        for (int b = 0; b < nblk; b++) {
            const float* w = W + (size_t)n * K + (size_t)b * ORC_BLK;
            float amax = 0.0f;
            for (int i = 0; i < ORC_BLK; i++) { float a = fabsf(w[i]); if (a > amax) amax = a; }
            float s = amax / 7.0f;
            if (!(s >= 1e-8f)) s = 1e-8f;                        /* np.maximum(., 1e-8) in f32 */
            sc_out[(size_t)n * nblk + b] = s;
            sc16[(size_t)b * N + n] = orc_f32_to_f16(s);
            for (int i = 0; i < ORC_BLK; i++) {
                float r = nearbyintf(w[i] / s) + 8.0f;
                if (r < 0.0f) r = 0.0f;
                if (r > 15.0f) r = 15.0f;
                uint32_t q = (uint32_t)r;
                int k = b * ORC_BLK + i;
                if (q_out) q_out[(size_t)n * K + k] = (uint8_t)q;
            }
        }
    }
    /* pack after the parallel loop so no two threads write one word */
#pragma omp parallel for schedule(static)
    for (int k = 0; k < K; k++) {
        for (int g = 0; g < N / 8; g++) {
            uint32_t word = 0;
            for (int j = 0; j < 8; j++) {
                int n = 8 * g + j;
                int b = k / ORC_BLK;
                float s = sc_out[(size_t)n * nblk + b];
                float r = nearbyintf(W[(size_t)n * K + k] / s) + 8.0f;
                if (r < 0.0f) r = 0.0f;
                if (r > 15.0f) r = 15.0f;
                word |= ((uint32_t)r & 15u) << (4 * j);
            }
            wp[(size_t)k * (N / 8) + g] = word;
        }
    }
}

/* src/vk_engine.py:133-137.  sc is [N, nblk] f32; writes [nblk, N] e4m3 bytes
 * and returns inv = 2^-shift. */
double orc_fp8_scales(const float* sc, int N, int nblk, uint8_t* e8) {
    float mx = 0.0f;
    for (size_t i = 0; i < (size_t)N * nblk; i++) if (sc[i] > mx) mx = sc[i];
    int shift = (mx > 0.0f) ? (int)floor(log2(256.0 / (double)mx)) : 0;
    float mul = (float)ldexp(1.0, shift);
    for (int n = 0; n < N; n++)
        for (int b = 0; b < nblk; b++) {
            float v = sc[(size_t)n * nblk + b] * mul;
            if (v < 0.0f) v = 0.0f;
            if (v > 448.0f) v = 448.0f;
            e8[(size_t)b * N + n] = orc_e4m3_encode(v);
        }
    return ldexp(1.0, -shift);
}

/* src/vk_engine.py:143-148: rows = ceil(N/8 / 64); want = max(1, ceil(384/rows));
 * the divisor of nblk closest to want, ties to the smaller divisor. */
int orc_split(int N, int nblk) {
    int rows = (N / 8 + 63) / 64;
    int r = rows > 1 ? rows : 1;
    int want = (384 + r - 1) / r;
    if (want < 1) want = 1;
    int best = 1, bestd = abs(1 - want);
    for (int s = 1; s <= nblk; s++) {
        if (nblk % s) continue;
        int d = abs(s - want);
        if (d < bestd) { best = s; bestd = d; }
    }
    return best;
}

/* src/vk_engine.py:152-157.  q is [N, K] nibbles, sc [N, nblk] f32.
 * w8t: [K, N] int8 = clip(rint(deqW / s_w), -127, 127) with deqW = (q - 8) * sc (f32)
 * sw16: [N] f16 bits of s_w = max(rowabsmax(deqW) / 127, 1e-12) */
void orc_w8a8_weights(const uint8_t* q, const float* sc, int N, int K, int8_t* w8t, uint16_t* sw16,
                      float* sw_f32) {
    int nblk = K / ORC_BLK;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; n++) {
        float amax = 0.0f;
        for (int k = 0; k < K; k++) {
            float d = ((float)q[(size_t)n * K + k] - 8.0f) * sc[(size_t)n * nblk + k / ORC_BLK];
            float a = fabsf(d); if (a > amax) amax = a;
        }
        float s = amax / 127.0f;
        if (!(s >= 1e-12f)) s = 1e-12f;
        if (sw_f32) sw_f32[n] = s;
        sw16[n] = orc_f32_to_f16(s);
        for (int k = 0; k < K; k++) {
            float d = ((float)q[(size_t)n * K + k] - 8.0f) * sc[(size_t)n * nblk + k / ORC_BLK];
            float r = nearbyintf(d / s);
            if (r < -127.0f) r = -127.0f;
            if (r > 127.0f) r = 127.0f;
            w8t[(size_t)k * N + n] = (int8_t)r;
        }
    }
}

/* benchmarks/coopgemm_w4a8.py:84: ratio[b, n] = f16(sc[n, b] / s_w[n]) */
void orc_w4a8_ratio(const float* sc, const float* sw_f32, int N, int nblk, uint16_t* ratio16) {
    for (int n = 0; n < N; n++)
        for (int b = 0; b < nblk; b++)
            ratio16[(size_t)b * N + n] = orc_f32_to_f16(sc[(size_t)n * nblk + b] / sw_f32[n]);
}

/* ------------------------------------------------------------------ GEMV */
static inline float scale_at(const void* scales, int fmt, int N, int b, int n) {
    if (fmt == 0) return orc_f16_to_f32(((const uint16_t*)scales)[(size_t)b * N + n]);
    return orc_e4m3_decode(((const uint8_t*)scales)[(size_t)b * N + n]);
}

/* vk/gemv.comp:11-33 (fmt 0, f16 scales) and vk/gemv_fp8.comp:20-40 (fmt 1,
 * e4m3 scales, output times inv).  x is f32 [M, K] (M tokens; the shader has
 * M = 1).  For each column n and K-slice c (bpc = nblk/split blocks):
 *     acc = 0; for each block: s = scale; for each k: acc += ((nib - 8) * s) * x[k]
 * partial[c, m, n] = acc (* inv for fp8).  If y is non-NULL, y[m, n] is the
 * reduce.comp sum over c ascending. */
void orc_gemv(const float* x, int M, const uint32_t* wp, const void* scales, int fmt, float inv,
              int N, int K, int split, float* partial, float* y) {
    int nblk = K / ORC_BLK, bpc = nblk / split, nb8 = N / 8;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; n++) {
        int g = n >> 3, j = n & 7;
        for (int m = 0; m < M; m++) {
            const float* xm = x + (size_t)m * K;
            float tot = 0.0f;
            for (int c = 0; c < split; c++) {
                float acc = 0.0f;
                for (int bi = 0; bi < bpc; bi++) {
                    int b = c * bpc + bi;
                    float s = scale_at(scales, fmt, N, b, n);
                    for (int kk = 0; kk < ORC_BLK; kk++) {
                        int k = b * ORC_BLK + kk;
                        uint32_t nib = (wp[(size_t)k * nb8 + g] >> (4 * j)) & 15u;
                        float w = ((float)nib - 8.0f) * s;
                        float t = w * xm[k];
                        acc = acc + t;
                    }
                }
                if (fmt == 1) acc = acc * inv;
                if (partial) partial[((size_t)c * M + m) * N + n] = acc;
                tot = tot + acc;                                   /* reduce.comp:11, c ascending */
            }
            if (y) y[(size_t)m * N + n] = tot;
        }
    }
}

/* vk/reduce.comp:8-12: y[n] = sum_{c=0}^{split-1} partial[c*N + n], c ascending. */
void orc_reduce(const float* partial, float* y, int N, int split) {
    for (int n = 0; n < N; n++) {
        float s = 0.0f;
        for (int c = 0; c < split; c++) s = s + partial[(size_t)c * N + n];
        y[n] = s;
    }
}

/* vk/coopgemm_i4h.comp:19-25: Wdeq[k, n] = f16((q - 8) * f32(f16 scale[k/32, n])).
 * fmt 1 (e4m3 scales) writes f32 (q - 8) * dec * inv instead (exact), for the
 * GEMV's fp8 weights.  out is [K, N] f16 bits (fmt 0) or f32 (fmt 1). */
void orc_dequant(const uint32_t* wp, const void* scales, int fmt, float inv, int N, int K, void* out) {
    int nb8 = N / 8;
#pragma omp parallel for schedule(static)
    for (int k = 0; k < K; k++) {
        for (int n = 0; n < N; n++) {
            uint32_t q = (wp[(size_t)k * nb8 + (n >> 3)] >> ((n & 7) * 4)) & 15u;
            float s = scale_at(scales, fmt, N, k / ORC_BLK, n);
            float v = ((float)q - 8.0f) * s;
            if (fmt == 0) ((uint16_t*)out)[(size_t)k * N + n] = orc_f32_to_f16(v);
            else ((float*)out)[(size_t)k * N + n] = v * inv;
        }
    }
}

/* W4A16 prefill GEMM, vk/coopgemm_i4h.comp:13-35: Y[M, N] = X16[M, K] @ Wdeq16[K, N],
 * accumulated in f32 in k order (the f32-accumulate form of vk/coopgemm_i4f.comp:16-32;
 * the i4h shader's own f16 accumulator is strictly less accurate).  X is given
 * as f16 bits [M, K]; Y is f32 [M, N]. */
void orc_gemm_i4(const uint16_t* X16, const uint32_t* wp, const uint16_t* sc16, int M, int N, int K,
                 float* Y) {
    int nb8 = N / 8;
    /* dequantise once: [K, N] f32 holding f16-rounded values */
    float* Wd = (float*)malloc(sizeof(float) * (size_t)K * N);
    float* Xf = (float*)malloc(sizeof(float) * (size_t)M * K);
#pragma omp parallel for schedule(static)
    for (int k = 0; k < K; k++)
        for (int n = 0; n < N; n++) {
            uint32_t q = (wp[(size_t)k * nb8 + (n >> 3)] >> ((n & 7) * 4)) & 15u;
            float s = orc_f16_to_f32(sc16[(size_t)(k / ORC_BLK) * N + n]);
            Wd[(size_t)k * N + n] = orc_f16_to_f32(orc_f32_to_f16(((float)q - 8.0f) * s));
        }
    for (size_t i = 0; i < (size_t)M * K; i++) Xf[i] = orc_f16_to_f32(X16[i]);
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; m++) {
        float* yr = Y + (size_t)m * N;
        for (int n = 0; n < N; n++) yr[n] = 0.0f;
        for (int k = 0; k < K; k++) {
            float a = Xf[(size_t)m * K + k];
            const float* wr = Wd + (size_t)k * N;
            for (int n = 0; n < N; n++) yr[n] = yr[n] + a * wr[n];
        }
    }
    free(Wd); free(Xf);
}

/* vk/cast_i8.comp:11-19, per row m of X [M, K] f32:
 *   amax = max |x| ; s = max(amax / 127, 1e-12) ; inv = 1 / s
 *   q = clamp(roundEven(x * inv), -127, 127) ; sa[m] = s */
void orc_cast_i8(const float* X, int M, int K, int8_t* A8, float* sa) {
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; m++) {
        const float* xr = X + (size_t)m * K;
        float mx = 0.0f;
        for (int i = 0; i < K; i++) { float a = fabsf(xr[i]); if (a > mx) mx = a; }
        float s = mx / 127.0f;
        if (!(s >= 1e-12f)) s = 1e-12f;
        float inv = 1.0f / s;
        sa[m] = s;
        for (int i = 0; i < K; i++) {
            float r = nearbyintf(xr[i] * inv);
            if (r < -127.0f) r = -127.0f;
            if (r > 127.0f) r = 127.0f;
            A8[(size_t)m * K + i] = (int8_t)r;
        }
    }
}

/* vk/coopgemm_w8a8.comp:18-37: C[m, n] = sum_k A8[m, k] * W8[k, n] (exact int32);
 * Y[m, n] = f16((float(C) * sa[m]) * f32(f16 sw[n])).  W8 is [K, N] row-major.
 * C (may be NULL) receives the raw accumulators, Y16 the f16 bits. */
void orc_gemm_w8a8(const int8_t* A8, const int8_t* W8, const float* sa, const uint16_t* sw16,
                   int M, int N, int K, int32_t* C, uint16_t* Y16) {
#pragma omp parallel
    {
        int32_t* acc = (int32_t*)malloc(sizeof(int32_t) * (size_t)N);
#pragma omp for schedule(static)
        for (int m = 0; m < M; m++) {
            for (int n = 0; n < N; n++) acc[n] = 0;
            for (int k = 0; k < K; k++) {
                int32_t a = A8[(size_t)m * K + k];
                const int8_t* wr = W8 + (size_t)k * N;
                for (int n = 0; n < N; n++) acc[n] += a * (int32_t)wr[n];
            }
            for (int n = 0; n < N; n++) {
                if (C) C[(size_t)m * N + n] = acc[n];
                float v = ((float)acc[n] * sa[m]) * orc_f16_to_f32(sw16[n]);
                if (Y16) Y16[(size_t)m * N + n] = orc_f32_to_f16(v);
            }
        }
        free(acc);
    }
}

/* vk/coopgemm_w4a8.comp:28-34: w8[k, n] = clamp(roundEven((q - 8) * f32(f16 ratio[k/32, n])), -127, 127) */
void orc_w4a8_requant(const uint32_t* wp, const uint16_t* ratio16, int N, int K, int8_t* w8) {
    int nb8 = N / 8;
#pragma omp parallel for schedule(static)
    for (int k = 0; k < K; k++)
        for (int n = 0; n < N; n++) {
            uint32_t q = (wp[(size_t)k * nb8 + (n >> 3)] >> ((n & 7) * 4)) & 15u;
            float r = orc_f16_to_f32(ratio16[(size_t)(k / ORC_BLK) * N + n]);
            float v = nearbyintf(((float)q - 8.0f) * r);
            if (v < -127.0f) v = -127.0f;
            if (v > 127.0f) v = 127.0f;
            w8[(size_t)k * N + n] = (int8_t)v;
        }
}

/* vk/coopgemm_w4a8.comp:21-50: requantise (orc_w4a8_requant), then the W8A8 GEMM and epilogue. */
void orc_gemm_w4a8(const int8_t* A8, const uint32_t* wp, const uint16_t* ratio16, const float* sa,
                   const uint16_t* sw16, int M, int N, int K, int32_t* C, uint16_t* Y16) {
    int8_t* w8 = (int8_t*)malloc((size_t)K * N);
    orc_w4a8_requant(wp, ratio16, N, K, w8);
    orc_gemm_w8a8(A8, w8, sa, sw16, M, N, K, C, Y16);
    free(w8);
}

/* The sum of squares as vk/rmsnorm.comp:9-10 and vk/normadd.comp:9-10 form it: 256
 * invocations each add the squares of elements t, t + 256, ... in order, then a
 * shared-memory tree folds the partials (sh[t] += sh[t + st] for st = 128 .. 1). */
static float orc_sumsq_256(const float* x, int D) {
    float sh[256];
    for (int t = 0; t < 256; t++) {
        float s = 0.0f;
        for (int i = t; i < D; i += 256) {
            const float v = x[i];
            s += v * v;
        }
        sh[t] = s;
    }
    for (int st = 128; st > 0; st >>= 1)
        for (int t = 0; t < st; t++) sh[t] += sh[t + st];
    return sh[0];
}

/* vk/rmsnorm.comp:8-12: y[i] = x[i] * inv * w[i], inv = inversesqrt(sum / D + eps). */
void orc_rmsnorm(const float* x, const float* w, float* y, int D, float eps) {
    const float inv = 1.0f / sqrtf(orc_sumsq_256(x, D) / (float)D + eps);
    for (int i = 0; i < D; i++) y[i] = x[i] * inv * w[i];
}

/* vk/normadd.comp:8-12: h[i] = (h[i] + x[i] * inv * w[i]) * sc (in place on h). */
void orc_normadd(const float* x, const float* w, float* h, int D, float sc, float eps) {
    const float inv = 1.0f / sqrtf(orc_sumsq_256(x, D) / (float)D + eps);
    for (int i = 0; i < D; i++) h[i] = (h[i] + x[i] * inv * w[i]) * sc;
}

/* vk/gelumul.comp:7-8: out[i] = 0.5 x (1 + tanh(0.7978845608028654 (x + 0.044715 x^3))) * up[i],
 * with the shader's left-to-right products. */
void orc_gelumul(const float* gate, const float* up, float* out, int n) {
    for (int i = 0; i < n; i++) {
        const float x = gate[i];
        const float g = 0.5f * x * (1.0f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
        out[i] = g * up[i];
    }
}

/* vk/prepkv.comp:14-31: every KV head's k (rmsnorm with knw, then RoPE) and v (rmsnorm without a weight)
 * into the f16 caches [nkv][stride][hd] at slot pos (pos % window for a sliding ring); keqv reads v at koff. */
void orc_attn_prepkv(const float* qkv, const float* knw, const float* cosb, const float* sinb, uint16_t* kc,
                     uint16_t* vc, int nkv, int hd, int koff, int voff, int keqv, int stride, int window, int pos) {
    const int hf = hd / 2, slot = window > 0 ? pos % window : pos;
    float hv[512];
    for (int h = 0; h < nkv; h++) {
        for (int i = 0; i < hd; i++) hv[i] = qkv[koff + h * hd + i];
        const float ik = 1.0f / sqrtf(orc_sumsq_256(hv, hd) / (float)hd + 1e-6f);
        for (int i = 0; i < hd; i++) hv[i] = hv[i] * ik * knw[i];
        for (int i = 0; i < hd; i++) {
            const float rh = i < hf ? -hv[i + hf] : hv[i - hf];
            kc[((size_t)h * stride + slot) * hd + i] = orc_f32_to_f16(hv[i] * cosb[i] + rh * sinb[i]);
        }
        const int vo = keqv ? koff : voff;
        for (int i = 0; i < hd; i++) hv[i] = qkv[vo + h * hd + i];
        const float iv = 1.0f / sqrtf(orc_sumsq_256(hv, hd) / (float)hd + 1e-6f);
        for (int i = 0; i < hd; i++) vc[((size_t)h * stride + slot) * hd + i] = orc_f32_to_f16(hv[i] * iv);
    }
}

/* vk/attn.comp:15-55: per query head, q = RoPE(rmsnorm(q, qnw)), then the online softmax over the keys
 * in tiles of 256 (tile max and sum by the shader's 256-lane tree), acc = acc * corr + sum_j p_j v_j in
 * key order, out = acc / l.  No 1/sqrt(hd) scale. */
void orc_attn_decode(const float* qkv, const float* qnw, const float* cosb, const float* sinb, const uint16_t* kc,
                     const uint16_t* vc, float* out, int nH, int nkv, int hd, int qoff, int stride, int window,
                     int pos) {
    const int grp = nH / nkv, hf = hd / 2;
    const int T = window > 0 ? (pos + 1 < window ? pos + 1 : window) : pos + 1;
#pragma omp parallel for schedule(static)
    for (int h = 0; h < nH; h++) {
        const int kvh = h / grp;
        float qr[512], acc[512], sc[256], red[256];
        for (int i = 0; i < hd; i++) qr[i] = qkv[qoff + h * hd + i];
        const float iq = 1.0f / sqrtf(orc_sumsq_256(qr, hd) / (float)hd + 1e-6f);
        for (int i = 0; i < hd; i++) qr[i] = qr[i] * iq * qnw[i];
        for (int i = 0; i < hd; i++) {
            const float rh = i < hf ? -qr[i + hf] : qr[i - hf];
            acc[i] = qr[i] * cosb[i] + rh * sinb[i];
        }
        for (int i = 0; i < hd; i++) {
            qr[i] = acc[i];
            acc[i] = 0.0f;
        }
        float msh = -1e30f, lsh = 0.0f;
        for (int tile = 0; tile < T; tile += 256) {
            const int tlen = T - tile < 256 ? T - tile : 256;
            for (int j = 0; j < tlen; j++) {
                const uint16_t* k = kc + ((size_t)kvh * stride + tile + j) * hd;
                float d2 = 0.0f;
                for (int i = 0; i < hd; i += 4)
                    d2 += qr[i] * orc_f16_to_f32(k[i]) + qr[i + 1] * orc_f16_to_f32(k[i + 1]) +
                          qr[i + 2] * orc_f16_to_f32(k[i + 2]) + qr[i + 3] * orc_f16_to_f32(k[i + 3]);
                sc[j] = d2;
            }
            float mx = -1e30f;
            for (int j = 0; j < tlen; j++) mx = sc[j] > mx ? sc[j] : mx;
            const float mn = msh > mx ? msh : mx;
            const float corr = expf(msh - mn);
            msh = mn;
            for (int t = 0; t < 256; t++) {
                red[t] = 0.0f;
                if (t < tlen) {
                    sc[t] = expf(sc[t] - mn);
                    red[t] = sc[t];
                }
            }
            for (int st = 128; st > 0; st >>= 1)
                for (int t = 0; t < st; t++) red[t] += red[t + st];
            lsh = lsh * corr + red[0];
            for (int i = 0; i < hd; i++) {
                float a = acc[i] * corr;
                for (int j = 0; j < tlen; j++) a += sc[j] * orc_f16_to_f32(vc[((size_t)kvh * stride + tile + j) * hd + i]);
                acc[i] = a;
            }
        }
        for (int i = 0; i < hd; i++) out[h * hd + i] = acc[i] / lsh;
    }
}

/* vk/pre_prepkv.comp:15-30: token m of a chunk of M at absolute position p0 + m writes its normed,
 * rotated k (row m of kin, at kvh * hd) and normed v into slot (p0 + m) (% window); cosM / sinM rows are
 * the tokens' own angles ([M, hd]).  kin / vin rows are nk = row_stride floats apart. */
void orc_attn_prefill_prepkv(const float* kin, const float* vin, const float* knw, const float* cosM,
                             const float* sinM, uint16_t* kc, uint16_t* vc, int M, int nkv, int hd, int row_stride,
                             int stride, int window, int p0) {
    const int hf = hd / 2;
    float hv[512];
    for (int m = 0; m < M; m++) {
        const int pos = p0 + m, slot = window > 0 ? pos % window : pos;
        const float* cb = cosM + (size_t)m * hd;
        const float* sb = sinM + (size_t)m * hd;
        for (int h = 0; h < nkv; h++) {
            const size_t kb = (size_t)m * row_stride + (size_t)h * hd;
            for (int i = 0; i < hd; i++) hv[i] = kin[kb + i];
            const float ik = 1.0f / sqrtf(orc_sumsq_256(hv, hd) / (float)hd + 1e-6f);
            for (int i = 0; i < hd; i++) hv[i] = hv[i] * ik * knw[i];
            for (int i = 0; i < hd; i++) {
                const float rh = i < hf ? -hv[i + hf] : hv[i - hf];
                kc[((size_t)h * stride + slot) * hd + i] = orc_f32_to_f16(hv[i] * cb[i] + rh * sb[i]);
            }
            for (int i = 0; i < hd; i++) hv[i] = vin[kb + i];
            const float iv = 1.0f / sqrtf(orc_sumsq_256(hv, hd) / (float)hd + 1e-6f);
            for (int i = 0; i < hd; i++) vc[((size_t)h * stride + slot) * hd + i] = orc_f32_to_f16(hv[i] * iv);
        }
    }
}

/* vk/pre_attn.comp:16-53: causal attention of token m (position pos = p0 + m) of a chunk of M, per
 * query head: q = RoPE(rmsnorm(q[m], qnw), cosM[m], sinM[m]); T = pos + 1 (or min(pos + 1, window)); the
 * keys are slots 0..T-1 in tiles of 256; on a sliding ring a slot's absolute position is
 * base - ((base + window - slot) % window) with base = p0 + M - 1 (the chunk's keys are all written
 * first), and keys after pos score -1e30.  The tile's max and sum follow the shader (strided lane sums,
 * 256-lane tree); acc = acc * corr + sum_j p_j v_j in key order; out = acc / l.  q / out rows are
 * row_stride floats apart; head h starts at h * hd. */
void orc_attn_prefill(const float* q, const float* qnw, const float* cosM, const float* sinM, const uint16_t* kc,
                      const uint16_t* vc, float* out, int M, int nH, int nkv, int hd, int row_stride, int stride,
                      int window, int p0) {
    const int grp = nH / nkv, hf = hd / 2;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int m = 0; m < M; m++)
        for (int h = 0; h < nH; h++) {
            const int kvh = h / grp;
            const int pos = p0 + m;
            const int T = window > 0 ? (pos + 1 < window ? pos + 1 : window) : pos + 1;
            const float* cb = cosM + (size_t)m * hd;
            const float* sb = sinM + (size_t)m * hd;
            float qr[512], acc[512], sc[256], red[256];
            const size_t qb = (size_t)m * row_stride + (size_t)h * hd;
            for (int i = 0; i < hd; i++) qr[i] = q[qb + i];
            const float iq = 1.0f / sqrtf(orc_sumsq_256(qr, hd) / (float)hd + 1e-6f);
            for (int i = 0; i < hd; i++) qr[i] = qr[i] * iq * qnw[i];
            for (int i = 0; i < hd; i++) {
                const float rh = i < hf ? -qr[i + hf] : qr[i - hf];
                acc[i] = qr[i] * cb[i] + rh * sb[i];
            }
            for (int i = 0; i < hd; i++) {
                qr[i] = acc[i];
                acc[i] = 0.0f;
            }
            float msh = -1e30f, lsh = 0.0f;
            for (int tile = 0; tile < T; tile += 256) {
                const int tlen = T - tile < 256 ? T - tile : 256;
                for (int j = 0; j < tlen; j++) {
                    const int slot = tile + j;
                    const uint16_t* k = kc + ((size_t)kvh * stride + slot) * hd;
                    float d2 = 0.0f;
                    for (int i = 0; i < hd; i += 4)
                        d2 += qr[i] * orc_f16_to_f32(k[i]) + qr[i + 1] * orc_f16_to_f32(k[i + 1]) +
                              qr[i + 2] * orc_f16_to_f32(k[i + 2]) + qr[i + 3] * orc_f16_to_f32(k[i + 3]);
                    if (window > 0) {
                        const long long base = (long long)p0 + M - 1;
                        const long long posn = base - ((base + window - slot) % window);
                        if (posn > pos) d2 = -1e30f;
                    }
                    sc[j] = d2;
                }
                float mx = -1e30f;
                for (int j = 0; j < tlen; j++) mx = sc[j] > mx ? sc[j] : mx;
                const float mn = msh > mx ? msh : mx;
                const float corr = expf(msh - mn);
                msh = mn;
                for (int t = 0; t < 256; t++) {
                    red[t] = 0.0f;
                    if (t < tlen) {
                        sc[t] = expf(sc[t] - mn);
                        red[t] = sc[t];
                    }
                }
                for (int st = 128; st > 0; st >>= 1)
                    for (int t = 0; t < st; t++) red[t] += red[t + st];
                lsh = lsh * corr + red[0];
                for (int i = 0; i < hd; i++) {
                    float a = acc[i] * corr;
                    for (int j = 0; j < tlen; j++)
                        a += sc[j] * orc_f16_to_f32(vc[((size_t)kvh * stride + tile + j) * hd + i]);
                    acc[i] = a;
                }
            }
            for (int i = 0; i < hd; i++) out[qb + i] = acc[i] / lsh;
        }
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
