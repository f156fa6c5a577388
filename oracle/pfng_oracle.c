/*
 * pfng_oracle.c -- CPU restatement of perf-framework-ng's scalar ggml path.
 *
 * TEST INFRASTRUCTURE ONLY (see pfng_oracle.h).  Compiled with
 * -ffp-contract=off and without fast-math so that every fp32 operation rounds
 * exactly as in the reference (bench/llama_reference/llama_reference.cpp).
 * Expressions keep the reference's association order; comments cite the
 * line each one restates.
 */
#include "pfng_oracle.h"

#include <math.h>
#include <string.h>

#include "iq2xxs_grid_codes.h"

/* ------------------------------------------------------------------------ */
/* fp16 codec (include/ggml.h:83-117).  The reference uses the FP16-library   */
/* bit trick; both directions are exact IEEE conversions (fp16->fp32 exact,   */
/* fp32->fp16 round-to-nearest-even), restated here with integer arithmetic. */
/* NaN maps to 0x7E00 | sign as in ggml.h:116.                                */
/* ------------------------------------------------------------------------ */

static float bits_to_float(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t float_to_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

float oracle_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exponent = (h >> 10) & 0x1fu;
    const uint32_t mantissa = h & 0x3ffu;
    if (exponent == 0x1f) {
        /* inf, or NaN (quietened, as an fp32 multiply in ggml.h:89 would). */
        return bits_to_float(sign | 0x7f800000u | (mantissa << 13) | (mantissa ? 0x00400000u : 0u));
    }
    if (exponent != 0) return bits_to_float(sign | ((exponent + 112u) << 23) | (mantissa << 13));
    /* zero or subnormal: mantissa * 2^-24, exact in fp32 */
    const float magnitude = (float)mantissa * 0x1.0p-24f;
    return bits_to_float(sign | float_to_bits(magnitude));
}

uint16_t oracle_fp32_to_fp16(float f) {
    const uint32_t x = float_to_bits(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);  /* NaN */
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 -> inf */
    if (ax >= 0x38800000u) {                                   /* fp16 normal */
        uint32_t h = ((((ax >> 23) - 112u) << 10) | ((ax & 0x7fffffu) >> 13));
        const uint32_t rest = ax & 0x1fffu;
        if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) ++h;
        return (uint16_t)(sign | h);
    }
    if (ax < 0x33000000u) return (uint16_t)sign; /* below 2^-25 (ties to even 0) */
    /* fp16 subnormal: value in units of 2^-24 is M * 2^(E-126), E <= 112 */
    const uint32_t e = ax >> 23;
    const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
    const uint32_t shift = 126u - e;
    uint32_t h = m >> shift;
    const uint32_t rest = m & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1u);
    if (rest > half || (rest == half && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
}

/* ------------------------------------------------------------------------ */
/* Quantizers                                                                */
/* ------------------------------------------------------------------------ */

/* llama_reference.cpp:13-36 */
void oracle_quantize_row_q4_0(const float *x, oracle_block_q4_0 *y, size_t k) {
    for (size_t b = 0; b < k / ORACLE_QK4_0; ++b) {
        const float *v = x + b * ORACLE_QK4_0;
        float absolute_max = 0.0f;
        float signed_max = 0.0f;
        for (size_t i = 0; i < ORACLE_QK4_0; ++i) {
            if (absolute_max < fabsf(v[i])) {
                absolute_max = fabsf(v[i]);
                signed_max = v[i];
            }
        }
        const float scale = signed_max / -8.0f;
        const float inverse_scale = scale != 0.0f ? 1.0f / scale : 0.0f;
        y[b].d = oracle_fp32_to_fp16(scale);
        for (size_t i = 0; i < ORACLE_QK4_0 / 2; ++i) {
            const float low = v[i] * inverse_scale;
            const float high = v[ORACLE_QK4_0 / 2 + i] * inverse_scale;
            int ql = (int8_t)(low + 8.5f);
            int qh = (int8_t)(high + 8.5f);
            if (ql > 15) ql = 15;
            if (qh > 15) qh = 15;
            y[b].qs[i] = (uint8_t)((uint8_t)ql | (uint8_t)(qh << 4));
        }
    }
}

/* llama_reference.cpp:38-52 (std::max(a, b) == (a < b) ? b : a) */
void oracle_quantize_row_q8_0(const float *x, oracle_block_q8_0 *y, size_t k) {
    for (size_t b = 0; b < k / ORACLE_QK8_0; ++b) {
        const float *v = x + b * ORACLE_QK8_0;
        float absolute_max = 0.0f;
        for (size_t i = 0; i < ORACLE_QK8_0; ++i) {
            const float a = fabsf(v[i]);
            absolute_max = absolute_max < a ? a : absolute_max;
        }
        const float scale = absolute_max / 127.0f;
        const float inverse_scale = scale != 0.0f ? 1.0f / scale : 0.0f;
        y[b].d = oracle_fp32_to_fp16(scale);
        for (size_t i = 0; i < ORACLE_QK8_0; ++i) y[b].qs[i] = (int8_t)roundf(v[i] * inverse_scale);
    }
}

/* llama_reference.cpp:54-70 */
void oracle_quantize_row_q8_K(const float *x, oracle_block_q8_K *y, size_t k) {
    for (size_t b = 0; b < k / ORACLE_QK_K; ++b) {
        const float *v = x + b * ORACLE_QK_K;
        float amax = 0.0f;
        for (size_t i = 0; i < ORACLE_QK_K; ++i) {
            const float a = fabsf(v[i]);
            amax = amax < a ? a : amax;
        }
        y[b].d = amax / 127.0f;
        const float inv = y[b].d != 0.0f ? 1.0f / y[b].d : 0.0f;
        for (size_t i = 0; i < ORACLE_QK_K; ++i) y[b].qs[i] = (int8_t)roundf(v[i] * inv);
        for (size_t i = 0; i < ORACLE_QK_K / 16; ++i) {
            y[b].bsums[i] = 0;
            for (size_t j = 0; j < 16; ++j) y[b].bsums[i] = (int16_t)(y[b].bsums[i] + y[b].qs[i * 16 + j]);
        }
    }
}

static int clamp_int(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* llama_reference.cpp:72-111 (std::min(a, b) == (b < a) ? b : a) */
void oracle_quantize_row_q4_K(const float *x, oracle_block_q4_K *y, size_t k) {
    for (size_t b = 0; b < k / ORACLE_QK_K; ++b) {
        const float *v = x + b * ORACLE_QK_K;
        oracle_block_q4_K *o = &y[b];
        float ls[8], lm[8], maxs = 0.0f, maxm = 0.0f;
        for (size_t sb = 0; sb < 8; ++sb) {
            float lo = v[sb * 32], hi = lo;
            for (size_t j = 1; j < 32; ++j) {
                const float t = v[sb * 32 + j];
                lo = t < lo ? t : lo;
                hi = hi < t ? t : hi;
            }
            ls[sb] = (hi - lo) / 15.0f;
            lm[sb] = -lo / (ls[sb] != 0.0f ? ls[sb] : 1.0f);
            maxs = maxs < ls[sb] ? ls[sb] : maxs;
            maxm = maxm < lm[sb] ? lm[sb] : maxm;
        }
        const float ds = maxs / 63.0f, dm = maxm / 63.0f;
        o->d = oracle_fp32_to_fp16(ds);
        o->dmin = oracle_fp32_to_fp16(dm);
        uint8_t s[8], m[8];
        for (size_t i = 0; i < 8; ++i) {
            const int si = (int)roundf(ls[i] / (ds != 0.0f ? ds : 1.0f));
            const int mi = (int)roundf(lm[i] / (dm != 0.0f ? dm : 1.0f));
            s[i] = (uint8_t)(si < 63 ? si : 63);
            m[i] = (uint8_t)(mi < 63 ? mi : 63);
        }
        for (size_t i = 0; i < 4; ++i) {
            o->scales[i] = (uint8_t)(s[i] | ((s[i + 4] & 3) << 6));
            o->scales[i + 4] = (uint8_t)(m[i] | ((m[i + 4] & 3) << 6));
            o->scales[i + 8] = (uint8_t)((s[i + 4] >> 2) | ((m[i + 4] >> 2) << 4));
        }
        for (size_t pair = 0; pair < 4; ++pair) {
            const size_t lo_sb = pair * 2, hi_sb = lo_sb + 1;
            for (size_t j = 0; j < 32; ++j) {
                const int low = clamp_int(
                    (int)roundf(v[lo_sb * 32 + j] / (ls[lo_sb] != 0.0f ? ls[lo_sb] : 1.0f) + lm[lo_sb]), 0, 15);
                const int high = clamp_int(
                    (int)roundf(v[hi_sb * 32 + j] / (ls[hi_sb] != 0.0f ? ls[hi_sb] : 1.0f) + lm[hi_sb]), 0, 15);
                o->qs[pair * 32 + j] = (uint8_t)(low | (high << 4));
            }
        }
    }
}

void oracle_quantize_q4_0(const float *x, void *y, size_t m, size_t k) {
    for (size_t r = 0; r < m; ++r)
        oracle_quantize_row_q4_0(x + r * k, (oracle_block_q4_0 *)y + r * (k / ORACLE_QK4_0), k);
}
void oracle_quantize_q8_0(const float *x, void *y, size_t m, size_t k) {
    for (size_t r = 0; r < m; ++r)
        oracle_quantize_row_q8_0(x + r * k, (oracle_block_q8_0 *)y + r * (k / ORACLE_QK8_0), k);
}
void oracle_quantize_q8_K(const float *x, void *y, size_t m, size_t k) {
    for (size_t r = 0; r < m; ++r)
        oracle_quantize_row_q8_K(x + r * k, (oracle_block_q8_K *)y + r * (k / ORACLE_QK_K), k);
}
void oracle_quantize_q4_K(const float *x, void *y, size_t m, size_t k) {
    for (size_t r = 0; r < m; ++r)
        oracle_quantize_row_q4_K(x + r * k, (oracle_block_q4_K *)y + r * (k / ORACLE_QK_K), k);
}

/* ------------------------------------------------------------------------ */
/* iq2_xxs decode (kernels/common/iq2_xxs.h:25-41) with the full grid.       */
/* ------------------------------------------------------------------------ */

uint64_t oracle_iq2_xxs_grid(unsigned index) {
    const uint16_t code = oracle_iq2xxs_grid_codes[index & 255u];
    static const uint8_t magnitude[3] = {0x08, 0x19, 0x2b};
    uint64_t point = 0;
    for (unsigned j = 0; j < 8; ++j) point |= (uint64_t)magnitude[(code >> (2 * j)) & 3u] << (8 * j);
    return point;
}

uint8_t oracle_iq2_xxs_sign_mask(unsigned index7) {
    const unsigned i = index7 & 0x7fu;
    return (uint8_t)(i | ((unsigned)__builtin_parity(i) << 7));
}

void oracle_iq2_xxs_decode_group(const uint8_t *packed, int8_t *values, int *scale) {
    uint32_t signs_and_scale;
    memcpy(&signs_and_scale, packed + 4, 4);
    for (unsigned group = 0; group < 4; ++group) {
        const uint64_t magnitudes = oracle_iq2_xxs_grid(packed[group]);
        const uint8_t signs = oracle_iq2_xxs_sign_mask((signs_and_scale >> (7 * group)) & 0x7fu);
        for (unsigned lane = 0; lane < 8; ++lane) {
            const int8_t mag = (int8_t)((magnitudes >> (lane * 8)) & 0xff);
            values[group * 8 + lane] = (signs & (1u << lane)) ? (int8_t)-mag : mag;
        }
    }
    *scale = 2 * (int)((signs_and_scale >> 28) & 0x0fu) + 1;
}

/* ------------------------------------------------------------------------ */
/* Dot products                                                              */
/* ------------------------------------------------------------------------ */

static int32_t isum_q4_0(const oracle_block_q4_0 *w, const oracle_block_q8_0 *a) {
    int32_t s = 0;
    for (size_t i = 0; i < ORACLE_QK4_0 / 2; ++i) {
        s += ((int)(w->qs[i] & 0x0f) - 8) * a->qs[i];
        s += ((int)(w->qs[i] >> 4) - 8) * a->qs[i + ORACLE_QK4_0 / 2];
    }
    return s;
}

/* llama_reference.cpp:134-146 */
float oracle_dot_q4_0_q8_0(const oracle_block_q4_0 *w, const oracle_block_q8_0 *a, size_t nblocks) {
    float sum = 0.0f;
    for (size_t b = 0; b < nblocks; ++b) {
        const int32_t integer_sum = isum_q4_0(&w[b], &a[b]);
        sum += integer_sum * oracle_fp16_to_fp32(w[b].d) * oracle_fp16_to_fp32(a[b].d);
    }
    return sum;
}

static void unpack_q4_K_scales(const oracle_block_q4_K *w, uint8_t *scales, uint8_t *mins) {
    /* llama_reference.cpp:116-121 */
    for (size_t i = 0; i < 4; ++i) {
        scales[i] = w->scales[i] & 63;
        scales[i + 4] = (uint8_t)((w->scales[i + 8] & 15) | ((w->scales[i] >> 6) << 4));
        mins[i] = w->scales[i + 4] & 63;
        mins[i + 4] = (uint8_t)((w->scales[i + 8] >> 4) | ((w->scales[i + 4] >> 6) << 4));
    }
}

static int q4_K_nibble(const oracle_block_q4_K *w, size_t sb, size_t j) {
    const uint8_t packed = w->qs[(sb / 2) * 32 + j];
    return sb % 2 == 0 ? (packed & 15) : (packed >> 4);
}

/* llama_reference.cpp:113-132 */
float oracle_dot_q4_K_q8_K(const oracle_block_q4_K *w, const oracle_block_q8_K *a) {
    uint8_t scales[8], mins[8];
    unpack_q4_K_scales(w, scales, mins);
    const float d = oracle_fp16_to_fp32(w->d);
    const float dmin = oracle_fp16_to_fp32(w->dmin);
    float sum = 0.0f;
    for (size_t sb = 0; sb < 8; ++sb)
        for (size_t j = 0; j < 32; ++j) {
            const int q = q4_K_nibble(w, sb, j);
            sum += a->qs[sb * 32 + j] * (d * scales[sb] * q - dmin * mins[sb]);
        }
    return a->d * sum;
}

/* llama_reference.cpp:148-161 */
float oracle_dot_iq2_xxs_q8_K(const oracle_block_iq2_xxs *w, const oracle_block_q8_K *a) {
    const uint8_t *packed = (const uint8_t *)w->qs;
    int32_t sum = 0;
    for (size_t sb = 0; sb < ORACLE_QK_K / 32; ++sb) {
        int8_t values[32];
        int scale;
        oracle_iq2_xxs_decode_group(packed + sb * 8, values, &scale);
        int32_t subblock_sum = 0;
        for (size_t i = 0; i < 32; ++i) subblock_sum += values[i] * a->qs[sb * 32 + i];
        sum += scale * subblock_sum;
    }
    return 0.125f * oracle_fp16_to_fp32(w->d) * a->d * sum;
}

/* ------------------------------------------------------------------------ */
/* Matrix products (llama_reference.cpp:165-205).  Rows of C are independent */
/* and each element is computed exactly as the reference does, so the outer */
/* loop may run on several threads without changing a single bit.           */
/* ------------------------------------------------------------------------ */

void oracle_mm_q4_0_q8_0(const void *w, const void *a, float *c, size_t m, size_t n, size_t k, size_t ldc) {
    const size_t nb = k / ORACLE_QK4_0;
    const oracle_block_q4_0 *W = (const oracle_block_q4_0 *)w;
    const oracle_block_q8_0 *A = (const oracle_block_q8_0 *)a;
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)m; ++i)
        for (size_t j = 0; j < n; ++j) c[i * ldc + j] = oracle_dot_q4_0_q8_0(W + j * nb, A + i * nb, nb);
}

void oracle_mm_q4_K_q8_K(const void *w, const void *a, float *c, size_t m, size_t n, size_t k, size_t ldc) {
    const size_t nb = k / ORACLE_QK_K;
    const oracle_block_q4_K *W = (const oracle_block_q4_K *)w;
    const oracle_block_q8_K *A = (const oracle_block_q8_K *)a;
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)m; ++i)
        for (size_t j = 0; j < n; ++j) {
            float acc = 0.0f;
            for (size_t b = 0; b < nb; ++b) acc += oracle_dot_q4_K_q8_K(&W[j * nb + b], &A[i * nb + b]);
            c[i * ldc + j] = acc;
        }
}

void oracle_mm_iq2_xxs_q8_K(const void *w, const void *a, float *c, size_t m, size_t n, size_t k, size_t ldc) {
    const size_t nb = k / ORACLE_QK_K;
    const oracle_block_iq2_xxs *W = (const oracle_block_iq2_xxs *)w;
    const oracle_block_q8_K *A = (const oracle_block_q8_K *)a;
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)m; ++i)
        for (size_t j = 0; j < n; ++j) {
            float acc = 0.0f;
            for (size_t b = 0; b < nb; ++b) acc += oracle_dot_iq2_xxs_q8_K(&W[j * nb + b], &A[i * nb + b]);
            c[i * ldc + j] = acc;
        }
}

#include <stdlib.h>

void oracle_compute_q4_0(const void *w, const float *x, float *c, size_t m, size_t n, size_t k) {
    void *a = malloc(m * (k / ORACLE_QK8_0) * sizeof(oracle_block_q8_0) + 1);
    oracle_quantize_q8_0(x, a, m, k);
    oracle_mm_q4_0_q8_0(w, a, c, m, n, k, n);
    free(a);
}

void oracle_compute_q4_K(const void *w, const float *x, float *c, size_t m, size_t n, size_t k) {
    void *a = malloc(m * (k / ORACLE_QK_K) * sizeof(oracle_block_q8_K) + 1);
    oracle_quantize_q8_K(x, a, m, k);
    oracle_mm_q4_K_q8_K(w, a, c, m, n, k, n);
    free(a);
}

void oracle_compute_iq2_xxs(const void *w, const float *x, float *c, size_t m, size_t n, size_t k) {
    void *a = malloc(m * (k / ORACLE_QK_K) * sizeof(oracle_block_q8_K) + 1);
    oracle_quantize_q8_K(x, a, m, k);
    oracle_mm_iq2_xxs_q8_K(w, a, c, m, n, k, n);
    free(a);
}

/* ------------------------------------------------------------------------ */
/* Integer partials and error scales                                         */
/* ------------------------------------------------------------------------ */

void oracle_partials_q4_0_q8_0(const void *w, const void *a, int32_t *out, size_t m, size_t n, size_t k) {
    const size_t nb = k / ORACLE_QK4_0;
    const oracle_block_q4_0 *W = (const oracle_block_q4_0 *)w;
    const oracle_block_q8_0 *A = (const oracle_block_q8_0 *)a;
    for (size_t i = 0; i < m; ++i)
        for (size_t j = 0; j < n; ++j)
            for (size_t b = 0; b < nb; ++b) out[(i * n + j) * nb + b] = isum_q4_0(&W[j * nb + b], &A[i * nb + b]);
}

void oracle_partials_q4_K_q8_K(const void *w, const void *a, int32_t *out, size_t m, size_t n, size_t k) {
    const size_t nb = k / ORACLE_QK_K;
    const oracle_block_q4_K *W = (const oracle_block_q4_K *)w;
    const oracle_block_q8_K *A = (const oracle_block_q8_K *)a;
    for (size_t i = 0; i < m; ++i)
        for (size_t j = 0; j < n; ++j)
            for (size_t b = 0; b < nb; ++b)
                for (size_t sb = 0; sb < 8; ++sb) {
                    int32_t s = 0;
                    for (size_t t = 0; t < 32; ++t)
                        s += A[i * nb + b].qs[sb * 32 + t] * q4_K_nibble(&W[j * nb + b], sb, t);
                    out[((i * n + j) * nb + b) * 8 + sb] = s;
                }
}

void oracle_partials_iq2_xxs_q8_K(const void *w, const void *a, int32_t *out, size_t m, size_t n, size_t k) {
    const size_t nb = k / ORACLE_QK_K;
    const oracle_block_iq2_xxs *W = (const oracle_block_iq2_xxs *)w;
    const oracle_block_q8_K *A = (const oracle_block_q8_K *)a;
    for (size_t i = 0; i < m; ++i)
        for (size_t j = 0; j < n; ++j)
            for (size_t b = 0; b < nb; ++b) {
                const uint8_t *packed = (const uint8_t *)W[j * nb + b].qs;
                for (size_t sb = 0; sb < 8; ++sb) {
                    int8_t values[32];
                    int scale;
                    oracle_iq2_xxs_decode_group(packed + sb * 8, values, &scale);
                    int32_t s = 0;
                    for (size_t t = 0; t < 32; ++t) s += values[t] * A[i * nb + b].qs[sb * 32 + t];
                    out[((i * n + j) * nb + b) * 8 + sb] = s;
                }
            }
}

void oracle_bound_q4_0_q8_0(const void *w, const void *a, double *out, size_t m, size_t n, size_t k) {
    const size_t nb = k / ORACLE_QK4_0;
    const oracle_block_q4_0 *W = (const oracle_block_q4_0 *)w;
    const oracle_block_q8_0 *A = (const oracle_block_q8_0 *)a;
    for (size_t i = 0; i < m; ++i)
        for (size_t j = 0; j < n; ++j) {
            double total = 0.0;
            for (size_t b = 0; b < nb; ++b) {
                const oracle_block_q4_0 *wb = &W[j * nb + b];
                const oracle_block_q8_0 *ab = &A[i * nb + b];
                long s = 0;
                for (size_t t = 0; t < 16; ++t) {
                    s += labs((long)((wb->qs[t] & 15) - 8) * ab->qs[t]);
                    s += labs((long)((wb->qs[t] >> 4) - 8) * ab->qs[t + 16]);
                }
                total += (double)s * fabs((double)oracle_fp16_to_fp32(wb->d) * oracle_fp16_to_fp32(ab->d));
            }
            out[i * n + j] = total;
        }
}

void oracle_bound_q4_K_q8_K(const void *w, const void *a, double *out, size_t m, size_t n, size_t k) {
    const size_t nb = k / ORACLE_QK_K;
    const oracle_block_q4_K *W = (const oracle_block_q4_K *)w;
    const oracle_block_q8_K *A = (const oracle_block_q8_K *)a;
    for (size_t i = 0; i < m; ++i)
        for (size_t j = 0; j < n; ++j) {
            double total = 0.0;
            for (size_t b = 0; b < nb; ++b) {
                const oracle_block_q4_K *wb = &W[j * nb + b];
                const oracle_block_q8_K *ab = &A[i * nb + b];
                uint8_t scales[8], mins[8];
                unpack_q4_K_scales(wb, scales, mins);
                const double d = oracle_fp16_to_fp32(wb->d), dmin = oracle_fp16_to_fp32(wb->dmin);
                for (size_t sb = 0; sb < 8; ++sb)
                    for (size_t t = 0; t < 32; ++t) {
                        const double wv = d * scales[sb] * q4_K_nibble(wb, sb, t) - dmin * mins[sb];
                        total += fabs(wv) * fabs((double)ab->d * ab->qs[sb * 32 + t]);
                    }
            }
            out[i * n + j] = total;
        }
}

void oracle_bound_iq2_xxs_q8_K(const void *w, const void *a, double *out, size_t m, size_t n, size_t k) {
    const size_t nb = k / ORACLE_QK_K;
    const oracle_block_iq2_xxs *W = (const oracle_block_iq2_xxs *)w;
    const oracle_block_q8_K *A = (const oracle_block_q8_K *)a;
    for (size_t i = 0; i < m; ++i)
        for (size_t j = 0; j < n; ++j) {
            double total = 0.0;
            for (size_t b = 0; b < nb; ++b) {
                const uint8_t *packed = (const uint8_t *)W[j * nb + b].qs;
                const oracle_block_q8_K *ab = &A[i * nb + b];
                const double d = 0.125 * oracle_fp16_to_fp32(W[j * nb + b].d);
                for (size_t sb = 0; sb < 8; ++sb) {
                    int8_t values[32];
                    int scale;
                    oracle_iq2_xxs_decode_group(packed + sb * 8, values, &scale);
                    long s = 0;
                    for (size_t t = 0; t < 32; ++t) s += labs((long)values[t] * ab->qs[sb * 32 + t]);
                    total += fabs(d * scale * ab->d) * (double)s;
                }
            }
            out[i * n + j] = total;
        }
}

/* ---- q4_0 planar row layout (a permutation of each row's bytes) ---------- */
void oracle_pack_q4_0_planar(const void *w, void *w_planar, size_t n, size_t k) {
    const size_t nb = k / ORACLE_QK4_0, rb = nb * sizeof(oracle_block_q4_0);
    for (size_t row = 0; row < n; ++row) {
        const oracle_block_q4_0 *src = (const oracle_block_q4_0 *)((const uint8_t *)w + row * rb);
        uint8_t *dst = (uint8_t *)w_planar + row * rb;
        for (size_t j = 0; j < nb; ++j) {
            memcpy(dst + 16 * j, src[j].qs, 16);
            memcpy(dst + 16 * nb + 2 * j, &src[j].d, 2);
        }
    }
}

void oracle_unpack_q4_0_planar(const void *w_planar, void *w, size_t n, size_t k) {
    const size_t nb = k / ORACLE_QK4_0, rb = nb * sizeof(oracle_block_q4_0);
    for (size_t row = 0; row < n; ++row) {
        const uint8_t *src = (const uint8_t *)w_planar + row * rb;
        oracle_block_q4_0 *dst = (oracle_block_q4_0 *)((uint8_t *)w + row * rb);
        for (size_t j = 0; j < nb; ++j) {
            memcpy(dst[j].qs, src + 16 * j, 16);
            memcpy(&dst[j].d, src + 16 * nb + 2 * j, 2);
        }
    }
}
