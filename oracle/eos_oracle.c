/*
 * oracle/eos_oracle.c -- CPU restatement of eosllm's quantized matmul path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product): see
 * eos_oracle.h.  Each function cites the reference file:line it restates.
 * Compile: gcc -std=c99 -O2 -ffp-contract=off (no FMA contraction, like the
 * reference's ISO-C99 build); the explicit fmaf() calls below stand for the
 * reference's explicit _mm256_fmadd_ps / _mm256_fmsub_ps.
 */
#define _POSIX_C_SOURCE 200809L
#include "eos_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ------------------------------------------------------------------ */
/* binary16 <-> binary32: restates src/util/f16.h:17-82                */
/* ------------------------------------------------------------------ */

/* Summation-order switch (orc_set_sum_order): 0 is the reference's order
 * everywhere; the other bits exist only to measure how far the reference's
 * algorithm itself moves under a rounding-level reordering of its sums. */
static int g_orc_sum_order = 0;

float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)(h & 0x8000u)) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t mant = h & 0x3FFu;
    uint32_t bits;
    float f;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            /* subnormal half: normalise the mantissa (f16.h:28-35) */
            uint32_t e = 113u; /* 127 - 14 */
            while ((mant & 0x400u) == 0) { mant <<= 1; e--; }
            bits = sign | (e << 23) | ((mant & 0x3FFu) << 13);
        }
    } else if (exp == 0x1Fu) {
        bits = sign | 0x7F800000u | (mant << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (mant << 13);
    }
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t orc_f32_to_f16(float f) {
    /* Same rounding as the reference encoder (f16.h:49-82): add the first
     * dropped bit (round half up in magnitude), flush f32 subnormals. */
    uint32_t bits, sign, exp, mant;
    int32_t e;
    memcpy(&bits, &f, 4);
    sign = (bits >> 16) & 0x8000u;
    exp = (bits >> 23) & 0xFFu;
    mant = bits & 0x7FFFFFu;
    if (exp == 0xFFu) return (uint16_t)(sign | 0x7C00u | (mant ? ((mant >> 13) | 0x200u) : 0u));
    if (exp == 0) return (uint16_t)sign;
    e = (int32_t)exp - 112;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        uint32_t sh;
        if (e < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        sh = (uint32_t)(14 - e);
        return (uint16_t)(sign | ((mant >> sh) + ((mant >> (sh - 1)) & 1u)));
    }
    return (uint16_t)(sign | ((((uint32_t)e << 10) | (mant >> 13)) + ((mant >> 12) & 1u)));
}

/* ------------------------------------------------------------------ */
/* Q4_K scale/min packing                                              */
/* ------------------------------------------------------------------ */

void orc_get_scale_min(int j, const uint8_t *q, uint8_t *sc, uint8_t *m) {
    /* src/kernels/avx2/matmul_q4_k_int8.c:58-67 (same at
     * src/kernels/scalar/matmul_q4_k.c:32-41, src/quant/q4_k.c:31-40) */
    if (j < 4) {
        *sc = (uint8_t)(q[j] & 63u);
        *m = (uint8_t)(q[j + 4] & 63u);
    } else {
        *sc = (uint8_t)((q[j + 4] & 15u) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

void orc_unpack_scale_min_batch(const uint8_t *q, size_t count, uint8_t *sc, uint8_t *m) {
    size_t i;
    int j;
    for (i = 0; i < count; ++i)
        for (j = 0; j < 8; ++j) orc_get_scale_min(j, q + 12 * i, &sc[8 * i + (size_t)j], &m[8 * i + (size_t)j]);
}

void orc_pack_q4k_scales(const uint8_t sc[8], const uint8_t m[8], uint8_t out[12]) {
    /* tests/unit/test_runner.c:716-725: low 6 bits of entries 0..3 in bytes
     * 0..7, entries 4..7 split into a low nibble (bytes 8..11) and two high
     * bits (top of bytes 0..7). */
    int j;
    for (j = 0; j < 4; ++j) {
        out[j] = (uint8_t)((sc[j] & 63u) | ((sc[j + 4] >> 4) << 6));
        out[j + 4] = (uint8_t)((m[j] & 63u) | ((m[j + 4] >> 4) << 6));
        out[j + 8] = (uint8_t)((sc[j + 4] & 15u) | ((m[j + 4] & 15u) << 4));
    }
}

/* ------------------------------------------------------------------ */
/* Activation packing: restates quantize_sub32,                        */
/* src/kernels/avx2/matmul_q4_k_int8.c:98-154                          */
/* ------------------------------------------------------------------ */

/* MAXPS/MAXSS: the first operand if it is greater, else the second --
 * so a NaN in either operand yields the second operand. */
static float x86_max(float a, float b) { return a > b ? a : b; }

/* CVTPS2DQ under the default MXCSR (round to nearest even); NaN and
 * out-of-range inputs give the "integer indefinite" 0x80000000. */
static int32_t x86_cvtps(float x) {
    if (x != x) return INT32_MIN;
    if (x >= 2147483648.0f || x < -2147483648.0f) return INT32_MIN;
    return (int32_t)rintf(x);
}

void orc_quantize_sub32(const float *aa, int8_t *aq, float *out_scale, int32_t *out_sum) {
    float ma[32], mx[8], m4[4], m2a, m2b, max_abs, scale, inv;
    uint32_t sum = 0;
    int i;
    for (i = 0; i < 32; ++i) {
        uint32_t b;
        memcpy(&b, &aa[i], 4);
        b &= 0x7FFFFFFFu; /* _mm256_and_ps with abs_mask (:103,108-111) */
        memcpy(&ma[i], &b, 4);
    }
    /* mx = max(max(ma0, ma1), max(ma2, ma3)) lane-wise (:112-113) */
    for (i = 0; i < 8; ++i)
        mx[i] = x86_max(x86_max(ma[i], ma[8 + i]), x86_max(ma[16 + i], ma[24 + i]));
    /* hmax_ps_8 (:84-94): halves, movehl, shuffle lane 1, max_ss */
    for (i = 0; i < 4; ++i) m4[i] = x86_max(mx[i], mx[i + 4]);
    m2a = x86_max(m4[0], m4[2]);
    m2b = x86_max(m4[1], m4[3]);
    max_abs = x86_max(m2a, m2b);

    if (max_abs > 0.0f) { /* :117-123 */
        scale = max_abs / 127.0f;
        inv = 127.0f / max_abs;
    } else {
        scale = 0.0f;
        inv = 0.0f;
    }
    for (i = 0; i < 32; ++i) {
        int32_t q = x86_cvtps(aa[i] * inv); /* :127-130 */
        sum += (uint32_t)q;                  /* wrapping i32 adds (:136-138) */
        /* packs_epi32 then packs_epi16 saturate: [-128, 127] (:145-149) */
        aq[i] = (int8_t)(q < -128 ? -128 : (q > 127 ? 127 : q));
    }
    *out_scale = scale;
    *out_sum = (int32_t)sum;
}

int orc_quantize_act(const float *a, uint32_t k, int8_t *aq, float *scales, int32_t *sums) {
    uint32_t g;
    if (!a || !aq || !scales || !sums) return ORC_E_INVALID_ARG;
    if (k % 32u) return ORC_E_INVALID_ARG;
    for (g = 0; g < k / 32u; ++g)
        orc_quantize_sub32(a + 32u * g, aq + 32u * g, &scales[g], &sums[g]);
    return ORC_OK;
}

/* ------------------------------------------------------------------ */
/* Q4_K matmuls                                                        */
/* ------------------------------------------------------------------ */

static void q4k_header(const uint8_t *blk, float *d, float *dmin) {
    uint16_t dh, mh;
    memcpy(&dh, blk, 2);
    memcpy(&mh, blk + 2, 2);
    *d = orc_f16_to_f32(dh);
    *dmin = orc_f16_to_f32(mh);
}

int orc_matmul_q4_k_avx2_f32(const float *a, const void *bq, float *c,
                             uint32_t m, uint32_t n, uint32_t k) {
    /* src/kernels/avx2/matmul_q4_k.c:70-153 */
    const uint8_t *bb = (const uint8_t *)bq;
    uint32_t nb, i, j, b;
    if (!a || !bq || !c) return ORC_E_INVALID_ARG;
    if (k % 256u) return ORC_E_INVALID_ARG;
    nb = k / 256u;
    for (i = 0; i < m; ++i) {
        const float *ar = a + (size_t)i * k;
        for (j = 0; j < n; ++j) {
            const uint8_t *br = bb + (size_t)j * nb * 144u;
            float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            float s0, s1, s2, s3;
            for (b = 0; b < nb; ++b, br += 144) {
                const float *aa = ar + (size_t)b * 256u;
                const uint8_t *qs = br + 16;
                float d, dmin;
                int sub, l, t;
                q4k_header(br, &d, &dmin);
                for (sub = 0; sub < 8; sub += 2, qs += 32) {
                    uint8_t sl, ml, sh, mh;
                    float d1, m1, d2, m2;
                    orc_get_scale_min(sub, br + 4, &sl, &ml);
                    orc_get_scale_min(sub + 1, br + 4, &sh, &mh);
                    d1 = d * (float)sl;
                    m1 = dmin * (float)ml;
                    d2 = d * (float)sh;
                    m2 = dmin * (float)mh;
                    for (l = 0; l < 32; l += 8) {
                        for (t = 0; t < 8; ++t) { /* fmsub then fmadd (:126-128) */
                            float w = fmaf(d1, (float)(qs[l + t] & 15u), -m1);
                            acc[t] = fmaf(aa[sub * 32 + l + t], w, acc[t]);
                        }
                        for (t = 0; t < 8; ++t) { /* (:131-133) */
                            float w = fmaf(d2, (float)(qs[l + t] >> 4), -m2);
                            acc[t] = fmaf(aa[(sub + 1) * 32 + l + t], w, acc[t]);
                        }
                    }
                }
            }
            /* SSE horizontal reduce (:139-149) */
            s0 = acc[0] + acc[4];
            s1 = acc[1] + acc[5];
            s2 = acc[2] + acc[6];
            s3 = acc[3] + acc[7];
            c[(size_t)i * n + j] = (s0 + s2) + (s1 + s3);
        }
    }
    return ORC_OK;
}

int orc_matmul_q4_k_int8(const float *a, const void *bq, float *c,
                         uint32_t m, uint32_t n, uint32_t k) {
    /* src/kernels/avx2/matmul_q4_k_int8.c:164-269 */
    const uint8_t *bb = (const uint8_t *)bq;
    uint32_t nb, i, j, b;
    if (!a || !bq || !c) return ORC_E_INVALID_ARG;
    if (k % 256u) return ORC_E_INVALID_ARG;
    if (n < 4) return orc_matmul_q4_k_avx2_f32(a, bq, c, m, n, k); /* :182-184 */
    nb = k / 256u;
    for (i = 0; i < m; ++i) {
        const float *ar = a + (size_t)i * k;
        float *cr = c + (size_t)i * n;
        for (j = 0; j < n; ++j) cr[j] = 0.0f; /* :194 */
        for (b = 0; b < nb; ++b) {
            int8_t aq[256];
            float as[8];
            int32_t sa[8];
            int sub;
            /* order bit 2: super-blocks (and below, sub-blocks) accumulated last to first */
            const uint32_t bo = (g_orc_sum_order & 2) ? nb - 1u - b : b;
            for (sub = 0; sub < 8; ++sub) /* :208-211 */
                orc_quantize_sub32(ar + (size_t)bo * 256u + 32u * sub, aq + 32 * sub, &as[sub], &sa[sub]);
            for (j = 0; j < n; ++j) {
                const uint8_t *br = bb + ((size_t)j * nb + bo) * 144u;
                const uint8_t *qs = br + 16;
                float d, dmin, partial = 0.0f, term[8];
                q4k_header(br, &d, &dmin);
                for (sub = 0; sub < 8; sub += 2, qs += 32) {
                    uint8_t sl, ml, sh, mh;
                    int32_t dl = 0, dh = 0;
                    int l;
                    orc_get_scale_min(sub, br + 4, &sl, &ml);
                    orc_get_scale_min(sub + 1, br + 4, &sh, &mh);
                    for (l = 0; l < 32; ++l) { /* exact u4 x i8 dots (:234-249) */
                        dl += (int32_t)(qs[l] & 15u) * aq[32 * sub + l];
                        dh += (int32_t)(qs[l] >> 4) * aq[32 * (sub + 1) + l];
                    }
                    /* rescale in the reference's evaluation order (:254-261) */
                    term[sub] = d * (float)sl * as[sub] * (float)dl
                              - dmin * (float)ml * as[sub] * (float)sa[sub];
                    term[sub + 1] = d * (float)sh * as[sub + 1] * (float)dh
                                  - dmin * (float)mh * as[sub + 1] * (float)sa[sub + 1];
                }
                /* partial += term, sub-block by sub-block (order bit 2: last to first) */
                for (sub = 0; sub < 8; ++sub) partial += term[(g_orc_sum_order & 2) ? 7 - sub : sub];
                cr[j] += partial; /* :264 */
            }
        }
    }
    return ORC_OK;
}

int orc_matmul_q4_k_scalar(const float *a, const void *bq, float *c,
                           uint32_t m, uint32_t n, uint32_t k) {
    /* src/kernels/scalar/matmul_q4_k.c:43-104 */
    const uint8_t *bb = (const uint8_t *)bq;
    uint32_t nb, i, j, b;
    if (!a || !bq || !c) return ORC_E_INVALID_ARG;
    if (k % 256u) return ORC_E_INVALID_ARG;
    nb = k / 256u;
    for (i = 0; i < m; ++i) {
        const float *ar = a + (size_t)i * k;
        for (j = 0; j < n; ++j) {
            const uint8_t *br = bb + (size_t)j * nb * 144u;
            float acc = 0.0f;
            for (b = 0; b < nb; ++b, br += 144) {
                const float *aa = ar + (size_t)b * 256u;
                const uint8_t *qs = br + 16;
                float d, dmin;
                int sub, l;
                q4k_header(br, &d, &dmin);
                for (sub = 0; sub < 8; sub += 2, qs += 32) {
                    uint8_t sl, ml, sh, mh;
                    float d1, m1, d2, m2;
                    orc_get_scale_min(sub, br + 4, &sl, &ml);
                    orc_get_scale_min(sub + 1, br + 4, &sh, &mh);
                    d1 = d * (float)sl;
                    m1 = dmin * (float)ml;
                    d2 = d * (float)sh;
                    m2 = dmin * (float)mh;
                    for (l = 0; l < 32; ++l) {
                        float w = d1 * (float)(qs[l] & 15u) - m1;
                        acc += aa[sub * 32 + l] * w;
                    }
                    for (l = 0; l < 32; ++l) {
                        float w = d2 * (float)(qs[l] >> 4) - m2;
                        acc += aa[(sub + 1) * 32 + l] * w;
                    }
                }
            }
            c[(size_t)i * n + j] = acc;
        }
    }
    return ORC_OK;
}

/* ------------------------------------------------------------------ */
/* Q8_0 and f32                                                        */
/* ------------------------------------------------------------------ */

int orc_matmul_q8_0(const float *a, const void *bq, float *c,
                    uint32_t m, uint32_t n, uint32_t k) {
    /* src/kernels/scalar/matmul_q8.c:21-58 */
    const uint8_t *bb = (const uint8_t *)bq;
    uint32_t nb, i, j, b;
    if (!a || !bq || !c) return ORC_E_INVALID_ARG;
    if (k % 32u) return ORC_E_INVALID_ARG;
    nb = k / 32u;
    for (i = 0; i < m; ++i) {
        const float *ar = a + (size_t)i * k;
        for (j = 0; j < n; ++j) {
            const uint8_t *br = bb + (size_t)j * nb * 34u;
            float acc = 0.0f;
            for (b = 0; b < nb; ++b) {
                /* order bit 2: blocks and their products accumulated last to first */
                const uint32_t bo = (g_orc_sum_order & 2) ? nb - 1u - b : b;
                const uint8_t *blk = br + (size_t)bo * 34u;
                uint16_t sh;
                float scale;
                int p;
                memcpy(&sh, blk, 2);
                scale = orc_f16_to_f32(sh);
                for (p = 0; p < 32; ++p) {
                    const int pe = (g_orc_sum_order & 2) ? 31 - p : p;
                    acc += ar[32u * bo + (uint32_t)pe] * ((float)(int8_t)blk[2 + pe] * scale);
                }
            }
            c[(size_t)i * n + j] = acc;
        }
    }
    return ORC_OK;
}

int orc_matmul_f32(const float *a, const float *b, float *c,
                   uint32_t m, uint32_t n, uint32_t k) {
    /* src/kernels/scalar/matmul_f32.c:14-32 */
    uint32_t i, j, p;
    if (!a || !b || !c) return ORC_E_INVALID_ARG;
    for (i = 0; i < m; ++i)
        for (j = 0; j < n; ++j) {
            float acc = 0.0f;
            for (p = 0; p < k; ++p) acc += a[(size_t)i * k + p] * b[(size_t)j * k + p];
            c[(size_t)i * n + j] = acc;
        }
    return ORC_OK;
}

int orc_matmul_q(const float *a, const void *b, int dtype, float *c,
                 uint32_t m, uint32_t n, uint32_t k) {
    /* src/kernels/avx2/matmul_q4_k.c:155-171 */
    switch (dtype) {
    case ORC_DT_Q4_K: return orc_matmul_q4_k_int8(a, b, c, m, n, k);
    case ORC_DT_Q8_0: return orc_matmul_q8_0(a, b, c, m, n, k);
    default: return ORC_E_UNSUPPORTED;
    }
}

/* Row-sharded threads around orc_matmul_q.  m == 1: split the n output
 * rows (each thread's c slice is contiguous); m > 1: split the m rows. */
typedef struct {
    const float *a;
    const uint8_t *b;
    int dtype;
    float *c;
    uint32_t m, n, k, n_total;
    size_t row_bytes;
    int rc;
} orc_job_t;

static void *orc_job_run(void *p) {
    orc_job_t *j = (orc_job_t *)p;
    j->rc = orc_matmul_q(j->a, j->b, j->dtype, j->c, j->m, j->n, j->k);
    return NULL;
}

int orc_matmul_q_threads(const float *a, const void *b, int dtype, float *c,
                         uint32_t m, uint32_t n, uint32_t k, int threads) {
    orc_job_t jobs[256];
    pthread_t tid[256];
    size_t row_bytes;
    uint32_t split, t;
    int rc = ORC_OK;
    if (!a || !b || !c) return ORC_E_INVALID_ARG;
    if (dtype == ORC_DT_Q4_K) {
        if (k % 256u) return ORC_E_INVALID_ARG;
        row_bytes = (size_t)(k / 256u) * 144u;
    } else if (dtype == ORC_DT_Q8_0) {
        if (k % 32u) return ORC_E_INVALID_ARG;
        row_bytes = (size_t)(k / 32u) * 34u;
    } else {
        return ORC_E_UNSUPPORTED;
    }
    if (threads <= 0) threads = (int)sysconf(_SC_NPROCESSORS_ONLN);
    if (threads > 256) threads = 256;
    if (threads < 1) threads = 1;
    split = (m == 1) ? n : m;
    if ((uint32_t)threads > split) threads = (int)(split ? split : 1);
    for (t = 0; t < (uint32_t)threads; ++t) {
        uint32_t lo = (uint32_t)(((uint64_t)split * t) / (uint32_t)threads);
        uint32_t hi = (uint32_t)(((uint64_t)split * (t + 1)) / (uint32_t)threads);
        orc_job_t *j = &jobs[t];
        j->dtype = dtype;
        j->k = k;
        j->rc = ORC_OK;
        if (m == 1) {
            j->a = a;
            j->b = (const uint8_t *)b + (size_t)lo * row_bytes;
            j->c = c + lo;
            j->m = 1;
            j->n = hi - lo;
        } else {
            j->a = a + (size_t)lo * k;
            j->b = (const uint8_t *)b;
            j->c = c + (size_t)lo * n;
            j->m = hi - lo;
            j->n = n;
        }
        if (pthread_create(&tid[t], NULL, orc_job_run, j) != 0) {
            orc_job_run(j);
            tid[t] = 0;
        }
    }
    for (t = 0; t < (uint32_t)threads; ++t) {
        if (tid[t]) pthread_join(tid[t], NULL);
        if (jobs[t].rc != ORC_OK) rc = jobs[t].rc;
    }
    return rc;
}

/* ------------------------------------------------------------------ */
/* Quant schemes                                                       */
/* ------------------------------------------------------------------ */

int orc_q4_k_dequantize(const void *src, float *dst, size_t n_el) {
    /* src/quant/q4_k.c:42-81 */
    const uint8_t *p = (const uint8_t *)src;
    size_t b;
    if (!src || !dst) return ORC_E_INVALID_ARG;
    if (n_el % 256u) return ORC_E_INVALID_ARG;
    for (b = 0; b < n_el / 256u; ++b, p += 144) {
        const uint8_t *qs = p + 16;
        float d, dmin;
        int sub, l;
        q4k_header(p, &d, &dmin);
        for (sub = 0; sub < 8; sub += 2, qs += 32) {
            uint8_t sl, ml, sh, mh;
            float d1, m1, d2, m2;
            orc_get_scale_min(sub, p + 4, &sl, &ml);
            orc_get_scale_min(sub + 1, p + 4, &sh, &mh);
            d1 = d * (float)sl;
            m1 = dmin * (float)ml;
            d2 = d * (float)sh;
            m2 = dmin * (float)mh;
            for (l = 0; l < 32; ++l) {
                dst[b * 256u + (size_t)sub * 32u + (size_t)l] = d1 * (float)(qs[l] & 15u) - m1;
                dst[b * 256u + (size_t)(sub + 1) * 32u + (size_t)l] = d2 * (float)(qs[l] >> 4) - m2;
            }
        }
    }
    return ORC_OK;
}

int orc_q8_0_dequantize(const void *src, float *dst, size_t n_el) {
    /* src/quant/q8_0.c:33-56 */
    const uint8_t *p = (const uint8_t *)src;
    size_t b;
    int i;
    if (!src || !dst) return ORC_E_INVALID_ARG;
    if (n_el % 32u) return ORC_E_INVALID_ARG;
    for (b = 0; b < n_el / 32u; ++b, p += 34) {
        uint16_t sh;
        float s;
        memcpy(&sh, p, 2);
        s = orc_f16_to_f32(sh);
        for (i = 0; i < 32; ++i) dst[b * 32u + (size_t)i] = (float)(int8_t)p[2 + i] * s;
    }
    return ORC_OK;
}

int orc_q8_0_quantize(const float *src, void *dst, size_t n_el) {
    /* src/quant/q8_0.c:58-93: amax/127 scale, round half away from zero,
     * clamp [-128, 127], fp16 scale via the reference encoder. */
    uint8_t *p = (uint8_t *)dst;
    size_t b;
    int i;
    if (!src || !dst) return ORC_E_INVALID_ARG;
    if (n_el % 32u) return ORC_E_INVALID_ARG;
    for (b = 0; b < n_el / 32u; ++b, p += 34) {
        const float *bs = src + b * 32u;
        float amax = 0.0f, scale, inv;
        uint16_t sh;
        for (i = 0; i < 32; ++i) {
            float v = bs[i] < 0.0f ? -bs[i] : bs[i];
            if (v > amax) amax = v;
        }
        scale = amax / 127.0f;
        inv = (scale > 0.0f) ? (1.0f / scale) : 0.0f;
        for (i = 0; i < 32; ++i) {
            float v = bs[i] * inv;
            int q = (int)(v < 0.0f ? v - 0.5f : v + 0.5f);
            if (q > 127) q = 127;
            if (q < -128) q = -128;
            p[2 + i] = (uint8_t)(int8_t)q;
        }
        sh = orc_f32_to_f16(scale);
        memcpy(p, &sh, 2);
    }
    return ORC_OK;
}

/* Own Q4_K quantizer (the reference has none).  Per sub-block j of 32:
 *   lo_j = min(0, min x), hi_j = max x, scale_j = (hi_j - lo_j)/15,
 *   min_j = -lo_j;  d = max scale_j / 63, dmin = max min_j / 63 (as fp16);
 *   sc_j = rint(scale_j/d), m_j = rint(min_j/dmin) in [0, 63];
 *   q = rint((x + dmin*m_j) / (d*sc_j)) in [0, 15].
 * Only IEEE add/sub/mul/div and round-to-nearest-even conversions, so the
 * device quantizer reproduces it bit-for-bit. */
static int orc_rint_clamp(float v, int hi) {
    int q;
    if (!(v > 0.0f)) return 0; /* negatives, zero and NaN */
    if (v >= (float)hi) return hi;
    q = (int)rintf(v);
    return q > hi ? hi : q;
}

static void orc_q4k_quantize_block(const float *x, uint8_t *blk) {
    float scale[8], mins[8], max_scale = 0.0f, max_min = 0.0f, d, dmin;
    uint8_t sc[8], mq[8], q[256];
    uint16_t dh, mh;
    int j, l;
    for (j = 0; j < 8; ++j) {
        float lo = x[32 * j], hi = x[32 * j];
        for (l = 1; l < 32; ++l) {
            float v = x[32 * j + l];
            if (v < lo) lo = v;
            if (v > hi) hi = v;
        }
        if (lo > 0.0f) lo = 0.0f;
        scale[j] = (hi - lo) / 15.0f;
        mins[j] = -lo;
        if (scale[j] > max_scale) max_scale = scale[j];
        if (mins[j] > max_min) max_min = mins[j];
    }
    dh = orc_f32_to_f16(max_scale / 63.0f);
    mh = orc_f32_to_f16(max_min / 63.0f);
    d = orc_f16_to_f32(dh);
    dmin = orc_f16_to_f32(mh);
    for (j = 0; j < 8; ++j) {
        float es, em;
        sc[j] = (uint8_t)(d > 0.0f ? orc_rint_clamp(scale[j] / d, 63) : 0);
        mq[j] = (uint8_t)(dmin > 0.0f ? orc_rint_clamp(mins[j] / dmin, 63) : 0);
        es = d * (float)sc[j];
        em = dmin * (float)mq[j];
        for (l = 0; l < 32; ++l)
            q[32 * j + l] = (uint8_t)(es > 0.0f ? orc_rint_clamp((x[32 * j + l] + em) / es, 15) : 0);
    }
    memcpy(blk, &dh, 2);
    memcpy(blk + 2, &mh, 2);
    orc_pack_q4k_scales(sc, mq, blk + 4);
    for (j = 0; j < 4; ++j)
        for (l = 0; l < 32; ++l)
            blk[16 + 32 * j + l] = (uint8_t)(q[64 * j + l] | (q[64 * j + 32 + l] << 4));
}

int orc_q4_k_quantize(const float *src, void *dst, size_t n_el) {
    size_t b;
    if (!src || !dst) return ORC_E_INVALID_ARG;
    if (n_el % 256u) return ORC_E_INVALID_ARG;
    for (b = 0; b < n_el / 256u; ++b)
        orc_q4k_quantize_block(src + 256u * b, (uint8_t *)dst + 144u * b);
    return ORC_OK;
}

/* ------------------------------------------------------------------ */
/* Synthetic inputs                                                    */
/* ------------------------------------------------------------------ */

static uint64_t orc_splitmix64(uint64_t z) {
    /* Steele, Lea & Flood, "Fast splittable pseudorandom number
     * generators" (OOPSLA 2014): golden-gamma increment + mix64. */
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

float orc_gauss(uint64_t seed, uint64_t index, float sigma) {
    uint64_t key = orc_splitmix64(seed ^ 0x6A09E667F3BCC909ull);
    int32_t s = 0;
    int h;
    for (h = 0; h < 4; ++h) {
        uint64_t r = orc_splitmix64(key + 4u * index + (uint64_t)h);
        s += (int32_t)(r & 0x1FFFFFu) + (int32_t)((r >> 21) & 0x1FFFFFu) +
             (int32_t)((r >> 42) & 0x1FFFFFu);
    }
    /* (sum - 6*2^21) is exact in f32; times 2^-21 is exact; one rounding
     * for sigma. */
    return ((float)(s - 6 * 2097152) * 4.76837158203125e-07f) * sigma;
}

void orc_fill_gauss(float *dst, size_t n, uint64_t seed, uint64_t offset, float sigma) {
    size_t i;
    for (i = 0; i < n; ++i) dst[i] = orc_gauss(seed, offset + i, sigma);
}

uint32_t orc_xorshift32(uint32_t *st) {
    /* tests/unit/test_runner.c:635-643 */
    uint32_t x = *st;
    x ^= x << 13;
    x ^= x >> 17;
    x ^= x << 5;
    *st = x;
    return x;
}

float orc_xs_rand_unit(uint32_t *st) {
    /* tests/unit/test_runner.c:644-646 */
    return ((float)(orc_xorshift32(st) & 0xFFFFFFu) / (float)0x800000) - 1.0f;
}

/* ------------------------------------------------------------------ */
/* Decoder ops                                                         */
/* ------------------------------------------------------------------ */

void orc_set_sum_order(int order) { g_orc_sum_order = order; }

/* Sum of squares in the order of a 256-thread reduction: thread t sums
 * elements t, t + 256, ...; then a xor butterfly (16, 8, 4, 2, 1) inside
 * each 32-thread warp; then the 8 warp totals in warp order. */
static float orc_sumsq_strided256(const float *x, uint32_t n) {
    float t[256], u[256], s;
    uint32_t i, j;
    int off;
    for (i = 0; i < 256; ++i) t[i] = 0.0f;
    for (j = 0; j < n; j += 256)
        for (i = 0; i < 256 && j + i < n; ++i) t[i] += x[j + i] * x[j + i];
    for (off = 16; off > 0; off >>= 1) {
        for (i = 0; i < 256; ++i) u[i] = t[i] + t[(i & ~31u) | ((i & 31u) ^ (uint32_t)off)];
        for (i = 0; i < 256; ++i) t[i] = u[i];
    }
    s = t[0];
    for (i = 1; i < 8; ++i) s += t[32 * i];
    return s;
}

int orc_rmsnorm(const float *x, const float *w, float eps, float *y,
                uint32_t rows, uint32_t cols) {
    /* src/kernels/scalar/rmsnorm.c:14-37 */
    uint32_t i, j;
    if (!x || !y || cols == 0) return ORC_E_INVALID_ARG;
    for (i = 0; i < rows; ++i) {
        const float *xr = x + (size_t)i * cols;
        float *yr = y + (size_t)i * cols;
        float ms = 0.0f, s;
        if (g_orc_sum_order & 1)
            ms = orc_sumsq_strided256(xr, cols);
        else
            for (j = 0; j < cols; ++j) ms += xr[j] * xr[j];
        ms /= (float)cols;
        s = 1.0f / sqrtf(ms + eps);
        for (j = 0; j < cols; ++j) yr[j] = xr[j] * s * (w ? w[j] : 1.0f);
    }
    return ORC_OK;
}

int orc_rope(float *x, uint32_t n_heads, uint32_t head_dim, uint32_t pos, float base) {
    /* src/kernels/scalar/rope.c:16-38 */
    uint32_t h, i;
    if (!x || head_dim == 0 || (head_dim & 1u)) return ORC_E_INVALID_ARG;
    for (h = 0; h < n_heads; ++h) {
        float *xh = x + (size_t)h * head_dim;
        for (i = 0; i + 1 < head_dim; i += 2) {
            float th = (float)pos * powf(base, -((float)i) / (float)head_dim);
            float cs = cosf(th), sn = sinf(th), p0 = xh[i], p1 = xh[i + 1];
            xh[i] = p0 * cs - p1 * sn;
            xh[i + 1] = p0 * sn + p1 * cs;
        }
    }
    return ORC_OK;
}

int orc_silu(const float *x, float *y, size_t n) {
    /* src/kernels/scalar/silu.c:12-23 */
    size_t i;
    if (!x || !y) return ORC_E_INVALID_ARG;
    for (i = 0; i < n; ++i) y[i] = x[i] * (1.0f / (1.0f + expf(-x[i])));
    return ORC_OK;
}

/* ------------------------------------------------------------------ */
/* Llama decoder step: restates src/modality/text/text.c:267-436       */
/* ------------------------------------------------------------------ */

struct orc_text {
    orc_llama_t m;
    uint32_t head_dim, pos;
    float *k_cache, *v_cache;  /* [n_layer][max_ctx][n_kv_head * head_dim] (text.c:220-226) */
    float *x, *xn, *q, *k, *v, *attn_out, *ff_gate, *ff_up, *ff_tmp;
};

int orc_text_open(const orc_llama_t *m, orc_text_t **out) {
    orc_text_t *st;
    size_t kvl;
    if (!m || !out || m->n_head == 0 || m->n_kv_head == 0) return ORC_E_INVALID_ARG;
    st = (orc_text_t *)calloc(1, sizeof(*st));
    if (!st) return ORC_E_OUT_OF_MEMORY;
    st->m = *m;
    st->head_dim = m->n_embd / m->n_head; /* text.c:147 */
    kvl = (size_t)m->max_ctx * m->n_kv_head * st->head_dim;
    st->k_cache = (float *)calloc((size_t)m->n_layer * kvl, sizeof(float));
    st->v_cache = (float *)calloc((size_t)m->n_layer * kvl, sizeof(float));
    st->x = (float *)calloc(m->n_embd, 4);
    st->xn = (float *)calloc(m->n_embd, 4);
    st->q = (float *)calloc(m->n_embd, 4);
    st->k = (float *)calloc((size_t)m->n_kv_head * st->head_dim, 4);
    st->v = (float *)calloc((size_t)m->n_kv_head * st->head_dim, 4);
    st->attn_out = (float *)calloc(m->n_embd, 4);
    /* ff_gate doubles as the attention score scratch (text.c:370), so it
     * must hold max_ctx entries too */
    st->ff_gate = (float *)calloc(m->n_ff > m->max_ctx ? m->n_ff : m->max_ctx, 4);
    st->ff_up = (float *)calloc(m->n_ff, 4);
    st->ff_tmp = (float *)calloc(m->n_ff > m->n_embd ? m->n_ff : m->n_embd, 4);
    if (!st->k_cache || !st->v_cache || !st->x || !st->xn || !st->q || !st->k || !st->v || !st->attn_out ||
        !st->ff_gate || !st->ff_up || !st->ff_tmp) {
        orc_text_close(st);
        return ORC_E_OUT_OF_MEMORY;
    }
    *out = st;
    return ORC_OK;
}

void orc_text_close(orc_text_t *st) {
    if (!st) return;
    free(st->k_cache); free(st->v_cache); free(st->x); free(st->xn); free(st->q); free(st->k);
    free(st->v); free(st->attn_out); free(st->ff_gate); free(st->ff_up); free(st->ff_tmp);
    free(st);
}

uint32_t orc_text_pos(const orc_text_t *st) { return st ? st->pos : 0; }

static int orc_mw(const orc_text_t *st, const float *x, const void *w, int dt, float *y, uint32_t out_dim,
                  uint32_t in_dim) {
    /* matmul_w for Q8_0 / Q4_K (text.c:75-99): matmul_q with m = 1 */
    (void)st;
    return orc_matmul_q(x, w, dt, y, 1, out_dim, in_dim);
}

int orc_text_step(orc_text_t *st, uint32_t token, float *logits) {
    const orc_llama_t *m;
    uint32_t n_embd, n_head, n_kvh, hd, n_ff, pos, L, h, p, i;
    size_t kv_stride;
    int r;
    if (!st || !logits) return ORC_E_INVALID_ARG;
    m = &st->m;
    if (token >= m->n_vocab) return ORC_E_INVALID_ARG;       /* text.c:277 */
    if (st->pos >= m->max_ctx) return ORC_E_OUT_OF_MEMORY;   /* text.c:278 */
    n_embd = m->n_embd; n_head = m->n_head; n_kvh = m->n_kv_head; hd = st->head_dim; n_ff = m->n_ff;
    pos = st->pos;
    kv_stride = (size_t)m->max_ctx * n_kvh * hd;

    /* 1. embedding row, F16 (text.c:317-320) */
    for (i = 0; i < n_embd; ++i) st->x[i] = orc_f16_to_f32(m->tok_embd[(size_t)token * n_embd + i]);

    for (L = 0; L < m->n_layer; ++L) {
        /* 2a-2b (text.c:344-352) */
        if ((r = orc_rmsnorm(st->x, m->attn_norm[L], m->rms_eps, st->xn, 1, n_embd))) return r;
        if ((r = orc_mw(st, st->xn, m->wq[L], m->wdtype, st->q, n_embd, n_embd))) return r;
        if ((r = orc_mw(st, st->xn, m->wk[L], m->wdtype, st->k, n_kvh * hd, n_embd))) return r;
        if ((r = orc_mw(st, st->xn, m->wv[L], m->wdtype, st->v, n_kvh * hd, n_embd))) return r;
        /* 2c (text.c:355-356) */
        if ((r = orc_rope(st->q, n_head, hd, pos, m->rope_base))) return r;
        if ((r = orc_rope(st->k, n_kvh, hd, pos, m->rope_base))) return r;
        /* 2d (text.c:359-362) */
        memcpy(&st->k_cache[L * kv_stride + (size_t)pos * n_kvh * hd], st->k, (size_t)n_kvh * hd * 4);
        memcpy(&st->v_cache[L * kv_stride + (size_t)pos * n_kvh * hd], st->v, (size_t)n_kvh * hd * 4);
        /* 2e: attention with GQA grouping (text.c:366-401) */
        {
            const float scale = 1.0f / sqrtf((float)hd);
            const float *Kc = &st->k_cache[L * kv_stride], *Vc = &st->v_cache[L * kv_stride];
            float *att = st->ff_gate;
            memset(st->attn_out, 0, (size_t)n_embd * 4);
            for (h = 0; h < n_head; ++h) {
                const uint32_t kvh = (h * n_kvh) / n_head;
                const float *qh = st->q + (size_t)h * hd;
                float maxv = -1e30f, sum = 0.0f;
                for (p = 0; p <= pos; ++p) {
                    const float *kp = Kc + (size_t)p * n_kvh * hd + (size_t)kvh * hd;
                    float dot = 0.0f;
                    for (i = 0; i < hd; ++i) dot += qh[i] * kp[i];
                    att[p] = dot * scale;
                    if (att[p] > maxv) maxv = att[p];
                }
                for (p = 0; p <= pos; ++p) {
                    att[p] = expf(att[p] - maxv);
                    sum += att[p];
                }
                if (sum > 0.0f) {
                    float inv = 1.0f / sum;
                    for (p = 0; p <= pos; ++p) att[p] *= inv;
                }
                for (p = 0; p <= pos; ++p) {
                    const float *vp = Vc + (size_t)p * n_kvh * hd + (size_t)kvh * hd;
                    float a = att[p];
                    for (i = 0; i < hd; ++i) st->attn_out[h * hd + i] += a * vp[i];
                }
            }
        }
        /* 2f (text.c:404-406) */
        if ((r = orc_mw(st, st->attn_out, m->wo[L], m->wdtype, st->ff_tmp, n_embd, n_embd))) return r;
        for (i = 0; i < n_embd; ++i) st->x[i] += st->ff_tmp[i];
        /* 2g-2h (text.c:409-417) */
        if ((r = orc_rmsnorm(st->x, m->ffn_norm[L], m->rms_eps, st->xn, 1, n_embd))) return r;
        if ((r = orc_mw(st, st->xn, m->wg[L], m->wdtype, st->ff_gate, n_ff, n_embd))) return r;
        if ((r = orc_mw(st, st->xn, m->wu[L], m->wdtype, st->ff_up, n_ff, n_embd))) return r;
        if ((r = orc_silu(st->ff_gate, st->ff_gate, n_ff))) return r;
        for (i = 0; i < n_ff; ++i) st->ff_tmp[i] = st->ff_gate[i] * st->ff_up[i];
        /* 2i (text.c:420-421) */
        if ((r = orc_mw(st, st->ff_tmp, m->wd[L], m->wdtype, st->attn_out, n_embd, n_ff))) return r;
        for (i = 0; i < n_embd; ++i) st->x[i] += st->attn_out[i];
    }
    /* 3. final norm + output projection (text.c:425-432) */
    if ((r = orc_rmsnorm(st->x, m->output_norm, m->rms_eps, st->xn, 1, n_embd))) return r;
    if ((r = orc_mw(st, st->xn, m->output_w, m->out_dtype, logits, m->n_vocab, n_embd))) return r;
    st->pos++;
    return ORC_OK;
}
