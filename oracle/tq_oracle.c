/*
 * tq_oracle.c — CPU restatement of LeanKV's TurboQuant hot path.
 * TEST INFRASTRUCTURE ONLY (see tq_oracle.h): the product never links it.
 *
 * Every function names the reference lines it restates.  Built by
 * oracle/Makefile with the reference's own flags (-O2 -std=c11, no fast-math)
 * so float32 arithmetic follows the same IEEE single-precision rules as the
 * reference build.
 */
#define _POSIX_C_SOURCE 200809L
#include "tq_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ── codebooks: src/ggml-tq.h:98-121 (values must be identical) ───────── */

const float ORC_TQ3_LEVELS[8] = {
    -1.0000000f, -0.6245203f, -0.3513239f, -0.1138989f,
    +0.1138989f, +0.3513239f, +0.6245203f, +1.0000000f,
};
const float ORC_TQ3_BOUNDS[7] = {
    -0.8122602f, -0.4879221f, -0.2326114f, +0.0000000f,
    +0.2326114f, +0.4879221f, +0.8122602f,
};
const float ORC_TQ2_LEVELS[4] = {-1.0000000f, -0.2997714f, +0.2997714f, +1.0000000f};
const float ORC_TQ4_LEVELS[16] = {
    -1.0000000f, -0.7573038f, -0.5923403f, -0.4599576f,
    -0.3450764f, -0.2405254f, -0.1421261f, -0.0470277f,
    +0.0470277f, +0.1421261f, +0.2405254f, +0.3450764f,
    +0.4599576f, +0.5923403f, +0.7573038f, +1.0000000f,
};
const float ORC_TQ4_BOUNDS[15] = {
    -0.8786519f, -0.6748221f, -0.5261490f, -0.4025170f,
    -0.2928009f, -0.1913257f, -0.0945769f, +0.0000000f,
    +0.0945769f, +0.1913257f, +0.2928009f, +0.4025170f,
    +0.5261490f, +0.6748221f, +0.8786519f,
};

/* scripts/tq3_rounding.py:18-26 parses these decimal literals as float64 */
static const double TQ3_LEVELS_F64[8] = {
    -1.0000000, -0.6245203, -0.3513239, -0.1138989,
    +0.1138989, +0.3513239, +0.6245203, +1.0000000,
};
static const double TQ3_BOUNDS_F64[7] = {
    -0.8122602, -0.4879221, -0.2326114, +0.0000000,
    +0.2326114, +0.4879221, +0.8122602,
};

/* ── fp16 codec of the standalone build: src/ggml-tq.h:39-64 ─────────── */

uint16_t orc_half_from_float(float f) {
    uint32_t u;
    memcpy(&u, &f, sizeof u);
    const uint16_t sign = (uint16_t)((u >> 31) << 15);
    const int e = (int)((u >> 23) & 0xFFu) - 112;      /* rebias 127 -> 15 */
    if (e <= 0) return sign;                            /* below normal range: signed zero */
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);     /* above range, inf, nan: signed inf */
    return (uint16_t)(sign | (uint32_t)e << 10 | ((u >> 13) & 0x3FFu)); /* mantissa truncated */
}

float orc_float_from_half(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t e = (h >> 10) & 31u;
    const uint32_t m = h & 0x3FFu;
    float f;
    if (e == 0) {
        /* zero or subnormal: exactly m * 2^-24 */
        f = (float)m * 0x1p-24f;
        return sign ? -f : f;
    }
    /* no inf/nan special case in the standalone decoder: e == 31 is 2^16 * 1.m */
    const uint32_t u = sign | ((e + 112u) << 23) | (m << 13);
    memcpy(&f, &u, sizeof f);
    return f;
}

/* ── FWHT: src/ggml-tq.c:361-381, :398-404 ────────────────────────────── */

void orc_fwht(float *x, int d) {
    /* stages in increasing distance h = 1, 2, 4, ... ; (a, b) -> (a + b, a - b) */
    for (int h = 1; h < d; h <<= 1) {
        for (int j = 0; j < d; ++j) {
            if (j & h) continue;
            const float a = x[j], b = x[j + h];
            x[j] = a + b;
            x[j + h] = a - b;
        }
    }
    const float norm = 1.0f / sqrtf((float)d);
    for (int j = 0; j < d; ++j) x[j] *= norm;
}

void orc_fwht_rows(float *x, int64_t n, int head_dim) {
    for (int64_t off = 0; off + head_dim <= n; off += head_dim) orc_fwht(x + off, head_dim);
}

/* ── nearest level: src/ggml-tq.c:112-154 ─────────────────────────────
 * Both reference searches return the number of boundaries strictly below xn
 * for ordered xn.  For NaN the TQ3 scan returns 0 and the TQ4 tree returns 15. */

int orc_tq3_nearest(float xn) {
    if (xn != xn) return 0;
    int c = 0;
    for (int b = 0; b < 7; ++b) c += ORC_TQ3_BOUNDS[b] < xn;
    return c;
}

int orc_tq4_nearest(float xn) {
    if (xn != xn) return 15;
    int c = 0;
    for (int b = 0; b < 15; ++b) c += ORC_TQ4_BOUNDS[b] < xn;
    return c;
}

static float clamp_unit(float v) {
    if (v < -1.0f) v = -1.0f;
    if (v > 1.0f) v = 1.0f;
    return v;
}

/* amax that ignores NaN exactly like `if (v > amax) amax = v` */
static float block_amax(const float *x) {
    float m = 0.0f;
    for (int j = 0; j < ORC_QK; ++j) {
        const float a = fabsf(x[j]);
        if (a > m) m = a;
    }
    return m;
}

static void put_half(uint8_t *p, uint16_t h) { p[0] = (uint8_t)(h & 0xFF); p[1] = (uint8_t)(h >> 8); }
static uint16_t get_half(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* ── 3-bit packing: src/ggml-tq.c:26-68 ───────────────────────────────
 * Each group of 8 codes is a little-endian 24-bit word with code i at bits 3i..3i+2. */

void orc_tq3_pack32(const uint8_t idx[32], uint8_t qs[12]) {
    for (int g = 0; g < 4; ++g) {
        uint32_t w = 0;
        for (int i = 0; i < 8; ++i) w |= (uint32_t)(idx[8 * g + i] & 7u) << (3 * i);
        qs[3 * g + 0] = (uint8_t)(w & 0xFF);
        qs[3 * g + 1] = (uint8_t)((w >> 8) & 0xFF);
        qs[3 * g + 2] = (uint8_t)((w >> 16) & 0xFF);
    }
}

void orc_tq3_unpack32(const uint8_t qs[12], uint8_t idx[32]) {
    for (int g = 0; g < 4; ++g) {
        const uint32_t w = (uint32_t)qs[3 * g] | (uint32_t)qs[3 * g + 1] << 8 | (uint32_t)qs[3 * g + 2] << 16;
        for (int i = 0; i < 8; ++i) idx[8 * g + i] = (uint8_t)((w >> (3 * i)) & 7u);
    }
}

/* ── TQ3_0: src/ggml-tq.c:215-265 ───────────────────────────────────── */

void orc_tq3_quantize(const float *x, uint8_t *blocks, int64_t k) {
    const int64_t nb = k / ORC_QK;
    for (int64_t i = 0; i < nb; ++i) {
        const float *src = x + ORC_QK * i;
        uint8_t *dst = blocks + ORC_TQ3_BYTES * i;
        const float amax = block_amax(src);
        const float inv = amax > 0.0f ? 1.0f / amax : 0.0f;
        put_half(dst, orc_half_from_float(amax));
        uint8_t idx[32];
        for (int j = 0; j < ORC_QK; ++j) idx[j] = (uint8_t)orc_tq3_nearest(clamp_unit(src[j] * inv));
        orc_tq3_pack32(idx, dst + 2);
    }
}

void orc_tq3_dequantize(const uint8_t *blocks, float *y, int64_t k) {
    const int64_t nb = k / ORC_QK;
    for (int64_t i = 0; i < nb; ++i) {
        const uint8_t *src = blocks + ORC_TQ3_BYTES * i;
        const float d = orc_float_from_half(get_half(src));
        uint8_t idx[32];
        orc_tq3_unpack32(src + 2, idx);
        for (int j = 0; j < ORC_QK; ++j) y[ORC_QK * i + j] = ORC_TQ3_LEVELS[idx[j]] * d;
    }
}

/* ── TQ2_0 decode: src/ggml-tq.c:191-207 ───────────────────────────────
 * Byte i of the codes holds elements 4i .. 4i+3, two bits each from the low end
 * (the unpack of src/ggml-tq.c:70-77); y = level * d. */
void orc_tq2_dequantize(const uint8_t *blocks, float *y, int64_t k) {
    const int64_t nb = k / ORC_QK;
    for (int64_t i = 0; i < nb; ++i) {
        const uint8_t *src = blocks + ORC_TQ2_BYTES * i;
        const float d = orc_float_from_half(get_half(src));
        for (int b = 0; b < 8; ++b)
            for (int e = 0; e < 4; ++e) y[ORC_QK * i + 4 * b + e] = ORC_TQ2_LEVELS[(src[2 + b] >> (2 * e)) & 3] * d;
    }
}

/* ── TQ4_0: src/ggml-tq.c:273-321 ───────────────────────────────────── */

void orc_tq4_quantize(const float *x, uint8_t *blocks, int64_t k) {
    const int64_t nb = k / ORC_QK;
    for (int64_t i = 0; i < nb; ++i) {
        const float *src = x + ORC_QK * i;
        uint8_t *dst = blocks + ORC_TQ4_BYTES * i;
        const float amax = block_amax(src);
        const float inv = amax > 0.0f ? 1.0f / amax : 0.0f;
        put_half(dst, orc_half_from_float(amax));
        for (int j = 0; j < 16; ++j) {
            const int lo = orc_tq4_nearest(clamp_unit(src[j] * inv));
            const int hi = orc_tq4_nearest(clamp_unit(src[j + 16] * inv));
            dst[2 + j] = (uint8_t)(lo | hi << 4);
        }
    }
}

void orc_tq4_dequantize(const uint8_t *blocks, float *y, int64_t k) {
    const int64_t nb = k / ORC_QK;
    for (int64_t i = 0; i < nb; ++i) {
        const uint8_t *src = blocks + ORC_TQ4_BYTES * i;
        const float d = orc_float_from_half(get_half(src));
        for (int j = 0; j < 16; ++j) {
            y[ORC_QK * i + j] = ORC_TQ4_LEVELS[src[2 + j] & 15] * d;
            y[ORC_QK * i + j + 16] = ORC_TQ4_LEVELS[src[2 + j] >> 4] * d;
        }
    }
}

/* ── TQ3 optimal rounding: scripts/tq3_rounding.py:51-57, :74-125 ─────── */

/* numpy's pairwise sum for 8 <= n < 128 (8 running partial sums, then a tree) */
static double np_pairwise_sum32(const double *a) {
    double r[8];
    for (int i = 0; i < 8; ++i) r[i] = a[i];
    for (int i = 8; i < 32; i += 8)
        for (int j = 0; j < 8; ++j) r[j] += a[i + j];
    return ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
}

/* optimal_scale: dot(block, L) / dot(L, L), 0 when the denominator is 0 */
static double ls_scale(const double *b, const uint8_t *idx) {
    double num = 0.0, den = 0.0;
    for (int j = 0; j < ORC_QK; ++j) {
        const double l = TQ3_LEVELS_F64[idx[j]];
        den += l * l;
        num += b[j] * l;
    }
    return den == 0.0 ? 0.0 : num / den;
}

/* block_mse: mean((block - L * scale)^2) */
static double block_mse(const double *b, const uint8_t *idx, double s) {
    double e[ORC_QK];
    for (int j = 0; j < ORC_QK; ++j) {
        const double r = b[j] - TQ3_LEVELS_F64[idx[j]] * s;
        e[j] = r * r;
    }
    return np_pairwise_sum32(e) / ORC_QK;
}

int orc_tq3_opt_block(const float x32[32], uint8_t idx[32], double *scale, int n_passes, int init_f64) {
    double b[ORC_QK];
    for (int j = 0; j < ORC_QK; ++j) b[j] = (double)x32[j];
    const float amax = block_amax(x32);
    if (amax == 0.0f) {
        memset(idx, 0, ORC_QK);
        *scale = 0.0;
        return 0;
    }
    if (init_f64) {
        for (int j = 0; j < ORC_QK; ++j) {
            double xn = b[j] / (double)amax;
            if (xn < -1.0) xn = -1.0;
            if (xn > 1.0) xn = 1.0;
            int c = 0;
            for (int t = 0; t < 7; ++t) c += xn > TQ3_BOUNDS_F64[t];
            idx[j] = (uint8_t)c;
        }
    } else {
        const float inv = 1.0f / amax;
        for (int j = 0; j < ORC_QK; ++j) idx[j] = (uint8_t)orc_tq3_nearest(clamp_unit(x32[j] * inv));
    }
    double d = ls_scale(b, idx);
    double best = block_mse(b, idx, d);
    int moves = 0;
    for (int pass = 0; pass < n_passes; ++pass) {
        int improved = 0;
        for (int j = 0; j < ORC_QK; ++j) {
            const uint8_t orig = idx[j];
            int cand[2], nc = 0;
            if (orig > 0) cand[nc++] = orig - 1;   /* the lower neighbour is tried first */
            if (orig < 7) cand[nc++] = orig + 1;
            for (int c = 0; c < nc; ++c) {
                idx[j] = (uint8_t)cand[c];
                const double nd = ls_scale(b, idx);
                const double nm = block_mse(b, idx, nd);
                if (nm < best) {                   /* first strict improvement wins */
                    best = nm;
                    d = nd;
                    improved = 1;
                    ++moves;
                    break;
                }
                idx[j] = orig;
            }
        }
        if (!improved) break;                      /* converged */
    }
    *scale = d;
    return moves;
}

int64_t orc_tq3_quantize_opt(const float *x, uint8_t *blocks, int64_t k, int n_passes, int init_f64) {
    const int64_t nb = k / ORC_QK;
    int64_t moves = 0;
    for (int64_t i = 0; i < nb; ++i) {
        uint8_t idx[32];
        double d;
        moves += orc_tq3_opt_block(x + ORC_QK * i, idx, &d, n_passes, init_f64);
        float df = (float)d;
        if (df != df) df = fabsf(df);   /* canonical positive NaN -> +inf scale field */
        uint8_t *dst = blocks + ORC_TQ3_BYTES * i;
        put_half(dst, orc_half_from_float(df));
        orc_tq3_pack32(idx, dst + 2);
    }
    return moves;
}

void orc_tq3_quantize_opt2_row(const void *x, void *blocks, int64_t k) {
    orc_tq3_quantize_opt((const float *)x, (uint8_t *)blocks, k, 2, 0);
}

/* ── decode attention (restated math, float64) ────────────────────────── */

static void dequant_row(const uint8_t *blocks, int type, float *y, int D) {
    if (type == 3) orc_tq3_dequantize(blocks, y, D);
    else if (type == 2) orc_tq2_dequantize(blocks, y, D);
    else orc_tq4_dequantize(blocks, y, D);
}

static void fwht_f64(double *x, int d) {
    for (int h = 1; h < d; h <<= 1)
        for (int j = 0; j < d; ++j) {
            if (j & h) continue;
            const double a = x[j], b = x[j + h];
            x[j] = a + b;
            x[j + h] = a - b;
        }
    const double norm = 1.0 / sqrt((double)d);
    for (int j = 0; j < d; ++j) x[j] *= norm;
}

typedef struct {
    int B, Hq, Hkv, D;
    int64_t T;
    const float *q;
    const uint8_t *k, *v;
    int k_type, v_type;
    const int64_t *kv_len;
    float sm_scale;
    int rotate_q, v_rotated;
    float *out, *lse;
    int64_t pair_begin, pair_end;
} attn_job;

static void attn_pair(const attn_job *J, int b, int g) {
    const int D = J->D, grp = J->Hq / J->Hkv;
    const int64_t n = J->kv_len ? J->kv_len[b] : J->T;
    const int kbytes = (J->k_type == 3 ? ORC_TQ3_BYTES : J->k_type == 2 ? ORC_TQ2_BYTES : ORC_TQ4_BYTES) * (D / ORC_QK);
    const int vbytes = (J->v_type == 3 ? ORC_TQ3_BYTES : ORC_TQ4_BYTES) * (D / ORC_QK);
    const uint8_t *kbase = J->k + ((int64_t)b * J->Hkv + g) * J->T * kbytes;
    const uint8_t *vbase = J->v + ((int64_t)b * J->Hkv + g) * J->T * vbytes;

    float *qr = malloc(sizeof(float) * (size_t)grp * D);
    double *s = malloc(sizeof(double) * (size_t)grp * (size_t)(n > 0 ? n : 1));
    double *acc = calloc((size_t)grp * D, sizeof(double));
    double *mx = malloc(sizeof(double) * grp);
    double *den = calloc(grp, sizeof(double));
    float *row = malloc(sizeof(float) * D);

    for (int h = 0; h < grp; ++h) {
        const float *src = J->q + ((int64_t)b * J->Hq + (int64_t)g * grp + h) * D;
        memcpy(qr + h * D, src, sizeof(float) * D);
        if (J->rotate_q) orc_fwht(qr + h * D, D);   /* hadamard_transform on the query */
        mx[h] = -INFINITY;
    }
    for (int64_t t = 0; t < n; ++t) {
        dequant_row(kbase + t * kbytes, J->k_type, row, D);
        for (int h = 0; h < grp; ++h) {
            double dot = 0.0;
            for (int e = 0; e < D; ++e) dot += (double)qr[h * D + e] * (double)row[e];
            const double sc = dot * (double)J->sm_scale;
            s[(size_t)h * n + t] = sc;
            if (sc > mx[h]) mx[h] = sc;
        }
    }
    for (int64_t t = 0; t < n; ++t) {
        dequant_row(vbase + t * vbytes, J->v_type, row, D);
        for (int h = 0; h < grp; ++h) {
            const double p = exp(s[(size_t)h * n + t] - mx[h]);
            den[h] += p;
            for (int e = 0; e < D; ++e) acc[h * D + e] += p * (double)row[e];
        }
    }
    for (int h = 0; h < grp; ++h) {
        const int64_t qh = (int64_t)b * J->Hq + (int64_t)g * grp + h;
        double *o = acc + h * D;
        if (n > 0) {
            for (int e = 0; e < D; ++e) o[e] /= den[h];
            if (J->v_rotated) fwht_f64(o, D);
        }
        for (int e = 0; e < D; ++e) J->out[qh * D + e] = n > 0 ? (float)o[e] : 0.0f;
        if (J->lse) J->lse[qh] = n > 0 ? (float)(mx[h] + log(den[h])) : -INFINITY;
    }
    free(qr); free(s); free(acc); free(mx); free(den); free(row);
}

static void *attn_worker(void *arg) {
    const attn_job *J = (const attn_job *)arg;
    for (int64_t p = J->pair_begin; p < J->pair_end; ++p) attn_pair(J, (int)(p / J->Hkv), (int)(p % J->Hkv));
    return NULL;
}

void orc_decode_attention(int B, int Hq, int Hkv, int D, int64_t T,
                          const float *q,
                          const uint8_t *k, int k_type,
                          const uint8_t *v, int v_type,
                          const int64_t *kv_len, float sm_scale,
                          int rotate_q, int v_rotated,
                          float *out, float *lse, int nthreads) {
    const int64_t pairs = (int64_t)B * Hkv;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > pairs) nthreads = (int)(pairs > 0 ? pairs : 1);
    attn_job base = {B, Hq, Hkv, D, T, q, k, v, k_type, v_type, kv_len, sm_scale,
                     rotate_q, v_rotated, out, lse, 0, pairs};
    if (nthreads == 1) { attn_worker(&base); return; }
    pthread_t *th = malloc(sizeof(pthread_t) * nthreads);
    attn_job *jobs = malloc(sizeof(attn_job) * nthreads);
    for (int i = 0; i < nthreads; ++i) {
        jobs[i] = base;
        jobs[i].pair_begin = pairs * i / nthreads;
        jobs[i].pair_end = pairs * (i + 1) / nthreads;
        pthread_create(&th[i], NULL, attn_worker, &jobs[i]);
    }
    for (int i = 0; i < nthreads; ++i) pthread_join(th[i], NULL);
    free(th); free(jobs);
}

void orc_lse_combine(int P, int64_t n, int D, const float *o, const float *lse,
                     float *out, float *lse_out) {
    for (int64_t i = 0; i < n; ++i) {
        double m = -INFINITY;
        for (int p = 0; p < P; ++p) if ((double)lse[(int64_t)p * n + i] > m) m = lse[(int64_t)p * n + i];
        if (m == -INFINITY) {
            for (int e = 0; e < D; ++e) out[i * D + e] = 0.0f;
            if (lse_out) lse_out[i] = -INFINITY;
            continue;
        }
        double wsum = 0.0;
        for (int e = 0; e < D; ++e) out[i * D + e] = 0.0f;
        double *acc = calloc(D, sizeof(double));
        for (int p = 0; p < P; ++p) {
            const double w = exp((double)lse[(int64_t)p * n + i] - m);
            wsum += w;
            for (int e = 0; e < D; ++e) acc[e] += w * (double)o[((int64_t)p * n + i) * D + e];
        }
        for (int e = 0; e < D; ++e) out[i * D + e] = (float)(acc[e] / wsum);
        if (lse_out) lse_out[i] = (float)(m + log(wsum));
        free(acc);
    }
}

/* ── row-parallel driver for CPU baselines ─────────────────────────────── */

typedef struct {
    orc_row_fn fn;
    orc_fwht_row_fn fwht;
    int head_dim, in_bf16;
    const uint8_t *in;
    int64_t in_row_bytes;
    uint8_t *out;
    int64_t out_row_bytes;
    int64_t r0, r1, row_elems;
} rows_job;

static void *rows_worker(void *arg) {
    const rows_job *J = (const rows_job *)arg;
    float *buf = NULL;
    if (J->head_dim > 0 || J->in_bf16) buf = malloc(sizeof(float) * (size_t)J->row_elems);
    for (int64_t r = J->r0; r < J->r1; ++r) {
        const uint8_t *src = J->in + r * J->in_row_bytes;
        const void *row = src;
        if (buf) {
            if (J->in_bf16) {
                const uint16_t *h = (const uint16_t *)src;
                for (int64_t e = 0; e < J->row_elems; ++e) {
                    const uint32_t u = (uint32_t)h[e] << 16;
                    memcpy(&buf[e], &u, sizeof(float));
                }
            } else {
                memcpy(buf, src, sizeof(float) * (size_t)J->row_elems);
            }
            if (J->head_dim > 0) J->fwht(buf, (int)J->row_elems, J->head_dim);
            row = buf;
        }
        J->fn(row, J->out + r * J->out_row_bytes, J->row_elems);
    }
    free(buf);
    return NULL;
}

void orc_parallel_rows(orc_row_fn fn, orc_fwht_row_fn fn_fwht_row, int fwht_head_dim,
                       int in_is_bf16,
                       const void *in, int64_t in_row_bytes,
                       void *out, int64_t out_row_bytes,
                       int64_t rows, int64_t row_elems, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > rows) nthreads = (int)(rows > 0 ? rows : 1);
    pthread_t *th = malloc(sizeof(pthread_t) * nthreads);
    rows_job *jobs = malloc(sizeof(rows_job) * nthreads);
    for (int i = 0; i < nthreads; ++i) {
        rows_job j = {fn, fn_fwht_row, fwht_head_dim, in_is_bf16, (const uint8_t *)in, in_row_bytes,
                      (uint8_t *)out, out_row_bytes, rows * i / nthreads, rows * (i + 1) / nthreads, row_elems};
        jobs[i] = j;
        pthread_create(&th[i], NULL, rows_worker, &jobs[i]);
    }
    for (int i = 0; i < nthreads; ++i) pthread_join(th[i], NULL);
    free(th); free(jobs);
}
