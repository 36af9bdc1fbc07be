/*
 * CPU oracle: plain-C restatement of the reference's quantized kernels.
 * TEST INFRASTRUCTURE ONLY (see quants_ref.h). Each function cites the
 * reference lines it restates (paths within the reference project).
 */
#include "quants_ref.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* quants.rs:44-72 — canonical IEEE half -> f32 by bit manipulation. */
float ora_f16_to_f32(uint16_t hh) {
    uint32_t h = hh;
    uint32_t sign = (h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1F;
    uint32_t frac = h & 0x3FF;
    uint32_t bits;
    if (exp == 0) {
        if (frac == 0) {
            bits = sign;
        } else {
            uint32_t e = 113, m = frac;
            while ((m & 0x400) == 0) {
                m <<= 1;
                e -= 1;
            }
            bits = sign | (e << 23) | ((m & 0x3FF) << 13);
        }
    } else if (exp == 0x1F) {
        bits = frac == 0 ? (sign | 0x7F800000u) : (sign | 0x7FC00000u);
    } else {
        bits = sign | ((exp + 112) << 23) | (frac << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static inline uint16_t f16_at(const uint8_t *b) { return (uint16_t)(b[0] | (b[1] << 8)); }

/* quants.rs:92-102 — 6-bit scale/min of group g from the 12 packed bytes. */
void ora_scale_min_k4(const uint8_t *s, int g, uint8_t *sc, uint8_t *m) {
    if (g < 4) {
        *sc = s[g] & 63;
        *m = s[g + 4] & 63;
    } else {
        *sc = (uint8_t)((s[g + 4] & 0xF) | ((s[g - 4] >> 6) << 4));
        *m = (uint8_t)((s[g + 4] >> 4) | ((s[g] >> 6) << 4));
    }
}

/* kernels.rs:27-42 — level-by-level pairs ((a0+a1)+(a2+a3))..., an odd tail
 * carries to the next level unpaired, the empty sum is 0. Same additions in
 * the same order; the levels are compacted in place instead of reallocated. */
double ora_pairwise_sum_f64(const double *v, size_t n) {
    if (n == 0) return 0.0;
    double stackbuf[512];
    double *lv = n <= 512 ? stackbuf : (double *)malloc(n * sizeof(double));
    memcpy(lv, v, n * sizeof(double));
    size_t len = n;
    while (len > 1) {
        size_t o = 0, i = 0;
        for (; i + 1 < len; i += 2) lv[o++] = lv[i] + lv[i + 1];
        if (i < len) lv[o++] = lv[i];
        len = o;
    }
    double r = lv[0];
    if (lv != stackbuf) free(lv);
    return r;
}

/* quants.rs:106-114 */
double ora_dot_f32(const float *x, const float *w, size_t n) {
    double *p = (double *)malloc((n ? n : 1) * sizeof(double));
    for (size_t i = 0; i < n; i++) p[i] = (double)x[i] * (double)w[i];
    double r = ora_pairwise_sum_f64(p, n);
    free(p);
    return r;
}

/* quants.rs:132-156 — exact f64 weight (d*sc)*nib - (dmin*m), f64 product,
 * pairwise sum. Element e of a block: group g=e/32, byte qs[32*(g/2)+e%32],
 * low nibble for even g. */
double ora_dot_q4_k(const float *x, const uint8_t *w, size_t n) {
    if (n % ORA_QK_K) return NAN;
    double *p = (double *)malloc((n ? n : 1) * sizeof(double));
    size_t nb = n / ORA_QK_K;
    for (size_t b = 0; b < nb; b++) {
        const uint8_t *blk = w + b * ORA_BLOCK_Q4_K;
        double d = (double)ora_f16_to_f32(f16_at(blk));
        double dmin = (double)ora_f16_to_f32(f16_at(blk + 2));
        const uint8_t *scales = blk + 4, *qs = blk + 16;
        for (int e = 0; e < ORA_QK_K; e++) {
            int g = e / 32;
            uint8_t sc, m;
            ora_scale_min_k4(scales, g, &sc, &m);
            uint8_t byte = qs[32 * (g / 2) + (e % 32)];
            uint8_t nib = (g % 2 == 0) ? (byte & 0xF) : (byte >> 4);
            double wv = (d * (double)sc) * (double)nib - (dmin * (double)m);
            p[b * ORA_QK_K + e] = (double)x[b * ORA_QK_K + e] * wv;
        }
    }
    double r = ora_pairwise_sum_f64(p, n);
    free(p);
    return r;
}

/* quants.rs:171-200 — block ql[128] | qh[64] | scales i8[16] | d f16 (at 208).
 * q = (nib | hi2<<4) - 32, w = d*(sc*q), exact in f64. */
static inline int q6_raw(const uint8_t *blk, int e) {
    const uint8_t *ql = blk, *qh = blk + 128;
    uint8_t byte = ql[64 * (e / 128) + (e % 64)];
    int nib = ((e / 64) % 2 == 0) ? (byte & 0xF) : (byte >> 4);
    int hi2 = (qh[(e % 32) + 32 * (e / 128)] >> (2 * ((e % 128) / 32))) & 3;
    return nib | (hi2 << 4);
}

double ora_dot_q6_k(const float *x, const uint8_t *w, size_t n) {
    if (n % ORA_QK_K) return NAN;
    double *p = (double *)malloc((n ? n : 1) * sizeof(double));
    size_t nb = n / ORA_QK_K;
    for (size_t b = 0; b < nb; b++) {
        const uint8_t *blk = w + b * ORA_BLOCK_Q6_K;
        const int8_t *scales = (const int8_t *)(blk + 192);
        double d = (double)ora_f16_to_f32(f16_at(blk + 208));
        for (int e = 0; e < ORA_QK_K; e++) {
            int q = q6_raw(blk, e) - 32;
            double wv = d * ((double)scales[e / 16] * (double)q);
            p[b * ORA_QK_K + e] = (double)x[b * ORA_QK_K + e] * wv;
        }
    }
    double r = ora_pairwise_sum_f64(p, n);
    free(p);
    return r;
}

/* Q8_0 has no kernel in the reference (gemv_quant panics for it at
 * quants.rs:446). Restated format: 34-byte blocks of f16 d then 32 int8 q
 * (row sizing min_forward.rs:56-63), w = d*q (exact), under the same f64
 * contract as dot_q4_k. */
double ora_dot_q8_0(const float *x, const uint8_t *w, size_t n) {
    if (n % ORA_QK8_0) return NAN;
    double *p = (double *)malloc((n ? n : 1) * sizeof(double));
    size_t nb = n / ORA_QK8_0;
    for (size_t b = 0; b < nb; b++) {
        const uint8_t *blk = w + b * ORA_BLOCK_Q8_0;
        double d = (double)ora_f16_to_f32(f16_at(blk));
        const int8_t *q = (const int8_t *)(blk + 2);
        for (int e = 0; e < ORA_QK8_0; e++)
            p[b * ORA_QK8_0 + e] = (double)x[b * ORA_QK8_0 + e] * (d * (double)q[e]);
    }
    double r = ora_pairwise_sum_f64(p, n);
    free(p);
    return r;
}

/* quants.rs:230-233 — magic-number rounding, ties to even. */
int32_t ora_nearest_int(float f) {
    float val = f + 12582912.0f;
    uint32_t bits;
    memcpy(&bits, &val, 4);
    return (int32_t)(bits & 0x007FFFFF) - 0x00400000;
}

/* quants.rs:250-290 — per 256: signed value at the first strict argmax of
 * |x|; amax == 0 gives d = 0, qs = 0, bsums = 0; otherwise
 * iscale = -127/max, qs = min(127, nearest_int(iscale*x)), bsums = sums of 16,
 * d = 1/iscale. */
int ora_quantize_q8_k(const float *x, size_t n, ora_q8k_block *out) {
    if (n % ORA_QK_K) return ORA_ERR_DIM;
    for (size_t b = 0; b < n / ORA_QK_K; b++) {
        const float *c = x + b * ORA_QK_K;
        ora_q8k_block *o = &out[b];
        float max = 0.0f, amax = 0.0f;
        for (int j = 0; j < ORA_QK_K; j++) {
            float ax = fabsf(c[j]);
            if (ax > amax) {
                amax = ax;
                max = c[j];
            }
        }
        memset(o, 0, sizeof(*o));
        if (amax == 0.0f) continue;
        float iscale = -127.0f / max;
        for (int j = 0; j < ORA_QK_K; j++) {
            int32_t v = ora_nearest_int(iscale * c[j]);
            o->qs[j] = (int8_t)(v < 127 ? v : 127);
        }
        for (int j = 0; j < 16; j++) {
            int32_t s = 0;
            for (int i = 0; i < 16; i++) s += o->qs[16 * j + i];
            o->bsums[j] = s;
        }
        o->d = 1.0f / iscale;
    }
    return ORA_OK;
}

/* quants.rs:312-360 — ggml generic q4_K x q8_K: eight i32 lanes by e%8,
 * per-block f32 epilogue with separate mul and add, dmin term subtracted per
 * block, final sequential s = sumf + sums[0] + ... + sums[7]. */
float ora_dot_q4_k_q8_k(const ora_q8k_block *x, const uint8_t *w, size_t nblocks) {
    float sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float sumf = 0.0f;
    for (size_t b = 0; b < nblocks; b++) {
        const ora_q8k_block *q8 = &x[b];
        const uint8_t *blk = w + b * ORA_BLOCK_Q4_K;
        uint8_t sc[8], m[8];
        for (int g = 0; g < 8; g++) ora_scale_min_k4(blk + 4, g, &sc[g], &m[g]);
        const uint8_t *qs = blk + 16;
        int32_t sumi[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int e = 0; e < ORA_QK_K; e++) {
            int pos = e % 64;
            uint8_t byte = qs[32 * (e / 64) + pos % 32];
            int a = pos < 32 ? (byte & 0xF) : (byte >> 4);
            sumi[e % 8] += (int32_t)sc[e / 32] * a * (int32_t)q8->qs[e];
        }
        float d = q8->d * ora_f16_to_f32(f16_at(blk));
        for (int k = 0; k < 8; k++) {
            float t = d * (float)sumi[k];
            sums[k] = sums[k] + t;
        }
        int32_t minsum = 0;
        for (int g = 0; g < 16; g++) minsum += q8->bsums[g] * (int32_t)m[g / 2];
        float dmin = ora_f16_to_f32(f16_at(blk + 2)) * q8->d;
        float t = dmin * (float)minsum;
        sumf = sumf - t;
    }
    float s = sumf;
    for (int k = 0; k < 8; k++) s = s + sums[k];
    return s;
}

/* quants.rs:371-412 — ggml generic q6_K x q8_K: a = raw6 - 32 inside the
 * lane sums, signed i8 scales per 16, s = sums[0] + ... + sums[7] from 0. */
float ora_dot_q6_k_q8_k(const ora_q8k_block *x, const uint8_t *w, size_t nblocks) {
    float sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (size_t b = 0; b < nblocks; b++) {
        const ora_q8k_block *q8 = &x[b];
        const uint8_t *blk = w + b * ORA_BLOCK_Q6_K;
        const uint8_t *ql = blk, *qh = blk + 128;
        const int8_t *scales = (const int8_t *)(blk + 192);
        int32_t sumi[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int e = 0; e < ORA_QK_K; e++) {
            int pos = e % 128;
            uint8_t byte = ql[64 * (e / 128) + pos % 64];
            int nib = pos < 64 ? (byte & 0xF) : (byte >> 4);
            int hi2 = (qh[32 * (e / 128) + pos % 32] >> (2 * (pos / 32))) & 3;
            int a = (nib | (hi2 << 4)) - 32;
            sumi[e % 8] += (int32_t)scales[e / 16] * a * (int32_t)q8->qs[e];
        }
        float d = q8->d * ora_f16_to_f32(f16_at(blk + 208));
        for (int k = 0; k < 8; k++) {
            float t = d * (float)sumi[k];
            sums[k] = sums[k] + t;
        }
    }
    float s = 0.0f;
    for (int k = 0; k < 8; k++) s = s + sums[k];
    return s;
}

size_t ora_row_bytes(int dtype, size_t dim_in) {
    switch (dtype) {
    case ORA_F32: return dim_in * 4;
    case ORA_Q4K: return dim_in % ORA_QK_K ? 0 : dim_in / ORA_QK_K * ORA_BLOCK_Q4_K;
    case ORA_Q6K: return dim_in % ORA_QK_K ? 0 : dim_in / ORA_QK_K * ORA_BLOCK_Q6_K;
    case ORA_Q8_0: return dim_in % ORA_QK8_0 ? 0 : dim_in / ORA_QK8_0 * ORA_BLOCK_Q8_0;
    default: return 0;
    }
}

/* ---- row-parallel driver: contiguous chunks of output rows per thread ---- */

typedef struct {
    int kind; /* 0 exact f32 out, 1 q8k, 2 exact f64 out */
    void *out;
    const float *x;
    const uint8_t *w;
    const ora_q8k_block *xq;
    size_t dim_in, row_bytes, r0, r1;
    int dtype;
} row_job;

static double exact_row(const row_job *j, const uint8_t *row) {
    switch (j->dtype) {
    case ORA_F32: return ora_dot_f32(j->x, (const float *)row, j->dim_in);
    case ORA_Q4K: return ora_dot_q4_k(j->x, row, j->dim_in);
    case ORA_Q6K: return ora_dot_q6_k(j->x, row, j->dim_in);
    default: return ora_dot_q8_0(j->x, row, j->dim_in);
    }
}

static void *row_worker(void *arg) {
    row_job *j = (row_job *)arg;
    for (size_t r = j->r0; r < j->r1; r++) {
        const uint8_t *row = j->w + r * j->row_bytes;
        if (j->kind == 0) {
            ((float *)j->out)[r] = (float)exact_row(j, row);
        } else if (j->kind == 2) {
            ((double *)j->out)[r] = exact_row(j, row);
        } else {
            size_t nb = j->dim_in / ORA_QK_K;
            ((float *)j->out)[r] = j->dtype == ORA_Q4K ? ora_dot_q4_k_q8_k(j->xq, row, nb)
                                                       : ora_dot_q6_k_q8_k(j->xq, row, nb);
        }
    }
    return NULL;
}

static void run_rows(row_job proto, size_t dim_out, int nthreads) {
    if (nthreads <= 1 || dim_out < 2) {
        proto.r0 = 0;
        proto.r1 = dim_out;
        row_worker(&proto);
        return;
    }
    if ((size_t)nthreads > dim_out) nthreads = (int)dim_out;
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * nthreads);
    row_job *jobs = (row_job *)malloc(sizeof(row_job) * nthreads);
    size_t per = (dim_out + nthreads - 1) / nthreads;
    int started = 0;
    for (int t = 0; t < nthreads; t++) {
        jobs[t] = proto;
        jobs[t].r0 = t * per;
        jobs[t].r1 = (t + 1) * per < dim_out ? (t + 1) * per : dim_out;
        if (jobs[t].r0 >= jobs[t].r1) break;
        if (pthread_create(&th[t], NULL, row_worker, &jobs[t]) != 0) {
            row_worker(&jobs[t]);
            jobs[t].r0 = jobs[t].r1; /* mark done inline */
            th[t] = 0;
        }
        started = t + 1;
    }
    for (int t = 0; t < started; t++)
        if (th[t]) pthread_join(th[t], NULL);
    free(th);
    free(jobs);
}

/* quants.rs:422-466: F32, Q4_K, Q6_K (and the restated Q8_0). */
static int gemv_exact(void *out, int kind, const float *x, const uint8_t *w, size_t w_len,
                      size_t dim_in, size_t dim_out, int dtype, int nthreads) {
    if (dtype != ORA_F32 && dtype != ORA_Q4K && dtype != ORA_Q6K && dtype != ORA_Q8_0)
        return ORA_ERR_DTYPE;
    size_t rb = ora_row_bytes(dtype, dim_in);
    if (rb == 0 && dim_in != 0) return ORA_ERR_DIM;
    if (w_len != rb * dim_out) return ORA_ERR_LEN;
    row_job j;
    memset(&j, 0, sizeof(j));
    j.kind = kind;
    j.out = out;
    j.x = x;
    j.w = w;
    j.dim_in = dim_in;
    j.row_bytes = rb;
    j.dtype = dtype;
    run_rows(j, dim_out, nthreads);
    return ORA_OK;
}

int ora_gemv_quant(float *out, const float *x, const uint8_t *w, size_t w_len, size_t dim_in,
                   size_t dim_out, int dtype, int nthreads) {
    return gemv_exact(out, 0, x, w, w_len, dim_in, dim_out, dtype, nthreads);
}

int ora_gemv_quant_f64(double *out, const float *x, const uint8_t *w, size_t w_len,
                       size_t dim_in, size_t dim_out, int dtype, int nthreads) {
    return gemv_exact(out, 2, x, w, w_len, dim_in, dim_out, dtype, nthreads);
}

/* quants.rs:474-515: x quantized to Q8_K once, then the q8_K dot per row.
 * Only Q4_K and Q6_K (the reference panics otherwise, :497-499). */
int ora_gemv_quant_q8k(float *out, const float *x, const uint8_t *w, size_t w_len,
                       size_t dim_in, size_t dim_out, int dtype, int nthreads) {
    if (dtype != ORA_Q4K && dtype != ORA_Q6K) return ORA_ERR_DTYPE;
    if (dim_in % ORA_QK_K) return ORA_ERR_DIM;
    size_t rb = ora_row_bytes(dtype, dim_in);
    if (w_len != rb * dim_out) return ORA_ERR_LEN;
    size_t nb = dim_in / ORA_QK_K;
    ora_q8k_block *xq = (ora_q8k_block *)malloc(sizeof(ora_q8k_block) * (nb ? nb : 1));
    ora_quantize_q8_k(x, dim_in, xq);
    row_job j;
    memset(&j, 0, sizeof(j));
    j.kind = 1;
    j.out = out;
    j.x = x;
    j.w = w;
    j.xq = xq;
    j.dim_in = dim_in;
    j.row_bytes = rb;
    j.dtype = dtype;
    run_rows(j, dim_out, nthreads);
    free(xq);
    return ORA_OK;
}

/* quants.rs:534-567: per group pair, d1 = d*sc, m1 = min*m (f32), then
 * d1*(q&0xF) - m1 for 32 elements and d2*(q>>4) - m2 for the next 32. */
int ora_dequantize_q4_k(float *out, const uint8_t *w, size_t n) {
    if (n % ORA_QK_K) return ORA_ERR_DIM;
    size_t e = 0;
    for (size_t b = 0; b < n / ORA_QK_K; b++) {
        const uint8_t *blk = w + b * ORA_BLOCK_Q4_K;
        float d = ora_f16_to_f32(f16_at(blk));
        float mn = ora_f16_to_f32(f16_at(blk + 2));
        const uint8_t *scales = blk + 4, *qs = blk + 16;
        for (int is = 0; is < 8; is += 2) {
            uint8_t sc0, m0, sc1, m1s;
            ora_scale_min_k4(scales, is, &sc0, &m0);
            float d1 = d * (float)sc0, m1 = mn * (float)m0;
            ora_scale_min_k4(scales, is + 1, &sc1, &m1s);
            float d2 = d * (float)sc1, m2 = mn * (float)m1s;
            for (int l = 0; l < 32; l++) {
                float t = d1 * (float)(qs[l] & 0xF);
                out[e++] = t - m1;
            }
            for (int l = 0; l < 32; l++) {
                float t = d2 * (float)(qs[l] >> 4);
                out[e++] = t - m2;
            }
            qs += 32;
        }
    }
    return ORA_OK;
}

/* Q6_K element value of dot_q6_k (quants.rs:186-195), d*(sc*q): the product
 * has at most 23 significant bits, so it is exact in f32. */
int ora_dequantize_q6_k(float *out, const uint8_t *w, size_t n) {
    if (n % ORA_QK_K) return ORA_ERR_DIM;
    for (size_t b = 0; b < n / ORA_QK_K; b++) {
        const uint8_t *blk = w + b * ORA_BLOCK_Q6_K;
        const int8_t *scales = (const int8_t *)(blk + 192);
        double d = (double)ora_f16_to_f32(f16_at(blk + 208));
        for (int e = 0; e < ORA_QK_K; e++) {
            int q = q6_raw(blk, e) - 32;
            out[b * ORA_QK_K + e] = (float)(d * ((double)scales[e / 16] * (double)q));
        }
    }
    return ORA_OK;
}

/* Q8_0 restated: w = f16(d) * q, exact in f32. */
int ora_dequantize_q8_0(float *out, const uint8_t *w, size_t n) {
    if (n % ORA_QK8_0) return ORA_ERR_DIM;
    for (size_t b = 0; b < n / ORA_QK8_0; b++) {
        const uint8_t *blk = w + b * ORA_BLOCK_Q8_0;
        float d = ora_f16_to_f32(f16_at(blk));
        const int8_t *q = (const int8_t *)(blk + 2);
        for (int e = 0; e < ORA_QK8_0; e++) out[b * ORA_QK8_0 + e] = d * (float)q[e];
    }
    return ORA_OK;
}

/* greedy.rs:18-27 — strict '>' keeps the first index of the maximum. */
size_t ora_argmax(const float *v, size_t n) {
    size_t best = 0;
    for (size_t i = 1; i < n; i++)
        if (v[i] > v[best]) best = i;
    return best;
}
