/*
 * CPU oracle of the synthetic Qwen3.5-style decode step: a plain-C
 * restatement of crates/unltd-generation/src/qwen35_forward.rs (step,
 * recr_layer, attn_layer, ffn) and of the f32 kernels it calls in
 * crates/unltd-tensor/src/kernels.rs. Every projection goes through
 * ora_gemv_quant_q8k, as the reference's forward does.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the GPU decode step and the CPU
 * baseline of the decode benchmark. The library never links it.
 *
 * One deliberate restatement: the reference's f32 exp/log come from the
 * platform libm (platform-specific in the last bit). Here they are the
 * correctly rounded f32 values, computed through double precision; the GPU
 * uses the same definition, so both sides agree bit for bit.
 */
#include "forward_ref.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#include "quants_ref.h"

float ora_expf(float x) { return (float)exp((double)x); }
float ora_logf(float x) { return (float)log((double)x); }

/* kernels.rs:61-78: squares in f32, sequential f64 sum, mean rounded to f32,
 * scale = 1/sqrtf(mean + eps), out = (x*scale)*w with two f32 multiplies. */
void ora_rmsnorm(float *out, const float *x, const float *w, int n, float eps) {
    if (n == 0) return;
    double sum = 0.0;
    for (int i = 0; i < n; i++) {
        float sq = x[i] * x[i];
        sum += (double)sq;
    }
    float mean = (float)(sum / (double)n);
    float scale = 1.0f / sqrtf(mean + eps);
    for (int i = 0; i < n; i++) {
        float norm = x[i] * scale;
        out[i] = norm * w[i];
    }
}

/* kernels.rs:198-203 sigmoid, 206-211 silu, 217-226 softplus, 174-182 swiglu */
static inline float sigmoid1(float x) { return 1.0f / (1.0f + ora_expf(-x)); }
static inline float silu1(float x) { return x / (1.0f + ora_expf(-x)); }
static inline float softplus1(float x) { return x > 20.0f ? x : ora_logf(1.0f + ora_expf(x)); }

void ora_sigmoid(float *out, const float *x, int n) { for (int i = 0; i < n; i++) out[i] = sigmoid1(x[i]); }
void ora_silu(float *out, const float *x, int n) { for (int i = 0; i < n; i++) out[i] = silu1(x[i]); }
void ora_softplus(float *out, const float *x, int n) { for (int i = 0; i < n; i++) out[i] = softplus1(x[i]); }
void ora_swiglu(float *out, const float *g, const float *u, int n) {
    for (int i = 0; i < n; i++) {
        float t = g[i];
        float s = t / (1.0f + ora_expf(-t));
        out[i] = s * u[i];
    }
}

/* kernels.rs:265-310: x is ncs rows of `channels`, kernel[tau*channels + c];
 * out has n_t = ncs - (d_conv - 1) rows; f32 multiply-add in tau order. */
void ora_ssm_conv(float *out, const float *x, int ncs, const float *kernel, int d_conv, int channels) {
    int n_t = ncs - (d_conv - 1);
    for (int t = 0; t < n_t; t++)
        for (int c = 0; c < channels; c++) {
            float sumf = 0.0f;
            for (int tau = 0; tau < d_conv; tau++) {
                float p = x[(size_t)(t + tau) * channels + c] * kernel[(size_t)tau * channels + c];
                sumf = sumf + p;
            }
            out[(size_t)t * channels + c] = sumf;
        }
}

/* kernels.rs:236-252: sequential f64 sum of f32 squares; scale =
 * 1 / max(sqrtf((float)sum), eps); y = x*scale. */
void ora_l2_norm_rows(float *data, int rows, int dim, float eps) {
    for (int r = 0; r < rows; r++) {
        float *row = data + (size_t)r * dim;
        double sum = 0.0;
        for (int i = 0; i < dim; i++) {
            float sq = row[i] * row[i];
            sum += (double)sq;
        }
        float nrm = sqrtf((float)sum);
        if (nrm < eps) nrm = eps;
        float scale = 1.0f / nrm;
        for (int i = 0; i < dim; i++) row[i] = row[i] * scale;
    }
}

/* kernels.rs:316-372: one fused GatedDeltaNet step of one v-head. */
void ora_gdn_step(float *state, float *out, const float *q, const float *k, const float *v, float gate,
                  float beta, float scale, int dim) {
    float g_exp = ora_expf(gate);
    for (int i = 0; i < dim * dim; i++) state[i] = state[i] * g_exp;
    float *d = (float *)malloc(sizeof(float) * dim);
    for (int j = 0; j < dim; j++) {
        double sum = 0.0;
        for (int i = 0; i < dim; i++) {
            float p = state[i * dim + j] * k[i];
            sum += (double)p;
        }
        float s = (float)sum;
        float t = v[j] - s;
        d[j] = t * beta;
    }
    for (int j = 0; j < dim; j++)
        for (int i = 0; i < dim; i++) {
            float p = k[i] * d[j];
            state[i * dim + j] = state[i * dim + j] + p;
        }
    for (int j = 0; j < dim; j++) {
        double sum = 0.0;
        for (int i = 0; i < dim; i++) {
            float p = state[i * dim + j] * q[i];
            sum += (double)p;
        }
        out[j] = (float)sum * scale;
    }
    free(d);
}

/* kernels.rs:381-400: IMROPE, pairs (ic, ic + n_rot/2) rotate when ic % 3 == 0. */
void ora_rope_imrope(float *x, int n_rot, double theta_scale, int pos) {
    int half = n_rot / 2;
    double angle = (double)pos;
    for (int ic = 0; ic < half; ic++) {
        if (ic % 3 == 0) {
            double s = sin(angle), c = cos(angle);
            double x0 = x[ic], x1 = x[ic + half];
            x[ic] = (float)fma(c, x0, -(s * x1));
            x[ic + half] = (float)fma(s, x0, c * x1);
        }
        angle = angle * theta_scale;
    }
}

/* kernels.rs:157-168 */
void ora_softmax(float *out, const float *x, int n, float scale) {
    if (n == 0) return;
    float max = -INFINITY;
    for (int i = 0; i < n; i++) max = fmaxf(max, x[i]);
    double *e = (double *)calloc((size_t)n, sizeof(double));
    float *ef = (float *)calloc((size_t)n, sizeof(float));
    for (int i = 0; i < n; i++) {
        float t = (x[i] - max) * scale;
        ef[i] = ora_expf(t);
        e[i] = (double)ef[i];
    }
    double sum = ora_pairwise_sum_f64(e, n);
    for (int i = 0; i < n; i++) out[i] = (float)((double)ef[i] / sum);
    free(e);
    free(ef);
}

/* ---------------------------------------------------------------------- */

static size_t rb(int dtype, int n) { return ora_row_bytes(dtype, (size_t)n); }

/* 0: every projection through gemv_quant_q8k, as the reference's forward
 * does. 1: through gemv_quant (f64 dots rounded once to f32) instead, to
 * measure how far the reference's own Q8_K activation quantization moves
 * the hidden state (the yardstick for sharded runs, whose rank-order sums
 * move it too). Test infrastructure only. */
static int g_exact_gemv = 0;

void ora_forward_exact_gemv(int on) { g_exact_gemv = on; }

static void gemv(float *out, const float *x, const uint8_t *w, int dtype, int din, int dout, int nthreads) {
    if (g_exact_gemv)
        ora_gemv_quant(out, x, w, rb(dtype, din) * (size_t)dout, (size_t)din, (size_t)dout, dtype, nthreads);
    else
        ora_gemv_quant_q8k(out, x, w, rb(dtype, din) * (size_t)dout, (size_t)din, (size_t)dout, dtype, nthreads);
}

/* Tensor parallelism over `g_split` ranks (test infrastructure): the
 * projections split by input columns (ffn_down, ssm_out, attn_output) as the
 * ranks compute them: rank r takes columns [r din / W, (r + 1) din / W) of
 * x and of every row (its own gemv_quant_q8k over that slice, the chain over
 * its blocks only), and the partial outputs are summed in rank order in f32,
 * y = ((p0 + p1) + p2) + ... Every other part of the step is the same on one
 * GPU and on W (heads, rows and vocab rows split whole). 1: one device. */
static int g_split = 1;

void ora_forward_row_split(int world) { g_split = world < 1 ? 1 : world; }

static void gemv_rowsplit(float *out, const float *x, const uint8_t *w, int dtype, int din, int dout, int nthreads) {
    if (g_split == 1 || g_exact_gemv) {
        gemv(out, x, w, dtype, din, dout, nthreads);
        return;
    }
    const int cols = din / g_split;
    const size_t rbf = rb(dtype, din), rbs = rb(dtype, cols);
    uint8_t *ws = (uint8_t *)malloc(rbs * (size_t)dout);
    float *part = (float *)malloc(sizeof(float) * dout);
    for (int r = 0; r < g_split; r++) {
        const size_t off = rb(dtype, cols * r);  /* the slice's first byte in a row */
        for (int row = 0; row < dout; row++) memcpy(ws + rbs * row, w + rbf * row + off, rbs);
        ora_gemv_quant_q8k(part, x + (size_t)cols * r, ws, rbs * (size_t)dout, (size_t)cols, (size_t)dout, dtype,
                           nthreads);
        for (int i = 0; i < dout; i++) out[i] = r == 0 ? part[i] : out[i] + part[i];
    }
    free(ws);
    free(part);
}

#define T(L, f) (tensors[ORA_T_GLOBALS + (L) * ORA_T_PER_LAYER + (f)])
#define D(L, f) (dtypes[ORA_T_GLOBALS + (L) * ORA_T_PER_LAYER + (f)])

/* qwen35_forward.rs:713-768 */
static void ffn(const ora_model_cfg *c, void **tensors, const int *dtypes, int il, const float *residual,
                float *f, int nthreads) {
    int n = c->n_embd, nff = c->n_ff;
    float *p = (float *)malloc(sizeof(float) * n);
    float *g = (float *)malloc(sizeof(float) * nff);
    float *u = (float *)malloc(sizeof(float) * nff);
    ora_rmsnorm(p, residual, (const float *)T(il, ORA_POST_NORM), n, c->rms_eps);
    gemv(g, p, (const uint8_t *)T(il, ORA_FFN_GATE), D(il, ORA_FFN_GATE), n, nff, nthreads);
    gemv(u, p, (const uint8_t *)T(il, ORA_FFN_UP), D(il, ORA_FFN_UP), n, nff, nthreads);
    ora_swiglu(g, g, u, nff);
    gemv_rowsplit(f, g, (const uint8_t *)T(il, ORA_FFN_DOWN), D(il, ORA_FFN_DOWN), nff, n, nthreads);
    free(p);
    free(g);
    free(u);
}

/* qwen35_forward.rs:333-543 */
static void recr_layer(const ora_model_cfg *c, void **tensors, const int *dtypes, int il, float *conv_ring,
                       float *gdn_state, const float *x_in, float *l_out, int nthreads) {
    int n = c->n_embd, nqk = c->group_count, hd = c->d_inner / (2 * c->group_count);
    int nv = c->d_inner / hd, dconv = 2 * c->d_inner, K = c->conv_kernel;
    float eps = c->rms_eps;
    float *x = (float *)malloc(sizeof(float) * n);
    float *qkv = (float *)malloc(sizeof(float) * dconv);
    float *z = (float *)malloc(sizeof(float) * n);
    float *beta_raw = (float *)malloc(sizeof(float) * nv);
    float *alpha = (float *)malloc(sizeof(float) * nv);
    ora_rmsnorm(x, x_in, (const float *)T(il, ORA_ATTN_NORM), n, eps);
    gemv(qkv, x, (const uint8_t *)T(il, ORA_ATTN_QKV), D(il, ORA_ATTN_QKV), n, dconv, nthreads);
    gemv(z, x, (const uint8_t *)T(il, ORA_ATTN_GATE), D(il, ORA_ATTN_GATE), n, n, nthreads);
    gemv(beta_raw, x, (const uint8_t *)T(il, ORA_SSM_BETA), D(il, ORA_SSM_BETA), n, nv, nthreads);
    gemv(alpha, x, (const uint8_t *)T(il, ORA_SSM_ALPHA), D(il, ORA_SSM_ALPHA), n, nv, nthreads);
    const float *dtb = (const float *)T(il, ORA_SSM_DT_BIAS), *ssa = (const float *)T(il, ORA_SSM_A);
    float *beta = (float *)malloc(sizeof(float) * nv), *gate = (float *)malloc(sizeof(float) * nv);
    for (int h = 0; h < nv; h++) {
        beta[h] = sigmoid1(beta_raw[h]);
        float biased = alpha[h] + dtb[h];
        gate[h] = softplus1(biased) * ssa[h];
    }
    /* conv over the window [ring rows 0..K-2, qkv]; the GGUF kernel is
     * [channel][tau], ssm_conv takes [tau][channel] (qwen35_forward.rs:421-437) */
    const float *kraw = (const float *)T(il, ORA_SSM_CONV1D);
    float *win = (float *)malloc(sizeof(float) * (size_t)K * dconv);
    float *kern = (float *)malloc(sizeof(float) * (size_t)K * dconv);
    memcpy(win, conv_ring, sizeof(float) * (size_t)(K - 1) * dconv);
    memcpy(win + (size_t)(K - 1) * dconv, qkv, sizeof(float) * dconv);
    for (int ch = 0; ch < dconv; ch++)
        for (int tau = 0; tau < K; tau++) kern[(size_t)tau * dconv + ch] = kraw[(size_t)ch * K + tau];
    float *conv_out = (float *)malloc(sizeof(float) * dconv);
    ora_ssm_conv(conv_out, win, K, kern, K, dconv);
    float *mix = (float *)malloc(sizeof(float) * dconv);
    ora_silu(mix, conv_out, dconv);
    free(win), free(kern), free(conv_out);
    memmove(conv_ring, conv_ring + dconv, sizeof(float) * (size_t)(K - 2) * dconv);
    memcpy(conv_ring + (size_t)(K - 2) * dconv, qkv, sizeof(float) * dconv);
    float *qc = mix, *kc = mix + nqk * hd, *vc = mix + 2 * nqk * hd;
    ora_l2_norm_rows(qc, nqk, hd, eps);
    ora_l2_norm_rows(kc, nqk, hd, eps);
    float *gdn_out = (float *)malloc(sizeof(float) * n);
    float scale = 1.0f / sqrtf((float)hd);
    for (int h = 0; h < nv; h++) {
        int qk = h % nqk;
        ora_gdn_step(gdn_state + (size_t)h * hd * hd, gdn_out + (size_t)h * hd, qc + (size_t)qk * hd,
                     kc + (size_t)qk * hd, vc + (size_t)h * hd, gate[h], beta[h], scale, hd);
    }
    float *y = (float *)malloc(sizeof(float) * n);
    const float *ssmn = (const float *)T(il, ORA_SSM_NORM);
    for (int h = 0; h < nv; h++) ora_rmsnorm(y + (size_t)h * hd, gdn_out + (size_t)h * hd, ssmn, hd, eps);
    for (int i = 0; i < n; i++) y[i] = y[i] * silu1(z[i]);
    float *attn_out = (float *)malloc(sizeof(float) * n);
    gemv_rowsplit(attn_out, y, (const uint8_t *)T(il, ORA_SSM_OUT), D(il, ORA_SSM_OUT), n, n, nthreads);
    float *residual = (float *)malloc(sizeof(float) * n);
    for (int i = 0; i < n; i++) residual[i] = x_in[i] + attn_out[i];
    float *f = (float *)malloc(sizeof(float) * n);
    ffn(c, tensors, dtypes, il, residual, f, nthreads);
    for (int i = 0; i < n; i++) l_out[i] = residual[i] + f[i];
    free(x), free(qkv), free(z), free(beta_raw), free(alpha), free(beta), free(gate), free(mix);
    free(gdn_out), free(y), free(attn_out), free(residual), free(f);
}

/* qwen35_forward.rs:546-710 */
static void attn_layer(const ora_model_cfg *c, void **tensors, const int *dtypes, int il, float *kcache,
                       float *vcache, int pos, const float *x_in, float *l_out, int nthreads) {
    int n = c->n_embd, nh = c->n_head, nhkv = c->n_head_kv, hdv = c->head_dim;
    float eps = c->rms_eps;
    int kvlen = nhkv * hdv;
    float *x = (float *)malloc(sizeof(float) * n);
    ora_rmsnorm(x, x_in, (const float *)T(il, ORA_ATTN_NORM), n, eps);
    float *qfull = (float *)malloc(sizeof(float) * 2 * nh * hdv);
    gemv(qfull, x, (const uint8_t *)T(il, ORA_ATTN_Q), D(il, ORA_ATTN_Q), n, 2 * nh * hdv, nthreads);
    float *q = (float *)malloc(sizeof(float) * nh * hdv), *gt = (float *)malloc(sizeof(float) * nh * hdv);
    const float *qnw = (const float *)T(il, ORA_ATTN_Q_NORM);
    for (int h = 0; h < nh; h++) {
        ora_rmsnorm(q + (size_t)h * hdv, qfull + (size_t)h * 2 * hdv, qnw, hdv, eps);
        memcpy(gt + (size_t)h * hdv, qfull + (size_t)h * 2 * hdv + hdv, sizeof(float) * hdv);
    }
    float *k = (float *)malloc(sizeof(float) * kvlen), *kn = (float *)malloc(sizeof(float) * kvlen);
    gemv(k, x, (const uint8_t *)T(il, ORA_ATTN_K), D(il, ORA_ATTN_K), n, kvlen, nthreads);
    const float *knw = (const float *)T(il, ORA_ATTN_K_NORM);
    for (int h = 0; h < nhkv; h++) ora_rmsnorm(kn + (size_t)h * hdv, k + (size_t)h * hdv, knw, hdv, eps);
    float *v = (float *)malloc(sizeof(float) * kvlen);
    gemv(v, x, (const uint8_t *)T(il, ORA_ATTN_V), D(il, ORA_ATTN_V), n, kvlen, nthreads);
    for (int h = 0; h < nh; h++) ora_rope_imrope(q + (size_t)h * hdv, c->n_rot, c->theta_scale, pos);
    for (int h = 0; h < nhkv; h++) ora_rope_imrope(kn + (size_t)h * hdv, c->n_rot, c->theta_scale, pos);
    memcpy(kcache + (size_t)pos * kvlen, kn, sizeof(float) * kvlen);
    memcpy(vcache + (size_t)pos * kvlen, v, sizeof(float) * kvlen);
    int nctx = pos + 1;
    float *scores = (float *)malloc(sizeof(float) * nctx), *soft = (float *)malloc(sizeof(float) * nctx);
    float *attn = (float *)malloc(sizeof(float) * n);
    float kq = 1.0f / sqrtf((float)c->head_dim);
    for (int h = 0; h < nh; h++) {
        int kv = h / (nh / nhkv);
        for (int p = 0; p < nctx; p++)
            scores[p] = (float)ora_dot_f32(q + (size_t)h * hdv, kcache + (size_t)p * kvlen + (size_t)kv * hdv, hdv);
        ora_softmax(soft, scores, nctx, kq);
        for (int i = 0; i < hdv; i++) {
            double sum = 0.0;
            for (int p = 0; p < nctx; p++) {
                double t = (double)soft[p] * (double)vcache[(size_t)p * kvlen + (size_t)kv * hdv + i];
                sum = sum + t;
            }
            attn[(size_t)h * hdv + i] = (float)sum;
        }
    }
    float *gated = (float *)malloc(sizeof(float) * n);
    for (int i = 0; i < n; i++) gated[i] = attn[i] * sigmoid1(gt[i]);
    float *attn_out = (float *)malloc(sizeof(float) * n);
    gemv_rowsplit(attn_out, gated, (const uint8_t *)T(il, ORA_ATTN_OUT), D(il, ORA_ATTN_OUT), n, n, nthreads);
    float *residual = (float *)malloc(sizeof(float) * n);
    for (int i = 0; i < n; i++) residual[i] = x_in[i] + attn_out[i];
    float *f = (float *)malloc(sizeof(float) * n);
    ffn(c, tensors, dtypes, il, residual, f, nthreads);
    for (int i = 0; i < n; i++) l_out[i] = residual[i] + f[i];
    free(x), free(qfull), free(q), free(gt), free(k), free(kn), free(v), free(scores), free(soft), free(attn);
    free(gated), free(attn_out), free(residual), free(f);
}

int ora_decode_token(const ora_model_cfg *c, void **tensors, const int *dtypes, float **conv, float **gdn,
                     float **kcache, float **vcache, int position, uint32_t token, float *logits, float *hidden_out,
                     int nthreads) {
    int n = c->n_embd;
    if (token >= (uint32_t)c->vocab || position >= c->ctx) return ORA_ERR_LEN;
    float *x = (float *)malloc(sizeof(float) * n), *y = (float *)malloc(sizeof(float) * n);
    /* min_forward.rs:160-184: the embedding row, dequantized (Q4_K) */
    const uint8_t *emb = (const uint8_t *)tensors[ORA_T_TOK_EMBD];
    size_t erb = rb(dtypes[ORA_T_TOK_EMBD], n);
    ora_dequantize_q4_k(x, emb + (size_t)token * erb, (size_t)n);
    int ir = 0, ia = 0;
    for (int il = 0; il < c->n_layer; il++) {
        if ((il + 1) % c->full_attn_interval == 0) {
            attn_layer(c, tensors, dtypes, il, kcache[ia], vcache[ia], position, x, y, nthreads);
            ia++;
        } else {
            recr_layer(c, tensors, dtypes, il, conv[ir], gdn[ir], x, y, nthreads);
            ir++;
        }
        float *t = x;
        x = y;
        y = t;
    }
    if (hidden_out) memcpy(hidden_out, x, sizeof(float) * n);
    /* qwen35_forward.rs:272-281 output norm, min_forward.rs:210-266 LM head */
    ora_rmsnorm(y, x, (const float *)tensors[ORA_T_OUTPUT_NORM], n, c->rms_eps);
    gemv(logits, y, (const uint8_t *)tensors[ORA_T_OUTPUT], dtypes[ORA_T_OUTPUT], n, c->vocab, nthreads);
    free(x);
    free(y);
    return ORA_OK;
}
