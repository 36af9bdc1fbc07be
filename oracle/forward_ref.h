/*
 * CPU oracle of the Qwen3.5-style hybrid decode step (test infrastructure).
 * Restates crates/unltd-generation/src/qwen35_forward.rs and the f32 kernels
 * of crates/unltd-tensor/src/kernels.rs; see forward_ref.c.
 */
#ifndef ORA_FORWARD_REF_H
#define ORA_FORWARD_REF_H

#include <stddef.h>
#include <stdint.h>

#include "quants_ref.h"

#ifdef __cplusplus
extern "C" {
#endif

/* crates/unltd-architectures/src/qwen35.rs:46-80 (the fields the step uses);
 * theta_scale = powf(freq_base, -2/n_rot) widened to f64 (qwen35.rs:283-285). */
typedef struct {
    int n_layer, n_embd, n_ff, n_head, n_head_kv, head_dim, n_rot;
    int conv_kernel, group_count, d_inner, full_attn_interval, vocab, ctx;
    float rms_eps;
    double theta_scale;
} ora_model_cfg;

/* Tensor slots: globals first, then ORA_T_PER_LAYER per layer. The names are
 * the GGUF tensor names of qwen35_forward.rs:139-221. */
enum {
    ORA_T_TOK_EMBD = 0,    /* token_embd.weight (Q4_K) */
    ORA_T_OUTPUT_NORM = 1, /* output_norm.weight (F32) */
    ORA_T_OUTPUT = 2,      /* output.weight (Q6_K / Q4_K) */
    ORA_T_GLOBALS = 3
};
enum {
    ORA_ATTN_NORM = 0,   /* blk.N.attn_norm.weight */
    ORA_POST_NORM,       /* blk.N.post_attention_norm.weight */
    ORA_FFN_GATE,        /* blk.N.ffn_gate.weight */
    ORA_FFN_UP,          /* blk.N.ffn_up.weight */
    ORA_FFN_DOWN,        /* blk.N.ffn_down.weight */
    ORA_ATTN_Q,          /* blk.N.attn_q.weight (full-attention layers) */
    ORA_ATTN_Q_NORM,     /* blk.N.attn_q_norm.weight */
    ORA_ATTN_K,          /* blk.N.attn_k.weight */
    ORA_ATTN_K_NORM,     /* blk.N.attn_k_norm.weight */
    ORA_ATTN_V,          /* blk.N.attn_v.weight */
    ORA_ATTN_OUT,        /* blk.N.attn_output.weight */
    ORA_ATTN_QKV,        /* blk.N.attn_qkv.weight (recurrent layers) */
    ORA_ATTN_GATE,       /* blk.N.attn_gate.weight */
    ORA_SSM_CONV1D,      /* blk.N.ssm_conv1d.weight, [channel][tau] */
    ORA_SSM_DT_BIAS,     /* blk.N.ssm_dt.bias */
    ORA_SSM_A,           /* blk.N.ssm_a */
    ORA_SSM_BETA,        /* blk.N.ssm_beta.weight */
    ORA_SSM_ALPHA,       /* blk.N.ssm_alpha.weight */
    ORA_SSM_NORM,        /* blk.N.ssm_norm.weight */
    ORA_SSM_OUT,         /* blk.N.ssm_out.weight */
    ORA_T_PER_LAYER
};

float ora_expf(float x);
float ora_logf(float x);
void ora_rmsnorm(float *out, const float *x, const float *w, int n, float eps);
void ora_l2_norm_rows(float *data, int rows, int dim, float eps);
void ora_gdn_step(float *state, float *out, const float *q, const float *k, const float *v, float gate,
                  float beta, float scale, int dim);
void ora_rope_imrope(float *x, int n_rot, double theta_scale, int pos);
void ora_softmax(float *out, const float *x, int n, float scale);
void ora_sigmoid(float *out, const float *x, int n);
void ora_silu(float *out, const float *x, int n);
void ora_softplus(float *out, const float *x, int n);
void ora_swiglu(float *out, const float *g, const float *u, int n);
void ora_ssm_conv(float *out, const float *x, int ncs, const float *kernel, int d_conv, int channels);

/* One token through all layers (qwen35_forward.rs:295-330), then the output
 * norm and the LM head (min_forward.rs:210-266). `conv[i]` ((K-1) x d_conv,
 * oldest row first) and `gdn[i]` (n_v x hd x hd) belong to the i-th recurrent
 * layer, `kcache/vcache[i]` (ctx x n_head_kv*head_dim) to the i-th attention
 * layer; all are updated in place. `hidden_out` (n_embd) may be NULL. */
/* Projections through gemv_quant (on = 1) instead of gemv_quant_q8k (0, the
 * default and the reference's choice); process-wide. */
void ora_forward_exact_gemv(int on);
/* The projections split by input columns (ffn_down, ssm_out, attn_output)
 * as `world` tensor-parallel ranks compute them: per-rank partial
 * gemv_quant_q8k over equal column slices, summed in rank order in f32
 * (1, the default: one device); process-wide. */
void ora_forward_row_split(int world);

int ora_decode_token(const ora_model_cfg *c, void **tensors, const int *dtypes, float **conv, float **gdn,
                     float **kcache, float **vcache, int position, uint32_t token, float *logits, float *hidden_out,
                     int nthreads);

#ifdef __cplusplus
}
#endif
#endif
