/*
 * CPU oracle for the quantized matrix-product path: a plain-C restatement of
 * the reference's scalar kernels (crates/unltd-tensor/src/quants.rs and the
 * pairwise reduction tree of crates/unltd-tensor/src/kernels.rs:27-42).
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker that the CUDA path is
 * compared against, and the timed CPU baseline. Nothing in the product links
 * it; the CUDA library never falls back to it.
 *
 * Build with -O2 -ffp-contract=off and no fast-math: the Q8_K dots need a
 * separate f32 multiply and add (quants.rs:305-306, 345-346).
 */
#ifndef UNLTD_ORACLE_QUANTS_REF_H
#define UNLTD_ORACLE_QUANTS_REF_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* DType ordinal, in the order of the reference enum (lib.rs:19-31). */
enum ora_dtype {
    ORA_F32 = 0,
    ORA_F16 = 1,
    ORA_BF16 = 2,
    ORA_I8 = 3,
    ORA_U8 = 4,
    ORA_Q4K = 5,
    ORA_Q6K = 6,
    ORA_Q8_0 = 7
};

#define ORA_QK_K 256
#define ORA_BLOCK_Q4_K 144
#define ORA_BLOCK_Q6_K 210
#define ORA_QK8_0 32
#define ORA_BLOCK_Q8_0 34

/* Q8_K activation block (quants.rs:237-242): f32 d, 256 int8, 16 int32 sums. */
typedef struct {
    float d;
    int8_t qs[256];
    int32_t bsums[16];
} ora_q8k_block;

/* Status codes: 0 ok, negative = the reference would have panicked. */
#define ORA_OK 0
#define ORA_ERR_LEN -1
#define ORA_ERR_DTYPE -2
#define ORA_ERR_DIM -3

float ora_f16_to_f32(uint16_t h);
void ora_scale_min_k4(const uint8_t *s, int g, uint8_t *sc, uint8_t *m);
double ora_pairwise_sum_f64(const double *v, size_t n);
int32_t ora_nearest_int(float f);

double ora_dot_f32(const float *x, const float *w, size_t n);
double ora_dot_q4_k(const float *x, const uint8_t *w, size_t n);
double ora_dot_q6_k(const float *x, const uint8_t *w, size_t n);
double ora_dot_q8_0(const float *x, const uint8_t *w, size_t n);

int ora_quantize_q8_k(const float *x, size_t n, ora_q8k_block *out);
float ora_dot_q4_k_q8_k(const ora_q8k_block *x, const uint8_t *w, size_t nblocks);
float ora_dot_q6_k_q8_k(const ora_q8k_block *x, const uint8_t *w, size_t nblocks);

/* Row GEMVs (quants.rs:422-515). nthreads <= 1 runs the single-threaded row
 * loop of the reference; nthreads > 1 splits output rows into contiguous
 * chunks (the rayon LM head, min_forward.rs:245-264). Results are identical
 * for every thread count: rows are independent. */
int ora_gemv_quant(float *out, const float *x, const uint8_t *w, size_t w_len,
                   size_t dim_in, size_t dim_out, int dtype, int nthreads);
int ora_gemv_quant_q8k(float *out, const float *x, const uint8_t *w, size_t w_len,
                       size_t dim_in, size_t dim_out, int dtype, int nthreads);

/* f64 ground truth of one output row, unrounded (for tolerance tests). */
int ora_gemv_quant_f64(double *out, const float *x, const uint8_t *w, size_t w_len,
                       size_t dim_in, size_t dim_out, int dtype, int nthreads);

/* Dequantization to f32 (quants.rs:534-567 for Q4_K; Q6_K and Q8_0 restate
 * the element formulas of dot_q6_k and the Q8_0 format; every value is exact
 * in f32, so the result is unique). n = number of elements. */
int ora_dequantize_q4_k(float *out, const uint8_t *w, size_t n);
int ora_dequantize_q6_k(float *out, const uint8_t *w, size_t n);
int ora_dequantize_q8_0(float *out, const uint8_t *w, size_t n);

/* First index of the maximum (greedy.rs:18-27). n must be > 0. */
size_t ora_argmax(const float *v, size_t n);

/* Bytes of one packed row of dim_in elements, or 0 if dim_in is not a
 * multiple of the block (min_forward.rs:52-80). */
size_t ora_row_bytes(int dtype, size_t dim_in);

#ifdef __cplusplus
}
#endif
#endif
