/*
 * unltd_gpu.h — C ABI of the B200 (sm_100a) quantized matrix-product path.
 *
 * This library replaces, for CUDA devices, the quantized matvec operators of
 * the reference crate `unltd-tensor` (crates/unltd-tensor/src/quants.rs).
 * Every function returns an int32 status (UNLTD_OK = 0) and never aborts;
 * `unltd_last_error()` gives a message for the calling thread. Argument
 * checks mirror the reference's `assert!`s one for one, so a call the
 * reference would panic on returns an error status here instead.
 *
 * Two layers:
 *  1. Handle API (device pointers, asynchronous on the context's stream):
 *     contexts, weight upload from a host view (an mmap'd GGUF tensor) with a
 *     lossless on-device repack, GEMV/argmax/GEMM/dequant launches, NCCL.
 *  2. Reference-signature API (host buffers, synchronous): the exact argument
 *     lists of `gemv_quant`, `gemv_quant_q8k` and `dequantize_q4_k`. The
 *     weight bytes are uploaded on first use and cached by host address, so a
 *     caller holding mmap views can switch without changing call sites.
 *
 * Conventions (quants.rs:414-417): W has `dim_out` rows of `dim_in` packed
 * elements, as GGUF writes it, so y = W.x; Y = X.W^T for the batched GEMM.
 * Thread safety: a context may be used from one host thread at a time;
 * separate contexts are independent. The reference-signature API uses one
 * default context per process (device selectable by unltd_set_default_device).
 */
#ifndef UNLTD_GPU_H
#define UNLTD_GPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define UNLTD_ABI_VERSION 1

/* Element types, same ordinals as the reference enum DType
 * (crates/unltd-tensor/src/lib.rs:19-31). Only F32 inputs and the packed
 * Q4_K / Q6_K / Q8_0 weights are accepted by the compute entry points. */
typedef enum {
    UNLTD_DTYPE_F32 = 0,
    UNLTD_DTYPE_F16 = 1,
    UNLTD_DTYPE_BF16 = 2,
    UNLTD_DTYPE_I8 = 3,
    UNLTD_DTYPE_U8 = 4,
    UNLTD_DTYPE_Q4K = 5,
    UNLTD_DTYPE_Q6K = 6,
    UNLTD_DTYPE_Q8_0 = 7
} unltd_dtype;

typedef enum {
    UNLTD_OK = 0,
    UNLTD_ERR_INVALID_ARG = 1,   /* null pointer, bad enum, bad handle */
    UNLTD_ERR_LENGTH = 2,        /* a buffer length that a reference assert rejects */
    UNLTD_ERR_DIM = 3,           /* dim_in not a multiple of the block size */
    UNLTD_ERR_UNSUPPORTED = 4,   /* dtype/mode pair with no kernel (the reference panics too) */
    UNLTD_ERR_CUDA = 5,          /* a CUDA runtime error; see unltd_last_error */
    UNLTD_ERR_OUT_OF_MEMORY = 6,
    UNLTD_ERR_NO_DEVICE = 7,
    UNLTD_ERR_NCCL = 8,
    UNLTD_ERR_TIMEOUT = 9
} unltd_status;

/* GEMV arithmetic modes.
 * F32X      — f32 activations, exact integer products over the packed weights
 *             with x held as 24-bit fixed point per 256-element block; within
 *             1e-4 max-rel of the f64-accumulated `gemv_quant`
 *             (quants.rs:422-466). Q4_K, Q6_K and Q8_0.
 * Q8K_EXACT — bit-identical to `gemv_quant_q8k` (quants.rs:474-515): x is
 *             quantized to Q8_K exactly as `quantize_q8_k` does, the integer
 *             lane sums are exact, and the per-block f32 epilogue runs in the
 *             reference's order without FMA. Q4_K and Q6_K only. */
typedef enum { UNLTD_MODE_F32X = 0, UNLTD_MODE_Q8K_EXACT = 1 } unltd_mode;

typedef struct unltd_ctx_s *unltd_ctx;
typedef struct unltd_weight_s *unltd_weight;

/* ---- errors and library info ---------------------------------------- */
const char *unltd_last_error(void);
int32_t unltd_abi_version(void);
/* Bytes of one packed row (min_forward.rs:52-80); 0 if dim_in is not a
 * multiple of the dtype's block or the dtype is not packed/F32. */
size_t unltd_row_bytes(int32_t dtype, size_t dim_in);

/* ---- contexts --------------------------------------------------------- */
/* A context owns a CUDA stream on `device`, its scratch memory and (after
 * unltd_comm_init) an NCCL communicator. */
int32_t unltd_ctx_create(int32_t device, unltd_ctx *out);
int32_t unltd_ctx_destroy(unltd_ctx ctx);
/* The cudaStream_t the context launches on, as void*. */
int32_t unltd_ctx_stream(unltd_ctx ctx, void **stream_out);
/* Launch on a caller-owned stream instead (NULL restores the own stream). */
int32_t unltd_ctx_set_stream(unltd_ctx ctx, void *stream);
int32_t unltd_ctx_synchronize(unltd_ctx ctx);
/* Number of kernels this context has launched so far. */
int64_t unltd_ctx_launch_count(unltd_ctx ctx);

/* ---- weights ------------------------------------------------------------ */
/* Copy a packed weight view (GGUF bytes, `dim_out` rows of `dim_in`
 * elements, `nbytes` = dim_out * row_bytes) to the device and repack it
 * losslessly into the kernels' row layout. Replaces the zero-copy `&[u8]`
 * view the reference passes to every call (weights.rs:55-61): the upload
 * happens once. Validates like gemv_quant (quants.rs:430-452). */
int32_t unltd_weight_upload(unltd_ctx ctx, const void *host_bytes, size_t nbytes, int32_t dtype,
                            size_t dim_in, size_t dim_out, unltd_weight *out);
/* Same, for a row range [row0, row0 + rows) of a host view whose full shape
 * is dim_out x dim_in (tensor-parallel column shards of a projection). */
int32_t unltd_weight_upload_rows(unltd_ctx ctx, const void *host_bytes, size_t nbytes, int32_t dtype,
                                 size_t dim_in, size_t dim_out, size_t row0, size_t rows,
                                 unltd_weight *out);
int32_t unltd_weight_free(unltd_weight w);
int32_t unltd_weight_info(unltd_weight w, int32_t *dtype, size_t *dim_in, size_t *dim_out,
                          size_t *device_bytes);

/* ---- compute (device pointers, async on the context stream) ------------- */
/* y[dim_out] = W . x[dim_in]; f32 in and out. Replaces gemv_quant
 * (quants.rs:422) for mode F32X and gemv_quant_q8k (quants.rs:474) for
 * mode Q8K_EXACT. */
int32_t unltd_gemv(unltd_ctx ctx, unltd_weight w, const float *x_dev, float *y_dev, int32_t mode);

/* LM head: logits = W . x, then the first index of the maximum
 * (min_forward.rs:210-266 followed by greedy.rs:18-27), fused. `logits_dev`
 * may be NULL. `token_dev` receives the index as uint32. A NaN logit never
 * wins except at index 0, as in the reference's strict '>' scan. */
int32_t unltd_gemv_argmax(unltd_ctx ctx, unltd_weight w, const float *x_dev, float *logits_dev,
                          uint32_t *token_dev, int32_t mode);

/* The LM head split by vocab rows across GPUs (min_forward.rs:210-266 with
 * greedy.rs:18-27 over all shards): `w` holds rows [row0, row0 + dim_out) of
 * the full head. Writes this shard's argmax as the 64-bit key
 * (orderable(logit) << 32) | (0xFFFFFFFF - global row) to `key_dev`; after
 * unltd_allreduce_max_u64 over the ranks, every rank holds the key of the
 * first-index maximum of the whole vocabulary, token = 0xFFFFFFFF - (key &
 * 0xFFFFFFFF). NaN rules as unltd_gemv_argmax (global row 0 only). */
int32_t unltd_gemv_argmax_shard(unltd_ctx ctx, unltd_weight w, const float *x_dev, float *logits_dev,
                                uint64_t *key_dev, uint32_t row0, int32_t mode);

/* Batch decode: y_s = W . x_s for n_seq (1..32) sequences that share W,
 * x_dev f32 [n_seq][dim_in], y_dev f32 [n_seq][dim_out]. Every y_s is the
 * bits of unltd_gemv(..., UNLTD_MODE_Q8K_EXACT) on x_s alone, i.e.
 * gemv_quant_q8k (quants.rs:474-515) per sequence; the reference decodes one
 * sequence per step (qwen35_forward.rs:289), so this is its operator applied
 * to each sequence of a batch, with W read from memory once. Q4_K and Q6_K
 * weights, Q8K_EXACT mode only. */
int32_t unltd_gemv_batch(unltd_ctx ctx, unltd_weight w, const float *x_dev, float *y_dev, int32_t n_seq,
                         int32_t mode);

/* The LM head of a batch: logits and greedy token of every sequence
 * (unltd_gemv_argmax per sequence, same NaN rules). `logits_dev` [n_seq][dim_out]
 * may be NULL; `tokens_dev` receives n_seq uint32 indices. */
int32_t unltd_gemv_argmax_batch(unltd_ctx ctx, unltd_weight w, const float *x_dev, float *logits_dev,
                                uint32_t *tokens_dev, int32_t n_seq, int32_t mode);

/* Batched prefill: Y[m][n] = sum_k X[m][k] * W[n][k] for m < m_tokens, X f32
 * row-major [m_tokens][dim_in], Y f32 row-major [m_tokens][dim_out]. This is
 * gemv_quant (quants.rs:422) applied to every token at once; the reference
 * runs prefill token by token (qwen35_forward.rs:8-12, greedy.rs:55-65).
 * Q4_K weights; tcgen05 tensor cores with fp16 operands (X rounded once to
 * fp16, |X| < 65504; W = q*fp16(d*sc) - fp16(dmin*m) in one fp16 FMA) and f32
 * accumulation: |Y - exact| <= 2^-9 * sum_k |X| (|W| + |d sc q| + |dmin m|)
 * per element. */
int32_t unltd_gemm(unltd_ctx ctx, unltd_weight w, const float *X_dev, float *Y_dev, size_t m_tokens);

/* The same product with the accuracy of gemv_quant (quants.rs:422): within
 * 1e-4 max-rel of the f64-accumulated truth. Each token row of X is scaled by
 * a power of two and split into fp16 hi + lo; W = d*sc*q - dmin*m is formed
 * in f32, scaled by 2^8 and split the same way (|W| < 256); three tcgen05
 * MMAs per K slice (Xh Wh + Xh Wl + Xl Wh, f32 accumulation), 128-token
 * tiles. Q4_K weights. */
int32_t unltd_gemm_f32x(unltd_ctx ctx, unltd_weight w, const float *X_dev, float *Y_dev, size_t m_tokens);

/* Dequantize all rows to f32, row-major [dim_out][dim_in]. Bit-exact with
 * dequantize_q4_k (quants.rs:534-567) for Q4_K and with the exact element
 * values of dot_q6_k (quants.rs:171-200) and of the Q8_0 format. */
int32_t unltd_dequant(unltd_ctx ctx, unltd_weight w, float *out_dev);

/* Same result as unltd_gemv (no counterpart in the reference), for callers
 * that cannot allocate GPU memory: code inside an allocator or memory pool,
 * hosts that reserve all device memory up front, or code that must not hit
 * the implicit synchronisation of cudaMalloc/cudaFree. Its scratch is a
 * fixed 64 KiB device array inside the library (held on every GPU that loads
 * the library until exit), so a call allocates nothing. Limits: dim_in <=
 * 16384 (larger is rejected with UNLTD_ERR_UNSUPPORTED); Q4_K, Q6_K, Q8_0.
 * All calls on a device share the array: calls whose kernels overlap on the
 * GPU race; order them on one stream. `stream` is a cudaStream_t (NULL = the
 * legacy default stream). The first call on a device sets up that device
 * (symbol address, kernel attributes); make it before any stream capture (a
 * failed set-up is retried by the next call). A kernel that gives up on a
 * bounded pipeline wait records the timeout in the error word of w's
 * context: after `stream` has finished, unltd_ctx_synchronize on that
 * context returns UNLTD_ERR_TIMEOUT (y is then not valid). */
int32_t unltd_gemv_noalloc(unltd_weight w, const float *x_dev, float *y_dev, int32_t mode, void *stream);

/* ---- NCCL communicators (tensor parallelism, one process per GPU) ----------
 * NCCL is loaded at run time (libnccl.so.2, the copy the process already has
 * if any). Rank 0 creates the 128-byte id, the caller distributes it (e.g. a
 * torch.distributed broadcast), every rank calls unltd_comm_init. */
int32_t unltd_comm_unique_id(void *id_out, size_t id_bytes);
int32_t unltd_comm_init(unltd_ctx ctx, int32_t rank, int32_t world, const void *id, size_t id_bytes);
/* Optional NVLink peer all-reduce (after unltd_comm_init): every rank calls
 * unltd_peer_export (64-byte CUDA IPC handle of its receive area), the
 * caller gathers the handles in rank order (e.g. torch.distributed
 * all_gather_object), every rank calls unltd_peer_import with all of them.
 * From then on the all-reduces below of up to 16384 elements run as one
 * kernel that exchanges the data over peer memory and sums in rank order
 * (identical bits on every rank); larger ones use NCCL. */
int32_t unltd_peer_export(unltd_ctx ctx, void *handle_out, size_t handle_bytes);
int32_t unltd_peer_import(unltd_ctx ctx, const void *handles, size_t handle_bytes);
/* In-place all-reduces on the context's stream. */
int32_t unltd_allreduce_sum_f32(unltd_ctx ctx, float *buf_dev, size_t count);
int32_t unltd_allreduce_max_u64(unltd_ctx ctx, uint64_t *buf_dev, size_t count);

/* ---- GGUF files (gguf.rs:353-520, weights.rs:32-92) ----------------------
 * unltd_gguf_open maps a GGUF (v2/v3) file read-only and parses its metadata
 * and tensor table, every field bounds-checked; tensors are zero-copy views
 * of the mapping, valid until unltd_gguf_close. dtype: the unltd ordinal of
 * the tensor's ggml type, -1 for a type this path does not read (data NULL).
 * ne: the dims, ne[0] fastest (a weight is ne = [dim_in, dim_out]). */
typedef struct unltd_gguf_s *unltd_gguf;
int32_t unltd_gguf_open(const char *path, unltd_gguf *out);
int32_t unltd_gguf_close(unltd_gguf g);
int64_t unltd_gguf_tensor_count(unltd_gguf g);
int32_t unltd_gguf_tensor_info(unltd_gguf g, int64_t index, const char **name, int32_t *dtype, int64_t ne[4],
                               int32_t *ndims, const void **data, size_t *nbytes);
int32_t unltd_gguf_find_tensor(unltd_gguf g, const char *name, int64_t *index);
/* Scalar metadata: integer types (bool as 0/1), f32/f64, strings. */
int32_t unltd_gguf_get_int(unltd_gguf g, const char *key, int64_t *out);
int32_t unltd_gguf_get_float(unltd_gguf g, const char *key, double *out);
int32_t unltd_gguf_get_string(unltd_gguf g, const char *key, const char **out);

/* ---- Qwen3.5-style hybrid decode step ------------------------------------
 * Replaces Qwen35Forward (crates/unltd-generation/src/qwen35_forward.rs):
 * open (139-232: every tensor checked for shape and dtype), new_session
 * (235-257), step (295-330) and, fused on the device, output_norm + the LM
 * head (min_forward.rs:210-266) + greedy argmax (greedy.rs:18-27). One CUDA
 * graph per token; the greedy token is fed back on the device. Every
 * projection is gemv_quant_q8k-exact and the f32 kernels between them keep
 * the reference's operation order, so hidden states and logits equal the
 * reference's (f32 exp/log correctly rounded). Kernel limits: linear head dim
 * 128, attention head_dim 128 or 256, d_inner == n_embd, ctx <= 16384. */
typedef struct {
    int32_t n_layer, n_embd, n_ff, n_head, n_head_kv, head_dim, head_dim_v, n_rot;
    int32_t conv_kernel, state_size, group_count, time_step_rank, d_inner, full_attn_interval, vocab;
    float freq_base, rms_eps;
} unltd_qwen35_config; /* qwen35.rs:46-80 */
/* Qwen35Config::from_gguf (qwen35.rs:23-42, 130-200): the qwen35.* keys, each
 * required with its type (rope.dimension_sections i32[4]); vocab = the rows of
 * token_embd.weight. The structural checks run in unltd_qwen35_create. */
int32_t unltd_qwen35_config_from_gguf(unltd_gguf g, unltd_qwen35_config *cfg);

typedef struct unltd_qwen35_s *unltd_qwen35;
typedef struct unltd_qwen35_session_s *unltd_qwen35_session;

int32_t unltd_qwen35_create(unltd_ctx ctx, const unltd_qwen35_config *cfg, unltd_qwen35 *out);
/* Tensor-parallel shard `rank` of `world` GPUs (one process per GPU; the
 * context needs a communicator, unltd_comm_init). set_tensor still takes the
 * full GGUF tensors and keeps this rank's part: q/k/v, qkv/z/beta/alpha and
 * gate/up by output rows (heads), ffn_down, ssm_out and attn_output by input
 * columns with an NCCL all-reduce of their partial outputs, the LM head by
 * vocab rows with a cross-GPU argmax (all-reduce MAX of 64-bit keys). */
int32_t unltd_qwen35_create_tp(unltd_ctx ctx, const unltd_qwen35_config *cfg, int32_t rank, int32_t world,
                               unltd_qwen35 *out);
/* Host-only (no GPU): the part of tensor `name` that rank `rank` of `world`
 * keeps, as source row ranges [ranges[2i], ranges[2i+1]) (element ranges for
 * F32 tensors), concatenated in order, each row restricted to input columns
 * [*in_begin, *in_end). */
int32_t unltd_qwen35_shard(const unltd_qwen35_config *cfg, int32_t rank, int32_t world, const char *name,
                           int64_t *ranges, int32_t max_ranges, int32_t *n_ranges, int64_t *in_begin,
                           int64_t *in_end);
/* Upload one GGUF tensor by its name ("blk.3.attn_q.weight", "output.weight",
 * ...): packed bytes or F32 values, checked against the configuration. */
int32_t unltd_qwen35_set_tensor(unltd_qwen35 m, const char *name, const void *host, size_t nbytes, int32_t dtype);
/* Check that every tensor is present and merge same-input projections
 * (qkv|z|beta|alpha, q|k|v, gate|up) into single GEMVs. */
int32_t unltd_qwen35_finalize(unltd_qwen35 m);
/* Every tensor of the model from an opened GGUF file (zero-copy views of its
 * mapping, checked for name, dtype and shape like set_tensor), then
 * finalize. weights.rs:32-92 + Qwen35Forward::open (qwen35_forward.rs:139-232). */
int32_t unltd_qwen35_load_gguf(unltd_qwen35 m, unltd_gguf g);
int32_t unltd_qwen35_destroy(unltd_qwen35 m);
/* A session: conv windows, GDN states and K/V cache for ctx_len positions,
 * all zero, position 0 (new_session). Has its own stream. */
int32_t unltd_qwen35_session_create(unltd_qwen35 m, int32_t ctx_len, unltd_qwen35_session *out);
int32_t unltd_qwen35_session_destroy(unltd_qwen35_session s);
/* Load a state at `position`: per recurrent layer (in layer order) the conv
 * window ((conv_kernel-1) x 2*d_inner, oldest row first) and the GDN
 * matrices (n_v x 128 x 128); per attention layer the first `position` rows
 * of K and V (n_head_kv*head_dim each). NULL arrays or entries mean zeros. */
int32_t unltd_qwen35_session_set_state(unltd_qwen35_session s, int32_t position, const float *const *conv,
                                       const float *const *gdn, const float *const *kcache,
                                       const float *const *vcache);
/* The inverse: copy the state at the current position out, same layout
 * (caller-allocated host buffers; NULL arrays or entries are skipped). */
int32_t unltd_qwen35_session_get_state(unltd_qwen35_session s, float *const *conv, float *const *gdn,
                                       float *const *kcache, float *const *vcache);
/* Teacher-forced steps over a prompt; *next_token (nullable) = the greedy
 * token after the last one. */
int32_t unltd_qwen35_feed(unltd_qwen35_session s, const uint32_t *tokens, int32_t n, uint32_t *next_token);
/* The same prompt as a batched prefill (one GPU, one-sequence session): the
 * prompt in chunks of up to 32 tokens, every projection one batched GEMV per
 * chunk (each weight read once per chunk), attention batched over the chunk's
 * tokens, the recurrence token by token. The state, the last token's logits
 * and hidden state, and *next_token are the bits unltd_qwen35_feed gives
 * (the reference prefills token by token, qwen35_forward.rs:8-12,
 * greedy.rs:55-65). */
int32_t unltd_qwen35_prefill(unltd_qwen35_session s, const uint32_t *tokens, int32_t n, uint32_t *next_token);
/* Greedy decode of n_steps tokens: step 0 consumes `token`, step i consumes
 * tokens_out[i-1]; tokens_out[i] = argmax of step i's logits. */
int32_t unltd_qwen35_decode(unltd_qwen35_session s, uint32_t token, int32_t n_steps, uint32_t *tokens_out);
/* Position, the session's cudaStream_t, kernels launched per step. */
int32_t unltd_qwen35_session_info(unltd_qwen35_session s, int32_t *position, void **stream,
                                  int64_t *launches_per_step);
/* Per-rank sizes: conv window row (channels), GDN heads, K/V row, and the
 * vocab rows [begin, end) whose logits this rank holds. */
int32_t unltd_qwen35_session_shape(unltd_qwen35_session s, int64_t *conv_row, int64_t *gdn_heads,
                                   int64_t *kv_row, int64_t *vocab_begin, int64_t *vocab_end);
/* Last step's logits (this rank's vocab rows) and hidden state (l_out of the
 * last layer, full n_embd on every rank). */
int32_t unltd_qwen35_session_read(unltd_qwen35_session s, float *logits, float *hidden);

/* Batch decode (batch 32): one session of n_seq (1..32)
 * independent sequences that share the model, each with its own state and
 * position; one step decodes every sequence, reading each weight matrix once
 * (unltd_gemv_batch). Every sequence's tokens, logits and hidden states are
 * those of a one-sequence session started from the same state: the
 * reference's qwen35_forward.rs:289 step, applied per sequence. One GPU. */
int32_t unltd_qwen35_session_create_batch(unltd_qwen35 m, int32_t ctx_len, int32_t n_seq,
                                          unltd_qwen35_session *out);
/* set_state / get_state / session_read of sequence `seq`. */
int32_t unltd_qwen35_batch_set_state(unltd_qwen35_session s, int32_t seq, int32_t position,
                                     const float *const *conv, const float *const *gdn,
                                     const float *const *kcache, const float *const *vcache);
int32_t unltd_qwen35_batch_get_state(unltd_qwen35_session s, int32_t seq, float *const *conv, float *const *gdn,
                                     float *const *kcache, float *const *vcache);
int32_t unltd_qwen35_batch_read(unltd_qwen35_session s, int32_t seq, float *logits, float *hidden);
/* n_steps greedy steps of every sequence: step 0 of sequence z consumes
 * tokens[z]; tokens_out[z * n_steps + i] = its token of step i. */
int32_t unltd_qwen35_batch_decode(unltd_qwen35_session s, const uint32_t *tokens, int32_t n_steps,
                                  uint32_t *tokens_out);
/* The session's sequence count and each sequence's position (may be NULL). */
int32_t unltd_qwen35_batch_info(unltd_qwen35_session s, int32_t *n_seq, int32_t *positions);

/* ---- reference-signature API (host buffers, synchronous) ---------------- */
/* quants.rs:422  pub fn gemv_quant(out, x, w, dim_in, dim_out, dtype) */
int32_t unltd_gemv_quant(float *out, size_t out_len, const float *x, size_t x_len, const uint8_t *w,
                         size_t w_len, size_t dim_in, size_t dim_out, int32_t dtype);
/* quants.rs:474  pub fn gemv_quant_q8k(out, x, w, dim_in, dim_out, dtype) */
int32_t unltd_gemv_quant_q8k(float *out, size_t out_len, const float *x, size_t x_len,
                             const uint8_t *w, size_t w_len, size_t dim_in, size_t dim_out,
                             int32_t dtype);
/* quants.rs:534  pub fn dequantize_q4_k(out, w) */
int32_t unltd_dequantize_q4_k(float *out, size_t out_len, const uint8_t *w, size_t w_len);
/* Device used by the reference-signature API (default 0). Must be called
 * before the first such call. */
int32_t unltd_set_default_device(int32_t device);
/* Drop every cached weight upload of the reference-signature API (call when
 * the mmap behind the cached host addresses goes away). */
int32_t unltd_forget_host_weights(void);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif /* UNLTD_GPU_H */
