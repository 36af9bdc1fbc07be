// C ABI of libunltd_gpu: contexts, weight upload, compute entry points and
// the reference-signature host-buffer API. See include/unltd_gpu.h.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>

#include "unltd_host.h"
#include "unltd_internal.cuh"

using namespace unltd;

namespace unltd {

static thread_local std::string g_err;

int32_t set_error(int32_t status, const std::string &msg) {
  g_err = msg;
  return status;
}

int32_t cuda_error(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return UNLTD_OK;
  cudaGetLastError();  // clear a non-sticky error
  return set_error(e == cudaErrorMemoryAllocation ? UNLTD_ERR_OUT_OF_MEMORY : UNLTD_ERR_CUDA,
                   std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

}  // namespace unltd

namespace {

bool packed_or_f32(int dtype) { return dtype == F32 || dtype == Q4K || dtype == Q6K || dtype == Q8_0; }

const char *dtype_name(int d) {
  switch (d) {
    case F32: return "F32";
    case F16: return "F16";
    case BF16: return "BF16";
    case I8: return "I8";
    case U8: return "U8";
    case Q4K: return "Q4K";
    case Q6K: return "Q6K";
    case Q8_0: return "Q8_0";
    default: return "?";
  }
}

// Shape checks of gemv_quant (quants.rs:430-452) on the packed view.
int32_t check_view(int dtype, size_t dim_in, size_t dim_out, size_t nbytes, const char *who) {
  if (!packed_or_f32(dtype))
    return set_error(UNLTD_ERR_UNSUPPORTED, std::string(who) + ": dtype " + dtype_name(dtype) + " has no kernel");
  if ((dtype == Q4K || dtype == Q6K) && dim_in % kQK)
    return set_error(UNLTD_ERR_DIM, std::string(who) + ": dim_in " + std::to_string(dim_in) + " is not a multiple of 256");
  if (dtype == Q8_0 && dim_in % kQ80Elems)
    return set_error(UNLTD_ERR_DIM, std::string(who) + ": dim_in " + std::to_string(dim_in) + " is not a multiple of 32");
  size_t rb = gguf_row_bytes(dtype, dim_in);
  if (nbytes != rb * dim_out)
    return set_error(UNLTD_ERR_LENGTH, std::string(who) + ": len(w) " + std::to_string(nbytes) +
                                           " != dim_out * row_bytes = " + std::to_string(rb * dim_out));
  return UNLTD_OK;
}

}  // namespace

namespace unltd {

// The error word is copied into pinned host memory behind the queued work, so
// one synchronisation covers the results and the error check.
int32_t sync_and_check(unltd_ctx c, cudaStream_t st, const char *who) {
  cudaError_t e = cudaMemcpyAsync(c->err_host, c->err, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_error(e, who);
  const int v = *c->err_host;
  if (v == 0) return UNLTD_OK;
  *c->err_host = 0;
  e = cudaMemsetAsync(c->err, 0, sizeof(int), st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_error(e, who);
  if (v == 2) return set_error(UNLTD_ERR_INVALID_ARG, std::string(who) + ": a token id outside the vocabulary reached the embedding");
  if (v == 3) return set_error(UNLTD_ERR_TIMEOUT, std::string(who) + ": a peer all-reduce gave up waiting for another rank");
  return set_error(UNLTD_ERR_TIMEOUT, std::string(who) + ": a kernel gave up waiting on a pipeline barrier");
}

}  // namespace unltd

extern "C" {

const char *unltd_last_error(void) { return g_err.c_str(); }

int32_t unltd_abi_version(void) { return UNLTD_ABI_VERSION; }

size_t unltd_row_bytes(int32_t dtype, size_t dim_in) { return packed_or_f32(dtype) ? gguf_row_bytes(dtype, dim_in) : 0; }

int32_t unltd_ctx_create(int32_t device, unltd_ctx *out) {
  if (!out) return set_error(UNLTD_ERR_INVALID_ARG, "ctx_create: out is NULL");
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) {
    cudaGetLastError();
    return set_error(UNLTD_ERR_NO_DEVICE, "ctx_create: no CUDA device");
  }
  if (device < 0 || device >= n)
    return set_error(UNLTD_ERR_INVALID_ARG, "ctx_create: device " + std::to_string(device) + " out of range");
  CtxGuard g(device);
  unltd_ctx c = new unltd_ctx_s();
  c->device = device;
  cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device);
  e = cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking);
  // [key | done | err | token | pad] then the batched argmax state: 32 keys,
  // a counter, 32 tokens
  if (e == cudaSuccess) e = cudaMalloc(&c->argmax_key, 512);
  if (e == cudaSuccess) {
    uint8_t *base = reinterpret_cast<uint8_t *>(c->argmax_key);
    c->argmax_done = reinterpret_cast<unsigned *>(base + 8);
    c->err = reinterpret_cast<int *>(base + 12);
    c->bkey = reinterpret_cast<unsigned long long *>(base + 64);
    c->bdone = reinterpret_cast<unsigned *>(base + 64 + 8 * kMaxBatch);
    c->btok = reinterpret_cast<uint32_t *>(base + 128 + 8 * kMaxBatch);
    e = cudaMemset(c->argmax_key, 0, 512);
  }
  if (e == cudaSuccess) {
    c->scratch_bytes = 256 * 1024;
    e = cudaMalloc(&c->scratch, c->scratch_bytes);
  }
  if (e == cudaSuccess) e = cudaHostAlloc(&c->err_host, 64, cudaHostAllocDefault);
  if (e == cudaSuccess) *c->err_host = 0;
  if (e != cudaSuccess) {
    int32_t rc = cuda_error(e, "ctx_create");
    if (c->own_stream) cudaStreamDestroy(c->own_stream);
    if (c->argmax_key) cudaFree(c->argmax_key);
    if (c->scratch) cudaFree(c->scratch);
    delete c;
    return rc;
  }
  c->stream = c->own_stream;
  *out = c;
  return UNLTD_OK;
}

int32_t unltd_ctx_destroy(unltd_ctx c) {
  if (!c) return UNLTD_OK;
  CtxGuard g(c->device);
  cudaStreamSynchronize(c->stream);
  comm_destroy(c);
  if (c->scratch) cudaFree(c->scratch);
  if (c->gemm_scratch) cudaFree(c->gemm_scratch);
  if (c->argmax_key) cudaFree(c->argmax_key);
  if (c->err_host) cudaFreeHost(c->err_host);
  if (c->own_stream) cudaStreamDestroy(c->own_stream);
  delete c;
  return UNLTD_OK;
}

int32_t unltd_ctx_stream(unltd_ctx c, void **s) {
  if (!c || !s) return set_error(UNLTD_ERR_INVALID_ARG, "ctx_stream: NULL argument");
  *s = (void *)c->stream;
  return UNLTD_OK;
}

int32_t unltd_ctx_set_stream(unltd_ctx c, void *s) {
  if (!c) return set_error(UNLTD_ERR_INVALID_ARG, "ctx_set_stream: NULL ctx");
  c->stream = s ? (cudaStream_t)s : c->own_stream;
  return UNLTD_OK;
}

int32_t unltd_ctx_synchronize(unltd_ctx c) {
  if (!c) return set_error(UNLTD_ERR_INVALID_ARG, "ctx_synchronize: NULL ctx");
  CtxGuard g(c->device);
  return sync_and_check(c, c->stream, "ctx_synchronize");
}

int64_t unltd_ctx_launch_count(unltd_ctx c) { return c ? c->launches.load() : -1; }

int32_t unltd_weight_upload_rows(unltd_ctx c, const void *host, size_t nbytes, int32_t dtype, size_t dim_in,
                                 size_t dim_out, size_t row0, size_t rows, unltd_weight *out) {
  if (!c || !host || !out) return set_error(UNLTD_ERR_INVALID_ARG, "weight_upload: NULL argument");
  *out = nullptr;
  int32_t rc = check_view(dtype, dim_in, dim_out, nbytes, "weight_upload");
  if (rc) return rc;
  if (row0 > dim_out || rows > dim_out - row0)
    return set_error(UNLTD_ERR_LENGTH, "weight_upload: row range outside the tensor");
  CtxGuard g(c->device);
  unltd_weight w = new unltd_weight_s();
  w->ctx = c;
  w->dtype = dtype;
  w->dim_in = dim_in;
  w->dim_out = rows;
  w->nb = dtype == Q8_0 ? dim_in / kQ80Elems : (dtype == F32 ? dim_in : dim_in / kQK);
  w->row_bytes = gguf_row_bytes(dtype, dim_in);
  w->row_stride = round_up(w->row_bytes, 16);
  size_t dev_bytes = std::max<size_t>(w->row_stride * rows, 16);
  cudaError_t e = cudaMalloc(&w->dev, dev_bytes);
  if (e != cudaSuccess) {
    delete w;
    return cuda_error(e, "weight_upload: device alloc");
  }
  if (w->row_stride != w->row_bytes) cudaMemsetAsync(w->dev, 0, dev_bytes, c->stream);
  // Stage raw rows through a bounded buffer, repacking each chunk on device.
  const size_t chunk_rows = std::max<size_t>(1, std::min<size_t>(rows, (64u << 20) / std::max<size_t>(w->row_bytes, 1)));
  uint8_t *staging = nullptr;
  if (rows) e = cudaMalloc(&staging, chunk_rows * w->row_bytes);
  const uint8_t *src = static_cast<const uint8_t *>(host) + row0 * w->row_bytes;
  for (size_t r = 0; e == cudaSuccess && r < rows; r += chunk_rows) {
    size_t n = std::min(chunk_rows, rows - r);
    e = cudaMemcpyAsync(staging, src + r * w->row_bytes, n * w->row_bytes, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = launch_repack(*w, staging, r, n, c->stream);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  if (staging) cudaFree(staging);
  if (e != cudaSuccess) {
    cudaFree(w->dev);
    delete w;
    return cuda_error(e, "weight_upload");
  }
  c->launches += (int64_t)((rows + chunk_rows - 1) / chunk_rows);
  *out = w;
  return UNLTD_OK;
}

int32_t unltd_weight_upload(unltd_ctx c, const void *host, size_t nbytes, int32_t dtype, size_t dim_in,
                            size_t dim_out, unltd_weight *out) {
  return unltd_weight_upload_rows(c, host, nbytes, dtype, dim_in, dim_out, 0, dim_out, out);
}

int32_t unltd_weight_free(unltd_weight w) {
  if (!w) return UNLTD_OK;
  CtxGuard g(w->ctx->device);
  cudaStreamSynchronize(w->ctx->stream);
  cudaFree(w->dev);
  if (w->dev_b) cudaFree(w->dev_b);
  delete w;
  return UNLTD_OK;
}

int32_t unltd_weight_info(unltd_weight w, int32_t *dtype, size_t *dim_in, size_t *dim_out, size_t *device_bytes) {
  if (!w) return set_error(UNLTD_ERR_INVALID_ARG, "weight_info: NULL weight");
  if (dtype) *dtype = w->dtype;
  if (dim_in) *dim_in = w->dim_in;
  if (dim_out) *dim_out = w->dim_out;
  if (device_bytes) *device_bytes = w->row_stride * w->dim_out;
  return UNLTD_OK;
}

static int32_t check_mode(unltd_weight w, int32_t mode, const char *who) {
  if (mode != MODE_F32X && mode != MODE_Q8K)
    return set_error(UNLTD_ERR_INVALID_ARG, std::string(who) + ": unknown mode " + std::to_string(mode));
  if (mode == MODE_Q8K && w->dtype != Q4K && w->dtype != Q6K)
    return set_error(UNLTD_ERR_UNSUPPORTED, std::string(who) + ": dtype " + dtype_name(w->dtype) +
                                                " has no Q8_K dot (gemv_quant_q8k accepts Q4_K and Q6_K only)");
  if (mode == MODE_Q8K && w->dtype == F32)
    return set_error(UNLTD_ERR_UNSUPPORTED, std::string(who) + ": F32 weights have no Q8_K path");
  return UNLTD_OK;
}

int32_t unltd_gemv(unltd_ctx c, unltd_weight w, const float *x, float *y, int32_t mode) {
  if (!c || !w || !x || !y) return set_error(UNLTD_ERR_INVALID_ARG, "gemv: NULL argument");
  if (w->ctx != c) return set_error(UNLTD_ERR_INVALID_ARG, "gemv: weight belongs to another context");
  int32_t rc = check_mode(w, mode, "gemv");
  if (rc) return rc;
  CtxGuard g(c->device);
  GemvArgs a{w, x, y, mode, nullptr, nullptr, nullptr};
  return gemv_launch(c, a);
}

int32_t unltd_gemv_argmax(unltd_ctx c, unltd_weight w, const float *x, float *logits, uint32_t *token,
                          int32_t mode) {
  if (!c || !w || !x || !token) return set_error(UNLTD_ERR_INVALID_ARG, "gemv_argmax: NULL argument");
  if (w->ctx != c) return set_error(UNLTD_ERR_INVALID_ARG, "gemv_argmax: weight belongs to another context");
  if (w->dim_out == 0) return set_error(UNLTD_ERR_LENGTH, "gemv_argmax: empty logits");
  int32_t rc = check_mode(w, mode, "gemv_argmax");
  if (rc) return rc;
  CtxGuard g(c->device);
  GemvArgs a{w, x, logits, mode, c->argmax_key, c->argmax_done, token};
  return gemv_launch(c, a);
}

int32_t unltd_gemv_argmax_shard(unltd_ctx c, unltd_weight w, const float *x, float *logits, uint64_t *key,
                                uint32_t row0, int32_t mode) {
  if (!c || !w || !x || !key) return set_error(UNLTD_ERR_INVALID_ARG, "gemv_argmax_shard: NULL argument");
  if (w->ctx != c) return set_error(UNLTD_ERR_INVALID_ARG, "gemv_argmax_shard: weight belongs to another context");
  if (w->dim_out == 0) return set_error(UNLTD_ERR_LENGTH, "gemv_argmax_shard: empty shard");
  if ((uint64_t)row0 + w->dim_out > 0x7FFFFFFFull)
    return set_error(UNLTD_ERR_LENGTH, "gemv_argmax_shard: global row index beyond 2^31");
  if (w->dtype == F32) return set_error(UNLTD_ERR_UNSUPPORTED, "gemv_argmax_shard: packed weights only");
  int32_t rc = check_mode(w, mode, "gemv_argmax_shard");
  if (rc) return rc;
  CtxGuard g(c->device);
  // the local token goes to a spare word of the context's argmax block
  uint32_t *tok = reinterpret_cast<uint32_t *>(reinterpret_cast<uint8_t *>(c->argmax_key) + 16);
  GemvArgs a{w, x, logits, mode, c->argmax_key, c->argmax_done, tok};
  a.argmax_row0 = (int)row0;
  a.key_out = reinterpret_cast<unsigned long long *>(key);
  return gemv_launch(c, a);
}

static int32_t check_batch(unltd_ctx c, unltd_weight w, int32_t n_seq, int32_t mode, const char *fn) {
  if (w->ctx != c) return set_error(UNLTD_ERR_INVALID_ARG, std::string(fn) + ": weight belongs to another context");
  if (n_seq < 1 || n_seq > kMaxBatch)
    return set_error(UNLTD_ERR_INVALID_ARG, std::string(fn) + ": n_seq must be 1..32");
  if (mode != MODE_Q8K) return set_error(UNLTD_ERR_UNSUPPORTED, std::string(fn) + ": Q8K_EXACT mode only");
  if (w->dtype != Q4K && w->dtype != Q6K)
    return set_error(UNLTD_ERR_UNSUPPORTED, std::string(fn) + ": Q4_K and Q6_K weights only");
  if (!gemv_batch_supported(c->device, *w))
    return set_error(UNLTD_ERR_UNSUPPORTED, std::string(fn) + ": rows too long for a shared-memory tile");
  return UNLTD_OK;
}

// Grows the context scratch to n_seq batched x images of w.
static int32_t reserve_batch(unltd_ctx c, unltd_weight w, int32_t n_seq) {
  const size_t need = gemv_batch_img_bytes(*w, n_seq);
  if (c->scratch_bytes >= need) return UNLTD_OK;
  if (c->scratch_fixed) return set_error(UNLTD_ERR_UNSUPPORTED, "gemv_batch: x images larger than the fixed scratch");
  cudaError_t e = cudaStreamSynchronize(c->stream);
  if (e == cudaSuccess && c->scratch) e = cudaFree(c->scratch);
  c->scratch = nullptr;
  c->scratch_bytes = 0;
  if (e == cudaSuccess) e = cudaMalloc(&c->scratch, need);
  if (e != cudaSuccess) return cuda_error(e, "gemv_batch scratch");
  c->scratch_bytes = need;
  return UNLTD_OK;
}

int32_t unltd_gemv_batch(unltd_ctx c, unltd_weight w, const float *x, float *y, int32_t n_seq, int32_t mode) {
  if (!c || !w || !x || !y) return set_error(UNLTD_ERR_INVALID_ARG, "gemv_batch: NULL argument");
  int32_t rc = check_batch(c, w, n_seq, mode, "gemv_batch");
  if (rc) return rc;
  CtxGuard g(c->device);
  if ((rc = reserve_batch(c, w, n_seq))) return rc;
  if ((rc = gemv_batch_prepare(c, w))) return rc;
  BatchGemvArgs a{w};
  a.x = x;
  a.xstride = w->dim_in;
  a.y = y;
  a.ystride = w->dim_out;
  a.nseq = n_seq;
  return gemv_batch_launch(c, a);
}

int32_t unltd_gemv_argmax_batch(unltd_ctx c, unltd_weight w, const float *x, float *logits, uint32_t *tokens,
                                int32_t n_seq, int32_t mode) {
  if (!c || !w || !x || !tokens) return set_error(UNLTD_ERR_INVALID_ARG, "gemv_argmax_batch: NULL argument");
  if (w->dim_out == 0) return set_error(UNLTD_ERR_LENGTH, "gemv_argmax_batch: empty logits");
  if (w->dim_out > 0x7FFFFFFFull) return set_error(UNLTD_ERR_LENGTH, "gemv_argmax_batch: vocab beyond 2^31");
  int32_t rc = check_batch(c, w, n_seq, mode, "gemv_argmax_batch");
  if (rc) return rc;
  CtxGuard g(c->device);
  if ((rc = reserve_batch(c, w, n_seq))) return rc;
  if ((rc = gemv_batch_prepare(c, w))) return rc;
  BatchGemvArgs a{w};
  a.x = x;
  a.xstride = w->dim_in;
  a.y = logits;
  a.ystride = w->dim_out;
  a.nseq = n_seq;
  a.key = c->bkey;
  a.done = c->bdone;
  a.token = tokens;
  return gemv_batch_launch(c, a);
}

int32_t unltd_gemm(unltd_ctx c, unltd_weight w, const float *X, float *Y, size_t m_tokens) {
  if (!c || !w || !X || !Y) return set_error(UNLTD_ERR_INVALID_ARG, "gemm: NULL argument");
  if (w->ctx != c) return set_error(UNLTD_ERR_INVALID_ARG, "gemm: weight belongs to another context");
  if (m_tokens > (size_t)1 << 24) return set_error(UNLTD_ERR_LENGTH, "gemm: m_tokens too large");
  CtxGuard g(c->device);
  return gemm_launch(c, *w, X, Y, m_tokens, false);
}

int32_t unltd_gemm_f32x(unltd_ctx c, unltd_weight w, const float *X, float *Y, size_t m_tokens) {
  if (!c || !w || !X || !Y) return set_error(UNLTD_ERR_INVALID_ARG, "gemm_f32x: NULL argument");
  if (w->ctx != c) return set_error(UNLTD_ERR_INVALID_ARG, "gemm_f32x: weight belongs to another context");
  if (m_tokens > (size_t)1 << 24) return set_error(UNLTD_ERR_LENGTH, "gemm_f32x: m_tokens too large");
  CtxGuard g(c->device);
  return gemm_launch(c, *w, X, Y, m_tokens, true);
}

int32_t unltd_dequant(unltd_ctx c, unltd_weight w, float *out) {
  if (!c || !w || !out) return set_error(UNLTD_ERR_INVALID_ARG, "dequant: NULL argument");
  CtxGuard g(c->device);
  cudaError_t e = launch_dequant(*w, out, c->stream);
  if (e == cudaSuccess) c->launches += 1;
  return cuda_error(e, "dequant");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Reference-signature API: one default context, weights cached by host view.
namespace {

struct HostState {
  std::mutex mu;
  int device = 0;
  unltd_ctx ctx = nullptr;
  struct Cached {
    unltd_weight w;
    uint64_t fp;  // sampled fingerprint of the bytes uploaded
  };
  std::map<std::tuple<const void *, size_t, int, size_t, size_t>, Cached> cache;
  float *xbuf = nullptr, *ybuf = nullptr;
  size_t xcap = 0, ycap = 0;
};

// FNV-1a over the first and last 64 bytes and 64 words spread over the view:
// a cheap check that the bytes behind a cached pointer are still the ones
// uploaded (an address freed and reused by other weights of the same size).
// The reference reads w afresh on every call; weights rewritten in place in
// only a few bytes are not caught, and need unltd_forget_host_weights.
uint64_t view_fingerprint(const uint8_t *w, size_t n) {
  uint64_t h = 1469598103934665603ull;
  auto mix = [&](const uint8_t *p, size_t len) {
    for (size_t i = 0; i < len; i++) h = (h ^ p[i]) * 1099511628211ull;
  };
  mix(w, std::min<size_t>(n, 64));
  if (n > 64) mix(w + n - std::min<size_t>(n - 64, 64), std::min<size_t>(n - 64, 64));
  if (n >= 8 * 64)
    for (size_t i = 0; i < 64; i++) mix(w + (n / 64) * i, 8);
  return h;
}

HostState &hs() {
  static HostState s;
  return s;
}

int32_t ensure_buf(float **p, size_t *cap, size_t n) {
  if (*cap >= n) return UNLTD_OK;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  cudaError_t e = cudaMalloc(p, std::max<size_t>(n, 1024) * sizeof(float));
  if (e != cudaSuccess) return cuda_error(e, "host api buffer");
  *cap = std::max<size_t>(n, 1024);
  return UNLTD_OK;
}

int32_t host_gemv(float *out, size_t out_len, const float *x, size_t x_len, const uint8_t *w, size_t w_len,
                  size_t dim_in, size_t dim_out, int32_t dtype, int mode, const char *who) {
  if (!out || !x || !w) return set_error(UNLTD_ERR_INVALID_ARG, std::string(who) + ": NULL argument");
  if (out_len != dim_out) return set_error(UNLTD_ERR_LENGTH, std::string(who) + ": len(out) != dim_out");
  if (x_len < dim_in) return set_error(UNLTD_ERR_LENGTH, std::string(who) + ": len(x) < dim_in");
  if (mode == MODE_Q8K && dtype != Q4K && dtype != Q6K)
    return set_error(UNLTD_ERR_UNSUPPORTED, std::string(who) + ": dtype " + dtype_name(dtype) +
                                                " does not use a Q8_K dot (the reference refuses it too)");
  int32_t rc = check_view(dtype, dim_in, dim_out, w_len, who);
  if (rc) return rc;
  HostState &s = hs();
  std::lock_guard<std::mutex> lk(s.mu);
  if (!s.ctx) {
    rc = unltd_ctx_create(s.device, &s.ctx);
    if (rc) return rc;
  }
  CtxGuard g(s.ctx->device);
  auto key = std::make_tuple((const void *)w, w_len, (int)dtype, dim_in, dim_out);
  auto it = s.cache.find(key);
  const uint64_t fp = view_fingerprint(w, w_len);
  if (it != s.cache.end() && it->second.fp != fp) {  // other bytes at this address: upload again
    unltd_weight_free(it->second.w);
    s.cache.erase(it);
    it = s.cache.end();
  }
  unltd_weight wh;
  if (it == s.cache.end()) {
    rc = unltd_weight_upload(s.ctx, w, w_len, dtype, dim_in, dim_out, &wh);
    if (rc) return rc;
    s.cache[key] = HostState::Cached{wh, fp};
  } else {
    wh = it->second.w;
  }
  if ((rc = ensure_buf(&s.xbuf, &s.xcap, dim_in))) return rc;
  // `out` in page-locked host memory mapped into the device's address space
  // (cudaHostAlloc / cudaHostRegister): the GEMV stores y there itself, over
  // the bus while it runs, and no copy follows; otherwise y goes through a
  // device buffer and one copy.
  float *ydev = nullptr;
  cudaPointerAttributes pa{};
  if (cudaPointerGetAttributes(&pa, out) == cudaSuccess && pa.type == cudaMemoryTypeHost && pa.devicePointer)
    ydev = static_cast<float *>(pa.devicePointer);
  else
    cudaGetLastError();  // pageable memory: not an error
  if (!ydev && (rc = ensure_buf(&s.ybuf, &s.ycap, dim_out))) return rc;
  cudaStream_t st = s.ctx->stream;
  cudaError_t e = cudaMemcpyAsync(s.xbuf, x, dim_in * sizeof(float), cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return cuda_error(e, who);
  GemvArgs a{wh, s.xbuf, ydev ? ydev : s.ybuf, mode, nullptr, nullptr, nullptr};
  if ((rc = gemv_launch(s.ctx, a))) return rc;
  if (!ydev) {
    e = cudaMemcpyAsync(out, s.ybuf, dim_out * sizeof(float), cudaMemcpyDeviceToHost, st);
    if ((rc = cuda_error(e, who))) return rc;
  }
  return sync_and_check(s.ctx, st, who);
}

}  // namespace

extern "C" {

int32_t unltd_set_default_device(int32_t device) {
  HostState &s = hs();
  std::lock_guard<std::mutex> lk(s.mu);
  if (s.ctx) return set_error(UNLTD_ERR_INVALID_ARG, "set_default_device: the default context already exists");
  s.device = device;
  return UNLTD_OK;
}

int32_t unltd_forget_host_weights(void) {
  HostState &s = hs();
  std::lock_guard<std::mutex> lk(s.mu);
  for (auto &kv : s.cache) unltd_weight_free(kv.second.w);
  s.cache.clear();
  return UNLTD_OK;
}

int32_t unltd_gemv_quant(float *out, size_t out_len, const float *x, size_t x_len, const uint8_t *w, size_t w_len,
                         size_t dim_in, size_t dim_out, int32_t dtype) {
  return host_gemv(out, out_len, x, x_len, w, w_len, dim_in, dim_out, dtype, MODE_F32X, "gemv_quant");
}

int32_t unltd_gemv_quant_q8k(float *out, size_t out_len, const float *x, size_t x_len, const uint8_t *w,
                             size_t w_len, size_t dim_in, size_t dim_out, int32_t dtype) {
  return host_gemv(out, out_len, x, x_len, w, w_len, dim_in, dim_out, dtype, MODE_Q8K, "gemv_quant_q8k");
}

int32_t unltd_dequantize_q4_k(float *out, size_t out_len, const uint8_t *w, size_t w_len) {
  if (!out || !w) return set_error(UNLTD_ERR_INVALID_ARG, "dequantize_q4_k: NULL argument");
  if (out_len % kQK || w_len != out_len / kQK * kQ4Bytes)
    return set_error(UNLTD_ERR_LENGTH, "dequantize_q4_k: len(w) != exact blocks for len(out)");
  if (out_len == 0) return UNLTD_OK;
  HostState &s = hs();
  std::lock_guard<std::mutex> lk(s.mu);
  int32_t rc;
  if (!s.ctx && (rc = unltd_ctx_create(s.device, &s.ctx))) return rc;
  CtxGuard g(s.ctx->device);
  // one row of out_len elements: uncached (embedding rows are looked up once)
  unltd_weight wh;
  if ((rc = unltd_weight_upload(s.ctx, w, w_len, Q4K, out_len, 1, &wh))) return rc;
  float *dout = nullptr;
  cudaError_t e = cudaMalloc(&dout, out_len * sizeof(float));
  if (e == cudaSuccess) e = launch_dequant(*wh, dout, s.ctx->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(out, dout, out_len * sizeof(float), cudaMemcpyDeviceToHost, s.ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s.ctx->stream);
  if (dout) cudaFree(dout);
  unltd_weight_free(wh);
  return cuda_error(e, "dequantize_q4_k");
}

}  // extern "C"
