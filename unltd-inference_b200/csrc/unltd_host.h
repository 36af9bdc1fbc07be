// Host-side internal interfaces of libunltd_gpu (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <atomic>
#include <string>

#include "../../include/unltd_gpu.h"

struct unltd_ctx_s {
  int device = 0;
  int num_sms = 0;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  // Scratch for per-call x images (grown on demand, never shrunk).
  uint8_t *scratch = nullptr;
  size_t scratch_bytes = 0;
  // The scratch is a fixed array the context does not own (unltd_gemv_noalloc):
  // gemv_reserve must neither free nor grow it.
  bool scratch_fixed = false;
  // Argmax reduction state: a 64-bit key and a CTA-completion counter.
  unsigned long long *argmax_key = nullptr;
  unsigned int *argmax_done = nullptr;
  // Per-sequence argmax state of the batched GEMV (kMaxBatch keys, a counter,
  // kMaxBatch tokens), inside the same allocation as argmax_key.
  unsigned long long *bkey = nullptr;
  unsigned int *bdone = nullptr;
  uint32_t *btok = nullptr;
  // Device error word: kernels write a nonzero code on a bounded-wait timeout.
  int *err = nullptr;
  // Pinned host copy of the error word: read back with the call's own results
  // so a synchronous call needs one stream synchronisation, not two.
  int *err_host = nullptr;
  // Scratch of the prefill GEMM (bf16 copy of X), grown on demand.
  uint8_t *gemm_scratch = nullptr;
  size_t gemm_scratch_bytes = 0;
  std::atomic<int64_t> launches{0};
  void *comm = nullptr;  // ncclComm_t once unltd_comm_init ran
  int rank = 0, world = 1;
  // Peer all-reduce over NVLink (comm.cu): this rank's receive area
  // (exported through CUDA IPC), every rank's area mapped into this process
  // (own = peer_area), and the device counter of all-reduces issued.
  void *peer_area = nullptr;
  void *peer_map[8] = {};
  unsigned *peer_ctr = nullptr;
  unsigned *peer_done = nullptr;  // CTAs of a sending GEMV that finished (reset by the last)
  bool peer_ok = false;
};

namespace unltd {
// Every rank's peer receive area: 64 flag words (flag[src] = the last
// all-reduce number rank src completed writing here), then two parities x
// kPeerMaxRanks source slots of kPeerMaxCount 8-byte words.
constexpr int kPeerMaxRanks = 8;
constexpr size_t kPeerMaxCount = 131072;  // floats (or u64) per all-reduce: 32 sequences x 4096
constexpr size_t kPeerFlagBytes = 256;
constexpr size_t kPeerSlotBytes = kPeerMaxCount * 8;
constexpr size_t kPeerAreaBytes = kPeerFlagBytes + 2 * kPeerMaxRanks * kPeerSlotBytes;
constexpr int kErrPeer = 3;
}  // namespace unltd

struct unltd_weight_s {
  unltd_ctx ctx = nullptr;
  int dtype = 0;
  size_t dim_in = 0, dim_out = 0;
  size_t nb = 0;          // blocks per row (256 elems for K-quants, 32 for Q8_0)
  size_t row_bytes = 0;   // GGUF bytes per row
  size_t row_stride = 0;  // device bytes per row (row_bytes rounded up to 16)
  uint8_t *dev = nullptr;
  // Q6_K for the batched GEMV (made on first batched use): per block, the
  // scaled quants v = sc * (q - 32) as two int8 digit planes (v = 128 w1 + w0)
  // in the MMA's operand order, then the block's f16 d; kBatch6Block bytes
  // per block, b_pitch per row.
  uint8_t *dev_b = nullptr;
  size_t b_pitch = 0;
};

namespace unltd {

// Makes `dev` the current device for a scope and restores the previous one.
struct CtxGuard {
  int prev = -1;
  explicit CtxGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~CtxGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// Thread-local error message behind unltd_last_error().
int32_t set_error(int32_t status, const std::string &msg);
int32_t cuda_error(cudaError_t e, const char *what);
// Waits for the work queued on `st` and reads c's device error word in the
// same round trip; a nonzero word is cleared and returned as an error status.
int32_t sync_and_check(unltd_ctx c, cudaStream_t st, const char *who);

// weights.cu
cudaError_t launch_repack(const unltd_weight_s &w, const uint8_t *raw_dev, size_t row0_local,
                          size_t rows, cudaStream_t s);
cudaError_t launch_dequant(const unltd_weight_s &w, float *out, cudaStream_t s);

// gemv.cu
struct GemvNorm {
  const float *a, *b;
  float *r_out;
  const float *w;
  float eps;
  uint8_t *img4_out, *img6_out;
  // b is the tensor-parallel row-split sum received over peer memory (b
  // null): the slots of the last all-reduce summed in rank order
  bool peer_recv = false;
};
struct GemvArgs {
  const unltd_weight_s *w;
  const float *x;
  float *y;
  int mode;
  unsigned long long *argmax_key;  // non-null: fused argmax
  unsigned int *argmax_done;
  uint32_t *token;
  // Non-null: the x image was already written (by a fused producer kernel
  // that ran before on the same stream, in this mode's layout); no prep.
  const uint8_t *img = nullptr;
  // Fused argmax of a vocab shard: global index of row 0, and where to store
  // the final 64-bit key (for the cross-GPU MAX) besides the token.
  int argmax_row0 = 0;
  unsigned long long *key_out = nullptr;
  // Non-null: RMSNorm fused into the GEMV's prologue (tensor-core Q4_K Q8K
  // path only, see gemv_norm_fusable): x = rmsnorm(a (+ b), w) is quantized
  // by every CTA into its own image; CTA 0 also stores r = a (+ b) to r_out
  // and the Q4_K / Q6_K images to img4_out / img6_out for later GEMVs.
  const GemvNorm *norm = nullptr;
  // Tensor parallelism with peer_import done: instead of y, store the rows
  // into this rank's slot of every rank's peer area and raise the flag (the
  // consumer's fused norm receives them with GemvNorm::peer_recv).
  bool peer_send = false;
};
int32_t gemv_launch(unltd_ctx ctx, const GemvArgs &a);

// gemv_batch.cu: y_s = W . x_s for nseq sequences (Q8K_EXACT, Q4_K / Q6_K),
// each y_s the bits of gemv_launch's on x_s alone.
constexpr int kMaxBatch = 32;
struct BatchGemvArgs {
  const unltd_weight_s *w;
  const float *x = nullptr;     // [nseq][xstride] f32 (null: img is given)
  size_t xstride = 0;
  const uint8_t *img = nullptr;  // non-null: the batched x images (kBImgBlock per span and sequence group)
  int nsg = 0;                   // sequence groups the images hold (their stride)
  float *y = nullptr;           // [nseq][ystride] (may be null with argmax)
  size_t ystride = 0;
  int nseq = 1;
  unsigned long long *key = nullptr;  // non-null: fused argmax, one key per sequence
  unsigned *done = nullptr;
  uint32_t *token = nullptr;
  size_t tstride = 1;                 // token of sequence s at token[s * tstride]
  // a vocab shard: the global index of row 0; non-null key_out: every
  // sequence's final argmax key there instead of its token
  int row0 = 0;
  unsigned long long *key_out = nullptr;
};
int32_t gemv_batch_launch(unltd_ctx ctx, const BatchGemvArgs &a);
// Bytes of the batched x images of nseq sequences for w.
size_t gemv_batch_img_bytes(const unltd_weight_s &w, int nseq);
bool gemv_batch_supported(int device, const unltd_weight_s &w);
cudaError_t gemv_batch_prewarm(int device);
// Makes w's batched-GEMV operands (Q6_K digit planes) if w needs them and
// they do not exist yet; allocates and synchronizes, so never inside a
// stream capture.
int32_t gemv_batch_prepare(unltd_ctx ctx, unltd_weight_s *w);
// True when gemv_launch can fuse an RMSNorm of length w.dim_in into w's GEMV.
bool gemv_norm_fusable(unltd_ctx ctx, const unltd_weight_s &w, int mode);
// True when w's GEMV runs on the tensor-core kernel (peer row-split sums).
bool gemv_tc_eligible(unltd_ctx ctx, const unltd_weight_s &w, int mode);
// Grow the context's x-image scratch for w (call before stream capture).
int32_t gemv_reserve(unltd_ctx ctx, const unltd_weight_s &w, int mode);
cudaError_t gemv_prewarm(int device);

// gguf.cu: a tensor of an opened GGUF file (data: a view into the mapping,
// null when its type is not one this path reads)
struct GgufTensorView {
  const void *data;
  size_t nbytes;
  int dtype;
  uint32_t ndims;
  int64_t ne[4];
};
bool gguf_tensor(unltd_gguf g, const std::string &name, GgufTensorView *out);

// comm.cu (NCCL through dlopen)
int32_t comm_allreduce(unltd_ctx c, cudaStream_t st, void *buf, size_t count, bool max_u64);
void comm_destroy(unltd_ctx c);

// gemm_tc.cu
// accurate: X and W as hi + lo fp16 pairs, three MMAs per K slice (1e-4 max-rel
// of the f64 truth); otherwise fp16 operands rounded once.
int32_t gemm_launch(unltd_ctx ctx, const unltd_weight_s &w, const float *X, float *Y, size_t M, bool accurate);

}  // namespace unltd
