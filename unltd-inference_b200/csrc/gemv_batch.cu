// Batched decode GEMV: y_s = W . x_s for up to 32 sequences that share the
// weights (batch decode), every y_s bit-identical to gemv_quant_q8k
// (crates/unltd-tensor/src/quants.rs:474-515) of its x_s alone, i.e. to
// dot_q4_k_q8_k / dot_q6_k_q8_k (quants.rs:312-412) per row: the per-class
// integer sums sumi[k] are exact, and the f32 chains sums[k] += d * sumi[k]
// (and Q4_K's sumf -= dmin * sum(m * bsums)) run in the reference's block
// order, then s = sumf + sums[0] + ... + sums[7].
//
// The weights stream through shared memory once for all sequences (bulk
// copies by a producer warp, as in the single-sequence kernels); each compute
// warp owns 16 rows x a group of 8 sequences for the whole row and keeps the
// f32 chains of its (row, class, sequence) triples in registers, so no chain
// buffer or chain warp is needed. x comes from the batched images
// (unltd_internal.cuh, bimg_*): per span and group of 8 sequences, laid out
// as this kernel's B fragments, read from global memory (L2) one block ahead.
//
// The sequences are the MMA's N dimension. For class k the K dimension is
// the class's 32 elements of the block (4 per scale group):
//  * Q4_K: each 4-element word of a group shares the group's 6-bit scale, so
//    the scale is folded into A as two digits, sc = sc_lo + 8 sc_hi (0..7
//    each): A_lo = q * sc_lo, A_hi = q * sc_hi (<= 105, one 32-bit multiply
//    per packed word, no carries), and sumi[k] = D_lo + 8 D_hi exactly. The
//    min term is an m16n8k16 MMA of the mins against the balanced low / high
//    bytes of the sequences' group sums.
//  * Q6_K: A comes from digit planes made once per weight (batch6_convert):
//    v = sc * (q - 32) = 128 w1 + w0, so sumi[k] = D0 + 128 D1 exactly.
#include <algorithm>
#include <mutex>
#include <vector>

#include "mma_frag.cuh"
#include "q8k_span.cuh"
#include "unltd_host.h"
#include "unltd_internal.cuh"

namespace unltd {
namespace {

constexpr int kBatchWarps = 8;                        // compute warps
constexpr int kBatchThreads = (kBatchWarps + 1) * 32;  // + one producer warp
constexpr int kBatchStages = 4;
constexpr int kBatchHdr = 512;  // barriers + per-sequence argmax keys

struct BParams {
  const uint8_t *W;
  size_t pitch;        // bytes per row in global memory
  int rows, nbc, nch;  // rows; blocks per unit; units per row
  int unit_bytes;      // bytes of one row's unit (a 16-block chunk or the whole row)
  int ps, stage_bytes, S;
  const uint8_t *img;  // batched x images: (block b, sequence group sg) at img + bimg_block(b, sg, nsg)
  int nsg;
  float *y;            // y of sequence s at y + s * ystride (may be null with argmax)
  size_t ystride;
  int nseq;
  unsigned long long *key;  // argmax: one key per sequence (null: no argmax)
  unsigned *done;
  uint32_t *token;     // token of sequence s at token[s * tstride]
  size_t tstride;
  int row0;                         // global index of row 0 (a vocab shard)
  unsigned long long *key_out;      // non-null: the final keys here instead of tokens
  int *err;
};

__device__ __forceinline__ uint2 ldg64(const uint8_t *p) { return __ldg(reinterpret_cast<const uint2 *>(p)); }
__device__ __forceinline__ uint32_t ldg32(const uint8_t *p) { return __ldg(reinterpret_cast<const uint32_t *>(p)); }
__device__ __forceinline__ float ldgf(const uint8_t *p) { return __ldg(reinterpret_cast<const float *>(p)); }

// ---- Q4_K: 16 rows x 8 sequences, one block -------------------------------
// Thread (gid, tig) builds A for rows gid and gid + 8 from qs segment tig
// (word k of a segment = class k; low nibbles = group 2 tig, high = group
// 2 tig + 1): K-word tig = group 2 tig, K-word tig + 4 = group 2 tig + 1. B:
// the x words (group 2 tig, class k) and (group 2 tig + 1, class k) of
// sequence gid. D: rows gid / gid + 8 x sequences 2 tig / 2 tig + 1.
struct Q4Chain {
  float s[8][4];  // [class][(row gid, seq 2tig), (gid, 2tig+1), (gid+8, 2tig), (gid+8, 2tig+1)]
  float m[4];     // sumf (min term), same order
};

// This lane's x operands of one block, from the batched image of its
// sequence group (one coalesced 8-byte load each): the B words of sequence
// gid for the eight classes, its min-term words, and the d of the two
// sequences of its D columns. Loaded one block ahead of their use. Slots of
// sequences past the batch are never written; they feed only D columns that
// are never emitted (and the min-term rows with tig >= 2 are zero in A).
struct Q4X {
  uint2 bx[8];
  uint32_t bml, bmh;
  float xd0, xd1;
};

template <bool MIN>
__device__ __forceinline__ void q4x_load(const uint8_t *blk, Q4X &x) {
  const int lane = threadIdx.x & 31, tig = lane & 3;
#pragma unroll
  for (int k = 0; k < 8; k++) x.bx[k] = ldg64(blk + 256 * k + 8 * lane);
  const uint2 bm = MIN && tig < 2 ? ldg64(blk + 2048 + 8 * lane) : make_uint2(0u, 0u);
  x.bml = bm.x;
  x.bmh = bm.y;
  const float2 xd = __ldg(reinterpret_cast<const float2 *>(blk + 2304 + 8 * tig));
  x.xd0 = xd.x;
  x.xd1 = xd.y;
}

__device__ __forceinline__ void q4k_batch_block(const uint8_t *row0, const uint8_t *row1, int nbc, int b,
                                                const Q4X &x, Q4Chain &c) {
  const int lane = threadIdx.x & 31, tig = lane & 3;
  const uint4 h0 = lds128(row0 + b * 16), h1 = lds128(row1 + b * 16);
  const uint8_t *q0p = row0 + nbc * 16 + b * 128 + 32 * tig, *q1p = row1 + nbc * 16 + b * 128 + 32 * tig;
  const uint4 q0a = lds128(q0p), q0b = lds128(q0p + 16), q1a = lds128(q1p), q1b = lds128(q1p + 16);
  const uint32_t w0[8] = {q0a.x, q0a.y, q0a.z, q0a.w, q0b.x, q0b.y, q0b.z, q0b.w};
  const uint32_t w1[8] = {q1a.x, q1a.y, q1a.z, q1a.w, q1b.x, q1b.y, q1b.z, q1b.w};
  // scales of groups 2 tig, 2 tig + 1 (get_scale_min_k4, quants.rs:92-102)
  const bool lo4 = tig < 2;
  const uint32_t SC0 = lo4 ? (h0.y & 0x3F3F3F3Fu) : ((h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u));
  const uint32_t SC1 = lo4 ? (h1.y & 0x3F3F3F3Fu) : ((h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u));
  const int bi = 2 * (tig & 1);
  const int s00 = byte_of(SC0, bi), s01 = byte_of(SC0, bi + 1);  // row gid: groups 2tig, 2tig+1
  const int s10 = byte_of(SC1, bi), s11 = byte_of(SC1, bi + 1);  // row gid + 8
  const uint32_t l00 = s00 & 7, l01 = s01 & 7, l10 = s10 & 7, l11 = s11 & 7;
  const uint32_t g00 = s00 >> 3, g01 = s01 >> 3, g10 = s10 >> 3, g11 = s11 >> 3;
  // the sequences' d and the block's f16 d / dmin
  const float xd0 = x.xd0, xd1 = x.xd1;
  const float df0 = h2f_bits(h0.x & 0xFFFFu), df1 = h2f_bits(h1.x & 0xFFFFu);
  const float dm0 = h2f_bits(h0.x >> 16), dm1 = h2f_bits(h1.x >> 16);
  const float d[4] = {__fmul_rn(xd0, df0), __fmul_rn(xd1, df0), __fmul_rn(xd0, df1), __fmul_rn(xd1, df1)};
  // min term: sum_g m[g] * bsums[g] (A: mins of groups 4 tig .. 4 tig + 3 for
  // tig < 2; B: the balanced low / high bytes of sequence gid's group sums)
  const uint32_t MA0 = h0.z & 0x3F3F3F3Fu, MB0 = ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u);
  const uint32_t MA1 = h1.z & 0x3F3F3F3Fu, MB1 = ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u);
  const uint32_t am0 = tig == 0 ? MA0 : (tig == 1 ? MB0 : 0u), am1 = tig == 0 ? MA1 : (tig == 1 ? MB1 : 0u);
  int ml[4], mh[4];
  mma_s8_k16(am0, am1, x.bml, ml[0], ml[1], ml[2], ml[3]);
  mma_s8_k16(am0, am1, x.bmh, mh[0], mh[1], mh[2], mh[3]);
  const float dmv[4] = {__fmul_rn(dm0, xd0), __fmul_rn(dm0, xd1), __fmul_rn(dm1, xd0), __fmul_rn(dm1, xd1)};
#pragma unroll
  for (int i = 0; i < 4; i++) c.m[i] = __fsub_rn(c.m[i], __fmul_rn(dmv[i], (float)(ml[i] + 256 * mh[i])));
  // x words of sequence gid: class k, groups 2 tig and 2 tig + 1
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const uint2 bx = x.bx[k];
    const uint32_t n0l = w0[k] & 0x0F0F0F0Fu, n0h = (w0[k] >> 4) & 0x0F0F0F0Fu;
    const uint32_t n1l = w1[k] & 0x0F0F0F0Fu, n1h = (w1[k] >> 4) & 0x0F0F0F0Fu;
    int L[4], H[4];
    mma_s8(n0l * l00, n1l * l10, n0h * l01, n1h * l11, bx.x, bx.y, L[0], L[1], L[2], L[3]);
    mma_s8(n0l * g00, n1l * g10, n0h * g01, n1h * g11, bx.x, bx.y, H[0], H[1], H[2], H[3]);
#pragma unroll
    for (int i = 0; i < 4; i++) c.s[k][i] = __fadd_rn(c.s[k][i], __fmul_rn(d[i], (float)(L[i] + 8 * H[i])));
  }
}

// ---- Q6_K: 16 rows x 8 sequences, one block, from the digit planes -------
// Per block kBatch6Block bytes: plane w0 (256 B), plane w1 (256 B), f16 d.
// v = sc * (q - 32) = 128 w1 + w0 (w0 in [0, 127], w1 in [-32, 32]), so
// sumi[k] = D0 + 128 D1 exactly with D_p = sum over class k of w_p * q8. In
// a plane, class pair j, lane tig's 16 bytes at 64 j + 16 tig hold classes
// 2j and 2j + 1, each as the words of groups 2 tig and 2 tig + 1 (byte i of
// a word: element 32 g + 8 i + k), the K order of the Q4_K x image.
constexpr int kBatch6Block = 528;

__host__ __device__ inline int batch6_byte(int e, int plane) {
  const int g = e >> 5, i = (e >> 3) & 3, k = e & 7;
  return plane * 256 + (k >> 1) * 64 + (g >> 1) * 16 + (k & 1) * 8 + (g & 1) * 4 + i;
}

__device__ __forceinline__ void q6d_batch_block(const uint8_t *row0, const uint8_t *row1, int b, const Q4X &x,
                                                Q4Chain &c) {
  const int tig = threadIdx.x & 3;
  const uint8_t *p0 = row0 + b * kBatch6Block + 16 * tig, *p1 = row1 + b * kBatch6Block + 16 * tig;
  const float df0 = h2f_bits(*reinterpret_cast<const unsigned short *>(row0 + b * kBatch6Block + 512));
  const float df1 = h2f_bits(*reinterpret_cast<const unsigned short *>(row1 + b * kBatch6Block + 512));
  const float d[4] = {__fmul_rn(x.xd0, df0), __fmul_rn(x.xd1, df0), __fmul_rn(x.xd0, df1), __fmul_rn(x.xd1, df1)};
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const uint4 a0 = lds128(p0 + 64 * j), a1 = lds128(p1 + 64 * j);              // w0: rows gid, gid + 8
    const uint4 b0 = lds128(p0 + 256 + 64 * j), b1 = lds128(p1 + 256 + 64 * j);  // w1
#pragma unroll
    for (int kk = 0; kk < 2; kk++) {
      const int k = 2 * j + kk;
      const uint32_t r0g0 = kk ? a0.z : a0.x, r0g1 = kk ? a0.w : a0.y;
      const uint32_t r1g0 = kk ? a1.z : a1.x, r1g1 = kk ? a1.w : a1.y;
      const uint32_t s0g0 = kk ? b0.z : b0.x, s0g1 = kk ? b0.w : b0.y;
      const uint32_t s1g0 = kk ? b1.z : b1.x, s1g1 = kk ? b1.w : b1.y;
      int L[4], H[4];
      mma_s8(r0g0, r1g0, r0g1, r1g1, x.bx[k].x, x.bx[k].y, L[0], L[1], L[2], L[3]);
      mma_s8(s0g0, s1g0, s0g1, s1g1, x.bx[k].x, x.bx[k].y, H[0], H[1], H[2], H[3]);
#pragma unroll
      for (int i = 0; i < 4; i++) c.s[k][i] = __fadd_rn(c.s[k][i], __fmul_rn(d[i], (float)(L[i] + 128 * H[i])));
    }
  }
}

// Digit planes of a repacked Q6_K tensor: one thread per (row, block, element).
__global__ void batch6_convert(const uint8_t *__restrict__ dev, size_t stride, size_t rows, size_t nb,
                               uint8_t *__restrict__ out, size_t pitch) {
  const size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= rows * nb * kQK) return;
  const size_t r = t / (nb * kQK), rem = t % (nb * kQK);
  const int e = (int)(rem % kQK);
  size_t off;
  int nbl, b;
  q6_locate(nb, rem / kQK, off, nbl, b);
  const uint8_t *row = dev + r * stride + off;
  const int h = e >> 7, pos = e & 127;
  const int qlo = 64 * h + (pos & 63), qho = 32 * h + (pos & 31);
  const uint8_t lb = row[b * 128 + 16 * (qlo >> 4) + q6_pic(qlo & 15)];
  const uint8_t hb = row[nbl * 128 + b * 64 + 16 * (qho >> 4) + q6_pic(qho & 15)] ^ 0xAAu;  // stored flipped
  const int nib = pos < 64 ? (lb & 0xF) : (lb >> 4);
  const int q = (nib | (((hb >> (2 * (pos >> 5))) & 3) << 4)) - 32;
  const int sc = (int8_t)row[nbl * 192 + b * 16 + (e >> 4)];
  const int v = sc * q;          // in [-4064, 4096]
  const int w1 = v >> 7;         // floor(v / 128), in [-32, 32]
  const int w0 = v - 128 * w1;   // in [0, 127]
  uint8_t *blk = out + r * pitch + (rem / kQK) * kBatch6Block;
  blk[batch6_byte(e, 0)] = (uint8_t)w0;
  blk[batch6_byte(e, 1)] = (uint8_t)(int8_t)w1;
  if (e == 0) {
    blk[512] = row[nbl * 208 + b * 2];
    blk[513] = row[nbl * 208 + b * 2 + 1];
  }
  if (e < 14) blk[514 + e] = 0;
}

__device__ __forceinline__ void batch_emit(const BParams &P, int row, int seq, float acc,
                                           unsigned long long *best) {
  if (P.y) P.y[(size_t)seq * P.ystride + row] = acc;
  if (P.key) atomicMax(best + seq, argmax_key(acc, P.row0 + row));
}

// T rows per tile (16 x the row groups); SB sequences per warp task. Warp w
// takes row group w % (T / 16) and sequence group w / (T / 16).
template <int FMT, int T, int SB>
__global__ void __launch_bounds__(kBatchThreads, 1) gemv_batch_kernel(BParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *full = reinterpret_cast<uint64_t *>(smem);
  uint64_t *empty = full + kBatchStages;
  unsigned long long *best = reinterpret_cast<unsigned long long *>(smem + 128);  // [32]
  uint8_t *stages = smem + kBatchHdr;
  const int S = P.S;
  pdl_trigger();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int rb = (int)((long long)P.rows * blockIdx.x / G);
  const int re = (int)((long long)P.rows * (blockIdx.x + 1) / G);
  const int ntiles = (re - rb + T - 1) / T;
  const int nunits = ntiles * P.nch;

  if (threadIdx.x == 0) {
    for (int st = 0; st < S; st++) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], kBatchWarps);
    }
    fence_mbar_init();
  }
  if (threadIdx.x < 32) best[threadIdx.x] = 0ull;
  __syncthreads();

  if (warp == kBatchWarps) {
    // ---------------- producer: one bulk copy per row and unit ---------------
    if (lane == 0) {
      int issued = 0;
      for (int u = 0; u < nunits; u++) {
        const int st = u % S;
        if (u >= S && !mbar_wait_bounded(&empty[st], ((u / S) - 1) & 1, P.err)) break;
        const int r0 = rb + (u / P.nch) * T;
        const int nr = min(T, re - r0);
        mbar_expect_tx(&full[st], (uint32_t)(nr * P.unit_bytes));
        const uint8_t *src = P.W + (size_t)r0 * P.pitch + (size_t)(u % P.nch) * P.unit_bytes;
        uint8_t *dst = stages + (size_t)st * P.stage_bytes;
        for (int rr = 0; rr < nr; rr++)
          bulk_g2s(dst + rr * P.ps, src + (size_t)rr * P.pitch, (uint32_t)P.unit_bytes, &full[st]);
        issued = u + 1;
      }
      for (int u = max(0, issued - S); u < issued; u++) mbar_wait_bounded(&full[u % S], (u / S) & 1, P.err);
    }
    return;
  }

  pdl_wait();
  constexpr int NG = T / 16;
  const int gid = lane >> 2, tig = lane & 3;
  const int g = warp % NG, sg = warp / NG;
  const int nsg = (P.nseq + SB - 1) / SB;
  const bool active = sg < nsg;
  const int nbc = P.nbc;
  static_assert(SB == 8, "the 8 sequences of a group are the MMA's N");
  const int sa = sg * 8 + 2 * tig, sb2 = sa + 1;  // D: sequences of this thread
  const uint8_t *img = P.img + (size_t)(active ? sg : 0) * kBImgBlock;  // block b at + b * nsg * kBImgBlock
  const size_t bstride = (size_t)P.nsg * kBImgBlock;
  Q4Chain ch;
  // x of the first block; then always one block ahead (units run in the
  // order tile, chunk, so the block after a unit's last is the next chunk's
  // first: block ((c + 1) % nch) * nbc)
  Q4X xc;
  if (active) q4x_load<FMT == Q4K>(img, xc);
  for (int u = 0; u < nunits; u++) {
    const int st = u % S, c = u % P.nch;
    if (!mbar_wait_bounded(&full[st], (u / S) & 1, P.err)) break;
    if (active) {
      if (c == 0) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
          ch.m[i] = 0.0f;
#pragma unroll
          for (int k = 0; k < 8; k++) ch.s[k][i] = 0.0f;
        }
      }
      const uint8_t *tile = stages + (size_t)st * P.stage_bytes;
      const uint8_t *row0 = tile + (16 * g + gid) * P.ps, *row1 = row0 + 8 * P.ps;
      const int nxt = ((c + 1) % P.nch) * nbc;
#pragma unroll 1
      for (int b = 0; b < nbc; b++) {
        const size_t xo = (size_t)(b + 1 < nbc ? c * nbc + b + 1 : nxt) * bstride;
        Q4X xn;
        q4x_load<FMT == Q4K>(img + xo, xn);
        if constexpr (FMT == Q4K) q4k_batch_block(row0, row1, nbc, b, xc, ch);
        else q6d_batch_block(row0, row1, b, xc, ch);
        xc = xn;
      }
      if (c == P.nch - 1) {
        const int r0 = rb + (u / P.nch) * T + 16 * g + gid;
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const int row = r0 + 8 * (i >> 1), seq = (i & 1) ? sb2 : sa;
          // s = sumf + sums[0] + ... + sums[7] (Q6_K: sumf = 0)
          float acc = ch.m[i];
#pragma unroll
          for (int k = 0; k < 8; k++) acc = __fadd_rn(acc, ch.s[k][i]);
          if (row < re && seq < P.nseq) batch_emit(P, row, seq, acc, best);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }

  if (P.key) {
    // per-sequence argmax: CTA best -> global MAX; the last CTA writes the tokens
    named_bar_sync(1, kBatchWarps * 32);
    if (warp == 0) {
      const int s = lane;
      if (s < P.nseq) atomicMax(P.key + s, best[s]);
      __threadfence();
      __syncwarp();
      unsigned prev = 0;
      if (lane == 0) prev = atomicAdd(P.done, 1u);
      prev = __shfl_sync(0xffffffffu, prev, 0);
      if (prev == gridDim.x - 1) {
        __threadfence();
        if (s < P.nseq) {
          const unsigned long long kf = atomicAdd(P.key + s, 0ull);
          if (P.key_out) P.key_out[s] = kf;
          else P.token[(size_t)s * P.tstride] = 0xffffffffu - (uint32_t)(kf & 0xffffffffull);
          P.key[s] = 0ull;
        }
        __syncwarp();
        if (lane == 0) *P.done = 0u;
      }
    }
  }
}

// Batched x images: quantize_q8_k of every span of every sequence (grid:
// spans x sequences), in the class-major layout of the Q4_K image, which the
// batched kernel reads for both formats.
__global__ void __launch_bounds__(256) prep_q8k_batch(const float *__restrict__ x, size_t dim_in, size_t xstride,
                                                      uint8_t *__restrict__ img, int nsg) {
  pdl_trigger();
  __shared__ Q8KSpanSmem sm;
  const size_t span = blockIdx.x, s = blockIdx.y;
  const size_t e = span * kQK + threadIdx.x;
  const float v = e < dim_in ? x[s * xstride + e] : 0.0f;
  q8k_span_write(v, nullptr, nullptr, sm, img + bimg_block(span, (int)(s >> 3), nsg), (int)(s & 7));
}

using BatchFn = void (*)(BParams);

struct BatchPlan {
  BatchFn fn = nullptr;
  int T = 0, S = 0, ps = 0, stage_bytes = 0, smem = 0, nch = 1, nbc = 0, unit_bytes = 0;
};

int max_smem_optin_b(int device) {
  static int cache[64] = {0};
  if (device >= 0 && device < 64 && cache[device]) return cache[device];
  int v = 0;
  cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  if (device >= 0 && device < 64) cache[device] = v;
  return v;
}

// Per (device, kernel) dynamic shared-memory limit, set once.
cudaError_t ensure_batch_attr(int device, BatchFn fn, int smem) {
  static std::mutex mu;
  static std::vector<std::pair<int, BatchFn>> done;
  std::lock_guard<std::mutex> lk(mu);
  for (auto &d : done)
    if (d.first == device && d.second == fn) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess) done.push_back({device, fn});
  return e;
}

// Q4_K: a unit is 32 rows x the whole row. Q6_K (digit planes): 32 rows x
// nbc consecutive blocks, nbc the largest divisor of the block count up to 4
// (the planes of consecutive blocks are contiguous). Shared-memory rows are
// padded past a multiple of 128 bytes so a warp's 128-bit loads (eight rows
// x four lanes) take the minimum four wavefronts: by 16 bytes for Q4_K
// (lanes read 16 bytes at 32 tig of their row), by 64 for the Q6_K planes
// (lanes read 16 bytes at 16 tig).
BatchPlan batch_plan(int device, const unltd_weight_s &w) {
  BatchPlan p;
  const bool q4 = w.dtype == Q4K;
  p.T = 32;
  if (q4) {
    p.nch = 1;
    p.nbc = (int)w.nb;
    p.unit_bytes = (int)w.row_stride;
  } else {
    int nbc = 1;
    for (int c = 4; c >= 1; c--)
      if (w.nb % c == 0) {
        nbc = c;
        break;
      }
    p.nbc = nbc;
    p.nch = (int)(w.nb / nbc);
    p.unit_bytes = nbc * kBatch6Block;
  }
  p.ps = (int)round_up((size_t)p.unit_bytes, 128) + (q4 ? 16 : 64);
  p.stage_bytes = (int)round_up((size_t)p.T * p.ps, 128);
  const int smem_max = max_smem_optin_b(device) - 1024;
  p.S = std::min(kBatchStages, (smem_max - kBatchHdr) / p.stage_bytes);
  if (p.S < 2) return p;
  p.smem = kBatchHdr + p.S * p.stage_bytes;
  p.fn = q4 ? gemv_batch_kernel<Q4K, 32, 8> : gemv_batch_kernel<Q6K, 32, 8>;
  return p;
}

}  // namespace

size_t gemv_batch_img_bytes(const unltd_weight_s &w, int nseq) {
  return w.nb * (size_t)((nseq + 7) / 8) * kBImgBlock;
}

int32_t gemv_batch_prepare(unltd_ctx ctx, unltd_weight_s *w) {
  if (w->dtype != Q6K || w->dev_b || w->dim_out == 0) return UNLTD_OK;
  const size_t pitch = w->nb * kBatch6Block;
  uint8_t *out = nullptr;
  cudaError_t e = cudaMalloc(&out, w->dim_out * pitch);
  if (e != cudaSuccess) return cuda_error(e, "gemv_batch: Q6_K digit planes");
  const size_t n = w->dim_out * w->nb * kQK;
  batch6_convert<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(w->dev, w->row_stride, w->dim_out, w->nb, out,
                                                                        pitch);
  e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) {
    cudaFree(out);
    return cuda_error(e, "gemv_batch: Q6_K digit planes");
  }
  w->dev_b = out;
  w->b_pitch = pitch;
  return UNLTD_OK;
}

int32_t gemv_batch_launch(unltd_ctx ctx, const BatchGemvArgs &a) {
  const unltd_weight_s &w = *a.w;
  if (w.dtype != Q4K && w.dtype != Q6K)
    return set_error(UNLTD_ERR_UNSUPPORTED, "gemv_batch: Q4_K and Q6_K weights only (Q8K_EXACT)");
  if (a.nseq < 1 || a.nseq > kMaxBatch) return set_error(UNLTD_ERR_INVALID_ARG, "gemv_batch: n_seq must be 1..32");
  if (w.dim_out == 0) return UNLTD_OK;
  if (w.dim_out > (size_t)INT32_MAX) return set_error(UNLTD_ERR_UNSUPPORTED, "gemv_batch: too many rows");
  const BatchPlan pl = batch_plan(ctx->device, w);
  if (!pl.fn) return set_error(UNLTD_ERR_UNSUPPORTED, "gemv_batch: rows too long for a shared-memory tile");
  if (w.dtype == Q6K && !w.dev_b) return set_error(UNLTD_ERR_INVALID_ARG, "gemv_batch: Q6_K weight not prepared");
  cudaStream_t st = ctx->stream;
  const int nsg = (a.nseq + 7) / 8;
  const uint8_t *img = a.img;
  if (!img) {
    if (!a.x) return set_error(UNLTD_ERR_INVALID_ARG, "gemv_batch: no x and no image");
    if (ctx->scratch_bytes < gemv_batch_img_bytes(w, a.nseq))
      return set_error(UNLTD_ERR_INVALID_ARG, "gemv_batch: scratch not reserved");
    const dim3 grid((unsigned)w.nb, (unsigned)a.nseq);
    prep_q8k_batch<<<grid, 256, 0, st>>>(a.x, w.dim_in, a.xstride, ctx->scratch, nsg);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, "gemv_batch prep");
    ctx->launches += 1;
    img = ctx->scratch;
  }
  if (cudaError_t e = ensure_batch_attr(ctx->device, pl.fn, max_smem_optin_b(ctx->device) - 1024); e != cudaSuccess)
    return cuda_error(e, "gemv_batch attribute");
  BParams P;
  P.W = w.dtype == Q6K ? w.dev_b : w.dev;
  P.pitch = w.dtype == Q6K ? w.b_pitch : w.row_stride;
  P.rows = (int)w.dim_out;
  P.nbc = pl.nbc;
  P.nch = pl.nch;
  P.unit_bytes = pl.unit_bytes;
  P.ps = pl.ps;
  P.stage_bytes = pl.stage_bytes;
  P.S = pl.S;
  P.img = img;
  P.nsg = a.img ? a.nsg : nsg;
  P.y = a.y;
  P.ystride = a.ystride;
  P.nseq = a.nseq;
  P.key = a.key;
  P.done = a.done;
  P.token = a.token;
  P.tstride = a.tstride;
  P.row0 = a.row0;
  P.key_out = a.key_out;
  P.err = ctx->err;
  const int grid = std::max(1, std::min(ctx->num_sms, (P.rows + pl.T - 1) / pl.T));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kBatchThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, pl.fn, P);
  if (e != cudaSuccess) return cuda_error(e, "gemv_batch launch");
  ctx->launches += 1;
  return UNLTD_OK;
}

// Sets both batched kernels' shared-memory limits on `device` (current), so
// that launches inside a graph capture find them set.
cudaError_t gemv_batch_prewarm(int device) {
  const int m = max_smem_optin_b(device) - 1024;
  cudaError_t e = ensure_batch_attr(device, gemv_batch_kernel<Q4K, 32, 8>, m);
  if (e == cudaSuccess) e = ensure_batch_attr(device, gemv_batch_kernel<Q6K, 32, 8>, m);
  return e;
}

bool gemv_batch_supported(int device, const unltd_weight_s &w) {
  return (w.dtype == Q4K || w.dtype == Q6K) && batch_plan(device, w).fn != nullptr;
}

}  // namespace unltd
