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
// warp owns 16 rows x a group of sequences for the whole row and keeps the
// f32 chains of its (row, class, sequence) triples in registers, so no chain
// buffer or chain warp is needed. The x images (one per sequence, the Q8_K
// layouts of unltd_internal.cuh) are read from global memory (L2).
//
//  * Q4_K: the sequences are the MMA's N dimension. For class k the K
//    dimension is the class's 32 elements of the block (4 per scale group);
//    each 4-element word of a group shares the group's 6-bit scale, so the
//    scale is folded into A as two digits, sc = sc_lo + 8 sc_hi (0..7 each):
//    A_lo = q * sc_lo, A_hi = q * sc_hi (<= 105, one 32-bit multiply per
//    packed word, no carries), and sumi[k] = D_lo + 8 D_hi exactly. The min
//    term is an m16n8k16 MMA of the mins against the balanced low / high
//    bytes of the sequences' group sums.
//  * Q6_K: per sequence, the class-masked MMAs of the single-sequence kernel
//    (A operands and scales built once per block and reused).
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
  const uint8_t *img;  // x images: sequence s at img + s * istride
  size_t istride;
  float *y;            // y of sequence s at y + s * ystride (may be null with argmax)
  size_t ystride;
  int nseq;
  unsigned long long *key;  // argmax: one key per sequence (null: no argmax)
  unsigned *done;
  uint32_t *token;     // token of sequence s at token[s * tstride]
  size_t tstride;
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

// This lane's x operands of one block (from global memory): the B words of
// sequence gid for the eight classes, its min-term words, and the d of the
// two sequences of its D columns. Loaded one block ahead of their use.
struct Q4X {
  uint2 bx[8];
  uint32_t bml, bmh;
  float xd0, xd1;
};

__device__ __forceinline__ void q4x_load(const uint8_t *xg, bool xv, const uint8_t *xs0, bool v0, const uint8_t *xs1,
                                         bool v1, Q4X &x) {
  const int tig = threadIdx.x & 3;
  const uint8_t *xw = xg + 128 * (tig >> 1) + 8 * (tig & 1);
#pragma unroll
  for (int k = 0; k < 8; k++) x.bx[k] = xv ? ldg64(xw + 16 * k) : make_uint2(0u, 0u);
  const bool bmv = xv && tig < 2;
  x.bml = bmv ? ldg32(xg + kImgQ8K4_BM + 4 * tig) : 0u;
  x.bmh = bmv ? ldg32(xg + kImgQ8K4_BM + 4 * (2 + tig)) : 0u;
  x.xd0 = v0 ? ldgf(xs0 + kImgQ8K4_D) : 0.0f;
  x.xd1 = v1 ? ldgf(xs1 + kImgQ8K4_D) : 0.0f;
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

// ---- Q6_K: 16 rows, one sequence at a time ---------------------------------
// The A operands (4 (raw6 - 32) as s8) and the sub-block scales of the block
// for rows gid, gid + 8, built once and kept in registers.
struct Q6Frag {
  uint32_t alo0[8], ahi0[8], alo1[8], ahi1[8];
  int s0[8], t0[8], s1[8], t1[8];
  float df0, df1;
};

__device__ __forceinline__ void q6k_batch_frag(const uint8_t *row0, const uint8_t *row1, int nbc, int b, Q6Frag &f) {
  const int lane = threadIdx.x & 31, tig = lane & 3;
  const int qlo = b * 128 + 4 * tig, qho = nbc * 128 + b * 64 + 4 * tig;
  uint32_t h0[4], h1[4];
#pragma unroll
  for (int c = 0; c < 4; c++) {
    h0[c] = *reinterpret_cast<const uint32_t *>(row0 + qho + 16 * c);
    h1[c] = *reinterpret_cast<const uint32_t *>(row1 + qho + 16 * c);
  }
  const uint4 sc0 = lds128(row0 + nbc * 192 + b * 16), sc1 = lds128(row1 + nbc * 192 + b * 16);
  const uint32_t S0[4] = {sc0.x, sc0.y, sc0.z, sc0.w}, S1[4] = {sc1.x, sc1.y, sc1.z, sc1.w};
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int h = j >> 2, u = j & 3, sl = 2 * (u >> 1), c = 2 * h + (u & 1);
    const int slo = 8 * h + u, shi = slo + 4;  // the chunk's two sub-blocks
    const uint32_t l0 = *reinterpret_cast<const uint32_t *>(row0 + qlo + 16 * j);
    const uint32_t l1 = *reinterpret_cast<const uint32_t *>(row1 + qlo + 16 * j);
    f.alo0[j] = q6_a4_lo(l0, h0[c], sl);
    f.ahi0[j] = q6_a4_hi(l0, h0[c], sl);
    f.alo1[j] = q6_a4_lo(l1, h1[c], sl);
    f.ahi1[j] = q6_a4_hi(l1, h1[c], sl);
    f.s0[j] = sbyte_of(S0[slo >> 2], slo & 3);
    f.t0[j] = sbyte_of(S0[shi >> 2], shi & 3);
    f.s1[j] = sbyte_of(S1[slo >> 2], slo & 3);
    f.t1[j] = sbyte_of(S1[shi >> 2], shi & 3);
  }
  f.df0 = h2f_bits(*reinterpret_cast<const unsigned short *>(row0 + nbc * 208 + b * 2));
  f.df1 = h2f_bits(*reinterpret_cast<const unsigned short *>(row1 + nbc * 208 + b * 2));
}

// One sequence's products of the block: the chains of (row gid, classes 2 tig,
// 2 tig + 1) and (row gid + 8, the same classes).
__device__ __forceinline__ void q6k_batch_seq(const Q6Frag &f, const XBlock6 &x, float (&s)[4]) {
  int acc0 = 0, acc1 = 0, acc2 = 0, acc3 = 0;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    int d0, d1, d2, d3, e0, e1, e2, e3;
    mma_s8_k16(f.alo0[j], f.alo1[j], x.b[2 * j], d0, d1, d2, d3);
    mma_s8_k16(f.ahi0[j], f.ahi1[j], x.b[2 * j + 1], e0, e1, e2, e3);
    acc0 += f.s0[j] * d0 + f.t0[j] * e0;
    acc1 += f.s0[j] * d1 + f.t0[j] * e1;
    acc2 += f.s1[j] * d2 + f.t1[j] * e2;
    acc3 += f.s1[j] * d3 + f.t1[j] * e3;
  }
  const float d0 = __fmul_rn(x.xd, f.df0), d1 = __fmul_rn(x.xd, f.df1);
  s[0] = __fadd_rn(s[0], __fmul_rn(d0, (float)(acc0 >> 2)));
  s[1] = __fadd_rn(s[1], __fmul_rn(d0, (float)(acc1 >> 2)));
  s[2] = __fadd_rn(s[2], __fmul_rn(d1, (float)(acc2 >> 2)));
  s[3] = __fadd_rn(s[3], __fmul_rn(d1, (float)(acc3 >> 2)));
}

__device__ __forceinline__ void batch_emit(const BParams &P, int row, int seq, float acc,
                                           unsigned long long *best) {
  if (P.y) P.y[(size_t)seq * P.ystride + row] = acc;
  if (P.key) atomicMax(best + seq, argmax_key(acc, row));
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
  if constexpr (FMT == Q4K) {
    static_assert(SB == 8, "Q4_K: the 8 sequences of a group are the MMA's N");
    const int sx = sg * 8 + gid;                          // B: sequence of column gid
    const int sa = sg * 8 + 2 * tig, sb2 = sa + 1;         // D: sequences of this thread
    const bool xv = sx < P.nseq, v0 = sa < P.nseq, v1 = sb2 < P.nseq;
    const uint8_t *imx = P.img + (size_t)(xv ? sx : 0) * P.istride;
    const uint8_t *im0 = P.img + (size_t)(v0 ? sa : 0) * P.istride;
    const uint8_t *im1 = P.img + (size_t)(v1 ? sb2 : 0) * P.istride;
    Q4Chain ch;
    // x of block 0 (Q4_K rows are never chunked: every unit runs blocks 0 .. nbc-1)
    Q4X xc;
    q4x_load(imx, xv, im0, v0, im1, v1, xc);
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
#pragma unroll 1
        for (int b = 0; b < nbc; b++) {
          // the next block's x (block 0 again after the last: the next tile's first)
          const size_t xo = (size_t)(b + 1 < nbc ? b + 1 : 0) * kImgQ8K4;
          Q4X xn;
          q4x_load(imx + xo, xv, im0 + xo, v0, im1 + xo, v1, xn);
          q4k_batch_block(row0, row1, nbc, b, xc, ch);
          xc = xn;
        }
        if (c == P.nch - 1) {
          const int r0 = rb + (u / P.nch) * T + 16 * g + gid;
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const int row = r0 + 8 * (i >> 1), seq = (i & 1) ? sb2 : sa;
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
  } else {
    float ch[SB][4];
    for (int u = 0; u < nunits; u++) {
      const int st = u % S, c = u % P.nch;
      if (!mbar_wait_bounded(&full[st], (u / S) & 1, P.err)) break;
      if (active) {
        if (c == 0) {
#pragma unroll
          for (int q = 0; q < SB; q++)
#pragma unroll
            for (int i = 0; i < 4; i++) ch[q][i] = 0.0f;
        }
        const uint8_t *tile = stages + (size_t)st * P.stage_bytes;
        const uint8_t *row0 = tile + (16 * g + gid) * P.ps, *row1 = row0 + 8 * P.ps;
        // sequence q's x of block b, loaded one (block, sequence) step ahead
        const int nvq = min(SB, P.nseq - sg * SB);  // this group's sequences (warp-uniform)
        auto xim = [&](int b, int q) {
          return P.img + (size_t)(sg * SB + q) * P.istride + (size_t)(c * nbc + b) * kImgQ8K6;
        };
        XBlock6 xc;
        load_xblock6(xim(0, 0), xc);
#pragma unroll 1
        for (int b = 0; b < nbc; b++) {
          Q6Frag f;
          q6k_batch_frag(row0, row1, nbc, b, f);
#pragma unroll
          for (int q = 0; q < SB; q++) {
            if (q < nvq) {
              const bool lastq = q + 1 >= nvq;
              const int bn = lastq ? b + 1 : b, qn = lastq ? 0 : q + 1;
              XBlock6 xn = xc;
              if (bn < nbc) load_xblock6(xim(bn, qn), xn);
              q6k_batch_seq(f, xc, ch[q]);
              xc = xn;
            }
          }
        }
        if (c == P.nch - 1) {
          // s = 0 + sums[0] + ... + sums[7]: the row's classes 2 t, 2 t + 1
          // are held by the lane with tig = t of its row quad
          const int r0 = rb + (u / P.nch) * T + 16 * g + gid;
#pragma unroll
          for (int q = 0; q < SB; q++) {
            const int seq = sg * SB + q;
#pragma unroll
            for (int half = 0; half < 2; half++) {
              float acc = 0.0f;
#pragma unroll
              for (int t = 0; t < 4; t++) {
                const float a = __shfl_sync(0xffffffffu, ch[q][2 * half], (lane & ~3) + t);
                const float b2 = __shfl_sync(0xffffffffu, ch[q][2 * half + 1], (lane & ~3) + t);
                acc = __fadd_rn(acc, a);
                acc = __fadd_rn(acc, b2);
              }
              const int row = r0 + 8 * half;
              if (tig == 0 && row < re && seq < P.nseq) batch_emit(P, row, seq, acc, best);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
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
          P.token[(size_t)s * P.tstride] = 0xffffffffu - (uint32_t)(kf & 0xffffffffull);
          P.key[s] = 0ull;
        }
        __syncwarp();
        if (lane == 0) *P.done = 0u;
      }
    }
  }
}

// Batched x images: quantize_q8_k of every span of every sequence (grid: spans x sequences).
template <int FMT>
__global__ void __launch_bounds__(256) prep_q8k_batch(const float *__restrict__ x, size_t dim_in,
                                                      size_t xstride, uint8_t *__restrict__ img, size_t istride) {
  pdl_trigger();
  __shared__ Q8KSpanSmem sm;
  const size_t span = blockIdx.x, s = blockIdx.y;
  const size_t e = span * kQK + threadIdx.x;
  const float v = e < dim_in ? x[s * xstride + e] : 0.0f;
  uint8_t *im = img + s * istride;
  if constexpr (FMT == Q4K) q8k_span_write(v, im + span * kImgQ8K4, nullptr, sm);
  else q8k_span_write(v, nullptr, im + span * kImgQ8K6, sm);
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

BatchPlan batch_plan(int device, const unltd_weight_s &w) {
  BatchPlan p;
  const bool q4 = w.dtype == Q4K;
  p.T = q4 ? 32 : 16;
  const bool chunked = !q4 && q6_chunked(w.nb) && w.row_stride == w.row_bytes;
  p.nch = chunked ? (int)(w.nb / kQ6Chunk) : 1;
  p.nbc = chunked ? kQ6Chunk : (int)w.nb;
  p.unit_bytes = chunked ? kQ6Chunk * kQ6Bytes : (int)w.row_stride;
  p.ps = (int)round_up((size_t)p.unit_bytes, 128) + (q4 ? 32 : 16);
  p.stage_bytes = (int)round_up((size_t)p.T * p.ps, 128);
  const int smem_max = max_smem_optin_b(device) - 1024;
  p.S = std::min(kBatchStages, (smem_max - kBatchHdr) / p.stage_bytes);
  if (p.S < 2) return p;
  p.smem = kBatchHdr + p.S * p.stage_bytes;
  p.fn = q4 ? gemv_batch_kernel<Q4K, 32, 8> : gemv_batch_kernel<Q6K, 16, 4>;
  return p;
}

}  // namespace

size_t gemv_batch_img_bytes(const unltd_weight_s &w) {
  return round_up(w.nb * (size_t)(w.dtype == Q4K ? kImgQ8K4 : kImgQ8K6), 256);
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
  cudaStream_t st = ctx->stream;
  const size_t istride = gemv_batch_img_bytes(w);
  const uint8_t *img = a.img;
  if (!img) {
    if (!a.x) return set_error(UNLTD_ERR_INVALID_ARG, "gemv_batch: no x and no image");
    if (ctx->scratch_bytes < istride * a.nseq)
      return set_error(UNLTD_ERR_INVALID_ARG, "gemv_batch: scratch not reserved");
    const dim3 grid((unsigned)w.nb, (unsigned)a.nseq);
    if (w.dtype == Q4K) prep_q8k_batch<Q4K><<<grid, 256, 0, st>>>(a.x, w.dim_in, a.xstride, ctx->scratch, istride);
    else prep_q8k_batch<Q6K><<<grid, 256, 0, st>>>(a.x, w.dim_in, a.xstride, ctx->scratch, istride);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, "gemv_batch prep");
    ctx->launches += 1;
    img = ctx->scratch;
  }
  if (cudaError_t e = ensure_batch_attr(ctx->device, pl.fn, max_smem_optin_b(ctx->device) - 1024); e != cudaSuccess)
    return cuda_error(e, "gemv_batch attribute");
  BParams P;
  P.W = w.dev;
  P.pitch = w.row_stride;
  P.rows = (int)w.dim_out;
  P.nbc = pl.nbc;
  P.nch = pl.nch;
  P.unit_bytes = pl.unit_bytes;
  P.ps = pl.ps;
  P.stage_bytes = pl.stage_bytes;
  P.S = pl.S;
  P.img = img;
  P.istride = a.img ? a.istride : istride;
  P.y = a.y;
  P.ystride = a.ystride;
  P.nseq = a.nseq;
  P.key = a.key;
  P.done = a.done;
  P.token = a.token;
  P.tstride = a.tstride;
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
  if (e == cudaSuccess) e = ensure_batch_attr(device, gemv_batch_kernel<Q6K, 16, 4>, m);
  return e;
}

bool gemv_batch_supported(int device, const unltd_weight_s &w) {
  return (w.dtype == Q4K || w.dtype == Q6K) && batch_plan(device, w).fn != nullptr;
}

}  // namespace unltd
