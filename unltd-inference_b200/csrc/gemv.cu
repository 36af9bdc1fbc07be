// Decode GEMV over packed Q4_K / Q6_K / Q8_0 rows, y = W.x, for one
// activation vector, plus the fused LM-head argmax.
//
// Each call runs two kernels on the context stream:
//  1. prep: x (f32) -> an "x image" per 256-element span, in the lane order
//     of the weight layout (unltd_internal.cuh). Mode F32X stores x as a
//     22-bit fixed-point integer per span split into three byte limbs (s8
//     hi, u8 mid, u8 lo) with a power-of-two scale; mode Q8K_EXACT stores
//     quantize_q8_k's output (quants.rs:250-290) bit for bit.
//  2. gemv: a persistent kernel, one CTA per SM over a contiguous range of
//     rows. A producer warp streams tiles of T rows (one contiguous chunk of
//     global memory each) into a ring of shared-memory stages with 1-D bulk
//     copies (TMA) completing on mbarriers; eight consumer warps process each
//     tile in two phases:
//       integer phase — each 8-lane subgroup takes (R rows, block) items; a
//         lane handles one 16-byte chunk of the block's packed quants and
//         forms exact integer dot products with DP4A against the x image;
//         F32X writes one f32 partial per (row, block), Q8K_EXACT writes the
//         reference's per-block products d * sumi[k] for its eight lane
//         classes k = e % 8 (quants.rs:337-346, 390-404) and dmin * minsum;
//       chain phase — per row, the sequential per-block epilogue in block
//         order: F32X sums its partials; Q8K_EXACT runs
//         sums[k] += ..., sumf -= ... and s = sumf + sums[0] + ... + sums[7]
//         without FMA (quants.rs:343-358, 402-411), bit for bit.
//     The weight stage is released right after the integer phase, so the
//     producer refills it while the chain phase runs.
// The gemv kernel is launched with programmatic dependent launch: its
// producer starts streaming weights while prep still runs; the consumers wait
// (griddepcontrol.wait) before reading the image. Every mbarrier wait is
// bounded in time and reports a timeout through the context error word.
#include <algorithm>
#include <cstdio>
#include <mutex>
#include <utility>
#include <type_traits>
#include <vector>

#include "mma_frag.cuh"
#include "q8k_span.cuh"
#include "unltd_host.h"
#include "unltd_internal.cuh"

namespace unltd {
namespace {

constexpr int kThreads = 256;  // prep kernels
constexpr int kConsumerWarps = 16;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kGemvThreads = kConsumers + 32;  // + one producer warp
static_assert(kGemvThreads <= 1024, "a CTA has at most 1024 threads");
constexpr int kMaxStages = 8;
constexpr int kBarBytes = 128;

// ---------------------------------------------------------------- prep ----

__device__ __forceinline__ float block_max(float v, float *red) {
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float r = red[0];
  for (int i = 1; i < 8; i++) r = fmaxf(r, red[i]);
  __syncthreads();
  return r;
}

template <int FMT>
__device__ __forceinline__ int f32x_pos(int t) {
  if constexpr (FMT == Q4K) return q4_xpos(t);
  else if constexpr (FMT == Q6K) return q6_xpos(t);
  else return q80_xpos(t);
}

template <int FMT>
__global__ void __launch_bounds__(kThreads) prep_f32x(const float *__restrict__ x, size_t dim_in,
                                                      uint8_t *__restrict__ img,
                                                      unsigned long long *key, unsigned *done) {
  pdl_trigger();
  __shared__ float red[8];
  __shared__ int hsum[16];
  __shared__ int bad_s;
  const int t = threadIdx.x;
  const size_t span = blockIdx.x;
  const size_t e = span * kQK + t;
  if (t < 16) hsum[t] = 0;
  if (t == 0) bad_s = 0;
  if (key && span == 0 && t == 0) {
    *key = 0ull;
    *done = 0u;
  }
  __syncthreads();
  float v = e < dim_in ? x[e] : 0.0f;
  if (!isfinite(v)) atomicOr(&bad_s, 1);
  float amax = block_max(fabsf(v), red);
  int ex = 0;
  frexpf(amax, &ex);  // amax = m * 2^ex, m in [0.5, 1) -> |x| < 2^ex
  int xi = 0;
  float xs = 0.0f;
  if (amax > 0.0f) {
    xi = __float2int_rn(ldexpf(v, 22 - ex));  // |xi| <= 2^22
    xs = ldexpf(1.0f, ex - 22);
  }
  if (bad_s) xs = __int_as_float(0x7fc00000);  // non-finite x: outputs become NaN
  const int pos = f32x_pos<FMT>(t);
  uint8_t *im = img + span * kImgF32X;
  im[pos] = (uint8_t)(xi >> 16);
  im[256 + pos] = (uint8_t)((xi >> 8) & 0xFF);
  im[512 + pos] = (uint8_t)(xi & 0xFF);
  if constexpr (FMT == Q4K) {
    // lane-half sums for the Q4_K min term: lane j = 2p + (k >= 4), half = nibble group
    int p = t >> 6, half = (t >> 5) & 1, k = t & 7;
    atomicAdd(&hsum[2 * (2 * p + (k >> 2)) + half], xi);
  }
  __syncthreads();
  if (t == 0) *reinterpret_cast<float *>(im + kImgF32X_XS) = xs;
  if constexpr (FMT == Q4K) {
    if (t < 16) reinterpret_cast<float *>(im + kImgF32X_XSUM)[t] = (float)hsum[t] * xs;
  }
}

// prep_f32x's arithmetic for one span by one warp, lane l holding elements
// 8l .. 8l+7 of v: the same amax, exponent, xi and scale (and, for Q4_K, the
// same integer half sums), so a GEMV whose prologue writes its image this way
// gives the same bits as one fed by prep_f32x.
template <int FMT>
__device__ __forceinline__ void f32x_span_write_warp(const float (&v)[8], int lane, uint8_t *im) {
  float amax = 0.0f;
  bool bad = false;
#pragma unroll
  for (int k = 0; k < 8; k++) {
    bad |= !isfinite(v[k]);
    amax = fmaxf(amax, fabsf(v[k]));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  bad = __any_sync(0xffffffffu, bad);
  int ex = 0;
  frexpf(amax, &ex);
  int xi[8];
#pragma unroll
  for (int k = 0; k < 8; k++) xi[k] = amax > 0.0f ? __float2int_rn(ldexpf(v[k], 22 - ex)) : 0;
  float xs = amax > 0.0f ? ldexpf(1.0f, ex - 22) : 0.0f;
  if (bad) xs = __int_as_float(0x7fc00000);
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const int pos = f32x_pos<FMT>(8 * lane + k);
    im[pos] = (uint8_t)(xi[k] >> 16);
    im[256 + pos] = (uint8_t)((xi[k] >> 8) & 0xFF);
    im[512 + pos] = (uint8_t)(xi[k] & 0xFF);
  }
  if (lane == 0) *reinterpret_cast<float *>(im + kImgF32X_XS) = xs;
  if constexpr (FMT == Q4K) {
    // half sums for the min term: elements of class < 4 / >= 4 of nibble
    // group (p, half); the four lanes l with the same l >> 2 share them
    int s0 = xi[0] + xi[1] + xi[2] + xi[3], s1 = xi[4] + xi[5] + xi[6] + xi[7];
    s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
    s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
    s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
    s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
    if ((lane & 3) == 0) {
      const int p = lane >> 3, half = (lane >> 2) & 1;
      float *xsum = reinterpret_cast<float *>(im + kImgF32X_XSUM);
      xsum[2 * (2 * p) + half] = (float)s0 * xs;
      xsum[2 * (2 * p + 1) + half] = (float)s1 * xs;
    }
  }
}

// F32X image of an f32 x (16-byte aligned) in a GEMV's prologue: warp w of
// nw takes spans w, w + nw, ...; elements past dim_in (a Q8_0 row whose last
// span is partial) are zero, as in prep_f32x.
template <int FMT>
__device__ __noinline__ void f32x_prologue(const float *__restrict__ x, int dim_in, int nsp, uint8_t *ximg, int nw) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int s0 = warp; s0 < nsp; s0 += 3 * nw) {
    float4 v[3][2];
#pragma unroll
    for (int q = 0; q < 3; q++) {
      const int e0 = (s0 + nw * q) * 256 + 8 * lane;
      v[q][0] = v[q][1] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (s0 + nw * q < nsp && e0 < dim_in) {  // dim_in is a multiple of 32: all 8 in or all out
        const float4 *p = reinterpret_cast<const float4 *>(x + e0);
        v[q][0] = p[0];
        v[q][1] = p[1];
      }
    }
#pragma unroll
    for (int q = 0; q < 3; q++) {
      const int span = s0 + nw * q;
      if (span >= nsp) break;
      const float e[8] = {v[q][0].x, v[q][0].y, v[q][0].z, v[q][0].w, v[q][1].x, v[q][1].y, v[q][1].z, v[q][1].w};
      f32x_span_write_warp<FMT>(e, lane, ximg + (size_t)span * kImgF32X);
    }
  }
}

// Exact restatement of quantize_q8_k (quants.rs:250-290), one span per CTA.
template <int FMT>
__global__ void __launch_bounds__(kThreads) prep_q8k(const float *__restrict__ x, size_t dim_in,
                                                     uint8_t *__restrict__ img,
                                                     unsigned long long *key, unsigned *done) {
  pdl_trigger();
  __shared__ Q8KSpanSmem sm;
  const int t = threadIdx.x;
  const size_t span = blockIdx.x;
  const size_t e = span * kQK + t;
  if (key && span == 0 && t == 0) {
    *key = 0ull;
    *done = 0u;
  }
  const float v = e < dim_in ? x[e] : 0.0f;
  if constexpr (FMT == Q4K) q8k_span_write(v, img + span * kImgQ8K4, nullptr, sm);
  else q8k_span_write(v, nullptr, img + span * kImgQ8K6, sm);
}

// ---------------------------------------------------------------- gemv ----

struct Params {
  const uint8_t *W;
  size_t stride;   // device bytes per row
  int nb;          // blocks per row (Q8_0: 32-element blocks)
  int nbu;         // work units per row: 256-element blocks (K-quants) or spans (Q8_0)
  int rows;
  const uint8_t *img;
  int img_bytes;
  float *y;
  unsigned long long *key;
  unsigned *done;
  uint32_t *token;
  unsigned long long *key_out;  // non-null: also store the final argmax key
  int row0;                     // global index of row 0 (vocab-split LM head)
  int *err;
  int pstride;     // shared-memory row stride in a stage (> stride: padded rows)
  int mma;         // Q4_K Q8K: integer phase on the tensor cores (T a multiple of 16)
  int T;           // rows per tile
  int S;           // stages
  int stage_bytes; // bytes per stage buffer (>= T * stride, multiple of 128)
  int rs;          // chain-buffer row stride in floats
  int cbuf_bytes;  // one chain buffer
  // fused RMSNorm of the input (tensor-core kernel; nn = its length, 0: none)
  const float *norm_a, *norm_b;
  float *norm_r;
  const float *norm_w;
  float norm_eps;
  uint8_t *norm_img4, *norm_img6;
  int nn;
  // non-null: x in f32 (dim_in elements, 16-byte aligned), quantized into the
  // CTA's image in the prologue instead of by a separate prep kernel
  const float *xq;
  // tensor-parallel row-split sum over NVLink peer memory, the all-reduce
  // protocol of the peer kernel split in two (peer_n > 0):
  // peer_send: the chain stores each y row into this rank's slot of every
  //   rank's receive area (not into y); the last CTA raises this rank's flag
  //   in every area and advances the all-reduce counter
  // peer_recv (with the fused norm): the prologue waits for every rank's
  //   flag and takes b = the slots summed in rank order
  uint8_t *peer_map[kPeerMaxRanks];
  unsigned *peer_ctr, *peer_done;
  int peer_rank, peer_n, peer_send, peer_recv;
};

__device__ __forceinline__ unsigned peer_ld_acquire(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void peer_st_release(unsigned *p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// slot `src` of parity (ep & 1) in the area `area`
__device__ __forceinline__ float *peer_slot(uint8_t *area, unsigned ep, int src) {
  return reinterpret_cast<float *>(area + kPeerFlagBytes + (size_t)(ep & 1u) * kPeerMaxRanks * kPeerSlotBytes +
                                   (size_t)src * kPeerSlotBytes);
}



// One block of the class-major Q8_K x image as the MMA B operands of this
// lane: column n of B is class n, and lane (gid, tig) holds B[k-quad tig][gid]
// (class 2 tig elements) and B[k-quad 4 + tig][gid] (class 2 tig + 1), nonzero
// only when gid is that class; plus the B operand of the min term's MMA and
// the block's d.
struct XBlock {
  uint32_t b0[8], b1[8];
  uint32_t bm;  // min term: B[k][0 | 1] = low / high byte of group sum k
  float xd;
};

__device__ __forceinline__ void load_xblock(const uint8_t *im, XBlock &x) {
  const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
  const bool own0 = gid == 2 * tig, own1 = gid == 2 * tig + 1;
  uint4 xa = make_uint4(0u, 0u, 0u, 0u), xb = xa;
  if (own0 || own1) {
    xa = lds128(im + 16 * gid);
    xb = lds128(im + 128 + 16 * gid);
  }
  const uint32_t xg[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
  for (int g = 0; g < 8; g++) {
    x.b0[g] = own0 ? xg[g] : 0u;
    x.b1[g] = own1 ? xg[g] : 0u;
  }
  // min term (m16n8k16): lane (gid, tig) holds B[4 tig .. 4 tig + 3][gid];
  // column 0 = the balanced low bytes bl = ((s + 128) & 255) - 128 of the
  // eight group sums s, column 1 = the high bytes (s - bl) / 256 (|s| <=
  // 32 * 127, so both fit s8); rows 8..15 and columns 2..7 are zero
  // (precomputed by the image writer, kImgQ8K4_BM)
  x.bm = (gid < 2 && tig < 2) ? *reinterpret_cast<const uint32_t *>(im + kImgQ8K4_BM + 4 * (2 * gid + tig)) : 0u;
  x.xd = *reinterpret_cast<const float *>(im + kImgQ8K4_D);
}

// Q8K, Q4_K on the tensor cores: one warp takes 16 rows x one block. For
// each scale group g an int8 MMA m16n8k32 multiplies the 16 rows' 32 quants
// of the group (A: thread (r, t) holds words 2t and 2t+1 of the row's 32-byte
// qs segment, i.e. classes 2t and 2t+1, each four elements) by the class-
// masked q8 values (XBlock), giving every (row, class) integer partial of the
// group at once; the group scales are applied per row in int32 (exact). The
// odd groups (high nibbles) enter as 16 x nibble and their scaled sum is
// divided by 16 at the end (exact: every term is a multiple of 16, and the
// sum stays below 2^31). The min term sum_g m_g * s_g (s_g: group sum of the
// q8 values) is one more int8 MMA m16n8k16: A[r][k] = the 6-bit min of group
// k of row r (k < 8), B = the group sums as two byte columns (XBlock::bm).
__device__ __forceinline__ void q4k_q8k_mma_item(const uint8_t *tile, int nr, int g16, int b, const XBlock &x,
                                                 const Params &P, float *tk, float *tm) {
  const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
  const int lr0 = g16 * 16 + gid, lr1 = lr0 + 8;
  const bool v0 = lr0 < nr, v1 = lr1 < nr;
  const uint8_t *row0 = tile + (v0 ? lr0 : 0) * P.pstride;
  const uint8_t *row1 = tile + (v1 ? lr1 : 0) * P.pstride;
  const uint4 h0 = lds128(row0 + b * 16), h1 = lds128(row1 + b * 16);
  const int qo = P.nb * 16 + b * 128 + 8 * tig;
  uint2 w0[4], w1[4];
#pragma unroll
  for (int p = 0; p < 4; p++) {
    w0[p] = lds64(row0 + qo + 32 * p);
    w1[p] = lds64(row1 + qo + 32 * p);
  }
  const uint32_t SCa0 = h0.y & 0x3F3F3F3Fu, SCb0 = (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u);
  const uint32_t SCa1 = h1.y & 0x3F3F3F3Fu, SCb1 = (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u);
  int lo0 = 0, lo1 = 0, lo2 = 0, lo3 = 0, hi0 = 0, hi1 = 0, hi2 = 0, hi3 = 0;
#pragma unroll
  for (int p = 0; p < 4; p++) {
    const uint32_t S0 = p < 2 ? SCa0 : SCb0, S1 = p < 2 ? SCa1 : SCb1;
    const int k = (2 * p) & 3;
    int d0, d1, d2, d3, e0, e1, e2, e3;
    mma_s8(w0[p].x & 0x0F0F0F0Fu, w1[p].x & 0x0F0F0F0Fu, w0[p].y & 0x0F0F0F0Fu, w1[p].y & 0x0F0F0F0Fu, x.b0[2 * p],
           x.b1[2 * p], d0, d1, d2, d3);
    mma_u8s8(w0[p].x & 0xF0F0F0F0u, w1[p].x & 0xF0F0F0F0u, w0[p].y & 0xF0F0F0F0u, w1[p].y & 0xF0F0F0F0u,
             x.b0[2 * p + 1], x.b1[2 * p + 1], e0, e1, e2, e3);
    const int s0 = byte_of(S0, k), s1 = byte_of(S1, k), t0 = byte_of(S0, k + 1), t1 = byte_of(S1, k + 1);
    lo0 += s0 * d0;
    lo1 += s0 * d1;
    lo2 += s1 * d2;
    lo3 += s1 * d3;
    hi0 += t0 * e0;
    hi1 += t0 * e1;
    hi2 += t1 * e2;
    hi3 += t1 * e3;
  }
  const int acc0 = lo0 + (hi0 >> 4), acc1 = lo1 + (hi1 >> 4), acc2 = lo2 + (hi2 >> 4), acc3 = lo3 + (hi3 >> 4);
  // min term: A k-quad 0 = mins of groups 0..3 (lanes tig 0), k-quad 1 = groups
  // 4..7 (tig 1), the rest zero; lanes tig 0 get minsum = D[r][0] + 256 D[r][1]
  const uint32_t MA0 = h0.z & 0x3F3F3F3Fu, MB0 = ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u);
  const uint32_t MA1 = h1.z & 0x3F3F3F3Fu, MB1 = ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u);
  int mn0, mn1, mn2, mn3;
  mma_s8_k16(tig == 0 ? MA0 : (tig == 1 ? MB0 : 0u), tig == 0 ? MA1 : (tig == 1 ? MB1 : 0u), x.bm, mn0, mn1, mn2,
             mn3);
  const int ms0 = mn0 + mn1 * 256, ms1 = mn2 + mn3 * 256;
  const int rs2 = P.rs / 8;
  if (v0) {
    const float d = __fmul_rn(x.xd, h2f_bits(h0.x & 0xFFFFu)), dm = __fmul_rn(h2f_bits(h0.x >> 16), x.xd);
    float *t = tk + lr0 * P.rs + 8 * b + 2 * tig;
    t[0] = __fmul_rn(d, (float)acc0);
    t[1] = __fmul_rn(d, (float)acc1);
    if (tig == 0) tm[lr0 * rs2 + b] = __fmul_rn(dm, (float)ms0);
  }
  if (v1) {
    const float d = __fmul_rn(x.xd, h2f_bits(h1.x & 0xFFFFu)), dm = __fmul_rn(h2f_bits(h1.x >> 16), x.xd);
    float *t = tk + lr1 * P.rs + 8 * b + 2 * tig;
    t[0] = __fmul_rn(d, (float)acc2);
    t[1] = __fmul_rn(d, (float)acc3);
    if (tig == 0) tm[lr1 * rs2 + b] = __fmul_rn(dm, (float)ms1);
  }
}



// Q8K, Q6_K on the tensor cores: one warp takes 16 rows x one block. Per
// sub-block (16 elements, one int8 scale) an int8 MMA m16n8k16 multiplies the
// 16 rows' quads (A: thread (r, t) holds word t of the row's ql/qh chunk as
// 4 (raw6 - 32) in s8) by the class-masked q8 values (XBlock6), giving every
// (row, class) partial of the sub-block; the per-row scales are applied in
// int32 and the 4x removed at the end (exact: every term is a multiple of 4
// and |sum| < 2^31). No min term (quants.rs:371-412).
template <bool R8>
__device__ __forceinline__ void q6k_q8k_mma_item(const uint8_t *tile, int nr, int g16, int b, const XBlock6 &x,
                                                 const Params &P, float *tk) {
  // R8: 8-row tiles; rows 8..15 of the MMA fragments stay zero and are not built
  const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
  const int lr0 = (R8 ? 8 : 16) * g16 + gid, lr1 = lr0 + 8;
  const bool v0 = lr0 < nr, v1 = !R8 && lr1 < nr;
  const uint8_t *row0 = tile + (v0 ? lr0 : 0) * P.pstride;
  const uint8_t *row1 = tile + (v1 ? lr1 : 0) * P.pstride;
  int nb;
  const int bl = q6_planes(row0, P.nb, b, nb);
  if (q6_chunked((size_t)P.nb)) row1 += (b / kQ6Chunk) * (kQ6Chunk * 210);
  const int qlo = bl * 128 + 4 * tig, qho = nb * 128 + bl * 64 + 4 * tig;
  uint32_t l0[8], l1[8], h0[4], h1[4];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    l0[j] = *reinterpret_cast<const uint32_t *>(row0 + qlo + 16 * j);
    l1[j] = R8 ? 0u : *reinterpret_cast<const uint32_t *>(row1 + qlo + 16 * j);
  }
#pragma unroll
  for (int c = 0; c < 4; c++) {
    h0[c] = *reinterpret_cast<const uint32_t *>(row0 + qho + 16 * c);
    h1[c] = R8 ? 0u : *reinterpret_cast<const uint32_t *>(row1 + qho + 16 * c);
  }
  const uint4 sc0 = lds128(row0 + nb * 192 + bl * 16);
  const uint4 sc1 = R8 ? make_uint4(0u, 0u, 0u, 0u) : lds128(row1 + nb * 192 + bl * 16);
  const uint32_t S0[4] = {sc0.x, sc0.y, sc0.z, sc0.w}, S1[4] = {sc1.x, sc1.y, sc1.z, sc1.w};
  const uint32_t db0 = *reinterpret_cast<const unsigned short *>(row0 + nb * 208 + bl * 2);
  const uint32_t db1 = R8 ? 0u : *reinterpret_cast<const unsigned short *>(row1 + nb * 208 + bl * 2);
  int acc0 = 0, acc1 = 0, acc2 = 0, acc3 = 0;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int h = j >> 2, u = j & 3, sl = 2 * (u >> 1), c = 2 * h + (u & 1);
    const int slo = 8 * h + u, shi = slo + 4;  // the chunk's two sub-blocks
    int d0, d1, d2, d3, e0, e1, e2, e3;
    mma_s8_k16(q6_a4_lo(l0[j], h0[c], sl), R8 ? 0u : q6_a4_lo(l1[j], h1[c], sl), x.b[2 * j], d0, d1, d2, d3);
    mma_s8_k16(q6_a4_hi(l0[j], h0[c], sl), R8 ? 0u : q6_a4_hi(l1[j], h1[c], sl), x.b[2 * j + 1], e0, e1, e2, e3);
    const int s0 = sbyte_of(S0[slo >> 2], slo & 3), t0 = sbyte_of(S0[shi >> 2], shi & 3);
    acc0 += s0 * d0 + t0 * e0;
    acc1 += s0 * d1 + t0 * e1;
    if (!R8) {
      const int s1 = sbyte_of(S1[slo >> 2], slo & 3), t1 = sbyte_of(S1[shi >> 2], shi & 3);
      acc2 += s1 * d2 + t1 * e2;
      acc3 += s1 * d3 + t1 * e3;
    }
  }
  if (v0) {
    const float d = __fmul_rn(x.xd, h2f_bits(db0));
    float *t = tk + lr0 * P.rs + 8 * b + 2 * tig;
    t[0] = __fmul_rn(d, (float)(acc0 >> 2));
    t[1] = __fmul_rn(d, (float)(acc1 >> 2));
  }
  if (v1) {
    const float d = __fmul_rn(x.xd, h2f_bits(db1));
    float *t = tk + lr1 * P.rs + 8 * b + 2 * tig;
    t[0] = __fmul_rn(d, (float)(acc2 >> 2));
    t[1] = __fmul_rn(d, (float)(acc3 >> 2));
  }
}



// Q4_K: sc/m of groups 2p and 2p+1 from the 12 packed bytes (hq.y, hq.z,
// hq.w), vectorized get_scale_min_k4 (quants.rs:92-102).
__device__ __forceinline__ void q4_scales(const uint4 &hq, int p, int &sc_lo, int &sc_hi, int &m_lo,
                                          int &m_hi) {
  uint32_t SC, MM;
  if (p < 2) {
    SC = hq.y & 0x3F3F3F3Fu;
    MM = hq.z & 0x3F3F3F3Fu;
  } else {
    SC = (hq.w & 0x0F0F0F0Fu) | ((hq.y >> 2) & 0x30303030u);
    MM = ((hq.w >> 4) & 0x0F0F0F0Fu) | ((hq.z >> 2) & 0x30303030u);
  }
  const int sh = (p & 1) * 16;
  sc_lo = (SC >> sh) & 0xFF;
  sc_hi = (SC >> (sh + 8)) & 0xFF;
  m_lo = (MM >> sh) & 0xFF;
  m_hi = (MM >> (sh + 8)) & 0xFF;
}

__device__ __forceinline__ float sub_sum(float v, unsigned m) {
  v += __shfl_xor_sync(m, v, 4);
  v += __shfl_xor_sync(m, v, 2);
  v += __shfl_xor_sync(m, v, 1);
  return v;
}

// One (R rows, block b) item of the integer phase for an 8-lane subgroup.
// rowp[r]: the rows in shared memory; im: the x image of block/span b.
// F32X: writes cb[r * rs + b]. Q8K: writes cb[r * rs + 8b + k] (d * sumi per
// class) and cm[r * rs/8 + b] (dmin * minsum). cb/cm point at the item's first row.
template <int FMT, int MODE, int R>
__device__ __forceinline__ void integer_item(const uint8_t *const (&rowp)[R], const bool (&rv)[R], int b,
                                             const uint8_t *im, const Params &P, float *cb, float *cm, int j,
                                             unsigned m) {
  const int nb = P.nb;
  if constexpr (MODE == MODE_F32X) {
    float acc[R];
    if constexpr (FMT == Q4K) {
      const int p = j >> 1, kh = j & 1;
      const uint4 xh0 = lds128(im + 16 * j), xh1 = lds128(im + 128 + 16 * j);
      const uint4 xm0 = lds128(im + 256 + 16 * j), xm1 = lds128(im + 384 + 16 * j);
      const uint4 xl0 = lds128(im + 512 + 16 * j), xl1 = lds128(im + 640 + 16 * j);
      const float xs = *reinterpret_cast<const float *>(im + kImgF32X_XS);
      const float xsl = reinterpret_cast<const float *>(im + kImgF32X_XSUM)[2 * j];
      const float xsh = reinterpret_cast<const float *>(im + kImgF32X_XSUM)[2 * j + 1];
      const uint32_t xh_lo[4] = {xh0.x, xh0.y, xh0.z, xh0.w}, xh_hi[4] = {xh1.x, xh1.y, xh1.z, xh1.w};
      const uint32_t xm_lo[4] = {xm0.x, xm0.y, xm0.z, xm0.w}, xm_hi[4] = {xm1.x, xm1.y, xm1.z, xm1.w};
      const uint32_t xl_lo[4] = {xl0.x, xl0.y, xl0.z, xl0.w}, xl_hi[4] = {xl1.x, xl1.y, xl1.z, xl1.w};
#pragma unroll
      for (int r = 0; r < R; r++) {
        const uint4 hq = lds128(rowp[r] + b * 16);
        const uint4 q = lds128(rowp[r] + nb * 16 + b * 128 + 32 * p + 16 * kh);
        int sc_lo, sc_hi, m_lo, m_hi;
        q4_scales(hq, p, sc_lo, sc_hi, m_lo, m_hi);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
        int shl = 0, sml = 0, sll = 0, shh = 0, smh = 0, slh = 0;
#pragma unroll
        for (int t = 0; t < 4; t++) {
          const uint32_t lo = w[t] & 0x0F0F0F0Fu, hi = (w[t] >> 4) & 0x0F0F0F0Fu;
          shl = dp4a_us(lo, xh_lo[t], shl);
          sml = dp4a_uu(lo, xm_lo[t], sml);
          sll = dp4a_uu(lo, xl_lo[t], sll);
          shh = dp4a_us(hi, xh_hi[t], shh);
          smh = dp4a_uu(hi, xm_hi[t], smh);
          slh = dp4a_uu(hi, xl_hi[t], slh);
        }
        const int ah = sc_lo * shl + sc_hi * shh;
        const int am = sc_lo * sml + sc_hi * smh;
        const int al = sc_lo * sll + sc_hi * slh;
        const float F = fmaf((float)ah, 65536.0f, fmaf((float)am, 256.0f, (float)al));
        const float d = h2f_bits(hq.x & 0xFFFFu), dmin = h2f_bits(hq.x >> 16);
        const float M = fmaf((float)m_lo, xsl, (float)m_hi * xsh);
        acc[r] = fmaf(d * xs, F, -dmin * M);
      }
    } else if constexpr (FMT == Q6K) {
      const int h = j >> 2, u = j & 3, sl = 2 * (u >> 1);
      const uint4 xh0 = lds128(im + 16 * j), xh1 = lds128(im + 128 + 16 * j);
      const uint4 xm0 = lds128(im + 256 + 16 * j), xm1 = lds128(im + 384 + 16 * j);
      const uint4 xl0 = lds128(im + 512 + 16 * j), xl1 = lds128(im + 640 + 16 * j);
      const float xs = *reinterpret_cast<const float *>(im + kImgF32X_XS);
      const uint32_t xh_lo[4] = {xh0.x, xh0.y, xh0.z, xh0.w}, xh_hi[4] = {xh1.x, xh1.y, xh1.z, xh1.w};
      const uint32_t xm_lo[4] = {xm0.x, xm0.y, xm0.z, xm0.w}, xm_hi[4] = {xm1.x, xm1.y, xm1.z, xm1.w};
      const uint32_t xl_lo[4] = {xl0.x, xl0.y, xl0.z, xl0.w}, xl_hi[4] = {xl1.x, xl1.y, xl1.z, xl1.w};
#pragma unroll
      for (int r = 0; r < R; r++) {
        const uint8_t *row = rowp[r];
        int nbl;
        const int bl = q6_planes(row, nb, b, nbl);
        const uint4 ql = lds128(row + bl * 128 + 16 * j);
        const uint4 qh = lds128(row + nbl * 128 + bl * 64 + 16 * (2 * h + (u & 1)));
        const int8_t *scp = reinterpret_cast<const int8_t *>(row + nbl * 192 + bl * 16);
        const int sc_lo = scp[8 * h + u], sc_hi = scp[8 * h + 4 + u];
        const float d = h2f_bits(*reinterpret_cast<const unsigned short *>(row + nbl * 208 + bl * 2));
        const uint32_t wl[4] = {ql.x, ql.y, ql.z, ql.w}, wh[4] = {qh.x, qh.y, qh.z, qh.w};
        int shl = 0, sml = 0, sll = 0, shh = 0, smh = 0, slh = 0;
#pragma unroll
        for (int t = 0; t < 4; t++) {
          const uint32_t lo = q6_a4_lo(wl[t], wh[t], sl), hi = q6_a4_hi(wl[t], wh[t], sl);
          shl = dp4a_ss(lo, xh_lo[t], shl);
          sml = dp4a_su(lo, xm_lo[t], sml);
          sll = dp4a_su(lo, xl_lo[t], sll);
          shh = dp4a_ss(hi, xh_hi[t], shh);
          smh = dp4a_su(hi, xm_hi[t], smh);
          slh = dp4a_su(hi, xl_hi[t], slh);
        }
        const int ah = sc_lo * shl + sc_hi * shh;
        const int am = sc_lo * sml + sc_hi * smh;
        const int al = sc_lo * sll + sc_hi * slh;
        const float F = fmaf((float)ah, 65536.0f, fmaf((float)am, 256.0f, (float)al));
        acc[r] = d * xs * 0.25f * F;
      }
    } else {  // Q8_0: lane j owns 32-element block 8b + j of span b
      const int b32 = 8 * b + j;
      const bool ok = b32 < nb;
      const uint4 xh0 = lds128(im + 16 * j), xh1 = lds128(im + 128 + 16 * j);
      const uint4 xm0 = lds128(im + 256 + 16 * j), xm1 = lds128(im + 384 + 16 * j);
      const uint4 xl0 = lds128(im + 512 + 16 * j), xl1 = lds128(im + 640 + 16 * j);
      const float xs = *reinterpret_cast<const float *>(im + kImgF32X_XS);
      const uint32_t xh[8] = {xh0.x, xh0.y, xh0.z, xh0.w, xh1.x, xh1.y, xh1.z, xh1.w};
      const uint32_t xm[8] = {xm0.x, xm0.y, xm0.z, xm0.w, xm1.x, xm1.y, xm1.z, xm1.w};
      const uint32_t xl[8] = {xl0.x, xl0.y, xl0.z, xl0.w, xl1.x, xl1.y, xl1.z, xl1.w};
      const int bb = ok ? b32 : 0;
#pragma unroll
      for (int r = 0; r < R; r++) {
        const uint4 q0 = lds128(rowp[r] + bb * 32), q1 = lds128(rowp[r] + bb * 32 + 16);
        const float d = h2f_bits(*reinterpret_cast<const unsigned short *>(rowp[r] + nb * 32 + bb * 2));
        const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        int sh = 0, sm = 0, sll = 0;
#pragma unroll
        for (int t = 0; t < 8; t++) {
          sh = dp4a_ss(w[t], xh[t], sh);
          sm = dp4a_su(w[t], xm[t], sm);
          sll = dp4a_su(w[t], xl[t], sll);
        }
        const float F = fmaf((float)sh, 65536.0f, fmaf((float)sm, 256.0f, (float)sll));
        acc[r] = ok ? d * xs * F : 0.0f;
      }
    }
#pragma unroll
    for (int r = 0; r < R; r++) {
      const float v = sub_sum(acc[r], m);
      if (j == 0 && rv[r]) cb[r * P.rs + b] = v;
    }
  } else {  // MODE_Q8K
    float *tk = cb;  // rows of rs floats: 8 per block
    float *tm = cm;  // rows of rs/8 floats: 1 per block
    const int rs2 = P.rs / 8;
    const float xd = *reinterpret_cast<const float *>(im + (FMT == Q4K ? kImgQ8K4_D : kImgQ8K6_D));
    if constexpr (FMT == Q4K) {
      // Lane j computes the class-j sum sumi[j] of the block by itself: its
      // four qs words at 32p + 4j hold class j's elements 64p + j + 8i of
      // groups 2p (low nibbles) and 2p+1 (high nibbles); the image's class-j
      // row holds the matching q8 words, one per group. The min term takes
      // group j per lane and is summed over the eight lanes.
      const uint4 xa = lds128(im + 16 * j), xb = lds128(im + 128 + 16 * j);
      const uint32_t xg[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
      const int bsj = reinterpret_cast<const int *>(im + kImgQ8K4_BS)[j];
#pragma unroll
      for (int r = 0; r < R; r++) {
        const uint4 hq = lds128(rowp[r] + b * 16);
        const uint8_t *qs = rowp[r] + nb * 16 + b * 128 + 4 * j;
        const uint32_t SC03 = hq.y & 0x3F3F3F3Fu, M03 = hq.z & 0x3F3F3F3Fu;
        const uint32_t SC47 = (hq.w & 0x0F0F0F0Fu) | ((hq.y >> 2) & 0x30303030u);
        const uint32_t M47 = ((hq.w >> 4) & 0x0F0F0F0Fu) | ((hq.z >> 2) & 0x30303030u);
        int acc = 0;
#pragma unroll
        for (int p = 0; p < 4; p++) {
          const uint32_t w = *reinterpret_cast<const uint32_t *>(qs + 32 * p);
          const uint32_t SC = p < 2 ? SC03 : SC47;
          const int sh = (p & 1) * 16;
          const int sc_lo = (SC >> sh) & 0xFF, sc_hi = (SC >> (sh + 8)) & 0xFF;
          acc += sc_lo * dp4a_us(w & 0x0F0F0F0Fu, xg[2 * p], 0) + sc_hi * dp4a_us((w >> 4) & 0x0F0F0F0Fu, xg[2 * p + 1], 0);
        }
        const uint32_t MM = j < 4 ? M03 : M47;
        int msum = (int)((MM >> (8 * (j & 3))) & 0xFFu) * bsj;
        msum += __shfl_xor_sync(m, msum, 4);
        msum += __shfl_xor_sync(m, msum, 2);
        msum += __shfl_xor_sync(m, msum, 1);
        const float d = __fmul_rn(xd, h2f_bits(hq.x & 0xFFFFu));   // q8.d * f16(d)
        const float dm = __fmul_rn(h2f_bits(hq.x >> 16), xd);      // f16(dmin) * q8.d
        if (rv[r]) {
          tk[r * P.rs + 8 * b + j] = __fmul_rn(d, (float)acc);
          if (j == 0) tm[r * rs2 + b] = __fmul_rn(dm, (float)msum);
        }
      }
    } else {  // Q6_K
      const int h = j >> 2, u = j & 3, sl = 2 * (u >> 1);
      const uint4 c0 = lds128(im + 16 * j), c1 = lds128(im + 128 + 16 * j);
      const uint4 c2 = lds128(im + 256 + 16 * j), c3 = lds128(im + 384 + 16 * j);
      const uint32_t qA_lo[4] = {c0.x, c0.z, c1.x, c1.z}, qB_lo[4] = {c0.y, c0.w, c1.y, c1.w};
      const uint32_t qA_hi[4] = {c2.x, c2.z, c3.x, c3.z}, qB_hi[4] = {c2.y, c2.w, c3.y, c3.w};
      const bool b2 = (j >> 2) & 1, b1 = (j >> 1) & 1, b0 = j & 1;
#pragma unroll
      for (int r = 0; r < R; r++) {
        const uint8_t *row = rowp[r];
        int nbl;
        const int bl = q6_planes(row, nb, b, nbl);
        const uint4 ql = lds128(row + bl * 128 + 16 * j);
        const uint4 qh = lds128(row + nbl * 128 + bl * 64 + 16 * (2 * h + (u & 1)));
        const int8_t *scp = reinterpret_cast<const int8_t *>(row + nbl * 192 + bl * 16);
        const int sc_lo = scp[8 * h + u], sc_hi = scp[8 * h + 4 + u];
        const uint32_t dbits = *reinterpret_cast<const unsigned short *>(row + nbl * 208 + bl * 2);
        const uint32_t wl[4] = {ql.x, ql.y, ql.z, ql.w}, wh[4] = {qh.x, qh.y, qh.z, qh.w};
        int P4[8];
#pragma unroll
        for (int t = 0; t < 4; t++) {
          const uint32_t lo = q6_a4_lo(wl[t], wh[t], sl), hi = q6_a4_hi(wl[t], wh[t], sl);
          P4[2 * t] = sc_lo * dp4a_ss(lo, qA_lo[t], 0) + sc_hi * dp4a_ss(hi, qA_hi[t], 0);
          P4[2 * t + 1] = sc_lo * dp4a_ss(lo, qB_lo[t], 0) + sc_hi * dp4a_ss(hi, qB_hi[t], 0);
        }
        // reduce-scatter over the 8 lanes: lane j ends with class k = j
        int v4[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const int keepv = b2 ? P4[4 + i] : P4[i];
          const int sendv = b2 ? P4[i] : P4[4 + i];
          v4[i] = keepv + __shfl_xor_sync(m, sendv, 4);
        }
        int v2[2];
#pragma unroll
        for (int i = 0; i < 2; i++) {
          const int keepv = b1 ? v4[2 + i] : v4[i];
          const int sendv = b1 ? v4[i] : v4[2 + i];
          v2[i] = keepv + __shfl_xor_sync(m, sendv, 2);
        }
        const int keepv = b0 ? v2[1] : v2[0];
        const int sendv = b0 ? v2[0] : v2[1];
        const int sumi = (keepv + __shfl_xor_sync(m, sendv, 1)) >> 2;
        const float d = __fmul_rn(xd, h2f_bits(dbits));
        if (rv[r]) tk[r * P.rs + 8 * b + j] = __fmul_rn(d, (float)sumi);
      }
    }
  }
}

template <int FMT, int MODE, int R, bool ARGMAX, int NW = kConsumerWarps>
__global__ void __launch_bounds__(NW * 32 + 32, 1) gemv_kernel(Params P) {
  constexpr int kCW = NW, kCons = NW * 32;  // consumer warps / threads
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *full = reinterpret_cast<uint64_t *>(smem);
  uint64_t *empty = full + kMaxStages;
  uint8_t *ximg = smem + kBarBytes;
  float *cbuf0 = reinterpret_cast<float *>(ximg + P.img_bytes);
  uint8_t *stages = reinterpret_cast<uint8_t *>(cbuf0) + 2 * P.cbuf_bytes;
  // let the next kernel of the stream get resident; it waits for this grid's
  // completion (griddepcontrol.wait) before touching anything this grid uses
  pdl_trigger();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int rb = (int)((long long)P.rows * blockIdx.x / G);
  const int re = (int)((long long)P.rows * (blockIdx.x + 1) / G);
  const int ntiles = (re - rb + P.T - 1) / P.T;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P.S; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCW);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kCW) {
    // ---------------- producer: one thread streams row tiles -------------
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      for (int i = 0; i < ntiles && ok; i++) {
        const int s = i % P.S;
        if (i >= P.S) ok = mbar_wait_bounded(&empty[s], ((i / P.S) - 1) & 1, P.err);
        if (!ok) break;
        const int r0 = rb + i * P.T;
        const int nr = min(P.T, re - r0);
        const uint32_t bytes = (uint32_t)(nr * P.stride);
        mbar_expect_tx(&full[s], bytes);
        if (P.pstride == (int)P.stride) {
          bulk_g2s(stages + (size_t)s * P.stage_bytes, P.W + (size_t)r0 * P.stride, bytes, &full[s]);
        } else {  // padded rows: one copy per row
          for (int rr = 0; rr < nr; rr++)
            bulk_g2s(stages + (size_t)s * P.stage_bytes + (size_t)rr * P.pstride, P.W + (size_t)(r0 + rr) * P.stride,
                     (uint32_t)P.stride, &full[s]);
        }
        issued = i + 1;
      }
      // never leave with copies in flight: wait (bounded) for the last copy of each stage
      for (int i = max(0, issued - P.S); i < issued; i++)
        mbar_wait_bounded(&full[i % P.S], (i / P.S) & 1, P.err);
    }
    return;
  }

  // ---------------- consumers ---------------------------------------------
  pdl_wait();
  if (MODE == MODE_F32X && P.xq) {
    f32x_prologue<FMT>(P.xq, FMT == Q8_0 ? 32 * P.nb : 256 * P.nb, P.nbu, ximg, kCW);
  } else {
    const uint4 *src = reinterpret_cast<const uint4 *>(P.img);
    uint4 *dst = reinterpret_cast<uint4 *>(ximg);
    for (int i = threadIdx.x; i < P.img_bytes / 16; i += kCons) dst[i] = src[i];
  }
  named_bar_sync(1, kCons);

  const int s_in = lane >> 3, j = lane & 7;
  const unsigned subm = 0xFFu << (lane & 24);
  const int sg = warp * 4 + s_in;  // subgroup id
  constexpr int kSubgroups = kCW * 4;
  unsigned long long best = 0ull;
  const int istr = MODE == MODE_F32X ? kImgF32X : (FMT == Q4K ? kImgQ8K4 : kImgQ8K6);

  // One named barrier per tile, between the phases. The chain phase of tile i
  // (a few warps) overlaps the integer phase of tile i+1 (the others); the
  // two chain buffers alternate, and barrier i+1 orders chain(i) before
  // anyone writes that buffer again at tile i+2.
  for (int i = 0; i < ntiles; i++) {
    const int s = i % P.S;
    const int r0 = rb + i * P.T;
    const int nr = min(P.T, re - r0);
    const bool got = mbar_wait_bounded(&full[s], (i / P.S) & 1, P.err);
    const uint8_t *tile = stages + (size_t)s * P.stage_bytes;
    float *cb = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(cbuf0) + (i & 1) * P.cbuf_bytes);

    // integer phase
    const int ngroups = (nr + R - 1) / R;
    const int nitems = got ? ngroups * P.nbu : 0;
    for (int it = sg; it < nitems; it += kSubgroups) {
      const int g = it / P.nbu, b = it - g * P.nbu;
      const uint8_t *rowp[R];
      bool rv[R];
#pragma unroll
      for (int r = 0; r < R; r++) {
        const int lr = g * R + r;
        rv[r] = lr < nr;
        rowp[r] = tile + (size_t)(rv[r] ? lr : 0) * P.pstride;
      }
      float *cbr = cb + g * R * P.rs;                       // this group's first chain row
      float *cmr = cb + P.T * P.rs + g * R * (P.rs / 8);    // Q8K: its dmin*minsum row
      integer_item<FMT, MODE, R>(rowp, rv, b, ximg + (size_t)b * istr, P, cbr, cmr, j, subm);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with the weight stage
    // uniform exit if any consumer timed out waiting for this tile
    if (!named_bar_red_and(1, kCons, got)) break;

    // chain phase: loads hoisted ahead of the dependent adds, 8 at a time
    if constexpr (MODE == MODE_F32X) {
      const int t = threadIdx.x;
      if (t < nr) {
        const float *fr = cb + t * P.rs;
        float v = 0.0f;
        for (int b = 0; b < P.nbu; b += 8) {
          float f[8];
#pragma unroll
          for (int q = 0; q < 8; q++) f[q] = b + q < P.nbu ? fr[b + q] : 0.0f;
#pragma unroll
          for (int q = 0; q < 8; q++) v += f[q];
        }
        const int row = r0 + t;
        if (P.y) P.y[row] = v;
        if (ARGMAX) {
          const unsigned long long kk = argmax_key(v, P.row0 + row);
          best = kk > best ? kk : best;
        }
      }
    } else {
      const int t = threadIdx.x, lr = t >> 3, k = t & 7;
      if (lr < nr) {
        const float *tk = cb + lr * P.rs + k;
        const float *tm = cb + P.T * P.rs + lr * (P.rs / 8);
        float sums = 0.0f, sumf = 0.0f;
        for (int b = 0; b < P.nbu; b += 8) {
          float a[8], mm[8];
#pragma unroll
          for (int q = 0; q < 8; q++) {
            const bool in = b + q < P.nbu;
            a[q] = in ? tk[8 * (b + q)] : 0.0f;
            if (FMT == Q4K) mm[q] = in ? tm[b + q] : 0.0f;
          }
#pragma unroll
          for (int q = 0; q < 8; q++) {
            if (b + q < P.nbu) {
              sums = __fadd_rn(sums, a[q]);
              if (FMT == Q4K) sumf = __fsub_rn(sumf, mm[q]);
            }
          }
        }
        const unsigned gm = 0xFFu << (lane & 24);
        float acc = sumf;  // Q6_K: sumf = 0, s = 0 + sums[0] + ...
#pragma unroll
        for (int kk = 0; kk < 8; kk++) acc = __fadd_rn(acc, __shfl_sync(gm, sums, (lane & 24) + kk));
        const int row = r0 + lr;
        if (k == 0) {
          if (P.y) P.y[row] = acc;
          if (ARGMAX) {
            const unsigned long long kk = argmax_key(acc, P.row0 + row);
            best = kk > best ? kk : best;
          }
        }
      }
    }
  }

  if constexpr (ARGMAX) {
    __shared__ unsigned long long cta_best[kCW];
    for (int o = 16; o; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if (lane == 0) cta_best[warp] = best;
    named_bar_sync(1, kCons);
    if (threadIdx.x == 0) {
      unsigned long long b = cta_best[0];
      for (int i = 1; i < kCW; i++) b = cta_best[i] > b ? cta_best[i] : b;
      atomicMax(P.key, b);
      __threadfence();
      const unsigned prev = atomicAdd(P.done, 1u);
      if (prev == gridDim.x - 1) {
        __threadfence();
        const unsigned long long k = atomicAdd(P.key, 0ull);
        *P.token = 0xffffffffu - (uint32_t)(k & 0xffffffffull);
        if (P.key_out) *P.key_out = k;
        *P.key = 0ull;
        *P.done = 0u;
      }
    }
  }
}

// Tensor-core Q4_K Q8K GEMV with the chain phase on warps of its own: the
// integer (MMA) warps hand each finished tile to the chain warps through an
// mbarrier and go on to the next tile; two chain buffers alternate, recycled
// through a second mbarrier pair. Nothing waits on a CTA-wide barrier per
// tile. Every wait is bounded.
// The warp counts are template parameters (NIW integer warps, NCW chain
// warps, one producer warp); the launches use kTcIntWarps / kTcChainWarps.
constexpr int kTcIntWarps = 16, kTcChainWarps = 3;
constexpr int kTcThreads = (kTcIntWarps + kTcChainWarps + 1) * 32;
constexpr int kTcBarBytes = 256;
// 256-element spans of a fused RMSNorm each integer warp keeps in registers.
constexpr int kNormSpans = 2;
static_assert(kTcThreads <= 1024, "a CTA has at most 1024 threads");
static_assert((2 * kMaxStages + 4) * 8 <= kTcBarBytes, "barrier area");

// RMSNorm (kernels.rs:61-78) of r = a (+ b) fused into the integer warps'
// prologue, after griddepcontrol.wait: every CTA sums the n squares itself
// (the reference's sequential f64 sum, resolved exactly as in the stand-alone
// norm kernel), then each warp quantizes whole spans of xn = rmsnorm(r, w)
// (quantize_q8_k) into the CTA's shared-memory image: warp w of NIW takes
// spans w and w + NIW, lane l their elements 8l .. 8l+7. CTA 0 also stores r and,
// when asked, the Q4_K / Q6_K images for later GEMVs. All pointers are
// 16-byte aligned (checked by gemv_launch).
template <int NIW>
__device__ __forceinline__ void tc_norm_prologue(const Params &P, uint8_t *ximg) {
  constexpr int NT = NIW * 32;
  __shared__ double red[NIW];
  __shared__ float s_mean;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31, n = P.nn, nsp = n >> 8;
  const bool cta0 = blockIdx.x == 0;
  if (P.peer_recv) {
    // every rank's partial rows must have landed here: wait (bounded) for its
    // flag to reach this all-reduce's number
    if (t < P.peer_n) {
      const unsigned ep = *P.peer_ctr;
      const unsigned *flag = reinterpret_cast<const unsigned *>(P.peer_map[P.peer_rank]) + t;
      if (peer_ld_acquire(flag) - ep > 0x7fffffffu) {
        const uint64_t t0 = global_ns();
        for (uint32_t it = 1;; ++it) {
          if (peer_ld_acquire(flag) - ep <= 0x7fffffffu) break;
          if ((it & 255u) == 0 && global_ns() - t0 > 2000000000ull) {
            atomicExch(P.err, kErrPeer);
            break;
          }
        }
      }
    }
    named_bar_sync(1, NT);
  }
  const bool has_b = P.norm_b || P.peer_recv;
  float r[kNormSpans][8], wv[kNormSpans][8];
#pragma unroll
  for (int u = 0; u < kNormSpans; u++) {
    const int e0 = (warp + NIW * u) * 256 + 8 * lane;
    float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0, b0 = a0, b1 = a0, w0 = a0, w1 = a0;
    if (e0 < n) {  // warp-uniform
      const float4 *pa = reinterpret_cast<const float4 *>(P.norm_a + e0);
      const float4 *pw = reinterpret_cast<const float4 *>(P.norm_w + e0);
      a0 = pa[0];
      a1 = pa[1];
      w0 = pw[0];
      w1 = pw[1];
      if (P.norm_b) {
        const float4 *pb = reinterpret_cast<const float4 *>(P.norm_b + e0);
        b0 = pb[0];
        b1 = pb[1];
      } else if (P.peer_recv) {  // b = the ranks' partial rows, summed in rank order
        const unsigned ep = *P.peer_ctr;
        const float *s0 = peer_slot(P.peer_map[P.peer_rank], ep, 0) + e0;
        b0 = __ldcv(reinterpret_cast<const float4 *>(s0));
        b1 = __ldcv(reinterpret_cast<const float4 *>(s0) + 1);
        for (int r = 1; r < P.peer_n; r++) {
          const float4 *sr = reinterpret_cast<const float4 *>(peer_slot(P.peer_map[P.peer_rank], ep, r) + e0);
          const float4 c0 = __ldcv(sr), c1 = __ldcv(sr + 1);
          b0 = make_float4(__fadd_rn(b0.x, c0.x), __fadd_rn(b0.y, c0.y), __fadd_rn(b0.z, c0.z), __fadd_rn(b0.w, c0.w));
          b1 = make_float4(__fadd_rn(b1.x, c1.x), __fadd_rn(b1.y, c1.y), __fadd_rn(b1.z, c1.z), __fadd_rn(b1.w, c1.w));
        }
      }
    }
    const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int k = 0; k < 8; k++) {
      r[u][k] = has_b ? __fadd_rn(av[k], bv[k]) : av[k];
      wv[u][k] = ww[k];
    }
  }
  double S = 0.0;
#pragma unroll
  for (int u = 0; u < kNormSpans; u++)
#pragma unroll
    for (int k = 0; k < 8; k++) S += (double)__fmul_rn(r[u][k], r[u][k]);
  if (cta0 && P.norm_r) {
#pragma unroll
    for (int u = 0; u < kNormSpans; u++) {
      const int e0 = (warp + NIW * u) * 256 + 8 * lane;
      if (e0 < n) {
        float4 *pr = reinterpret_cast<float4 *>(P.norm_r + e0);
        pr[0] = make_float4(r[u][0], r[u][1], r[u][2], r[u][3]);
        pr[1] = make_float4(r[u][4], r[u][5], r[u][6], r[u][7]);
      }
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);
  if (lane == 0) red[warp] = S;
  named_bar_sync(1, NT);
  S = 0.0;
#pragma unroll
  for (int w = 0; w < NIW; w++) S += red[w];
  float mean;
  const MeanOf f{n};
  if (!resolve_sum(S, S, n, f, &mean)) {  // S is the same in every thread
    if (t == 0) {
      double q = 0.0;
#pragma unroll 1
      for (int i = 0; i < n; i++) {
        float b = 0.0f;
        if (P.norm_b) {
          b = P.norm_b[i];
        } else if (P.peer_recv) {
          const unsigned ep = *P.peer_ctr;
          b = __ldcv(peer_slot(P.peer_map[P.peer_rank], ep, 0) + i);
          for (int rr = 1; rr < P.peer_n; rr++) b = __fadd_rn(b, __ldcv(peer_slot(P.peer_map[P.peer_rank], ep, rr) + i));
        }
        const float v = has_b ? __fadd_rn(P.norm_a[i], b) : P.norm_a[i];
        q = __dadd_rn(q, (double)__fmul_rn(v, v));
      }
      s_mean = f(q);
    }
    named_bar_sync(1, NT);
    mean = s_mean;
  }
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, P.norm_eps)));
#pragma unroll
  for (int u = 0; u < kNormSpans; u++) {
    const int span = warp + NIW * u;
    if (span < nsp) {  // warp-uniform
      float xn[8];
#pragma unroll
      for (int k = 0; k < 8; k++) xn[k] = __fmul_rn(__fmul_rn(r[u][k], scale), wv[u][k]);
      q8k_span_write_warp(xn, lane, ximg + (size_t)span * kImgQ8K4,
                          cta0 && P.norm_img6 ? P.norm_img6 + (size_t)span * kImgQ8K6 : nullptr);
    }
  }
  named_bar_sync(1, NT);
  if (cta0 && P.norm_img4) {
    const uint4 *src = reinterpret_cast<const uint4 *>(ximg);
    uint4 *dst = reinterpret_cast<uint4 *>(P.norm_img4);
    for (int k = t; k < P.img_bytes / 16; k += NT) dst[k] = src[k];
  }
}

// quantize_q8_k of x (quants.rs:250-290) in the integer warps' prologue,
// after griddepcontrol.wait, while the producer already streams weights:
// warp w of NIW takes spans w, w + NIW, ... (lane l: elements 8l .. 8l+7),
// loads of up to three spans in flight.
template <int FMT, int NIW>
__device__ __noinline__ void tc_quant_prologue(const float *__restrict__ x, int nsp, uint8_t *ximg) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int s0 = warp; s0 < nsp; s0 += 3 * NIW) {
    float4 v[3][2];
#pragma unroll
    for (int q = 0; q < 3; q++) {
      const int span = s0 + NIW * q;
      v[q][0] = v[q][1] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (span < nsp) {
        const float4 *p = reinterpret_cast<const float4 *>(x + (size_t)span * 256 + 8 * lane);
        v[q][0] = p[0];
        v[q][1] = p[1];
      }
    }
#pragma unroll
    for (int q = 0; q < 3; q++) {
      const int span = s0 + NIW * q;
      if (span >= nsp) break;
      const float e[8] = {v[q][0].x, v[q][0].y, v[q][0].z, v[q][0].w, v[q][1].x, v[q][1].y, v[q][1].z, v[q][1].w};
      if constexpr (FMT == Q4K) q8k_span_write_warp(e, lane, ximg + (size_t)span * kImgQ8K4, nullptr);
      else q8k_span_write_warp(e, lane, nullptr, ximg + (size_t)span * kImgQ8K6);
    }
  }
  named_bar_sync(1, NIW * 32);
}

template <int FMT, bool ARGMAX, bool R8, int NIW, int NCW, int MINB>
__global__ void __launch_bounds__((NIW + NCW + 1) * 32, MINB) gemv_tc_kernel(Params P) {
  constexpr int kImg = FMT == Q4K ? kImgQ8K4 : kImgQ8K6;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *full = reinterpret_cast<uint64_t *>(smem);
  uint64_t *empty = full + kMaxStages;
  uint64_t *intdone = empty + kMaxStages;  // [2]: a tile's integer results are in its chain buffer
  uint64_t *chaindone = intdone + 2;       // [2]: the chain buffer is free again
  uint8_t *ximg = smem + kTcBarBytes;
  float *cbuf0 = reinterpret_cast<float *>(ximg + P.img_bytes);
  uint8_t *stages = reinterpret_cast<uint8_t *>(cbuf0) + 2 * P.cbuf_bytes;
  pdl_trigger();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int rb = (int)((long long)P.rows * blockIdx.x / G);
  const int re = (int)((long long)P.rows * (blockIdx.x + 1) / G);
  const int ntiles = (re - rb + P.T - 1) / P.T;

  if (threadIdx.x == 0) {
    for (int st = 0; st < P.S; st++) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], NIW);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&intdone[b], NIW);
      mbar_init(&chaindone[b], NCW);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == NIW + NCW) {
    // ---------------- producer: padded rows, one bulk copy per row ----------
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      for (int i = 0; i < ntiles && ok; i++) {
        const int st = i % P.S;
        if (i >= P.S) ok = mbar_wait_bounded(&empty[st], ((i / P.S) - 1) & 1, P.err);
        if (!ok) break;
        const int r0 = rb + i * P.T;
        const int nr = min(P.T, re - r0);
        mbar_expect_tx(&full[st], (uint32_t)(nr * P.stride));
        for (int rr = 0; rr < nr; rr++)
          bulk_g2s(stages + (size_t)st * P.stage_bytes + (size_t)rr * P.pstride, P.W + (size_t)(r0 + rr) * P.stride,
                   (uint32_t)P.stride, &full[st]);
        issued = i + 1;
      }
      for (int i = max(0, issued - P.S); i < issued; i++)
        mbar_wait_bounded(&full[i % P.S], (i / P.S) & 1, P.err);
    }
    return;
  }

  pdl_wait();
  if (warp < NIW) {
    // ---------------- integer warps -------------------------------------------
    if (FMT == Q4K && P.nn) {
      tc_norm_prologue<NIW>(P, ximg);
    } else if (P.xq) {
      tc_quant_prologue<FMT, NIW>(P.xq, P.nbu, ximg);
    } else {
      const uint4 *src = reinterpret_cast<const uint4 *>(P.img);
      uint4 *dst = reinterpret_cast<uint4 *>(ximg);
      for (int k = threadIdx.x; k < P.img_bytes / 16; k += NIW * 32) dst[k] = src[k];
      named_bar_sync(1, NIW * 32);
    }
    // when the block count divides the warp count, a warp always takes the
    // same block (row groups rg0, rg0 + rgs, ...): its x operands stay in
    // registers for the whole kernel
    const bool fixed = NIW % P.nbu == 0;
    const int myb = warp % P.nbu, rg0 = warp / P.nbu, rgs = NIW / P.nbu;
    using XB = std::conditional_t<FMT == Q4K, XBlock, XBlock6>;
    XB xb;
    auto load_xb = [&](int b, XB &x) {
      if constexpr (FMT == Q4K) load_xblock(ximg + (size_t)b * kImg, x);
      else load_xblock6(ximg + (size_t)b * kImg, x);
    };
    auto item = [&](const uint8_t *tile, int nr, int g16, int b, const XB &x, float *cb, float *cm) {
      if constexpr (FMT == Q4K) q4k_q8k_mma_item(tile, nr, g16, b, x, P, cb, cm);
      else q6k_q8k_mma_item<R8>(tile, nr, g16, b, x, P, cb);
    };
    if (fixed) load_xb(myb, xb);
    for (int i = 0; i < ntiles; i++) {
      const int st = i % P.S;
      const int r0 = rb + i * P.T;
      const int nr = min(P.T, re - r0);
      if (!mbar_wait_bounded(&full[st], (i / P.S) & 1, P.err)) break;
      if (i >= 2 && !mbar_wait_bounded(&chaindone[i & 1], ((i >> 1) - 1) & 1, P.err)) break;
      const uint8_t *tile = stages + (size_t)st * P.stage_bytes;
      float *cb = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(cbuf0) + (i & 1) * P.cbuf_bytes);
      float *cm = cb + P.T * P.rs;
      const int ng = R8 ? (nr + 7) / 8 : (nr + 15) / 16;  // row groups of the item
      if (fixed) {
        for (int g16 = rg0; g16 < ng; g16 += rgs) item(tile, nr, g16, myb, xb, cb, cm);
      } else {
        for (int it = warp; it < ng * P.nbu; it += NIW) {
          const int g16 = it / P.nbu, b = it - g16 * P.nbu;
          XB xv;
          load_xb(b, xv);
          item(tile, nr, g16, b, xv, cb, cm);
        }
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&empty[st]);     // weight stage free
        mbar_arrive(&intdone[i & 1]);  // integer results ready
      }
    }
    return;
  }

  // ---------------- chain warps: the sequential per-row epilogue ------------
  const int ct = threadIdx.x - NIW * 32;  // 0 .. 32 * NCW - 1
  const int k = ct & 7;
  const unsigned gm = 0xFFu << (lane & 24);
  unsigned long long best = 0ull;
  const unsigned send_ep = P.peer_send ? *P.peer_ctr + 1u : 0u;  // the all-reduce this GEMV feeds
  for (int i = 0; i < ntiles; i++) {
    if (!mbar_wait_bounded(&intdone[i & 1], (i >> 1) & 1, P.err)) break;
    const int r0 = rb + i * P.T;
    const int nr = min(P.T, re - r0);
    const float *cb = reinterpret_cast<const float *>(reinterpret_cast<const uint8_t *>(cbuf0) + (i & 1) * P.cbuf_bytes);
    for (int lr = ct >> 3; lr < nr; lr += NCW * 4) {
      const float *tk = cb + lr * P.rs + k;
      const float *tm = cb + P.T * P.rs + lr * (P.rs / 8);
      float sums = 0.0f, sumf = 0.0f;
      for (int b = 0; b < P.nbu; b += 8) {
        float a[8], mm[8];
#pragma unroll
        for (int q = 0; q < 8; q++) {
          const bool in = b + q < P.nbu;
          a[q] = in ? tk[8 * (b + q)] : 0.0f;
          mm[q] = (FMT == Q4K && in) ? tm[b + q] : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < 8; q++) {
          if (b + q < P.nbu) {
            sums = __fadd_rn(sums, a[q]);
            if (FMT == Q4K) sumf = __fsub_rn(sumf, mm[q]);  // Q6_K: no min term, s starts at 0
          }
        }
      }
      float acc = sumf;
#pragma unroll
      for (int kk = 0; kk < 8; kk++) acc = __fadd_rn(acc, __shfl_sync(gm, sums, (lane & 24) + kk));
      if (k == 0) {
        const int row = r0 + lr;
        if (P.y) P.y[row] = acc;
        if (P.peer_send)  // this rank's partial row into every rank's slot
          for (int rr = 0; rr < P.peer_n; rr++) peer_slot(P.peer_map[rr], send_ep, P.peer_rank)[row] = acc;
        if (ARGMAX) {
          const unsigned long long kk2 = argmax_key(acc, P.row0 + row);
          best = kk2 > best ? kk2 : best;
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&chaindone[i & 1]);
  }
  if (P.peer_send) {
    // the last CTA to finish raises this rank's flag in every area (after a
    // system fence) and advances the all-reduce counter
    __threadfence_system();
    named_bar_sync(2, NCW * 32);
    if (ct == 0) {
      const unsigned prev = atomicAdd(P.peer_done, 1u);
      if (prev == gridDim.x - 1) {
        __threadfence_system();
        for (int rr = 0; rr < P.peer_n; rr++)
          peer_st_release(reinterpret_cast<unsigned *>(P.peer_map[rr]) + P.peer_rank, send_ep);
        *P.peer_ctr = send_ep;
        *P.peer_done = 0u;
      }
    }
  }
  if constexpr (ARGMAX) {
    __shared__ unsigned long long cta_best[NCW];
    for (int o = 16; o; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if (lane == 0) cta_best[warp - NIW] = best;
    named_bar_sync(2, NCW * 32);
    if (ct == 0) {
      unsigned long long b = cta_best[0];
      for (int w2 = 1; w2 < NCW; w2++) b = cta_best[w2] > b ? cta_best[w2] : b;
      atomicMax(P.key, b);
      __threadfence();
      const unsigned prev = atomicAdd(P.done, 1u);
      if (prev == gridDim.x - 1) {
        __threadfence();
        const unsigned long long kf = atomicAdd(P.key, 0ull);
        *P.token = 0xffffffffu - (uint32_t)(kf & 0xffffffffull);
        if (P.key_out) *P.key_out = kf;
        *P.key = 0ull;
        *P.done = 0u;
      }
    }
  }
}

// ---------------------------------------------------------------- lean ----
// The tensor-core GEMV specialised on its shape: blocks per row (NBU), rows
// per tile (T) and the padded shared-memory row stride are compile-time
// constants, so every shared-memory address is a register plus an immediate
// and the loops unroll without bounds checks. Used for the decode step's
// shapes (4096 or 12288 inputs); other shapes take gemv_tc_kernel. The same
// arithmetic, so the same bits.
//
//  * integer warps: with NBU == NIW a warp owns one block for the whole
//    kernel (its x operands stay in registers) and runs that block for every
//    16-row group of a tile; otherwise it takes blocks warp, warp + NIW, ...
//    and loads the block's x operands per item. Rows past the end of a
//    partial tile compute on stale shared memory; the chain never reads them.
//  * chain warp(s): T >= 16: lane = row, each lane runs the nine sequential
//    f32 chains of its row (sums[0..7] and the min term) over the blocks with
//    128-bit loads of the row's eight class products per block; T == 8:
//    lane = (row, class) as in gemv_tc_kernel.
//  * chunked Q6_K rows (12288 inputs): a work unit is a 16-row tile of one
//    16-block chunk (3360 bytes per row, one bulk copy each), so a stage
//    holds full-height MMA items for 16 rows in 55 KB; the tile's three
//    chunks run in order and the chain carries sums[0..7] across them.
template <int FMT, int NBU>
struct LeanShape {
  static constexpr int kRowBytes = NBU * (FMT == Q4K ? 144 : 210);
  static constexpr int kPs = (kRowBytes + 127) / 128 * 128 + (FMT == Q4K ? 32 : 16);
  static constexpr int kImg = FMT == Q4K ? kImgQ8K4 : kImgQ8K6;
  static constexpr int kRs = 8 * NBU + 4;   // chain row: eight class products per block (+4: bank spread)
  static constexpr int kRsm = NBU + 1;      // Q4_K min-term row
};

template <int FMT, int NBU, int T>
constexpr int lean_cbuf_bytes() {
  return ((T * LeanShape<FMT, NBU>::kRs + (FMT == Q4K ? T * LeanShape<FMT, NBU>::kRsm : 0)) * 4 + 127) / 128 * 128;
}

template <int NBU, int PS, int RS, int RSM>
__device__ __forceinline__ void q4k_item_lean(const uint8_t *tile, int g16, int b, const XBlock &x, float *tk,
                                              float *tm) {
  const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
  const int lr0 = g16 * 16 + gid;
  const uint8_t *row0 = tile + lr0 * PS;
  const uint8_t *row1 = row0 + 8 * PS;
  const uint4 h0 = lds128(row0 + b * 16), h1 = lds128(row1 + b * 16);
  const int qo = NBU * 16 + b * 128 + 8 * tig;
  uint2 w0[4], w1[4];
#pragma unroll
  for (int p = 0; p < 4; p++) {
    w0[p] = lds64(row0 + qo + 32 * p);
    w1[p] = lds64(row1 + qo + 32 * p);
  }
  const uint32_t SCa0 = h0.y & 0x3F3F3F3Fu, SCb0 = (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u);
  const uint32_t SCa1 = h1.y & 0x3F3F3F3Fu, SCb1 = (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u);
  int lo0 = 0, lo1 = 0, lo2 = 0, lo3 = 0, hi0 = 0, hi1 = 0, hi2 = 0, hi3 = 0;
#pragma unroll
  for (int p = 0; p < 4; p++) {
    const uint32_t S0 = p < 2 ? SCa0 : SCb0, S1 = p < 2 ? SCa1 : SCb1;
    const int k = (2 * p) & 3;
    int d0, d1, d2, d3, e0, e1, e2, e3;
    mma_s8(w0[p].x & 0x0F0F0F0Fu, w1[p].x & 0x0F0F0F0Fu, w0[p].y & 0x0F0F0F0Fu, w1[p].y & 0x0F0F0F0Fu, x.b0[2 * p],
           x.b1[2 * p], d0, d1, d2, d3);
    mma_u8s8(w0[p].x & 0xF0F0F0F0u, w1[p].x & 0xF0F0F0F0u, w0[p].y & 0xF0F0F0F0u, w1[p].y & 0xF0F0F0F0u,
             x.b0[2 * p + 1], x.b1[2 * p + 1], e0, e1, e2, e3);
    const int s0 = byte_of(S0, k), s1 = byte_of(S1, k), t0 = byte_of(S0, k + 1), t1 = byte_of(S1, k + 1);
    lo0 += s0 * d0;
    lo1 += s0 * d1;
    lo2 += s1 * d2;
    lo3 += s1 * d3;
    hi0 += t0 * e0;
    hi1 += t0 * e1;
    hi2 += t1 * e2;
    hi3 += t1 * e3;
  }
  const int acc0 = lo0 + (hi0 >> 4), acc1 = lo1 + (hi1 >> 4), acc2 = lo2 + (hi2 >> 4), acc3 = lo3 + (hi3 >> 4);
  const uint32_t MA0 = h0.z & 0x3F3F3F3Fu, MB0 = ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u);
  const uint32_t MA1 = h1.z & 0x3F3F3F3Fu, MB1 = ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u);
  int mn0, mn1, mn2, mn3;
  mma_s8_k16(tig == 0 ? MA0 : (tig == 1 ? MB0 : 0u), tig == 0 ? MA1 : (tig == 1 ? MB1 : 0u), x.bm, mn0, mn1, mn2,
             mn3);
  const float d0 = __fmul_rn(x.xd, h2f_bits(h0.x & 0xFFFFu)), dm0 = __fmul_rn(h2f_bits(h0.x >> 16), x.xd);
  const float d1 = __fmul_rn(x.xd, h2f_bits(h1.x & 0xFFFFu)), dm1 = __fmul_rn(h2f_bits(h1.x >> 16), x.xd);
  *reinterpret_cast<float2 *>(tk + lr0 * RS + 8 * b + 2 * tig) =
      make_float2(__fmul_rn(d0, (float)acc0), __fmul_rn(d0, (float)acc1));
  *reinterpret_cast<float2 *>(tk + (lr0 + 8) * RS + 8 * b + 2 * tig) =
      make_float2(__fmul_rn(d1, (float)acc2), __fmul_rn(d1, (float)acc3));
  if (tig == 0) {
    tm[lr0 * RSM + b] = __fmul_rn(dm0, (float)(mn0 + mn1 * 256));
    tm[(lr0 + 8) * RSM + b] = __fmul_rn(dm1, (float)(mn2 + mn3 * 256));
  }
}

template <bool R8, int NBU, int PS, int RS>
__device__ __forceinline__ void q6k_item_lean(const uint8_t *tile, int g16, int b, const XBlock6 &x, float *tk) {
  const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
  const int lr0 = (R8 ? 8 : 16) * g16 + gid;
  const uint8_t *row0 = tile + lr0 * PS;
  const uint8_t *row1 = row0 + 8 * PS;
  const int qlo = b * 128 + 4 * tig, qho = NBU * 128 + b * 64 + 4 * tig;
  uint32_t l0[8], l1[8], h0[4], h1[4];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    l0[j] = *reinterpret_cast<const uint32_t *>(row0 + qlo + 16 * j);
    l1[j] = R8 ? 0u : *reinterpret_cast<const uint32_t *>(row1 + qlo + 16 * j);
  }
#pragma unroll
  for (int c = 0; c < 4; c++) {
    h0[c] = *reinterpret_cast<const uint32_t *>(row0 + qho + 16 * c);
    h1[c] = R8 ? 0u : *reinterpret_cast<const uint32_t *>(row1 + qho + 16 * c);
  }
  const uint4 sc0 = lds128(row0 + NBU * 192 + b * 16);
  const uint4 sc1 = R8 ? make_uint4(0u, 0u, 0u, 0u) : lds128(row1 + NBU * 192 + b * 16);
  const uint32_t S0[4] = {sc0.x, sc0.y, sc0.z, sc0.w}, S1[4] = {sc1.x, sc1.y, sc1.z, sc1.w};
  const uint32_t db0 = *reinterpret_cast<const unsigned short *>(row0 + NBU * 208 + b * 2);
  const uint32_t db1 = R8 ? 0u : *reinterpret_cast<const unsigned short *>(row1 + NBU * 208 + b * 2);
  int acc0 = 0, acc1 = 0, acc2 = 0, acc3 = 0;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int h = j >> 2, u = j & 3, sl = 2 * (u >> 1), c = 2 * h + (u & 1);
    const int slo = 8 * h + u, shi = slo + 4;
    int d0, d1, d2, d3, e0, e1, e2, e3;
    mma_s8_k16(q6_a4_lo(l0[j], h0[c], sl), R8 ? 0u : q6_a4_lo(l1[j], h1[c], sl), x.b[2 * j], d0, d1, d2, d3);
    mma_s8_k16(q6_a4_hi(l0[j], h0[c], sl), R8 ? 0u : q6_a4_hi(l1[j], h1[c], sl), x.b[2 * j + 1], e0, e1, e2, e3);
    const int s0 = sbyte_of(S0[slo >> 2], slo & 3), t0 = sbyte_of(S0[shi >> 2], shi & 3);
    acc0 += s0 * d0 + t0 * e0;
    acc1 += s0 * d1 + t0 * e1;
    if (!R8) {
      const int s1 = sbyte_of(S1[slo >> 2], slo & 3), t1 = sbyte_of(S1[shi >> 2], shi & 3);
      acc2 += s1 * d2 + t1 * e2;
      acc3 += s1 * d3 + t1 * e3;
    }
  }
  const float d0 = __fmul_rn(x.xd, h2f_bits(db0));
  *reinterpret_cast<float2 *>(tk + lr0 * RS + 8 * b + 2 * tig) =
      make_float2(__fmul_rn(d0, (float)(acc0 >> 2)), __fmul_rn(d0, (float)(acc1 >> 2)));
  if (!R8) {
    const float d1 = __fmul_rn(x.xd, h2f_bits(db1));
    *reinterpret_cast<float2 *>(tk + (lr0 + 8) * RS + 8 * b + 2 * tig) =
        make_float2(__fmul_rn(d1, (float)(acc2 >> 2)), __fmul_rn(d1, (float)(acc3 >> 2)));
  }
}

// Emits one finished row: y, this rank's slot of every peer area, the argmax key.
template <bool ARGMAX>
__device__ __forceinline__ void lean_emit_row(const Params &P, int row, float acc, unsigned send_ep,
                                              unsigned long long &best) {
  if (P.y) P.y[row] = acc;
  if (P.peer_send)
    for (int rr = 0; rr < P.peer_n; rr++) peer_slot(P.peer_map[rr], send_ep, P.peer_rank)[row] = acc;
  if (ARGMAX) {
    const unsigned long long k2 = argmax_key(acc, P.row0 + row);
    best = k2 > best ? k2 : best;
  }
}

template <int FMT, int NBU, int T, int NIW, int NCW, bool ARGMAX, int MINB, int NBC>
__global__ void __launch_bounds__((NIW + NCW + 1) * 32, MINB) gemv_lean_kernel(Params P) {
  // A work unit is one tile of T rows by NBC blocks: the whole row, or one
  // 16-block chunk of a chunked Q6_K row (NBC = 16 < NBU), the tile's chunks
  // in order so the chain keeps the reference's block order.
  using Sh = LeanShape<FMT, NBC>;
  constexpr bool R8 = T == 8;
  constexpr int NCH = NBU / NBC;
  constexpr int kFullRow = NBU * (FMT == Q4K ? 144 : 210);
  static_assert(NBU % NBC == 0 && (NCH == 1 || (FMT == Q6K && NBC == kQ6Chunk && !R8)), "chunked units: Q6_K only");
  static_assert(R8 || T <= NCW * 32, "the chain takes one row per lane");
  constexpr int PS = Sh::kPs, RS = Sh::kRs, RSM = Sh::kRsm;
  constexpr int STAGE = (T * PS + 127) / 128 * 128;
  constexpr int CBUF = lean_cbuf_bytes<FMT, NBC, T>();
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *full = reinterpret_cast<uint64_t *>(smem);
  uint64_t *empty = full + kMaxStages;
  uint64_t *intdone = empty + kMaxStages;
  uint64_t *chaindone = intdone + 2;
  uint8_t *ximg = smem + kTcBarBytes;
  uint8_t *cbase = ximg + NBU * Sh::kImg;
  uint8_t *stages = cbase + 2 * CBUF;
  const int S = P.S;
  pdl_trigger();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int rb = (int)((long long)P.rows * blockIdx.x / G);
  const int re = (int)((long long)P.rows * (blockIdx.x + 1) / G);
  const int ntiles = (re - rb + T - 1) / T;
  const int nunits = ntiles * NCH;

  if (threadIdx.x == 0) {
    for (int st = 0; st < S; st++) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], NIW);
    }
    for (int bb = 0; bb < 2; bb++) {
      mbar_init(&intdone[bb], NIW);
      mbar_init(&chaindone[bb], NCW);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == NIW + NCW) {
    // ---------------- producer: one bulk copy per (padded) row --------------
    if (lane == 0) {
      int issued = 0;
      for (int u = 0; u < nunits; u++) {
        const int st = u % S;
        if (u >= S && !mbar_wait_bounded(&empty[st], ((u / S) - 1) & 1, P.err)) break;
        const int r0 = rb + (u / NCH) * T;
        const int nr = min(T, re - r0);
        mbar_expect_tx(&full[st], (uint32_t)(nr * Sh::kRowBytes));
        const uint8_t *src = P.W + (size_t)r0 * kFullRow + (size_t)(u % NCH) * Sh::kRowBytes;
        uint8_t *dst = stages + (size_t)st * STAGE;
        for (int rr = 0; rr < nr; rr++) bulk_g2s(dst + rr * PS, src + (size_t)rr * kFullRow, Sh::kRowBytes, &full[st]);
        issued = u + 1;
      }
      for (int i = max(0, issued - S); i < issued; i++) mbar_wait_bounded(&full[i % S], (i / S) & 1, P.err);
    }
    return;
  }

  pdl_wait();
  if (warp < NIW) {
    // ---------------- integer warps -------------------------------------------
    if (FMT == Q4K && P.nn) {
      tc_norm_prologue<NIW>(P, ximg);
    } else if (P.xq) {
      tc_quant_prologue<FMT, NIW>(P.xq, NBU, ximg);
    } else {
      const uint4 *src = reinterpret_cast<const uint4 *>(P.img);
      uint4 *dst = reinterpret_cast<uint4 *>(ximg);
      for (int k = threadIdx.x; k < NBU * Sh::kImg / 16; k += NIW * 32) dst[k] = src[k];
      named_bar_sync(1, NIW * 32);
    }
    using XB = std::conditional_t<FMT == Q4K, XBlock, XBlock6>;
    auto load_xb = [&](int b, XB &x) {
      if constexpr (FMT == Q4K) load_xblock(ximg + (size_t)b * Sh::kImg, x);
      else load_xblock6(ximg + (size_t)b * Sh::kImg, x);
    };
    constexpr int NG = R8 ? 1 : T / 16;  // 16-row groups of a tile (R8: one half-height group)
    constexpr bool kFixed = NBC == NIW;
    XB xb;
    if (kFixed && NCH == 1) load_xb(warp, xb);
    for (int u = 0; u < nunits; u++) {
      const int st = u % S, cb = (u % NCH) * NBC;  // cb: the unit's first block
      if (!mbar_wait_bounded(&full[st], (u / S) & 1, P.err)) break;
      if (u >= 2 && !mbar_wait_bounded(&chaindone[u & 1], ((u >> 1) - 1) & 1, P.err)) break;
      const uint8_t *tile = stages + (size_t)st * STAGE;
      float *tk = reinterpret_cast<float *>(cbase + (u & 1) * CBUF);
      float *tm = tk + T * RS;
      if constexpr (kFixed) {
        if constexpr (NCH > 1) load_xb(cb + warp, xb);
#pragma unroll
        for (int g = 0; g < NG; g++) {
          if constexpr (FMT == Q4K) q4k_item_lean<NBC, PS, RS, RSM>(tile, g, warp, xb, tk, tm);
          else q6k_item_lean<R8, NBC, PS, RS>(tile, g, warp, xb, tk);
        }
      } else {
#pragma unroll 1
        for (int b = warp; b < NBC; b += NIW) {
          XB xv;
          load_xb(cb + b, xv);
#pragma unroll
          for (int g = 0; g < NG; g++) {
            if constexpr (FMT == Q4K) q4k_item_lean<NBC, PS, RS, RSM>(tile, g, b, xv, tk, tm);
            else q6k_item_lean<R8, NBC, PS, RS>(tile, g, b, xv, tk);
          }
        }
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&empty[st]);
        mbar_arrive(&intdone[u & 1]);
      }
    }
    return;
  }

  // ---------------- chain warp(s): the sequential per-row epilogue -----------
  const int ct = threadIdx.x - NIW * 32;
  unsigned long long best = 0ull;
  const unsigned send_ep = P.peer_send ? *P.peer_ctr + 1u : 0u;
  // lane = row (T >= 16): the row's chains, carried across its chunks
  float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float sumf = 0.0f;
  for (int u = 0; u < nunits; u++) {
    if (!mbar_wait_bounded(&intdone[u & 1], (u >> 1) & 1, P.err)) break;
    const int r0 = rb + (u / NCH) * T, c = u % NCH;
    const int nr = min(T, re - r0);
    const float *tk = reinterpret_cast<const float *>(cbase + (u & 1) * CBUF);
    const float *tm = tk + T * RS;
    if constexpr (!R8) {
      // lane = row: sums[k] += d * sumi[k] over the blocks (the products are
      // in tk), sumf -= dmin * minsum, then s = sumf + sums[0] + ... + sums[7]
      const int lr = ct;
      if (lr < nr) {
        const float *row = tk + lr * RS;
        if (c == 0) {
#pragma unroll
          for (int k = 0; k < 8; k++) s[k] = 0.0f;
          sumf = 0.0f;
        }
#pragma unroll
        for (int b = 0; b < NBC; b++) {
          const float4 a = *reinterpret_cast<const float4 *>(row + 8 * b);
          const float4 c = *reinterpret_cast<const float4 *>(row + 8 * b + 4);
          s[0] = __fadd_rn(s[0], a.x);
          s[1] = __fadd_rn(s[1], a.y);
          s[2] = __fadd_rn(s[2], a.z);
          s[3] = __fadd_rn(s[3], a.w);
          s[4] = __fadd_rn(s[4], c.x);
          s[5] = __fadd_rn(s[5], c.y);
          s[6] = __fadd_rn(s[6], c.z);
          s[7] = __fadd_rn(s[7], c.w);
          if constexpr (FMT == Q4K) sumf = __fsub_rn(sumf, tm[lr * RSM + b]);
        }
        if (c == NCH - 1) {
          float acc = sumf;
#pragma unroll
          for (int k = 0; k < 8; k++) acc = __fadd_rn(acc, s[k]);
          lean_emit_row<ARGMAX>(P, r0 + lr, acc, send_ep, best);
        }
      }
    } else {
      // lane = (row, class): 8-row tiles of long rows (Q6_K, no min term)
      const int k = ct & 7;
      const unsigned gm = 0xFFu << (lane & 24);
      for (int lr = ct >> 3; lr < T; lr += NCW * 4) {
        const float *tkr = tk + lr * RS + k;
        float sums = 0.0f;
#pragma unroll 16
        for (int b = 0; b < NBC; b++) sums = __fadd_rn(sums, tkr[8 * b]);
        float acc = 0.0f;
#pragma unroll
        for (int kk = 0; kk < 8; kk++) acc = __fadd_rn(acc, __shfl_sync(gm, sums, (lane & 24) + kk));
        if (k == 0 && lr < nr) lean_emit_row<ARGMAX>(P, r0 + lr, acc, send_ep, best);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&chaindone[u & 1]);
  }
  if (P.peer_send) {
    __threadfence_system();
    named_bar_sync(2, NCW * 32);
    if (ct == 0) {
      const unsigned prev = atomicAdd(P.peer_done, 1u);
      if (prev == gridDim.x - 1) {
        __threadfence_system();
        for (int rr = 0; rr < P.peer_n; rr++)
          peer_st_release(reinterpret_cast<unsigned *>(P.peer_map[rr]) + P.peer_rank, send_ep);
        *P.peer_ctr = send_ep;
        *P.peer_done = 0u;
      }
    }
  }
  if constexpr (ARGMAX) {
    __shared__ unsigned long long cta_best[NCW];
    for (int o = 16; o; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if (lane == 0) cta_best[warp - NIW] = best;
    named_bar_sync(2, NCW * 32);
    if (ct == 0) {
      unsigned long long bb = cta_best[0];
      for (int w2 = 1; w2 < NCW; w2++) bb = cta_best[w2] > bb ? cta_best[w2] : bb;
      atomicMax(P.key, bb);
      __threadfence();
      const unsigned prev = atomicAdd(P.done, 1u);
      if (prev == gridDim.x - 1) {
        __threadfence();
        const unsigned long long kf = atomicAdd(P.key, 0ull);
        *P.token = 0xffffffffu - (uint32_t)(kf & 0xffffffffull);
        if (P.key_out) *P.key_out = kf;
        *P.key = 0ull;
        *P.done = 0u;
      }
    }
  }
}

// Plain f32 weights (gemv_quant's F32 case): one warp per row, f32 FMA.
__global__ void __launch_bounds__(kThreads) gemv_f32_kernel(const uint8_t *__restrict__ W, size_t stride,
                                                            int dim_in, int rows, const float *__restrict__ x,
                                                            float *__restrict__ y, unsigned long long *key,
                                                            unsigned *done, uint32_t *token) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gw = blockIdx.x * (kThreads / 32) + warp, nw = gridDim.x * (kThreads / 32);
  unsigned long long best = 0ull;
  for (int row = gw; row < rows; row += nw) {
    const float *wr = reinterpret_cast<const float *>(W + (size_t)row * stride);
    float acc = 0.0f;
    for (int i = lane; i < dim_in; i += 32) acc = fmaf(wr[i], x[i], acc);
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0 && y) y[row] = acc;
    if (key) {
      const unsigned long long k = argmax_key(acc, row);
      best = k > best ? k : best;
    }
  }
  if (key) {
    __shared__ unsigned long long cta_best[kThreads / 32];
    if (lane == 0) cta_best[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long b = cta_best[0];
      for (int i = 1; i < kThreads / 32; i++) b = cta_best[i] > b ? cta_best[i] : b;
      atomicMax(key, b);
      __threadfence();
      const unsigned prev = atomicAdd(done, 1u);
      if (prev == gridDim.x - 1) {
        __threadfence();
        const unsigned long long k = atomicAdd(key, 0ull);
        *token = 0xffffffffu - (uint32_t)(k & 0xffffffffull);
        *key = 0ull;
        *done = 0u;
      }
    }
  }
}

// --------------------------------------------------------------- dispatch --

using GemvFn = void (*)(Params);

template <int FMT, int MODE, bool AM>
GemvFn pick_r(int R) {
  return R == 1 ? gemv_kernel<FMT, MODE, 1, AM> : gemv_kernel<FMT, MODE, 2, AM>;
}

// mma: 0 DP4A kernel; tensor-core kernel 1 (16-row MMA items), 2 with 8-row
// tiles (Q6_K)
template <bool AM>
GemvFn pick(int fmt, int mode, int R, int mma = 0) {
  constexpr int FI = kTcIntWarps, FC = kTcChainWarps;
  if (mma == 2) return gemv_tc_kernel<Q6K, AM, true, FI, FC, 1>;  // 8-row tiles (Q6_K only)
  if (mma) return fmt == Q4K ? gemv_tc_kernel<Q4K, AM, false, FI, FC, 1> : gemv_tc_kernel<Q6K, AM, false, FI, FC, 1>;
  if (mode == MODE_F32X) {
    if (fmt == Q4K) return pick_r<Q4K, MODE_F32X, AM>(R);
    if (fmt == Q6K) return pick_r<Q6K, MODE_F32X, AM>(R);
    return pick_r<Q8_0, MODE_F32X, AM>(R);
  }
  if (fmt == Q4K) return pick_r<Q4K, MODE_Q8K, AM>(R);
  return pick_r<Q6K, MODE_Q8K, AM>(R);
}

int device_attr_cached(int device, cudaDeviceAttr attr) {
  static std::mutex mu;
  static std::vector<std::pair<std::pair<int, int>, int>> cache;
  std::lock_guard<std::mutex> lk(mu);
  for (auto &e : cache)
    if (e.first.first == device && e.first.second == (int)attr) return e.second;
  int v = 0;
  cudaDeviceGetAttribute(&v, attr, device);
  cache.push_back({{device, (int)attr}, v});
  return v;
}

int max_smem_optin(int device) { return device_attr_cached(device, cudaDevAttrMaxSharedMemoryPerBlockOptin); }


// cudaFuncSetAttribute applies to the current device's context, so the cache
// is keyed by (device, kernel): a process that drives several GPUs sets the
// limit on each of them.
cudaError_t ensure_smem_attr(int device, GemvFn fn, int smem) {
  struct Entry {
    int device;
    GemvFn fn;
    int smem;
  };
  static std::mutex mu;
  static std::vector<Entry> done;
  std::lock_guard<std::mutex> lk(mu);
  for (auto &e : done)
    if (e.device == device && e.fn == fn && e.smem >= smem) return cudaSuccess;
  const cudaError_t err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (err == cudaSuccess) done.push_back({device, fn, smem});
  return err;
}

// The shape-specialised kernel for w in Q8K mode, or null: Q4_K or Q6_K rows
// of 4096 inputs, Q6_K rows of 12288, every row a whole number of blocks
// with no padding. Fills the tile rows, stages, dynamic shared memory and
// block size of its launch.
struct LeanPlan {
  GemvFn fn = nullptr;
  int T = 0, S = 0, smem = 0, threads = 0, img_bytes = 0;
};

template <int FMT, int NBU, int T, int NBC = NBU, int NIW = kTcIntWarps, int MINB = 1>
LeanPlan lean_plan(bool am, int smem_max) {
  using Sh = LeanShape<FMT, NBC>;
  constexpr int stage = (T * Sh::kPs + 127) / 128 * 128;
  constexpr int fixed = kTcBarBytes + NBU * Sh::kImg + 2 * lean_cbuf_bytes<FMT, NBC, T>();
  LeanPlan p;
  p.S = std::min(kMaxStages, (smem_max - fixed) / stage);
  if (p.S < 2) return p;
  p.fn = am ? gemv_lean_kernel<FMT, NBU, T, NIW, 1, true, MINB, NBC>
            : gemv_lean_kernel<FMT, NBU, T, NIW, 1, false, MINB, NBC>;
  p.T = T;
  p.smem = fixed + p.S * stage;
  p.threads = (NIW + 2) * 32;
  p.img_bytes = NBU * Sh::kImg;
  return p;
}

LeanPlan lean_for(int device, const unltd_weight_s &w, int mode, bool am) {
  if (mode != MODE_Q8K || w.row_stride != w.row_bytes) return LeanPlan();
  const int smem_max = max_smem_optin(device) - 1024;
  if (w.dtype == Q4K && w.dim_in == 4096) return lean_plan<Q4K, 16, 32>(am, smem_max);
  if (w.dtype == Q6K && w.dim_in == 4096) return lean_plan<Q6K, 16, 16>(am, smem_max);
  if (w.dtype == Q6K && w.dim_in == 12288) return lean_plan<Q6K, 48, 16, kQ6Chunk>(am, smem_max);
  return LeanPlan();
}

}  // namespace

// Sets the dynamic shared-memory limit of every quantized GEMV kernel to the
// largest plan gemv_launch can choose on `device` (which must be current), so
// later launches find their attribute already set (no host-side cache growth
// on the hot path). Returns the first error of cudaFuncSetAttribute.
cudaError_t gemv_prewarm(int device) {
  const int m = max_smem_optin(device) - 1024;
  const int fmts[3] = {Q4K, Q6K, Q8_0};
  cudaError_t first = cudaSuccess;
  auto set = [&](GemvFn fn) {
    const cudaError_t e = ensure_smem_attr(device, fn, m);
    if (first == cudaSuccess) first = e;
  };
  for (int fmt : fmts)
    for (int mode = MODE_F32X; mode <= MODE_Q8K; mode++) {
      if (mode == MODE_Q8K && fmt == Q8_0) continue;
      for (int r = 1; r <= 2; r++) {
        set(pick<false>(fmt, mode, r));
        set(pick<true>(fmt, mode, r));
        if (fmt != Q8_0 && mode == MODE_Q8K) {
          for (int mma = 1; mma <= 2; mma++) {
            if (mma == 2 && fmt != Q6K) continue;
            set(pick<false>(fmt, mode, r, mma));
            set(pick<true>(fmt, mode, r, mma));
          }
        }
      }
    }
  for (int am = 0; am < 2; am++) {
    const GemvFn lean[3] = {lean_plan<Q4K, 16, 32>(am, m).fn, lean_plan<Q6K, 16, 16>(am, m).fn,
                            lean_plan<Q6K, 48, 16, kQ6Chunk>(am, m).fn};
    for (GemvFn fn : lean)
      if (fn) set(fn);
  }
  return first;
}

int32_t gemv_reserve(unltd_ctx ctx, const unltd_weight_s &w, int mode) {
  if (w.dtype == F32 || w.dim_out == 0) return UNLTD_OK;
  const int nspans = w.dtype == Q8_0 ? (int)((w.nb + 7) / 8) : (int)w.nb;
  const size_t img_bytes = (size_t)nspans * img_stride(w.dtype, mode);
  if (ctx->scratch_bytes >= img_bytes) return UNLTD_OK;
  if (ctx->scratch_fixed)  // a fixed array the context does not own: never freed or grown
    return set_error(UNLTD_ERR_UNSUPPORTED, "gemv: x image larger than the fixed scratch");
  if (ctx->scratch) cudaFree(ctx->scratch);
  ctx->scratch = nullptr;
  ctx->scratch_bytes = 0;
  cudaError_t e = cudaMalloc(&ctx->scratch, img_bytes);
  if (e != cudaSuccess) return cuda_error(e, "scratch alloc");
  ctx->scratch_bytes = img_bytes;
  return UNLTD_OK;
}

// Tile plan of a quantized GEMV: rows per tile T (R rows per work item),
// stages S, shared-memory layout, grid. S < 2: the row does not fit.
struct Plan {
  int nbu, img_bytes, rows, R, T, S, stage_bytes, cbuf, pstride, mma, rs, smem, grid, threads, niw;
};

Plan plan_gemv(unltd_ctx ctx, const unltd_weight_s &w, int mode) {
  const int fmt = w.dtype;
  const int nspans = fmt == Q8_0 ? (int)((w.nb + 7) / 8) : (int)w.nb;
  const int nbu = nspans;
  const int img_bytes = nspans * img_stride(fmt, mode);

  // ---- tiling: rows per tile T, stages S, shared-memory plan ----
  const int rows = (int)w.dim_out;
  const int stride = (int)w.row_stride;
  const int smem_max = max_smem_optin(ctx->device) - 1024;
  const int rs = mode == MODE_F32X ? (nbu | 1) : 8 * (nbu | 1);  // floats per chain row
  auto cbuf_for = [&](int T) {
    int f = mode == MODE_F32X ? T * rs : T * rs + T * (rs / 8);
    return (int)round_up((size_t)f * 4, 128);
  };
  // Pick rows per tile T: stages of at most 56 KB, at least 2 (preferably 3+)
  // stages in flight, and (T/R) * nbu items a multiple of the 64 subgroups so
  // the integer phase is balanced; then the largest such T.
  int R = 1, T = 0, S = 0, stage_bytes = 0, cbuf = 0, pstride = stride, mma = 0;
  double best_score = -1.0;
  const int nsub = kConsumerWarps * 4;
  // Q4_K / Q6_K Q8K: tensor-core tiles of 16 rows; rows padded in shared
  // memory so the eight rows of an MMA fragment load from distinct banks (a
  // stride of 32 mod 128 bytes for the 8-byte Q4_K loads, 16 for the 4-byte
  // Q6_K loads)
  if ((fmt == Q4K || fmt == Q6K) && mode == MODE_Q8K && !mma) {
    const int ps = (int)round_up((size_t)stride, 128) + (fmt == Q4K ? 32 : 16);
    // 32-row tiles (two MMA row groups per block item) measured faster than
    // 16-row tiles with deeper rings; Q6_K rows too long for two 16-row
    // stages take 8-row tiles (half-height MMA items)
    for (int t = fmt == Q6K ? 8 : 16; t <= 32; t *= 2) {
      const int sb = (int)round_up((size_t)t * ps, 128);
      const int cb = cbuf_for(t);
      const int fixed = kTcBarBytes + img_bytes + 2 * cb;
      const int s = std::min(kMaxStages, (smem_max - fixed) / sb);
      if (s < 2) continue;
      const int items = (t < 16 ? 1 : t / 16) * nbu;
      const double score = (items % kTcIntWarps == 0 ? 2.0 : 0.0) + (items >= kTcIntWarps ? 1.0 : 0.0) + t / 16.0 -
                           (t < 16 ? 4.0 : 0.0);
      if (score > best_score) {
        best_score = score;
        T = t;
        R = 2;
        S = s;
        stage_bytes = sb;
        cbuf = cb;
        pstride = ps;
        mma = t < 16 ? 2 : 1;
      }
    }
  }
  for (int t = 1; t <= 32 && !mma; t++) {
    const int r = t >= 2 ? 2 : 1;
    if (t % r) continue;
    const int sb = (int)round_up((size_t)t * stride, 128);
    if (sb > 56 * 1024 && t > 1) continue;
    const int cb = cbuf_for(t);
    const int fixed = kBarBytes + img_bytes + 2 * cb;
    const int s = std::min(kMaxStages, (smem_max - fixed) / sb);
    if (s < 2) continue;
    const int items = (t / r) * nbu;
    const double score = (s >= 3 ? 4.0 : 0.0) + (items % nsub == 0 ? 2.0 : 0.0) + (items >= nsub ? 1.0 : 0.0) +
                         t / 64.0;
    if (score > best_score) {
      best_score = score;
      T = t;
      R = r;
      S = s;
      stage_bytes = sb;
      cbuf = cb;
    }
  }
  Plan p;
  p.nbu = nbu;
  p.img_bytes = img_bytes;
  p.rows = rows;
  p.R = R;
  p.T = T;
  p.S = S;
  p.stage_bytes = stage_bytes;
  p.cbuf = cbuf;
  p.pstride = pstride;
  p.mma = mma;
  p.rs = rs;
  p.smem = (mma ? kTcBarBytes : kBarBytes) + img_bytes + 2 * cbuf + S * stage_bytes;
  p.grid = T ? std::max(1, std::min(ctx->num_sms, (rows + T - 1) / T)) : 1;
  p.threads = mma ? kTcThreads : kGemvThreads;
  p.niw = kTcIntWarps;
  return p;
}

bool gemv_tc_eligible(unltd_ctx ctx, const unltd_weight_s &w, int mode) {
  if (w.dtype == F32 || w.dim_out == 0) return false;
  const Plan p = plan_gemv(ctx, w, mode);
  return p.S >= 2 && p.mma;
}

bool gemv_norm_fusable(unltd_ctx ctx, const unltd_weight_s &w, int mode) {
  if (w.dtype != Q4K || mode != MODE_Q8K || w.dim_out == 0) return false;
  const Plan p = plan_gemv(ctx, w, mode);
  return p.S >= 2 && p.mma && w.dim_in <= (size_t)kNormSpans * p.niw * 256;
}

int32_t gemv_launch(unltd_ctx ctx, const GemvArgs &a) {
  const unltd_weight_s &w = *a.w;
  cudaStream_t st = ctx->stream;
  const bool am = a.argmax_key != nullptr;
  if (w.dim_out == 0) return UNLTD_OK;

  if (w.dtype == F32) {
    if (am) {
      cudaError_t e = cudaMemsetAsync(a.argmax_key, 0, sizeof(unsigned long long), st);
      if (e == cudaSuccess) e = cudaMemsetAsync(a.argmax_done, 0, sizeof(unsigned), st);
      if (e != cudaSuccess) return cuda_error(e, "argmax reset");
    }
    const int rows = (int)w.dim_out;
    int grid = std::min((rows + 7) / 8, ctx->num_sms * 8);
    gemv_f32_kernel<<<grid, kThreads, 0, st>>>(w.dev, w.row_stride, (int)w.dim_in, rows, a.x, a.y,
                                               a.argmax_key, a.argmax_done, a.token);
    ctx->launches += 1;
    return cuda_error(cudaGetLastError(), "gemv_f32");
  }

  const int fmt = w.dtype, mode = a.mode;
  const bool fuse = a.norm != nullptr;
  if (fuse && (am || !gemv_norm_fusable(ctx, w, mode)))
    return set_error(UNLTD_ERR_INVALID_ARG, "gemv: RMSNorm fusion needs a tensor-core Q4_K Q8K GEMV without argmax");
  if (fuse) {
    const GemvNorm &g = *a.norm;
    const void *ptrs[6] = {g.a, g.b, g.r_out, g.w, g.img4_out, g.img6_out};
    for (const void *p : ptrs)
      if ((uintptr_t)p % 16) return set_error(UNLTD_ERR_INVALID_ARG, "gemv: fused RMSNorm pointers must be 16-byte aligned");
    if (!g.a || !g.w) return set_error(UNLTD_ERR_INVALID_ARG, "gemv: fused RMSNorm needs a and w");
  }
  const Plan pl = plan_gemv(ctx, w, mode);
  // a plain f32 x is quantized in the GEMV's own prologue (Q8_K images on the
  // tensor-core kernel, F32X images on the DP4A kernel), no prep launch. The
  // argmax state needs no reset there: the last CTA of every argmax GEMV
  // leaves it zero, and the context starts with it zero.
  const bool xpro = !a.img && !fuse && a.x && (uintptr_t)a.x % 16 == 0 &&
                    ((pl.mma && mode == MODE_Q8K) || (!pl.mma && mode == MODE_F32X));
  if (!a.img && !fuse && !xpro) {
    if (int32_t rc = gemv_reserve(ctx, w, mode)) return rc;
  }
  if (pl.S < 2)
    return set_error(UNLTD_ERR_UNSUPPORTED, "gemv: row too long for the shared-memory pipeline (dim_in too large)");
  const int nspans = pl.nbu, nbu = pl.nbu, img_bytes = pl.img_bytes, rows = pl.rows;
  const int R = pl.R, T = pl.T, S = pl.S, stage_bytes = pl.stage_bytes, cbuf = pl.cbuf, pstride = pl.pstride;
  const int mma = pl.mma, rs = pl.rs, smem = pl.smem, grid = pl.grid;

  // 1) prep (skipped when the caller's kernel already wrote the image, or
  // when the GEMV's own prologue quantizes a fused RMSNorm)
  unsigned long long *key = am ? a.argmax_key : nullptr;
  unsigned *done = am ? a.argmax_done : nullptr;
  cudaError_t e = cudaSuccess;
  if (a.img || fuse || xpro) {
  } else if (mode == MODE_F32X) {
    if (fmt == Q4K) prep_f32x<Q4K><<<nspans, kThreads, 0, st>>>(a.x, w.dim_in, ctx->scratch, key, done);
    else if (fmt == Q6K) prep_f32x<Q6K><<<nspans, kThreads, 0, st>>>(a.x, w.dim_in, ctx->scratch, key, done);
    else prep_f32x<Q8_0><<<nspans, kThreads, 0, st>>>(a.x, w.dim_in, ctx->scratch, key, done);
  } else {
    if (fmt == Q4K) prep_q8k<Q4K><<<nspans, kThreads, 0, st>>>(a.x, w.dim_in, ctx->scratch, key, done);
    else prep_q8k<Q6K><<<nspans, kThreads, 0, st>>>(a.x, w.dim_in, ctx->scratch, key, done);
  }
  if (!a.img && !fuse && !xpro) {
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, "gemv prep");
    ctx->launches += 1;
  }

  // 2) gemv, programmatic dependent launch: the shape-specialised kernel
  // when there is one for w, else the generic one of the plan
  GemvFn fn = am ? pick<true>(fmt, mode, R, mma) : pick<false>(fmt, mode, R, mma);
  int launch_smem = smem, launch_grid = grid, launch_threads = pl.threads, launch_S = S;
  if (pl.mma) {
    const LeanPlan lp = lean_for(ctx->device, w, mode, am);
    if (lp.fn && lp.img_bytes == img_bytes) {
      fn = lp.fn;
      launch_smem = lp.smem;
      launch_threads = lp.threads;
      launch_S = lp.S;
      launch_grid = std::max(1, std::min(ctx->num_sms, (rows + lp.T - 1) / lp.T));
    }
  }
  e = ensure_smem_attr(ctx->device, fn, launch_smem);
  if (e != cudaSuccess) return cuda_error(e, "gemv: shared-memory attribute");

  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  Params P;
  P.W = w.dev;
  P.stride = w.row_stride;
  P.nb = (int)w.nb;
  P.nbu = nbu;
  P.rows = rows;
  P.img = a.img ? a.img : ctx->scratch;
  P.img_bytes = img_bytes;
  P.y = a.y;
  P.key = a.argmax_key;
  P.done = a.argmax_done;
  P.token = a.token;
  P.key_out = a.key_out;
  P.row0 = a.argmax_row0;
  P.err = ctx->err;
  P.pstride = pstride;
  P.mma = mma;
  P.T = T;
  P.S = launch_S;
  P.stage_bytes = stage_bytes;
  P.rs = rs;
  P.cbuf_bytes = cbuf;
  P.norm_a = fuse ? a.norm->a : nullptr;
  P.norm_b = fuse ? a.norm->b : nullptr;
  P.norm_r = fuse ? a.norm->r_out : nullptr;
  P.norm_w = fuse ? a.norm->w : nullptr;
  P.norm_eps = fuse ? a.norm->eps : 0.0f;
  P.norm_img4 = fuse ? a.norm->img4_out : nullptr;
  P.norm_img6 = fuse ? a.norm->img6_out : nullptr;
  P.nn = fuse ? (int)w.dim_in : 0;
  P.xq = xpro ? a.x : nullptr;
  const bool send = a.peer_send, recv = fuse && a.norm->peer_recv;
  if ((send || recv) && (!pl.mma || am || !ctx->peer_ok || w.dim_out > kPeerMaxCount || w.dim_in > kPeerMaxCount))
    return set_error(UNLTD_ERR_INVALID_ARG, "gemv: the peer row-split sum needs a tensor-core GEMV and peer_import");
  for (int r = 0; r < kPeerMaxRanks; r++) P.peer_map[r] = static_cast<uint8_t *>(ctx->peer_map[r]);
  P.peer_ctr = ctx->peer_ctr;
  P.peer_done = ctx->peer_done;
  P.peer_rank = ctx->rank;
  P.peer_n = ctx->world;
  P.peer_send = send;
  P.peer_recv = recv;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(launch_grid);
  cfg.blockDim = dim3(launch_threads);
  cfg.dynamicSmemBytes = launch_smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, fn, P);
  if (e != cudaSuccess) return cuda_error(e, "gemv launch");
  ctx->launches += 1;
  return UNLTD_OK;
}

}  // namespace unltd
