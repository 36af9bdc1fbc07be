// Decode GEMV over packed Q4_K / Q6_K / Q8_0 rows, y = W.x, for one
// activation vector, plus the fused LM-head argmax.
//
// Each call runs two kernels on the context stream:
//  1. prep: x (f32) -> an "x image" per 256-element span, in the lane order
//     of the weight layout (unltd_internal.cuh). Mode F32X stores x as a
//     22-bit fixed-point integer per span split into three byte limbs (s8
//     hi, u8 mid, u8 lo) with a power-of-two scale; mode Q8K_EXACT stores
//     quantize_q8_k's output (quants.rs:250-290) bit for bit.
//  2. gemv: each warp owns R output rows; its four 8-lane subgroups walk
//     consecutive blocks of those rows, one 16-byte chunk of packed quants
//     per lane per row, and form exact integer dot products with DP4A
//     against the image held in shared memory. F32X combines the integer
//     limb sums in f32 per block; Q8K_EXACT reproduces the reference's
//     per-lane (e % 8) integer sums and then its sequential f32 epilogue
//     (quants.rs:343-358, 402-411) without FMA, block by block in order.
// The gemv kernel is launched with programmatic dependent launch so its
// CTAs become resident while prep runs; it waits (griddepcontrol.wait)
// before reading the image.
#include <algorithm>
#include <cstdio>
#include <mutex>
#include <utility>
#include <vector>

#include "unltd_host.h"
#include "unltd_internal.cuh"

namespace unltd {
namespace {

constexpr int kThreads = 256;

// ---------------------------------------------------------------- prep ----

// Block-wide reductions for the 256-thread prep kernels.
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
  int pos;
  if constexpr (FMT == Q4K) pos = q4_xpos(t);
  else if constexpr (FMT == Q6K) pos = q6_xpos(t);
  else pos = t;
  uint8_t *im = img + span * kImgF32X;
  im[pos] = (uint8_t)(xi >> 16);
  im[256 + pos] = (uint8_t)((xi >> 8) & 0xFF);
  im[512 + pos] = (uint8_t)(xi & 0xFF);
  if constexpr (FMT == Q4K) {
    // lane-half sums for the Q4_K min term: lane j = 2p + (k>=4), half = nibble group
    int p = t >> 6, half = (t >> 5) & 1, k = t & 7;
    atomicAdd(&hsum[2 * (2 * p + (k >> 2)) + half], xi);
  }
  __syncthreads();
  if (t == 0) *reinterpret_cast<float *>(im + kImgF32X_XS) = xs;
  if constexpr (FMT == Q4K) {
    if (t < 16) reinterpret_cast<float *>(im + kImgF32X_XSUM)[t] = (float)hsum[t] * xs;
  }
}

// Exact restatement of quantize_q8_k (quants.rs:250-290) for one span per CTA.
template <int FMT>
__global__ void __launch_bounds__(kThreads) prep_q8k(const float *__restrict__ x, size_t dim_in,
                                                     uint8_t *__restrict__ img,
                                                     unsigned long long *key, unsigned *done) {
  pdl_trigger();
  __shared__ float red_a[8];
  __shared__ int red_i[8];
  __shared__ int hsum[16];
  const int t = threadIdx.x;
  const size_t span = blockIdx.x;
  const size_t e = span * kQK + t;
  if (t < 16) hsum[t] = 0;
  if (key && span == 0 && t == 0) {
    *key = 0ull;
    *done = 0u;
  }
  float v = e < dim_in ? x[e] : 0.0f;
  // first strict argmax of |x|; NaN never wins (the reference's `ax > amax`)
  float a = fabsf(v);
  if (isnan(a)) a = -1.0f;
  int idx = t;
  for (int o = 16; o; o >>= 1) {
    float oa = __shfl_xor_sync(0xffffffffu, a, o);
    int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (oa > a || (oa == a && oi < idx)) {
      a = oa;
      idx = oi;
    }
  }
  if ((t & 31) == 0) {
    red_a[t >> 5] = a;
    red_i[t >> 5] = idx;
  }
  __syncthreads();
  float amax = red_a[0];
  int imax = red_i[0];
  for (int w = 1; w < 8; w++) {
    if (red_a[w] > amax || (red_a[w] == amax && red_i[w] < imax)) {
      amax = red_a[w];
      imax = red_i[w];
    }
  }
  int q = 0;
  float d = 0.0f;
  if (amax > 0.0f) {
    size_t em = span * kQK + imax;
    float mx = em < dim_in ? x[em] : 0.0f;
    float iscale = __fdiv_rn(-127.0f, mx);
    float prod = __fmul_rn(iscale, v);
    int ni = (__float_as_int(__fadd_rn(prod, 12582912.0f)) & 0x007fffff) - 0x00400000;
    q = ni < 127 ? ni : 127;
    d = __fdiv_rn(1.0f, iscale);
  }
  if constexpr (FMT == Q4K) {
    uint8_t *im = img + span * kImgQ8K4;
    im[q4_xpos(t)] = (uint8_t)(int8_t)q;
    int p = t >> 6, half = (t >> 5) & 1, k = t & 7;
    atomicAdd(&hsum[2 * (2 * p + (k >> 2)) + half], q);
    __syncthreads();
    if (t == 0) *reinterpret_cast<float *>(im + kImgQ8K4_D) = d;
    if (t < 16) reinterpret_cast<int *>(im + kImgQ8K4_BS)[t] = hsum[t];
  } else {
    // Q6_K: element -> (lane j, half hh, run position ipos); word w = (ipos%8)/2
    // holds run positions (2w, 2w+8 | 2w+1, 2w+9); masked copies A (bytes 0,1)
    // and B (bytes 2,3). Each element writes its byte into one copy and a zero
    // into the same byte of the other, so every byte is written once.
    uint8_t *im = img + span * kImgQ8K6;
    int h = t >> 7, pos = t & 127, hh = pos >> 6, c = pos & 63, u = c >> 4, ipos = c & 15;
    int j = 4 * h + u;
    int pic = q6_pic(ipos);
    int w = pic >> 2, bpos = pic & 3;
    int base = (((j * 2 + hh) * 4 + w) * 2) * 4;  // byte offset of word A
    int own = bpos < 2 ? 0 : 4;
    im[base + own + bpos] = (uint8_t)(int8_t)q;
    im[base + (4 - own) + bpos] = 0;
    if (t == 0) *reinterpret_cast<float *>(im + kImgQ8K6_D) = d;
  }
}

// ---------------------------------------------------------------- gemv ----

struct Params {
  const uint8_t *W;
  size_t stride;
  int nb;       // blocks per row (Q8_0: 32-element blocks)
  int nspans;   // 256-element spans
  int rows;
  const uint8_t *img;
  float *y;
  unsigned long long *key;
  unsigned *done;
  uint32_t *token;
};

__device__ __forceinline__ float warp_sum(float v) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ unsigned long long argmax_key(float v, int row) {
  if (isnan(v)) return row == 0 ? ~0ull : 0ull;
  return ((unsigned long long)orderable(v) << 32) | (0xffffffffu - (uint32_t)row);
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
  int sh = (p & 1) * 16;
  sc_lo = (SC >> sh) & 0xFF;
  sc_hi = (SC >> (sh + 8)) & 0xFF;
  m_lo = (MM >> sh) & 0xFF;
  m_hi = (MM >> (sh + 8)) & 0xFF;
}

// Q6_K: four words of 4*(raw6 - 32) as s8 from ql/qh words (shift of the
// 2-bit field in qh: s for the low-nibble half, s+4 for the high half).
__device__ __forceinline__ uint32_t q6_a4_lo(uint32_t ql, uint32_t qh, int sl) {
  return (((ql << 2) & 0x3C3C3C3Cu) | ((qh << (6 - sl)) & 0xC0C0C0C0u)) ^ 0x80808080u;
}
__device__ __forceinline__ uint32_t q6_a4_hi(uint32_t ql, uint32_t qh, int sl) {
  return (((ql >> 2) & 0x3C3C3C3Cu) | ((qh << (2 - sl)) & 0xC0C0C0C0u)) ^ 0x80808080u;
}

template <int FMT, int MODE, int R, bool ARGMAX>
__global__ void __launch_bounds__(kThreads) gemv_kernel(Params P) {
  extern __shared__ uint4 smem4[];
  const uint8_t *simg = reinterpret_cast<const uint8_t *>(smem4);
  constexpr int ISTR = (MODE == MODE_F32X) ? kImgF32X : (FMT == Q4K ? kImgQ8K4 : kImgQ8K6);

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int s = lane >> 3, j = lane & 7;
  const int ntasks = (P.rows + R - 1) / R;
  const int gw = blockIdx.x * (kThreads / 32) + warp, nw = gridDim.x * (kThreads / 32);

  pdl_wait();
  {
    const uint4 *src = reinterpret_cast<const uint4 *>(P.img);
    uint4 *dst = smem4;
    const int n16 = P.nspans * ISTR / 16;
    for (int i = threadIdx.x; i < n16; i += kThreads) dst[i] = src[i];
  }
  __syncthreads();

  unsigned long long best = 0ull;
  const int nsteps = (FMT == Q8_0) ? (P.nspans + 3) / 4 : (P.nb + 3) / 4;

  for (int task = gw; task < ntasks; task += nw) {
    const int row0 = task * R;
    const uint8_t *Wr[R];
#pragma unroll
    for (int r = 0; r < R; r++) Wr[r] = P.W + (size_t)min(row0 + r, P.rows - 1) * P.stride;

    if constexpr (MODE == MODE_F32X) {
      float acc[R];
#pragma unroll
      for (int r = 0; r < R; r++) acc[r] = 0.0f;
      for (int st = 0; st < nsteps; st++) {
        if constexpr (FMT == Q4K) {
          const int b = 4 * st + s;
          if (b < P.nb) {
            const int p = j >> 1, kh = j & 1;
            const uint8_t *im = simg + b * kImgF32X;
            const int o_lo = 64 * p + 16 * kh, o_hi = o_lo + 32;
            const uint4 xh0 = *reinterpret_cast<const uint4 *>(im + o_lo);
            const uint4 xh1 = *reinterpret_cast<const uint4 *>(im + o_hi);
            const uint4 xm0 = *reinterpret_cast<const uint4 *>(im + 256 + o_lo);
            const uint4 xm1 = *reinterpret_cast<const uint4 *>(im + 256 + o_hi);
            const uint4 xl0 = *reinterpret_cast<const uint4 *>(im + 512 + o_lo);
            const uint4 xl1 = *reinterpret_cast<const uint4 *>(im + 512 + o_hi);
            const float xs = *reinterpret_cast<const float *>(im + kImgF32X_XS);
            const float xsl = reinterpret_cast<const float *>(im + kImgF32X_XSUM)[2 * j];
            const float xsh = reinterpret_cast<const float *>(im + kImgF32X_XSUM)[2 * j + 1];
            uint4 hq[R], q[R];
#pragma unroll
            for (int r = 0; r < R; r++) {
              hq[r] = __ldg(reinterpret_cast<const uint4 *>(Wr[r] + b * 16));
              q[r] = ldg_stream(Wr[r] + (size_t)P.nb * 16 + b * 128 + 32 * p + 16 * kh);
            }
#pragma unroll
            for (int r = 0; r < R; r++) {
              int sc_lo, sc_hi, m_lo, m_hi;
              q4_scales(hq[r], p, sc_lo, sc_hi, m_lo, m_hi);
              const uint32_t w[4] = {q[r].x, q[r].y, q[r].z, q[r].w};
              const uint32_t xh_lo[4] = {xh0.x, xh0.y, xh0.z, xh0.w}, xh_hi[4] = {xh1.x, xh1.y, xh1.z, xh1.w};
              const uint32_t xm_lo[4] = {xm0.x, xm0.y, xm0.z, xm0.w}, xm_hi[4] = {xm1.x, xm1.y, xm1.z, xm1.w};
              const uint32_t xl_lo[4] = {xl0.x, xl0.y, xl0.z, xl0.w}, xl_hi[4] = {xl1.x, xl1.y, xl1.z, xl1.w};
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
              const float d = h2f_bits(hq[r].x & 0xFFFFu), dmin = h2f_bits(hq[r].x >> 16);
              const float M = fmaf((float)m_lo, xsl, (float)m_hi * xsh);
              acc[r] = fmaf(d * xs, F, acc[r]);
              acc[r] = fmaf(-dmin, M, acc[r]);
            }
          }
        } else if constexpr (FMT == Q6K) {
          const int b = 4 * st + s;
          if (b < P.nb) {
            const int h = j >> 2, u = j & 3, sl = 2 * (u >> 1);
            const uint8_t *im = simg + b * kImgF32X;
            const int o_lo = 32 * j, o_hi = o_lo + 16;
            const uint4 xh0 = *reinterpret_cast<const uint4 *>(im + o_lo);
            const uint4 xh1 = *reinterpret_cast<const uint4 *>(im + o_hi);
            const uint4 xm0 = *reinterpret_cast<const uint4 *>(im + 256 + o_lo);
            const uint4 xm1 = *reinterpret_cast<const uint4 *>(im + 256 + o_hi);
            const uint4 xl0 = *reinterpret_cast<const uint4 *>(im + 512 + o_lo);
            const uint4 xl1 = *reinterpret_cast<const uint4 *>(im + 512 + o_hi);
            const float xs = *reinterpret_cast<const float *>(im + kImgF32X_XS);
            uint4 ql[R], qh[R];
            int sc_lo[R], sc_hi[R];
            uint32_t dbits[R];
#pragma unroll
            for (int r = 0; r < R; r++) {
              ql[r] = ldg_stream(Wr[r] + b * 128 + 16 * j);
              qh[r] = ldg_stream(Wr[r] + (size_t)P.nb * 128 + b * 64 + 16 * (2 * h + (u & 1)));
              const int8_t *scp = reinterpret_cast<const int8_t *>(Wr[r] + (size_t)P.nb * 192 + b * 16);
              sc_lo[r] = __ldg(scp + 8 * h + u);
              sc_hi[r] = __ldg(scp + 8 * h + 4 + u);
              dbits[r] = __ldg(reinterpret_cast<const unsigned short *>(Wr[r] + (size_t)P.nb * 208 + b * 2));
            }
#pragma unroll
            for (int r = 0; r < R; r++) {
              const uint32_t wl[4] = {ql[r].x, ql[r].y, ql[r].z, ql[r].w};
              const uint32_t wh[4] = {qh[r].x, qh[r].y, qh[r].z, qh[r].w};
              const uint32_t xh_lo[4] = {xh0.x, xh0.y, xh0.z, xh0.w}, xh_hi[4] = {xh1.x, xh1.y, xh1.z, xh1.w};
              const uint32_t xm_lo[4] = {xm0.x, xm0.y, xm0.z, xm0.w}, xm_hi[4] = {xm1.x, xm1.y, xm1.z, xm1.w};
              const uint32_t xl_lo[4] = {xl0.x, xl0.y, xl0.z, xl0.w}, xl_hi[4] = {xl1.x, xl1.y, xl1.z, xl1.w};
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
              const int ah = sc_lo[r] * shl + sc_hi[r] * shh;
              const int am = sc_lo[r] * sml + sc_hi[r] * smh;
              const int al = sc_lo[r] * sll + sc_hi[r] * slh;
              const float F = fmaf((float)ah, 65536.0f, fmaf((float)am, 256.0f, (float)al));
              const float d = h2f_bits(dbits[r]);
              acc[r] = fmaf(d * xs * 0.25f, F, acc[r]);
            }
          }
        } else {  // Q8_0: 8 lanes = 8 blocks of 32 in a 256-span
          const int span = 4 * st + s;
          const int b32 = 8 * span + j;
          if (b32 < P.nb) {
            const uint8_t *im = simg + span * kImgF32X;
            const int o = 32 * j;
            const uint4 xh0 = *reinterpret_cast<const uint4 *>(im + o);
            const uint4 xh1 = *reinterpret_cast<const uint4 *>(im + o + 16);
            const uint4 xm0 = *reinterpret_cast<const uint4 *>(im + 256 + o);
            const uint4 xm1 = *reinterpret_cast<const uint4 *>(im + 256 + o + 16);
            const uint4 xl0 = *reinterpret_cast<const uint4 *>(im + 512 + o);
            const uint4 xl1 = *reinterpret_cast<const uint4 *>(im + 512 + o + 16);
            const float xs = *reinterpret_cast<const float *>(im + kImgF32X_XS);
            uint4 q0[R], q1[R];
            uint32_t dbits[R];
#pragma unroll
            for (int r = 0; r < R; r++) {
              q0[r] = ldg_stream(Wr[r] + (size_t)b32 * 32);
              q1[r] = ldg_stream(Wr[r] + (size_t)b32 * 32 + 16);
              dbits[r] = __ldg(reinterpret_cast<const unsigned short *>(Wr[r] + (size_t)P.nb * 32 + b32 * 2));
            }
#pragma unroll
            for (int r = 0; r < R; r++) {
              const uint32_t w[8] = {q0[r].x, q0[r].y, q0[r].z, q0[r].w, q1[r].x, q1[r].y, q1[r].z, q1[r].w};
              const uint32_t xh[8] = {xh0.x, xh0.y, xh0.z, xh0.w, xh1.x, xh1.y, xh1.z, xh1.w};
              const uint32_t xm[8] = {xm0.x, xm0.y, xm0.z, xm0.w, xm1.x, xm1.y, xm1.z, xm1.w};
              const uint32_t xl[8] = {xl0.x, xl0.y, xl0.z, xl0.w, xl1.x, xl1.y, xl1.z, xl1.w};
              int sh = 0, sm = 0, sll = 0;
#pragma unroll
              for (int t = 0; t < 8; t++) {
                sh = dp4a_ss(w[t], xh[t], sh);
                sm = dp4a_su(w[t], xm[t], sm);
                sll = dp4a_su(w[t], xl[t], sll);
              }
              const float F = fmaf((float)sh, 65536.0f, fmaf((float)sm, 256.0f, (float)sll));
              acc[r] = fmaf(h2f_bits(dbits[r]) * xs, F, acc[r]);
            }
          }
        }
      }
#pragma unroll
      for (int r = 0; r < R; r++) {
        const float v = warp_sum(acc[r]);
        const int row = row0 + r;
        if (row < P.rows) {
          if (lane == 0 && P.y) P.y[row] = v;
          if (ARGMAX) {
            const unsigned long long k = argmax_key(v, row);
            best = k > best ? k : best;
          }
        }
      }
    } else {  // MODE_Q8K: bit-exact with gemv_quant_q8k
      float sums[R], sumf[R];
#pragma unroll
      for (int r = 0; r < R; r++) {
        sums[r] = 0.0f;
        sumf[r] = 0.0f;
      }
      for (int st = 0; st < nsteps; st++) {
        const int b = 4 * st + s;
        const bool valid = b < P.nb;
        const int bb = valid ? b : P.nb - 1;  // clamp loads; results masked below
        const uint8_t *im = simg + bb * ISTR;
        const float xd = *reinterpret_cast<const float *>(im + (FMT == Q4K ? kImgQ8K4_D : kImgQ8K6_D));
        float tk[R], tm[R];
        if constexpr (FMT == Q4K) {
          const int p = j >> 1, kh = j & 1;
          const uint4 q80 = *reinterpret_cast<const uint4 *>(im + 64 * p + 16 * kh);
          const uint4 q81 = *reinterpret_cast<const uint4 *>(im + 64 * p + 32 + 16 * kh);
          const int bs_lo = reinterpret_cast<const int *>(im + kImgQ8K4_BS)[2 * j];
          const int bs_hi = reinterpret_cast<const int *>(im + kImgQ8K4_BS)[2 * j + 1];
          uint4 hq[R], q[R];
#pragma unroll
          for (int r = 0; r < R; r++) {
            hq[r] = __ldg(reinterpret_cast<const uint4 *>(Wr[r] + bb * 16));
            q[r] = ldg_stream(Wr[r] + (size_t)P.nb * 16 + bb * 128 + 32 * p + 16 * kh);
          }
#pragma unroll
          for (int r = 0; r < R; r++) {
            int sc_lo, sc_hi, m_lo, m_hi;
            q4_scales(hq[r], p, sc_lo, sc_hi, m_lo, m_hi);
            const uint32_t w[4] = {q[r].x, q[r].y, q[r].z, q[r].w};
            const uint32_t qa[4] = {q80.x, q80.y, q80.z, q80.w}, qb[4] = {q81.x, q81.y, q81.z, q81.w};
            int P4[4];
#pragma unroll
            for (int t = 0; t < 4; t++) {
              const uint32_t lo = w[t] & 0x0F0F0F0Fu, hi = (w[t] >> 4) & 0x0F0F0F0Fu;
              P4[t] = sc_lo * dp4a_us(lo, qa[t], 0) + sc_hi * dp4a_us(hi, qb[t], 0);
            }
            int msum = m_lo * bs_lo + m_hi * bs_hi;
            // reduce over the four lanes sharing kh (lane bits 1, 2): recursive halving
            const bool b2 = (j >> 2) & 1, b1 = (j >> 1) & 1;
            int k0 = b2 ? P4[2] : P4[0], k1 = b2 ? P4[3] : P4[1];
            const int s0 = b2 ? P4[0] : P4[2], s1 = b2 ? P4[1] : P4[3];
            k0 += __shfl_xor_sync(0xffffffffu, s0, 4);
            k1 += __shfl_xor_sync(0xffffffffu, s1, 4);
            int keep = b1 ? k1 : k0;
            const int send = b1 ? k0 : k1;
            keep += __shfl_xor_sync(0xffffffffu, send, 2);
            msum += __shfl_xor_sync(0xffffffffu, msum, 4);
            msum += __shfl_xor_sync(0xffffffffu, msum, 2);
            msum += __shfl_xor_sync(0xffffffffu, msum, 1);
            const float d = __fmul_rn(xd, h2f_bits(hq[r].x & 0xFFFFu));   // q8.d * f16(d)
            const float dm = __fmul_rn(h2f_bits(hq[r].x >> 16), xd);      // f16(dmin) * q8.d
            tk[r] = __fmul_rn(d, (float)keep);
            tm[r] = __fmul_rn(dm, (float)msum);
          }
        } else {  // Q6K
          const int h = j >> 2, u = j & 3, sl = 2 * (u >> 1);
          const uint4 *qw = reinterpret_cast<const uint4 *>(im + j * 64);
          const uint4 A0 = qw[0], A1 = qw[1], B0 = qw[2], B1 = qw[3];  // (A,B) word pairs, halves 0/1
          const uint32_t qA_lo[4] = {A0.x, A0.z, A1.x, A1.z}, qB_lo[4] = {A0.y, A0.w, A1.y, A1.w};
          const uint32_t qA_hi[4] = {B0.x, B0.z, B1.x, B1.z}, qB_hi[4] = {B0.y, B0.w, B1.y, B1.w};
          uint4 ql[R], qh[R];
          int sc_lo[R], sc_hi[R];
          uint32_t dbits[R];
#pragma unroll
          for (int r = 0; r < R; r++) {
            ql[r] = ldg_stream(Wr[r] + bb * 128 + 16 * j);
            qh[r] = ldg_stream(Wr[r] + (size_t)P.nb * 128 + bb * 64 + 16 * (2 * h + (u & 1)));
            const int8_t *scp = reinterpret_cast<const int8_t *>(Wr[r] + (size_t)P.nb * 192 + bb * 16);
            sc_lo[r] = __ldg(scp + 8 * h + u);
            sc_hi[r] = __ldg(scp + 8 * h + 4 + u);
            dbits[r] = __ldg(reinterpret_cast<const unsigned short *>(Wr[r] + (size_t)P.nb * 208 + bb * 2));
          }
#pragma unroll
          for (int r = 0; r < R; r++) {
            const uint32_t wl[4] = {ql[r].x, ql[r].y, ql[r].z, ql[r].w};
            const uint32_t wh[4] = {qh[r].x, qh[r].y, qh[r].z, qh[r].w};
            int P4[8];
#pragma unroll
            for (int t = 0; t < 4; t++) {
              const uint32_t lo = q6_a4_lo(wl[t], wh[t], sl), hi = q6_a4_hi(wl[t], wh[t], sl);
              P4[2 * t] = sc_lo[r] * dp4a_ss(lo, qA_lo[t], 0) + sc_hi[r] * dp4a_ss(hi, qA_hi[t], 0);
              P4[2 * t + 1] = sc_lo[r] * dp4a_ss(lo, qB_lo[t], 0) + sc_hi[r] * dp4a_ss(hi, qB_hi[t], 0);
            }
            // reduce-scatter over the 8 lanes: lane j ends with class k = j
            const bool b2 = (j >> 2) & 1, b1 = (j >> 1) & 1, b0 = j & 1;
            int v4[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
              const int keepv = b2 ? P4[4 + i] : P4[i];
              const int sendv = b2 ? P4[i] : P4[4 + i];
              v4[i] = keepv + __shfl_xor_sync(0xffffffffu, sendv, 4);
            }
            int v2[2];
#pragma unroll
            for (int i = 0; i < 2; i++) {
              const int keepv = b1 ? v4[2 + i] : v4[i];
              const int sendv = b1 ? v4[i] : v4[2 + i];
              v2[i] = keepv + __shfl_xor_sync(0xffffffffu, sendv, 2);
            }
            const int keepv = b0 ? v2[1] : v2[0];
            const int sendv = b0 ? v2[0] : v2[1];
            const int sumi = (keepv + __shfl_xor_sync(0xffffffffu, sendv, 1)) >> 2;
            const float d = __fmul_rn(xd, h2f_bits(dbits[r]));
            tk[r] = __fmul_rn(d, (float)sumi);
            tm[r] = 0.0f;
          }
        }
        // sequential per-block epilogue, blocks 4*st .. 4*st+3 in order
#pragma unroll
        for (int sp = 0; sp < 4; sp++) {
          const bool ok = 4 * st + sp < P.nb;
#pragma unroll
          for (int r = 0; r < R; r++) {
            const float a = __shfl_sync(0xffffffffu, tk[r], 8 * sp + j);
            const float m = __shfl_sync(0xffffffffu, tm[r], 8 * sp + j);
            if (ok) {
              sums[r] = __fadd_rn(sums[r], a);
              if (FMT == Q4K) sumf[r] = __fsub_rn(sumf[r], m);
            }
          }
        }
        (void)valid;
      }
      // s = sumf + sums[0] + ... + sums[7] (Q6_K: sumf = 0)
#pragma unroll
      for (int r = 0; r < R; r++) {
        float acc = sumf[r];
#pragma unroll
        for (int k = 0; k < 8; k++) {
          int src;
          if (FMT == Q4K) src = ((k >> 2) & 1) + 4 * ((k >> 1) & 1) + 2 * (k & 1);
          else src = k;
          acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, sums[r], src));
        }
        const int row = row0 + r;
        if (row < P.rows) {
          if (lane == 0 && P.y) P.y[row] = acc;
          if (ARGMAX) {
            const unsigned long long k = argmax_key(acc, row);
            best = k > best ? k : best;
          }
        }
      }
    }
  }

  if constexpr (ARGMAX) {
    __shared__ unsigned long long cta_best[kThreads / 32];
    if (lane == 0) cta_best[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long b = cta_best[0];
      for (int i = 1; i < kThreads / 32; i++) b = cta_best[i] > b ? cta_best[i] : b;
      atomicMax(P.key, b);
      __threadfence();
      const unsigned prev = atomicAdd(P.done, 1u);
      if (prev == gridDim.x - 1) {
        __threadfence();
        const unsigned long long k = atomicAdd(P.key, 0ull);
        *P.token = 0xffffffffu - (uint32_t)(k & 0xffffffffull);
        *P.key = 0ull;
        *P.done = 0u;
      }
    }
  }
}

// Plain f32 weights (gemv_quant's F32 case): one warp per row, f32 FMA.
__global__ void __launch_bounds__(kThreads) gemv_f32_kernel(const uint8_t *__restrict__ W, size_t stride,
                                                            int dim_in, int rows, const float *__restrict__ x,
                                                            float *__restrict__ y,
                                                            unsigned long long *key, unsigned *done,
                                                            uint32_t *token) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gw = blockIdx.x * (kThreads / 32) + warp, nw = gridDim.x * (kThreads / 32);
  unsigned long long best = 0ull;
  if (key && blockIdx.x == 0 && threadIdx.x == 0) {
    // reset is done by the host memset before launch
  }
  for (int row = gw; row < rows; row += nw) {
    const float *wr = reinterpret_cast<const float *>(W + (size_t)row * stride);
    float acc = 0.0f;
    for (int i = lane; i < dim_in; i += 32) acc = fmaf(wr[i], x[i], acc);
    acc = warp_sum(acc);
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
  switch (R) {
    case 1: return gemv_kernel<FMT, MODE, 1, AM>;
    case 2: return gemv_kernel<FMT, MODE, 2, AM>;
    default: return gemv_kernel<FMT, MODE, 4, AM>;
  }
}

template <bool AM>
GemvFn pick(int fmt, int mode, int R) {
  if (mode == MODE_F32X) {
    if (fmt == Q4K) return pick_r<Q4K, MODE_F32X, AM>(R);
    if (fmt == Q6K) return pick_r<Q6K, MODE_F32X, AM>(R);
    return pick_r<Q8_0, MODE_F32X, AM>(R);
  }
  if (fmt == Q4K) return pick_r<Q4K, MODE_Q8K, AM>(R);
  return pick_r<Q6K, MODE_Q8K, AM>(R);
}

int choose_r(int rows) {
  if (rows >= 32768) return 4;
  if (rows >= 8192) return 2;
  return 1;
}

struct OccKey {
  GemvFn fn;
  int smem;
  bool operator==(const OccKey &o) const { return fn == o.fn && smem == o.smem; }
};

int blocks_per_sm(GemvFn fn, int smem) {
  static std::mutex mu;
  static std::vector<std::pair<OccKey, int>> cache;
  std::lock_guard<std::mutex> lk(mu);
  for (auto &e : cache)
    if (e.first == OccKey{fn, smem}) return e.second;
  if (smem > 48 * 1024) cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, kThreads, smem) != cudaSuccess || n < 1) n = 1;
  cache.push_back({OccKey{fn, smem}, n});
  return n;
}

}  // namespace

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
  const int nspans = fmt == Q8_0 ? (int)((w.nb + 7) / 8) : (int)w.nb;
  const int istr = img_stride(fmt, mode);
  const size_t img_bytes = (size_t)nspans * istr;
  if (img_bytes > 200 * 1024)
    return set_error(UNLTD_ERR_UNSUPPORTED, "gemv: dim_in too large for the shared-memory x image (max 61440 for F32X)");
  if (ctx->scratch_bytes < img_bytes) {
    if (ctx->scratch) cudaFree(ctx->scratch);
    ctx->scratch = nullptr;
    ctx->scratch_bytes = 0;
    cudaError_t e = cudaMalloc(&ctx->scratch, img_bytes);
    if (e != cudaSuccess) return cuda_error(e, "scratch alloc");
    ctx->scratch_bytes = img_bytes;
  }

  // 1) prep
  unsigned long long *key = am ? a.argmax_key : nullptr;
  unsigned *done = am ? a.argmax_done : nullptr;
  if (mode == MODE_F32X) {
    if (fmt == Q4K) prep_f32x<Q4K><<<nspans, kThreads, 0, st>>>(a.x, w.dim_in, ctx->scratch, key, done);
    else if (fmt == Q6K) prep_f32x<Q6K><<<nspans, kThreads, 0, st>>>(a.x, w.dim_in, ctx->scratch, key, done);
    else prep_f32x<Q8_0><<<nspans, kThreads, 0, st>>>(a.x, w.dim_in, ctx->scratch, key, done);
  } else {
    if (fmt == Q4K) prep_q8k<Q4K><<<nspans, kThreads, 0, st>>>(a.x, w.dim_in, ctx->scratch, key, done);
    else prep_q8k<Q6K><<<nspans, kThreads, 0, st>>>(a.x, w.dim_in, ctx->scratch, key, done);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "gemv prep");
  ctx->launches += 1;

  // 2) gemv, programmatic dependent launch
  const int rows = (int)w.dim_out;
  const int R = choose_r(rows);
  GemvFn fn = am ? pick<true>(fmt, mode, R) : pick<false>(fmt, mode, R);
  const int smem = (int)img_bytes;
  const int bps = blocks_per_sm(fn, smem);
  const int tasks = (rows + R - 1) / R;
  const int grid = std::max(1, std::min((tasks + 7) / 8, ctx->num_sms * bps));

  Params P;
  P.W = w.dev;
  P.stride = w.row_stride;
  P.nb = (int)w.nb;
  P.nspans = nspans;
  P.rows = rows;
  P.img = ctx->scratch;
  P.y = a.y;
  P.key = a.argmax_key;
  P.done = a.argmax_done;
  P.token = a.token;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, fn, P);
  if (e != cudaSuccess) return cuda_error(e, "gemv launch");
  ctx->launches += 1;
  return UNLTD_OK;
}

}  // namespace unltd
