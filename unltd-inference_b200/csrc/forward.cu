// Greedy decode step of the Qwen3.5-style hybrid model on one GPU: the f32
// kernels between the quantized projections, and the model/session runner
// that chains them with the Q8_K-exact GEMVs of gemv.cu into one CUDA graph
// per token.
//
// Follows crates/unltd-generation/src/qwen35_forward.rs (step 295-330,
// recr_layer 333-543, attn_layer 546-710, ffn 713-768), the LM head of
// min_forward.rs:210-266 and greedy.rs:18-27. Every f32/f64 operation of the
// reference is reproduced in the same order with explicit round-to-nearest
// intrinsics (no contraction), so the hidden states match the reference's
// bit for bit, with one stated exception: f32 exp/log are the correctly
// rounded values (computed through double precision), where the reference
// inherits its platform libm's last bit.
//
// Sequential f64 sums (rmsnorm, l2_norm_rows, the attention value sum) are
// evaluated in parallel and resolved exactly: the reference's left-to-right
// sum and the parallel sum both lie within (n-1)*2^-53*sum|t| of the exact
// sum, so when every value within twice that bound rounds to the same f32
// result, that result is the reference's; otherwise (rare: the interval
// straddles an f32 rounding boundary) one thread recomputes the sum
// left-to-right.
#include <cmath>
#include <cstring>
#include <type_traits>
#include <map>
#include <string>
#include <vector>

#include "q8k_span.cuh"
#include "unltd_host.h"
#include "unltd_internal.cuh"

namespace unltd {
namespace {

[[maybe_unused]] constexpr int kErrTimeout = 1;
constexpr int kErrToken = 2;

// ---- scalar functions (kernels.rs:198-226, 174-182) ----------------------
__device__ __forceinline__ float exp_cr(float x) { return (float)exp((double)x); }
__device__ __forceinline__ float log_cr(float x) { return (float)log((double)x); }
__device__ __forceinline__ float sigmoid_f(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_cr(-x))); }
__device__ __forceinline__ float silu_f(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, exp_cr(-x))); }
__device__ __forceinline__ float softplus_f(float x) {
  return x > 20.0f ? x : log_cr(__fadd_rn(1.0f, exp_cr(x)));
}

// ---- batch of sequences ---------------------------------------------------
// A session of n_seq sequences keeps every per-sequence buffer in its own
// arena; the arenas are ss bytes apart, so sequence z's copy of a buffer is
// the pointer of sequence 0 plus z * ss. Kernels take the sequence from
// blockIdx.z (grids are at most 2-D otherwise).
template <class T>
__device__ __forceinline__ T *seq_ptr(T *p, size_t off) {
  return p ? reinterpret_cast<T *>(reinterpret_cast<uintptr_t>(p) + off) : p;
}
__device__ __forceinline__ size_t seq_off(size_t ss) { return (size_t)blockIdx.z * ss; }
// A batch session's producers write the batched x images (shared by the
// sequences, kBImgBlock per span and group of 8 sequences): the block of
// this CTA's sequence (seq0 + blockIdx.z; a prefill launches the per-token
// kernels one token at a time with seq0 = the token) for `span`, or null
// without a batched image.
__device__ __forceinline__ uint8_t *seq_bimg(uint8_t *bimg, int nsg, int seq0, int span) {
  return bimg ? bimg + bimg_block((size_t)span, (int)((seq0 + blockIdx.z) >> 3), nsg) : nullptr;
}
__device__ __forceinline__ int seq_sl(int seq0) { return (int)((seq0 + blockIdx.z) & 7); }

// ---- reductions -----------------------------------------------------------
// Sum of a and b over the block; every thread receives the same values.
template <int NT>
__device__ __forceinline__ void block_sum2(double &a, double &b, double *red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    a += __shfl_xor_sync(~0u, a, o);
    b += __shfl_xor_sync(~0u, b, o);
  }
  constexpr int NW = NT / 32;
  if constexpr (NW > 1) {
    const int w = threadIdx.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) {
      red[w] = a;
      red[NW + w] = b;
    }
    __syncthreads();
    a = 0.0;
    b = 0.0;
#pragma unroll
    for (int i = 0; i < NW; i++) {
      a += red[i];
      b += red[NW + i];
    }
  }
}

template <int NT>
__device__ __forceinline__ float block_max(float v, float *red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(~0u, v, o));
  constexpr int NW = NT / 32;
  if constexpr (NW > 1) {
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    v = red[0];
#pragma unroll
    for (int i = 1; i < NW; i++) v = fmaxf(v, red[i]);
  }
  return v;
}

// ---- RMSNorm (kernels.rs:61-78) fused with the Q8_K image of its output ---
// r = a (+ b); r_out = r (when non-null); xn = rmsnorm(r, w), quantized
// (quantize_q8_k) straight into the x images of the GEMVs that consume it.
// One CTA per 256-element span; each CTA sums all n squares itself.
struct NormArgs {
  const float *a, *b;
  float *r_out;
  const float *w;
  int n;
  float eps;
  uint8_t *img4, *img6;     // Q4_K / Q6_K image (either may be null)
  unsigned long long *key;  // non-null: reset the LM-head argmax state
  unsigned *done;
  size_t ss = 0;            // bytes between the sequences' arenas (a, b, r_out, images)
  size_t bss = 0;           // b's own stride when it is not in the arenas (0: ss)
  uint8_t *bimg = nullptr;  // batch session: the batched x images (then img4 = img6 = null)
  int nsg = 0;
};

__global__ void __launch_bounds__(256) norm_quant_kernel(NormArgs p) {
  pdl_trigger();
  __shared__ double red[16];
  __shared__ float s_mean;
  __shared__ Q8KSpanSmem sm;
  pdl_wait();
  {
    const size_t so = seq_off(p.ss);
    p.a = seq_ptr(p.a, so);
    p.b = seq_ptr(p.b, p.bss ? seq_off(p.bss) : so);
    p.r_out = seq_ptr(p.r_out, so);
    p.img4 = seq_ptr(p.img4, so);
    p.img6 = seq_ptr(p.img6, so);
  }
  const int t = threadIdx.x, span = blockIdx.x;
  auto R = [&](int i) { return p.b ? __fadd_rn(p.a[i], p.b[i]) : p.a[i]; };
  double S = 0.0, A = 0.0;
  // loads in batches of 8 per thread, all in flight before they are used
  for (int i0 = t; i0 < p.n; i0 += 8 * 256) {
    float ra[8], rb[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int i = i0 + u * 256;
      ra[u] = i < p.n ? p.a[i] : 0.0f;
      rb[u] = (i < p.n && p.b) ? p.b[i] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const float r = p.b ? __fadd_rn(ra[u], rb[u]) : ra[u];
      S += (double)__fmul_rn(r, r);
    }
  }
  block_sum2<256>(S, A, red);
  float mean;
  const MeanOf f{p.n};
  if (!resolve_sum(S, S, p.n, f, &mean)) {
    if (t == 0) {
      double s = 0.0;
#pragma unroll 1
      for (int i = 0; i < p.n; i++) {
        const float r = R(i);
        s = __dadd_rn(s, (double)__fmul_rn(r, r));
      }
      s_mean = f(s);
    }
    __syncthreads();
    mean = s_mean;
  }
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
  const int e = span * 256 + t;
  const float r = R(e);
  if (p.r_out) p.r_out[e] = r;
  const float xn = __fmul_rn(__fmul_rn(r, scale), p.w[e]);
  q8k_span_write(xn, p.img4 ? p.img4 + (size_t)span * kImgQ8K4 : nullptr,
                 p.img6 ? p.img6 + (size_t)span * kImgQ8K6 : nullptr, sm, seq_bimg(p.bimg, p.nsg, 0, span), seq_sl(0));
  if (p.key && span == 0 && t == 0) {
    *p.key = 0ull;
    *p.done = 0u;
  }
}

// ---- token embedding: one Q4_K row, dequantized (min_forward.rs:160-184) --
__global__ void embed_q4k_kernel(const uint8_t *table, size_t stride, size_t nb, const uint32_t *token,
                                 uint32_t vocab, float *x, int n, int *err, size_t ss, size_t tss) {
  pdl_trigger();
  pdl_wait();
  token = seq_ptr(token, seq_off(tss));
  x = seq_ptr(x, seq_off(ss));
  uint32_t t = *token;
  if (t >= vocab) {
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(err, kErrToken);
    t = 0;
  }
  const uint8_t *row = table + (size_t)t * stride;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < n; e += gridDim.x * blockDim.x)
    x[e] = q4k_row_elem(row, nb, (size_t)e);
}

// ---- SwiGLU (kernels.rs:174-182) fused with the Q8_K image of its output ---
__global__ void __launch_bounds__(256) swiglu_quant_kernel(const float *g, const float *u, uint8_t *img4,
                                                           uint8_t *img6, size_t ss, uint8_t *bimg, int nsg) {
  pdl_trigger();
  __shared__ Q8KSpanSmem sm;
  pdl_wait();
  g = seq_ptr(g, seq_off(ss));
  u = seq_ptr(u, seq_off(ss));
  img4 = seq_ptr(img4, seq_off(ss));
  img6 = seq_ptr(img6, seq_off(ss));
  const int span = blockIdx.x, e = span * 256 + threadIdx.x;
  const float t = g[e];
  const float s = __fdiv_rn(t, __fadd_rn(1.0f, exp_cr(-t)));
  q8k_span_write(__fmul_rn(s, u[e]), img4 ? img4 + (size_t)span * kImgQ8K4 : nullptr,
                 img6 ? img6 + (size_t)span * kImgQ8K6 : nullptr, sm, seq_bimg(bimg, nsg, 0, span), seq_sl(0));
}

// ---- recurrent layer between the projections (qwen35_forward.rs:390-508) --
struct RecrArgs {
  const float *proj;    // [qkv (dconv) | z (nv*HD) | beta_raw (nv) | alpha (nv)]
  float *ring;          // K slots x dconv; row tau of the window at slot (pos+tau) % K
  const float *convw;   // ssm_conv1d.weight as stored, [channel][tau]
  const float *dt_bias, *ssm_a, *ssm_norm;
  float *state;         // nv x HD x HD, state[h][i][j]
  float *y;             // nv*HD GDN output (before the gated norm)
  const int *pos;
  int K, nqk, nv, dconv, z_off, beta_off, alpha_off;
  float eps;
  // per 256-element span of y: CTAs done (the last one runs the gated norm
  // and writes the span's Q8_K image(s) of ssm_out's input, then resets it)
  unsigned *span_ctr;
  uint8_t *img4, *img6;
  size_t ss = 0;  // bytes between the sequences' arenas
  uint8_t *bimg = nullptr;  // batch session: the batched x images (then img4 = img6 = null)
  int nsg = 0, seq0 = 0;    // the image slot of this launch's sequence z is seq0 + z
};

// One CTA per (v-head h, quarter of its columns), one thread per channel of
// the head: the conv, silu and l2 norms of the head's q and k (recomputed by
// each quarter; the window update is written by quarter 0 only) and the
// head's beta/gate; then gdn_fused_step (kernels.rs:316-372) for the
// quarter's 32 state columns. Column j is touched only through the dots over
// i, so a thread owns a column: its two dots are the reference's sequential
// f64 sums. The quarter's state slice (HD x 32) is staged in shared memory.
// Output: the head's GDN output before the gated norm.
constexpr int kGdnCols = 32;

// One dot of gdn_fused_step, sum_i (double)(st_i * x_i) in the reference's
// left-to-right f64 order, rounded to f32: four lanes (w = 0..3) each sum RW
// consecutive terms in order, the chunks are combined in order and resolved
// with the running-error bound (see attn_combine_quant_kernel); when the
// bound cannot decide, the column's terms go through shared memory and lane
// w == 0 sums all of them left to right.
// q and k of a head in shared memory hold their four quarter chunks (HD / 4
// channels each) kChunkPad floats apart, so the four lanes of a state column
// (one chunk each) read different banks, with 128-bit loads
constexpr int kChunkPad = 8;
template <int HD>
__device__ __forceinline__ int chunk_at(int i) {
  return i + (i / (HD / 4)) * kChunkPad;
}

template <int RW, int XP = 0>  // XP: x holds its four chunks RW + XP floats apart
__device__ __forceinline__ float gdn_dot(const float (&st)[RW], const float *xw, const float *x, float *fb, int w) {
  double Sw = 0.0, Qw = 0.0;
#pragma unroll
  for (int ii = 0; ii < RW; ii++) {
    Sw = __dadd_rn(Sw, (double)__fmul_rn(st[ii], xw[ii]));
    Qw = __dadd_rn(Qw, fabs(Sw));
  }
  const int base = threadIdx.x & ~3;  // lane of chunk 0 of this column (same warp)
  double O = 0.0, T1 = 0.0, T2 = 0.0, T3 = 0.0;
#pragma unroll
  for (int c = 0; c < 4; c++) {
    const double Sc = __shfl_sync(~0u, Sw, (base + c) & 31), Qc = __shfl_sync(~0u, Qw, (base + c) & 31);
    T1 += Qc;
    T2 += (double)RW * fabs(O);
    O = __dadd_rn(O, Sc);
    T3 += fabs(O);
  }
  const double B = 0x1p-51 * (2.0 * T1 + T2 + T3);
  float r = (float)(O - B);
  const bool amb = r != (float)(O + B);
  if (__any_sync(~0u, amb)) {  // rare: sequential sum of the column's terms
    if (amb) {
#pragma unroll
      for (int ii = 0; ii < RW; ii++) fb[RW * w + ii] = st[ii];
    }
    __syncwarp();
    if (amb && w == 0) {
      double s = 0.0;
#pragma unroll 1
      for (int i = 0; i < 4 * RW; i++) s = __dadd_rn(s, (double)__fmul_rn(fb[i], x[i + (i / RW) * XP]));
      fb[0] = (float)s;
    }
    __syncwarp();
    if (amb) r = fb[0];
    __syncwarp();
  }
  return r;
}

// The gated norm of the recurrent output (qwen35_forward.rs:482-498) for one
// 256-element span of y (two heads of HD = 128), by the CTA that completed
// the span: per head rmsnorm with ssm_norm (the reference's f64 sum of
// squares, resolved exactly), times silu(z), then the span's Q8_K image(s)
// (quantize_q8_k) by warp 0. Thread j takes column j of both heads.
template <int HD>
__device__ __noinline__ void gated_norm_span(const float *y, const float *z, const float *ssm_norm, float eps,
                                             uint8_t *img4, uint8_t *img6, int span, uint8_t *imb, int sl) {
  static_assert(HD == 128, "a span holds two heads of 128");
  __shared__ double red2[2][HD / 32];
  __shared__ float so[256];
  __shared__ float s_mean2[2];
  const int j = threadIdx.x, lane = j & 31, wp = j >> 5;
  const size_t e0 = (size_t)span * 256;
  float x[2];
  double S[2];
#pragma unroll
  for (int hh = 0; hh < 2; hh++) {
    x[hh] = __ldcg(y + e0 + hh * HD + j);  // written by other CTAs of this grid
    so[hh * HD + j] = x[hh];
    S[hh] = (double)__fmul_rn(x[hh], x[hh]);
#pragma unroll
    for (int off = 16; off; off >>= 1) S[hh] += __shfl_xor_sync(~0u, S[hh], off);
    if (lane == 0) red2[hh][wp] = S[hh];
  }
  __syncthreads();
  const MeanOf f{HD};
  float mean[2];
  bool ok[2];
#pragma unroll
  for (int hh = 0; hh < 2; hh++) {
    S[hh] = 0.0;
#pragma unroll
    for (int w = 0; w < HD / 32; w++) S[hh] += red2[hh][w];
    ok[hh] = resolve_sum(S[hh], S[hh], HD, f, &mean[hh]);  // uniform over the CTA
  }
  if (!ok[0] || !ok[1]) {
    if (j < 2 && !ok[j]) {  // rare: the reference's left-to-right sum
      double q = 0.0;
#pragma unroll 1
      for (int i = 0; i < HD; i++) q = __dadd_rn(q, (double)__fmul_rn(so[j * HD + i], so[j * HD + i]));
      s_mean2[j] = f(q);
    }
    __syncthreads();
    if (!ok[0]) mean[0] = s_mean2[0];
    if (!ok[1]) mean[1] = s_mean2[1];
  }
  __syncthreads();  // so[] is overwritten below
  const float wj = ssm_norm[j];
#pragma unroll
  for (int hh = 0; hh < 2; hh++) {
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean[hh], eps)));
    const float yn = __fmul_rn(__fmul_rn(x[hh], scale), wj);
    so[hh * HD + j] = __fmul_rn(yn, silu_f(z[e0 + hh * HD + j]));
  }
  __syncthreads();
  if (wp == 0) {
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; k++) v[k] = so[8 * lane + k];
    q8k_span_write_warp(v, lane, img4 ? img4 + (size_t)span * kImgQ8K4 : nullptr,
                        img6 ? img6 + (size_t)span * kImgQ8K6 : nullptr, imb, sl);
  }
}

template <int HD, int KT>  // KT: conv_kernel known at compile time (0: a.K at run time)
__global__ void __launch_bounds__(HD) recr_mid_kernel(RecrArgs a) {
  pdl_trigger();
  __shared__ __align__(16) float qs[HD + 4 * kChunkPad], ks[HD + 4 * kChunkPad];  // chunk_at layout
  __shared__ float gdn_fb[kGdnCols * HD];  // fallback of gdn_dot: one column's terms
  __shared__ double red[2 * HD / 32];
  __shared__ float s_f[2];
  pdl_wait();
  {
    const size_t so = seq_off(a.ss);
    a.proj = seq_ptr(a.proj, so);
    a.ring = seq_ptr(a.ring, so);
    a.state = seq_ptr(a.state, so);
    a.y = seq_ptr(a.y, so);
    a.pos = seq_ptr(a.pos, so);
    a.span_ctr = seq_ptr(a.span_ctr, so);
    a.img4 = seq_ptr(a.img4, so);
    a.img6 = seq_ptr(a.img6, so);
  }
  const int h = blockIdx.x, quarter = blockIdx.y, j = threadIdx.x;
  const int qk = h % a.nqk;  // periodic qk-head of v-head h (qwen35_forward.rs:464)
  const int pos = *a.pos, K = a.K;
  const int c0 = quarter * kGdnCols;
  const int chq = qk * HD + j, chk = a.nqk * HD + qk * HD + j;
  // this thread's state chunk: column c0 + j/4, rows [RW w, RW w + RW); loaded
  // first so the loads overlap the conv and norms
  const int jc = j >> 2, w = j & 3;
  constexpr int RW = HD / 4;
  float *S = a.state + (size_t)h * HD * HD + c0 + jc;
  float st[RW];
#pragma unroll
  for (int ii = 0; ii < RW; ii++) st[ii] = S[(size_t)(RW * w + ii) * HD];

  // the head's beta/alpha inputs, loaded with everything else
  const float beta_raw = a.proj[a.beta_off + h], alpha = a.proj[a.alpha_off + h];
  const float dtb = a.dt_bias[h], ssa = a.ssm_a[h];

  // depthwise conv over [window rows, current qkv] (kernels.rs:265-310), silu
  const int chv = 2 * a.nqk * HD + h * HD + c0 + (j & (kGdnCols - 1));
  float q, k, v = 0.0f;
  if constexpr (KT > 0) {
    // every ring slot is loaded (no wait on pos for the addresses), then the
    // window is taken in slot order (pos + tau) % K
    float xr[3][KT], wr[3][KT], cur[3];
    const int chs[3] = {chq, chk, chv};
#pragma unroll
    for (int c = 0; c < 3; c++) {
#pragma unroll
      for (int sl = 0; sl < KT; sl++) {
        xr[c][sl] = a.ring[(size_t)sl * a.dconv + chs[c]];
        wr[c][sl] = a.convw[(size_t)chs[c] * KT + sl];
      }
      cur[c] = a.proj[chs[c]];
    }
    float r3[3];
#pragma unroll
    for (int c = 0; c < 3; c++) {
      float sacc = 0.0f;
#pragma unroll
      for (int tau = 0; tau < KT; tau++) {
        float xv = cur[c];
        if (tau < KT - 1) {
          const int sl = (pos + tau) % KT;
#pragma unroll
          for (int u = 0; u < KT; u++)
            if (u == sl) xv = xr[c][u];
        }
        sacc = __fadd_rn(sacc, __fmul_rn(xv, wr[c][tau]));
      }
      r3[c] = sacc;
    }
    q = silu_f(r3[0]);
    k = silu_f(r3[1]);
    if (j < kGdnCols) v = silu_f(r3[2]);
  } else {
    auto conv = [&](int ch) {
      float sacc = 0.0f;
      for (int tau = 0; tau < K; tau++) {
        const float xv = tau < K - 1 ? a.ring[(size_t)((pos + tau) % K) * a.dconv + ch] : a.proj[ch];
        sacc = __fadd_rn(sacc, __fmul_rn(xv, a.convw[(size_t)ch * K + tau]));
      }
      return sacc;
    };
    q = silu_f(conv(chq));
    k = silu_f(conv(chk));
    if (j < kGdnCols) v = silu_f(conv(chv));
  }
  // the current row enters the window: it becomes row K-2 of the next step
  const size_t ws = (size_t)((pos + K - 1) % K) * a.dconv;
  // (all slots were loaded above; slot ws is not part of this window, and
  // only its owner CTA rewrites a channel's slot, after its own loads)
  if (j < kGdnCols) a.ring[ws + chv] = a.proj[chv];
  if (h < a.nqk && quarter == 0) {
    a.ring[ws + chq] = a.proj[chq];
    a.ring[ws + chk] = a.proj[chk];
  }

  // l2_norm_rows of q and k (kernels.rs:236-252)
  const int jp = chunk_at<HD>(j);
  qs[jp] = q;
  ks[jp] = k;
  double Sq = (double)__fmul_rn(q, q), Sk = (double)__fmul_rn(k, k);
  block_sum2<HD>(Sq, Sk, red);
  float fq, fk;
  const bool okq = resolve_sum(Sq, Sq, HD, ToF32{}, &fq);
  const bool okk = resolve_sum(Sk, Sk, HD, ToF32{}, &fk);
  if (!okq || !okk) {
    __syncthreads();
    if (j < 2 && !(j == 0 ? okq : okk)) {
      const float *src = j == 0 ? qs : ks;
      double s = 0.0;
#pragma unroll 1
      for (int i = 0; i < HD; i++) {
        const float xi = src[chunk_at<HD>(i)];
        s = __dadd_rn(s, (double)__fmul_rn(xi, xi));
      }
      s_f[j] = (float)s;
    }
    __syncthreads();
    if (!okq) fq = s_f[0];
    if (!okk) fk = s_f[1];
  }
  q = __fmul_rn(q, __fdiv_rn(1.0f, fmaxf(__fsqrt_rn(fq), a.eps)));
  k = __fmul_rn(k, __fdiv_rn(1.0f, fmaxf(__fsqrt_rn(fk), a.eps)));
  __syncthreads();
  qs[jp] = q;
  ks[jp] = k;

  // beta = sigmoid(beta_raw); gate = softplus(alpha + dt_bias) * ssm_a
  const float beta = sigmoid_f(beta_raw);
  const float gate = __fmul_rn(softplus_f(__fadd_rn(alpha, dtb)), ssa);
  const float g = exp_cr(gate);
  // v of the column this thread works on (computed above by threads j < 32)
  __shared__ float vs[kGdnCols];
  if (j < kGdnCols) vs[j] = v;
  __syncthreads();

  // gdn_fused_step: column jc = c0 + j/4; rows [32w, 32w+32) in registers,
  // w = j % 4. Each dot over i is evaluated as four in-order chunk sums whose
  // combination is resolved exactly (gdn_dot); the four lanes of a column
  // hold the same results.
  float kx[RW], qx[RW];  // this lane's chunk of k, then of q (128-bit loads)
#pragma unroll
  for (int ii = 0; ii < RW; ii += 4)
    *reinterpret_cast<float4 *>(&kx[ii]) = *reinterpret_cast<const float4 *>(ks + chunk_at<HD>(RW * w) + ii);
#pragma unroll
  for (int ii = 0; ii < RW; ii++) st[ii] = __fmul_rn(st[ii], g);
  const float dk = gdn_dot<RW, kChunkPad>(st, kx, ks, gdn_fb + jc * HD, w);
  const float d = __fmul_rn(__fsub_rn(vs[jc], dk), beta);
#pragma unroll
  for (int ii = 0; ii < RW; ii++) st[ii] = __fadd_rn(st[ii], __fmul_rn(kx[ii], d));
#pragma unroll
  for (int ii = 0; ii < RW; ii += 4)
    *reinterpret_cast<float4 *>(&qx[ii]) = *reinterpret_cast<const float4 *>(qs + chunk_at<HD>(RW * w) + ii);
  const float dq = gdn_dot<RW, kChunkPad>(st, qx, qs, gdn_fb + jc * HD, w);
  if (w == 0) a.y[h * HD + c0 + jc] = __fmul_rn(dq, __fdiv_rn(1.0f, __fsqrt_rn((float)HD)));
#pragma unroll
  for (int ii = 0; ii < RW; ii++) S[(size_t)(RW * w + ii) * HD] = st[ii];

  // the last of the CTAs writing this 256-element span of y (its 256 / HD
  // heads x the quarters) runs the gated norm of the span: y is published by
  // a fence before the count, read after it (no waiting on other CTAs)
  __shared__ unsigned s_last;
  const int span = (h * HD) >> 8;
  __threadfence();
  __syncthreads();
  if (j == 0) {
    const unsigned n = (256 / HD) * gridDim.y;
    const unsigned prev = atomicAdd(a.span_ctr + span, 1u);
    s_last = prev == n - 1;
    if (prev == n - 1) a.span_ctr[span] = 0u;  // every CTA of the span has counted
  }
  __syncthreads();
  if (s_last) {
    __threadfence();
    gated_norm_span<HD>(a.y, a.proj + a.z_off, a.ssm_norm, a.eps, a.img4, a.img6, span,
                        seq_bimg(a.bimg, a.nsg, a.seq0, span), seq_sl(a.seq0));
  }
}

// The recurrent layer for a prefill chunk of T tokens in one launch, with
// the operations of recr_mid_kernel per token. Each CTA (v-head h, quarter of
// its columns) works in two phases:
//  A. what does not depend on the GDN state, for every token at once (warp
//     w takes tokens w, w + 4, ...): the conv (the window rows of earlier
//     chunk tokens from their projections, pss bytes apart, older rows from
//     the ring, which this kernel does not write), silu, the l2 norms of q
//     and k (warp sums resolved exactly as in block_sum2 + resolve_sum),
//     beta and the gate, into shared memory;
//  B. the state recurrence token by token: each warp owns eight columns of
//     the state slice (registers), so the loop needs no block barrier;
//     y of token t goes to its activations.
// The gated norm of every (span, token) runs afterwards (prefill_gnorm_kernel)
// and the ring is updated after that (prefill_ring_kernel).
struct RecrChunkArgs {
  RecrArgs r;   // r.proj / r.y: token 0's; r.pos: the session's position (the chunk's first)
  size_t pss;   // bytes between consecutive tokens' activations
  int T;
};

constexpr int kChunkTok = 32;  // tokens of a prefill chunk (kPrefillLanes)

template <int HD>
struct RecrChunkSmem {
  static constexpr int kRow = HD + 4 * kChunkPad;
  static __device__ __forceinline__ int at(int i) { return chunk_at<HD>(i); }
  float q[kChunkTok][kRow], k[kChunkTok][kRow], v[kChunkTok][kGdnCols];
  float beta[kChunkTok], g[kChunkTok];
};

template <int HD, int KT>  // KT: conv_kernel known at compile time (0: c.r.K at run time)
__global__ void __launch_bounds__(HD) recr_chunk_kernel(RecrChunkArgs c) {
  static_assert(HD == 128, "four warps, four channels per lane");
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t csm[];
  RecrChunkSmem<HD> &sm = *reinterpret_cast<RecrChunkSmem<HD> *>(csm);
  __shared__ float gdn_fb[kGdnCols * HD];
  pdl_wait();
  const RecrArgs &a = c.r;
  const int h = blockIdx.x, quarter = blockIdx.y, j = threadIdx.x;
  const int warp = j >> 5, lane = j & 31;
  const int qk = h % a.nqk;
  const int pos0 = *a.pos, K = KT > 0 ? KT : a.K;
  const int c0 = quarter * kGdnCols;
  constexpr int RW = HD / 4;
  const int jc = j >> 2, w = j & 3;
  float *S = a.state + (size_t)h * HD * HD + c0 + jc;
  float st[RW];
#pragma unroll
  for (int ii = 0; ii < RW; ii++) st[ii] = S[(size_t)(RW * w + ii) * HD];
  const float dtb = a.dt_bias[h], ssa = a.ssm_a[h];
  auto proj_of = [&](int t) {
    return reinterpret_cast<const float *>(reinterpret_cast<const uint8_t *>(a.proj) + (size_t)t * c.pss);
  };

  // ---- A0: the chunk's q, k, v channels of this CTA into shared memory
  // (independent loads, column j by thread j); beta and the gate of token
  // t by thread t ----
  const int chq0 = qk * HD, chk0 = a.nqk * HD + qk * HD, chv0 = 2 * a.nqk * HD + h * HD + c0;
  using Sm = RecrChunkSmem<HD>;
  const int jp = Sm::at(j);
#pragma unroll 4
  for (int t = 0; t < c.T; t++) {
    const float *pr = proj_of(t);
    sm.q[t][jp] = pr[chq0 + j];
    sm.k[t][jp] = pr[chk0 + j];
    if (j < kGdnCols) sm.v[t][j] = pr[chv0 + j];
  }
  if (j < c.T) {
    const float *pr = proj_of(j);
    const float beta_raw = pr[a.beta_off + h], alpha = pr[a.alpha_off + h];
    sm.beta[j] = sigmoid_f(beta_raw);
    sm.g[j] = exp_cr(__fmul_rn(softplus_f(__fadd_rn(alpha, dtb)), ssa));
  }
  // ---- A1: depthwise conv over [window rows, current qkv] (kernels.rs:265-310)
  // and silu, in place: thread j owns column j, tokens in descending order, so
  // the rows token t reads (its own and the K-1 before it, or the ring's for
  // positions before the chunk) are still the raw projections ----
  {
    // NC columns of one stride at once, four tokens per pass: the loads of a
    // pass precede its stores, and its 4 x NC silu are independent
    auto conv_cols = [&](auto ncs, float *const *col, int stride, const int *ch) {
      constexpr int NC = decltype(ncs)::value;
      [[maybe_unused]] float wr[NC][KT > 0 ? KT : 1];  // KT == 0: the weights are read per tap
      if constexpr (KT > 0) {
#pragma unroll
        for (int n = 0; n < NC; n++)
#pragma unroll
          for (int tau = 0; tau < KT; tau++) wr[n][tau] = a.convw[(size_t)ch[n] * KT + tau];
      }
#pragma unroll 1
      for (int t0 = c.T - 1; t0 >= 0; t0 -= 4) {
        float r[4][NC];
#pragma unroll
        for (int u = 0; u < 4; u++) {
          const int t = t0 - u, pos = pos0 + t;
#pragma unroll
          for (int n = 0; n < NC; n++) {
            float sacc = 0.0f;
            if (t >= 0) {
              if constexpr (KT > 0) {
#pragma unroll
                for (int tau = 0; tau < KT; tau++) {
                  const int qp = pos - (KT - 1) + tau;  // the row's position
                  const float xv = qp >= pos0 ? col[n][(qp - pos0) * stride]
                                              : a.ring[(size_t)((pos + tau) % KT) * a.dconv + ch[n]];
                  sacc = __fadd_rn(sacc, __fmul_rn(xv, wr[n][tau]));
                }
              } else {
                for (int tau = 0; tau < K; tau++) {
                  const int qp = pos - (K - 1) + tau;
                  const float xv = qp >= pos0 ? col[n][(qp - pos0) * stride]
                                              : a.ring[(size_t)((pos + tau) % K) * a.dconv + ch[n]];
                  sacc = __fadd_rn(sacc, __fmul_rn(xv, a.convw[(size_t)ch[n] * K + tau]));
                }
              }
            }
            r[u][n] = sacc;
          }
        }
#pragma unroll
        for (int u = 0; u < 4; u++)
#pragma unroll
          for (int n = 0; n < NC; n++)
            if (t0 - u >= 0) col[n][(t0 - u) * stride] = silu_f(r[u][n]);
      }
    };
    {
      float *const cols[2] = {&sm.q[0][jp], &sm.k[0][jp]};
      const int chs[2] = {chq0 + j, chk0 + j};
      conv_cols(std::integral_constant<int, 2>{}, cols, Sm::kRow, chs);
    }
    if (j < kGdnCols) {
      float *const cols[1] = {&sm.v[0][j]};
      const int chs[1] = {chv0 + j};
      conv_cols(std::integral_constant<int, 1>{}, cols, kGdnCols, chs);
    }
  }
  __syncthreads();
  // ---- A2: l2_norm_rows of q and k (kernels.rs:236-252): warp w takes tokens
  // w, w + 4, ...; the sums of squares resolved exactly; rare ambiguity: lane 0
  // sums the squares left to right ----
  for (int t = warp; t < c.T; t += 4) {
    float q[4], k[4];
    double Sq = 0.0, Sk = 0.0;
#pragma unroll
    for (int m = 0; m < 4; m++) {
      q[m] = sm.q[t][Sm::at(lane + 32 * m)];
      k[m] = sm.k[t][Sm::at(lane + 32 * m)];
      Sq += (double)__fmul_rn(q[m], q[m]);
      Sk += (double)__fmul_rn(k[m], k[m]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      Sq += __shfl_xor_sync(~0u, Sq, o);
      Sk += __shfl_xor_sync(~0u, Sk, o);
    }
    float fq, fk;
    const bool okq = resolve_sum(Sq, Sq, HD, ToF32{}, &fq);
    const bool okk = resolve_sum(Sk, Sk, HD, ToF32{}, &fk);
    if (!okq || !okk) {
      float f2[2] = {fq, fk};
      if (lane == 0) {
        for (int which = 0; which < 2; which++) {
          if (which == 0 ? okq : okk) continue;
          const float *src = which == 0 ? sm.q[t] : sm.k[t];
          double s2 = 0.0;
#pragma unroll 1
          for (int i = 0; i < HD; i++) s2 = __dadd_rn(s2, (double)__fmul_rn(src[Sm::at(i)], src[Sm::at(i)]));
          f2[which] = (float)s2;
        }
      }
      fq = __shfl_sync(~0u, f2[0], 0);
      fk = __shfl_sync(~0u, f2[1], 0);
    }
    const float iq = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn(fq), a.eps));
    const float ik = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn(fk), a.eps));
    __syncwarp();
#pragma unroll
    for (int m = 0; m < 4; m++) {
      sm.q[t][Sm::at(lane + 32 * m)] = __fmul_rn(q[m], iq);
      sm.k[t][Sm::at(lane + 32 * m)] = __fmul_rn(k[m], ik);
    }
  }
  __syncthreads();

  // ---- B: gdn_fused_step token by token (as recr_mid_kernel) ----
#pragma unroll 1
  for (int t = 0; t < c.T; t++) {
    const float g = sm.g[t], beta = sm.beta[t];
    const float *ks = sm.k[t], *qs = sm.q[t];
    float kx[RW], qx[RW];  // this lane's chunk of k, then of q (128-bit loads)
#pragma unroll
    for (int ii = 0; ii < RW; ii += 4)
      *reinterpret_cast<float4 *>(&kx[ii]) = *reinterpret_cast<const float4 *>(ks + Sm::at(RW * w) + ii);
#pragma unroll
    for (int ii = 0; ii < RW; ii++) st[ii] = __fmul_rn(st[ii], g);
    const float dk = gdn_dot<RW, kChunkPad>(st, kx, ks, gdn_fb + jc * HD, w);
    const float d = __fmul_rn(__fsub_rn(sm.v[t][jc], dk), beta);
#pragma unroll
    for (int ii = 0; ii < RW; ii++) st[ii] = __fadd_rn(st[ii], __fmul_rn(kx[ii], d));
#pragma unroll
    for (int ii = 0; ii < RW; ii += 4)
      *reinterpret_cast<float4 *>(&qx[ii]) = *reinterpret_cast<const float4 *>(qs + Sm::at(RW * w) + ii);
    const float dq = gdn_dot<RW, kChunkPad>(st, qx, qs, gdn_fb + jc * HD, w);
    float *yt = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(a.y) + (size_t)t * c.pss);
    if (w == 0) yt[h * HD + c0 + jc] = __fmul_rn(dq, __fdiv_rn(1.0f, __fsqrt_rn((float)HD)));
  }
#pragma unroll
  for (int ii = 0; ii < RW; ii++) S[(size_t)(RW * w + ii) * HD] = st[ii];
}

// The gated norm of the recurrent output and its Q8_K image, for every
// (span, token) of a prefill chunk (grid spans x T; gated_norm_span).
template <int HD>
__global__ void __launch_bounds__(HD) prefill_gnorm_kernel(const float *y, const float *proj, size_t pss, int z_off,
                                                           const float *ssm_norm, float eps, uint8_t *bimg, int nsg) {
  pdl_trigger();
  pdl_wait();
  const int span = blockIdx.x, t = blockIdx.y;
  const float *yt = reinterpret_cast<const float *>(reinterpret_cast<const uint8_t *>(y) + (size_t)t * pss);
  const float *pr = reinterpret_cast<const float *>(reinterpret_cast<const uint8_t *>(proj) + (size_t)t * pss);
  gated_norm_span<HD>(yt, pr + z_off, ssm_norm, eps, nullptr, nullptr, span,
                      bimg + bimg_block((size_t)span, t >> 3, nsg), t & 7);
}

// The conv windows after a prefill chunk: the chunk's last K positions'
// qkv rows, each in its ring slot (pos + K - 1) % K, as the one-token steps
// leave them. One thread per (position, channel).
__global__ void prefill_ring_kernel(const float *proj, size_t pss, int T, float *ring, int dconv, int K,
                                    const int *pos) {
  pdl_trigger();
  pdl_wait();
  const int t0 = max(0, T - K), nrow = T - t0;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nrow * dconv) return;
  const int t = t0 + i / dconv, ch = i % dconv;
  const float *pr = reinterpret_cast<const float *>(reinterpret_cast<const uint8_t *>(proj) + (size_t)t * pss);
  ring[(size_t)((*pos + t + K - 1) % K) * dconv + ch] = pr[ch];
}

// ---- full-attention layer (qwen35_forward.rs:584-686) ----------------------
constexpr int kChunk = 64;    // positions per value-pass CTA
constexpr int kMaxGroup = 8;  // q heads per kv head

struct AttnArgs {
  const float *qk;      // [qfull (nh x 2HDV: q | gate per head) | k (nkv x HDV)]
  const float *v;       // nkv x HDV
  const float *q_norm, *k_norm;
  const double2 *rope;  // [ctx][nrp] (cos, sin) of the rotated pairs
  float *q;             // nh x HDV, normed and rotated
  float *kcache, *vcache;  // ctx x (nkv*HDV)
  float *scores;        // nh x ctx: scores, then softmax weights in place
  double2 *part;        // nh x nsplit x HDV: per-chunk (sum, sum |running sum|)
  uint8_t *img4, *img6; // x image(s) of attn_output's input
  const int *pos;
  int nh, nkv, n_rot, nrp, ctx, nsplit;
  float eps, kq_scale;
  size_t ss = 0;     // bytes between the sequences' arenas
  size_t kv_ss = 0;  // the same for the caches (0: a prefill chunk's tokens share one cache)
  uint8_t *bimg = nullptr;  // batch session: the batched x images (then img4 = img6 = null)
  int nsg = 0, seq0 = 0;    // the image slot of this launch's sequence z is seq0 + z
};

// This CTA's sequence's copies of the per-sequence buffers.
__device__ __forceinline__ void attn_at_seq(AttnArgs &a) {
  const size_t so = seq_off(a.ss);
  a.qk = seq_ptr(a.qk, so);
  a.v = seq_ptr(a.v, so);
  a.q = seq_ptr(a.q, so);
  a.kcache = seq_ptr(a.kcache, seq_off(a.kv_ss));
  a.vcache = seq_ptr(a.vcache, seq_off(a.kv_ss));
  a.scores = seq_ptr(a.scores, so);
  a.part = seq_ptr(a.part, so);
  a.img4 = seq_ptr(a.img4, so);
  a.img6 = seq_ptr(a.img6, so);
  a.pos = seq_ptr(a.pos, so);
}

// q/k head norms, IMROPE (kernels.rs:381-400) and the cache write. One CTA
// per q head and per kv head.
template <int HDV>
__global__ void __launch_bounds__(HDV) attn_pre_kernel(AttnArgs a) {
  pdl_trigger();
  __shared__ double red[2 * HDV / 32];
  __shared__ float sx[HDV];
  __shared__ float s_mean;
  pdl_wait();
  attn_at_seq(a);
  const int b = blockIdx.x, j = threadIdx.x;
  const bool isq = b < a.nh;
  const int hh = isq ? b : b - a.nh;
  const int pos = *a.pos;
  const float *src = isq ? a.qk + (size_t)hh * 2 * HDV : a.qk + (size_t)a.nh * 2 * HDV + (size_t)hh * HDV;
  const float *wn = isq ? a.q_norm : a.k_norm;
  const float x = src[j];
  sx[j] = x;
  double S = (double)__fmul_rn(x, x), dummy = 0.0;
  block_sum2<HDV>(S, dummy, red);
  float mean;
  const MeanOf f{HDV};
  if (!resolve_sum(S, S, HDV, f, &mean)) {
    __syncthreads();
    if (j == 0) {
      double s = 0.0;
#pragma unroll 1
      for (int i = 0; i < HDV; i++) s = __dadd_rn(s, (double)__fmul_rn(sx[i], sx[i]));
      s_mean = f(s);
    }
    __syncthreads();
    mean = s_mean;
  }
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
  const float xn = __fmul_rn(__fmul_rn(x, scale), wn[j]);
  __syncthreads();
  sx[j] = xn;
  __syncthreads();
  float out = xn;
  const int half = a.n_rot / 2;
  if (j < a.n_rot) {
    const int ic = j < half ? j : j - half;
    if (ic % 3 == 0) {
      const double2 cs = a.rope[(size_t)pos * a.nrp + ic / 3];
      const double x0 = sx[ic], x1 = sx[ic + half];
      out = j < half ? (float)fma(cs.x, x0, -__dmul_rn(cs.y, x1)) : (float)fma(cs.y, x0, __dmul_rn(cs.x, x1));
    }
  }
  const size_t kvlen = (size_t)a.nkv * HDV;
  if (isq) {
    a.q[(size_t)hh * HDV + j] = out;
  } else {
    a.kcache[(size_t)pos * kvlen + (size_t)hh * HDV + j] = out;
    a.vcache[(size_t)pos * kvlen + (size_t)hh * HDV + j] = a.v[(size_t)hh * HDV + j];
  }
}

// Across-lane part of the pairwise tree for L scores held by every lane
// (v[i]: this lane's subtree sum of score i): levels pair lanes xor 1, 2, 4,
// 8, 16 in that order, exactly as the tree pairs (2j, 2j+1) of the previous
// level. While a lane holds more than one score it keeps half of them and
// sends the other half to its partner (recursive halving): 5 levels cost
// L - 1 + (5 - log2 L) f64 exchanges instead of 5 L. Returns the full sum of
// score `idx`; lanes < L hold distinct scores.
template <int LEN, int B>
__device__ __forceinline__ void tree_level(double (&v)[16], int lane, int &base) {
  if constexpr (B < 5) {
    constexpr int m = 1 << B;
    const bool hi = (lane & m) != 0;
    if constexpr (LEN > 1) {
      constexpr int half = LEN / 2;
#pragma unroll
      for (int i = 0; i < half; i++) {
        const double send = hi ? v[i] : v[half + i];
        const double keep = hi ? v[half + i] : v[i];
        v[i] = __dadd_rn(keep, __shfl_xor_sync(~0u, send, m));
      }
      if (hi) base += half;
      tree_level<half, B + 1>(v, lane, base);
    } else {
      v[0] = __dadd_rn(v[0], __shfl_xor_sync(~0u, v[0], m));
      tree_level<1, B + 1>(v, lane, base);
    }
  }
}

template <int L>
__device__ __forceinline__ double tree_reduce_lanes(double (&v)[16], int lane, int &idx) {
  int base = 0;
  tree_level<L, 0>(v, lane, base);
  idx = base;
  return v[0];
}

// One pass of the score kernel over heads g0 .. g0 + gn - 1 (gn <= GN) and
// the warp's four positions: slot r * GN + gi holds (position r, head gi).
template <int HDV, int GN>
__device__ __forceinline__ void score_pass(const double *qsm, const float (&kv)[4][HDV / 32], const AttnArgs &a,
                                           int kvh, int G, int g0, int gn, int p0, int n_ctx, int warp, int lane) {
  constexpr int E = HDV / 32, L = 4 * GN;
  static_assert(E % 2 == 0, "tree level 1 pairs elements");
  double v[16];
#pragma unroll
  for (int i = 0; i < 16; i++) v[i] = 0.0;
  // head-major: a head's q slice is read from shared memory once for the
  // warp's four positions (each k element converted per use)
#pragma unroll
  for (int gi = 0; gi < GN; gi++) {
    if (gi < gn) {
      const double2 *qg2 = reinterpret_cast<const double2 *>(qsm + (g0 + gi) * HDV + lane * E);
      double qd[E];
#pragma unroll
      for (int t = 0; t < E; t += 2) {
        const double2 q2 = qg2[t / 2];
        qd[t] = q2.x;
        qd[t + 1] = q2.y;
      }
#pragma unroll
      for (int r = 0; r < 4; r++) {
        // tree level 1 as fma: q k of two f32 values is exact in f64, so
        // fma(q_t, k_t, q_t+1 k_t+1) rounds exactly as the pair's add does
        double pr[E];
#pragma unroll
        for (int t = 0; t < E; t += 2)
          pr[t] = __fma_rn(qd[t], (double)kv[r][t], __dmul_rn(qd[t + 1], (double)kv[r][t + 1]));
#pragma unroll
        for (int w = 2; w < E; w <<= 1)
#pragma unroll
          for (int t = 0; t < E; t += 2 * w) pr[t] = __dadd_rn(pr[t], pr[t + w]);
        v[r * GN + gi] = pr[0];
      }
    }
  }
  int idx = 0;
  const double sum = tree_reduce_lanes<L>(v, lane, idx);
  if (lane < L) {
    const int r = idx / GN, gi = idx % GN;
    const int p = p0 + warp + 8 * r;
    if (gi < gn && p < n_ctx) a.scores[(size_t)(kvh * G + g0 + gi) * a.ctx + p] = (float)sum;
  }
}

// scores[h][p] = dot_f32(q_h, k_p) as f32 (quants.rs:106-114): exact f64
// products summed by the pairwise tree, which for HDV = 32 * E (E a power of
// two) is lane-local subtrees over E contiguous elements and then the lanes
// (tree_reduce_lanes). A warp takes four positions (all loads issued first)
// and the q heads of the kv group, up to four at a time; 32 positions per
// CTA. q is converted to double once per CTA, each k row once per position.
template <int HDV>
__global__ void __launch_bounds__(256, 2) attn_scores_kernel(AttnArgs a) {
  constexpr int E = HDV / 32;
  pdl_trigger();
  extern __shared__ double qsm[];  // G x HDV
  pdl_wait();
  attn_at_seq(a);
  const int kvh = blockIdx.x, G = a.nh / a.nkv;
  const int n_ctx = *a.pos + 1;
  const int p0 = blockIdx.y * 32;
  if (p0 >= n_ctx) return;
#pragma unroll 4
  for (int i = threadIdx.x; i < G * HDV; i += 256) qsm[i] = (double)a.q[(size_t)(kvh * G) * HDV + i];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t kvlen = (size_t)a.nkv * HDV;
  float kv[4][E];
#pragma unroll
  for (int r = 0; r < 4; r++) {
    const int p = min(p0 + warp + 8 * r, n_ctx - 1);
    const float *kr = a.kcache + (size_t)p * kvlen + (size_t)kvh * HDV + lane * E;
#pragma unroll
    for (int t = 0; t < E; t += 4) {
      const float4 v4 = *reinterpret_cast<const float4 *>(kr + t);
      kv[r][t] = v4.x, kv[r][t + 1] = v4.y, kv[r][t + 2] = v4.z, kv[r][t + 3] = v4.w;
    }
  }
  __syncthreads();
  for (int g0 = 0; g0 < G; g0 += 4) {
    const int gn = min(4, G - g0);  // heads in this pass
    if (gn > 2) score_pass<HDV, 4>(qsm, kv, a, kvh, G, g0, gn, p0, n_ctx, warp, lane);
    else if (gn == 2) score_pass<HDV, 2>(qsm, kv, a, kvh, G, g0, gn, p0, n_ctx, warp, lane);
    else score_pass<HDV, 1>(qsm, kv, a, kvh, G, g0, gn, p0, n_ctx, warp, lane);
  }
}

// softmax (kernels.rs:157-168) of one head's scores, in place. 256 threads.
__global__ void __launch_bounds__(256) attn_softmax_kernel(AttnArgs a) {
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t sm[];
  __shared__ float redf[8];
  pdl_wait();
  attn_at_seq(a);
  const int h = blockIdx.x, tid = threadIdx.x;
  const int n = *a.pos + 1;
  float *e = reinterpret_cast<float *>(sm);
  double *l0 = reinterpret_cast<double *>(sm + round_up((size_t)a.ctx * 4, 16));
  double *l1 = l0 + (a.ctx + 1) / 2;
  float *sc = a.scores + (size_t)h * a.ctx;
  float m = -INFINITY;
#pragma unroll 8
  for (int p = tid; p < n; p += 256) {
    const float v = sc[p];
    e[p] = v;
    m = fmaxf(m, v);
  }
  m = block_max<256>(m, redf);
  for (int p = tid; p < n; p += 256) e[p] = exp_cr(__fmul_rn(__fsub_rn(e[p], m), a.kq_scale));
  __syncthreads();
  // pairwise_sum_f64 (kernels.rs:24-38): pairs (2i, 2i+1) per level, odd tail carried
  int len = (n + 1) / 2;
  for (int i = tid; i < len; i += 256)
    l0[i] = 2 * i + 1 < n ? __dadd_rn((double)e[2 * i], (double)e[2 * i + 1]) : (double)e[2 * i];
  __syncthreads();
  double *cur = l0, *nxt = l1;
  while (len > 1) {
    const int nl = (len + 1) / 2;
    for (int i = tid; i < nl; i += 256) nxt[i] = 2 * i + 1 < len ? __dadd_rn(cur[2 * i], cur[2 * i + 1]) : cur[2 * i];
    __syncthreads();
    double *t = cur;
    cur = nxt;
    nxt = t;
    len = nl;
  }
  const double sum = cur[0];
  for (int p = tid; p < n; p += 256) sc[p] = (float)__ddiv_rn((double)e[p], sum);
}

// Value pass over one chunk of kChunk positions for the G q heads of one kv
// head: per (head, column) the chunk's left-to-right f64 sum of
// soft[p] * v[p] (qwen35_forward.rs:660-672) and the sum of |running sum|,
// which bounds that chunk's rounding error. The chunk's V rows are staged in
// shared memory once for all G heads. Grid (nkv, nsplit), thread = column.
template <int HDV>
__global__ void __launch_bounds__(HDV) attn_values_kernel(AttnArgs a) {
  pdl_trigger();
  extern __shared__ __align__(16) float vsm[];  // kChunk x HDV
  __shared__ double ssoft[kMaxGroup][kChunk];  // converted once, not per column
  pdl_wait();
  attn_at_seq(a);
  const int kvh = blockIdx.x, split = blockIdx.y, c = threadIdx.x;
  const int n = *a.pos + 1, G = a.nh / a.nkv;
  const int p0 = split * kChunk;
  if (p0 >= n) return;
  const int len = min(kChunk, n - p0);
  const size_t kvlen = (size_t)a.nkv * HDV;
  constexpr int V4 = kChunk / 4;  // float4 loads per thread: kChunk * HDV / 4 / HDV
  float4 buf[V4];
#pragma unroll
  for (int i = 0; i < V4; i++) {
    const int idx = i * HDV + c;  // float4 index within the chunk
    const int p = idx / (HDV / 4), col4 = idx % (HDV / 4);
    buf[i] = p < len ? *reinterpret_cast<const float4 *>(a.vcache + (size_t)(p0 + p) * kvlen + (size_t)kvh * HDV +
                                                         col4 * 4)
                     : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int i = c; i < G * kChunk; i += HDV) {
    const int g = i / kChunk, pp = i % kChunk;
    ssoft[g][pp] = pp < len ? (double)a.scores[(size_t)(kvh * G + g) * a.ctx + p0 + pp] : 0.0;
  }
#pragma unroll
  for (int i = 0; i < V4; i++) reinterpret_cast<float4 *>(vsm)[i * HDV + c] = buf[i];
  __syncthreads();
  double S[kMaxGroup], Q[kMaxGroup];
#pragma unroll
  for (int g = 0; g < kMaxGroup; g++) S[g] = Q[g] = 0.0;
  // soft[p] * v[p] of two f32 values is exact in f64, so one fma rounds
  // exactly as the reference's add of the product does
  for (int p = 0; p < len; p++) {
    const double v = (double)vsm[p * HDV + c];
#pragma unroll
    for (int g = 0; g < kMaxGroup; g++) {
      if (g < G) {
        S[g] = __fma_rn(ssoft[g][p], v, S[g]);
        Q[g] = __dadd_rn(Q[g], fabs(S[g]));
      }
    }
  }
#pragma unroll
  for (int g = 0; g < kMaxGroup; g++)
    if (g < G) a.part[((size_t)(kvh * G + g) * a.nsplit + split) * HDV + c] = make_double2(S[g], Q[g]);
}

// Combine the chunks in position order, resolve the reference's sequential
// f64 sum exactly, gate with sigmoid (qwen35_forward.rs:676-686) and write the
// x image of attn_output's input. One CTA per 256-element span.
//
// Bound: the reference's left-to-right sum s^ of n terms satisfies
// |s^ - s| <= u' * sum_k |s^_k| <= u' (1 + O(nu)) sum_k |s_k| (s_k the exact
// prefix sums, u' = u / (1 - u)); with the exact total O_w before chunk w and
// in-chunk running sums q, sum_k |s_k| <= sum_w (len_w |O_w| + sum |q|). The
// chunked sum computed here is off by at most u' (sum_w sum |q| +
// sum_w |O_{w+1}|). B is their sum with a factor 4 (2^-51 instead of 2^-53)
// that covers every second-order term and the rounding of S +- B.
template <int HDV>
__global__ void __launch_bounds__(256) attn_combine_quant_kernel(AttnArgs a) {
  pdl_trigger();
  __shared__ Q8KSpanSmem sm;
  pdl_wait();
  attn_at_seq(a);
  const int span = blockIdx.x, t = threadIdx.x;
  const int e = span * 256 + t, h = e / HDV, c = e % HDV;
  const int n = *a.pos + 1;
  const int nw = (n + kChunk - 1) / kChunk;
  const double2 *pp = a.part + (size_t)h * a.nsplit * HDV + c;
  double O = 0.0, T1 = 0.0, T2 = 0.0, T3 = 0.0;
  for (int w0 = 0; w0 < nw; w0 += 8) {  // 8 chunks' partials in flight at a time
    double2 sq[8];
#pragma unroll
    for (int u = 0; u < 8; u++) sq[u] = w0 + u < nw ? pp[(size_t)(w0 + u) * HDV] : make_double2(0.0, 0.0);
#pragma unroll
    for (int u = 0; u < 8; u++) {
      if (w0 + u < nw) {
        const int len = min(kChunk, n - (w0 + u) * kChunk);
        T1 += sq[u].y;
        T2 += (double)len * fabs(O);
        O = __dadd_rn(O, sq[u].x);
        T3 += fabs(O);
      }
    }
  }
  const double B = 0x1p-51 * (2.0 * T1 + T2 + T3);
  float attn = (float)(O - B);
  const bool need = attn != (float)(O + B);
  if (__syncthreads_or(need)) {
    // some column's value is not resolved by the bound: its left-to-right
    // f64 sum is recomputed. For each such column (in turn), the whole CTA
    // forms its products soft[p] * v[p][c] into shared memory, 2048
    // positions at a time (each thread a few strided loads, all in flight at
    // once), and the column's own thread adds them up in order.
    constexpr int kFbChunk = 2048;
    __shared__ double fb_prod[kFbChunk];
    __shared__ int fb_list[256];
    __shared__ int fb_count;
    if (t == 0) fb_count = 0;
    __syncthreads();
    if (need) fb_list[atomicAdd(&fb_count, 1)] = t;
    __syncthreads();
    const int nfb = fb_count;
    const size_t kvlen = (size_t)a.nkv * HDV;
    for (int j = 0; j < nfb; j++) {
      const int owner = fb_list[j];
      const int eo = span * 256 + owner, ho = eo / HDV, co = eo % HDV;
      const float *vcol = a.vcache + (size_t)(ho / (a.nh / a.nkv)) * HDV + co;
      const float *soft = a.scores + (size_t)ho * a.ctx;
      double s = 0.0;
      for (int p0 = 0; p0 < n; p0 += kFbChunk) {
        const int len = min(kFbChunk, n - p0);
        for (int q = t; q < len; q += 256)
          fb_prod[q] = __dmul_rn((double)soft[p0 + q], (double)vcol[(size_t)(p0 + q) * kvlen]);
        __syncthreads();
        if (t == owner)
          for (int q = 0; q < len; q++) s = __dadd_rn(s, fb_prod[q]);
        __syncthreads();
      }
      if (t == owner) attn = (float)s;
    }
  }
  const float gate = a.qk[(size_t)h * 2 * HDV + HDV + c];
  q8k_span_write(__fmul_rn(attn, sigmoid_f(gate)), a.img4 ? a.img4 + (size_t)span * kImgQ8K4 : nullptr,
                 a.img6 ? a.img6 + (size_t)span * kImgQ8K6 : nullptr, sm, seq_bimg(a.bimg, a.nsg, a.seq0, span),
                 seq_sl(a.seq0));
}

// greedy token from the cross-GPU maximum of the argmax keys
// (orderable(logit) << 32 | ~global_row): the first index of the maximum
__global__ void key_to_token_kernel(const unsigned long long *key, uint32_t *token, size_t tss) {
  pdl_trigger();
  pdl_wait();
  key += blockIdx.z;  // a batch: one key per sequence, its token in its arena
  token = seq_ptr(token, seq_off(tss));
  *token = 0xffffffffu - (uint32_t)(*key & 0xffffffffull);
}

// A prefill chunk of T tokens: token t of the chunk sits at position
// *pos + t (the session's position before the chunk).
__global__ void prefill_begin_kernel(const int *pos, int *lane_pos, size_t lane_ss, int T) {
  pdl_trigger();
  pdl_wait();
  const int t = threadIdx.x;
  if (t < T) *reinterpret_cast<int *>(reinterpret_cast<uint8_t *>(lane_pos) + (size_t)t * lane_ss) = *pos + t;
}
// ... and after it: the session's position advances by T; with the LM head,
// its current token becomes the greedy token after the chunk's last token.
__global__ void prefill_end_kernel(int *pos, int T, uint32_t *cur_token, const uint32_t *last) {
  pdl_trigger();
  pdl_wait();
  *pos += T;
  if (last) *cur_token = *last;
}

// token bookkeeping at the end of a step
__global__ void step_end_kernel(const uint32_t *cur, uint32_t *hist, int *counter, int *pos, size_t ss) {
  pdl_trigger();
  pdl_wait();
  cur = seq_ptr(cur, seq_off(ss));
  hist = seq_ptr(hist, seq_off(ss));
  counter = seq_ptr(counter, seq_off(ss));
  pos = seq_ptr(pos, seq_off(ss));
  hist[*counter] = *cur;
  *counter += 1;
  *pos += 1;
}

}  // namespace
}  // namespace unltd

// ===========================================================================
// Host side: model (weights) and session (state + graph).
// ===========================================================================
using namespace unltd;

namespace {

struct Derived {
  int n, nff, nh, nkv, hdv, n_rot, K, nqk, hd, nv, dconv, kvlen, vocab, n_layer, interval, nrp;
  float eps, kq_scale;
  double theta_scale;
  // tensor-parallel shard of this rank (rank 0 of 1: the whole model)
  int rank = 0, world = 1;
  int nvl, nqkl, dconvl;   // recurrent: local v heads, local qk heads, local conv channels
  int vh0;                 // first local v head
  int nhl, nkvl, kvlenl;   // attention: local q heads, local kv heads
  int qh0, kv0;            // first local q head / kv head
  int nffl;                // local FFN width
  int v0, v1;              // local vocab rows [v0, v1)
};

struct Part {
  std::string name;
  size_t dim_in, dim_out;
  std::vector<int> dtypes;  // allowed
};

// One projection: consecutive same-dtype parts merged into one weight each.
struct Proj {
  std::vector<unltd_weight_s *> w;
  std::vector<size_t> off;  // output offset of each merged weight
  size_t rows = 0;
};

struct Layer {
  bool attn = false;
  int slot = 0;  // index among layers of the same kind
  float *attn_norm = nullptr, *post_norm = nullptr;
  Proj in;        // recurrent: qkv|z|beta|alpha; attention: q|k|v
  unltd_weight_s *out = nullptr;  // ssm_out / attn_output
  Proj gate_up;
  unltd_weight_s *down = nullptr;
  float *convw = nullptr, *dt_bias = nullptr, *ssm_a = nullptr, *ssm_norm = nullptr;  // recurrent
  float *q_norm = nullptr, *k_norm = nullptr;                                        // attention
};

struct Staged {
  int dtype = 0;
  unltd_weight_s *w = nullptr;
  float *f = nullptr;
};

}  // namespace

struct unltd_qwen35_s {
  unltd_ctx ctx = nullptr;
  unltd_qwen35_config cfg{};
  Derived d{};
  std::map<std::string, Staged> staged;
  bool finalized = false;
  std::vector<Layer> layers;
  unltd_weight_s *embd = nullptr, *output = nullptr;
  float *out_norm = nullptr;
  std::vector<void *> f32_bufs;
  int n_recr = 0, n_attn = 0;
  size_t proj_rows = 0;
};

struct unltd_qwen35_session_s {
  unltd_qwen35 m = nullptr;
  unltd_ctx ctx = nullptr;  // own context: stream, GEMV scratch, argmax state
  int ctx_len = 0;
  int host_pos = 0;
  // batch decode: n_seq sequences, every per-sequence buffer in the
  // sequence's arena (the pointers below are sequence 0's; sequence z's are
  // ss bytes further per z), positions tracked per sequence on the host
  int nseq = 1;
  size_t ss = 0;
  uint8_t *arena = nullptr;
  uint8_t *bimg = nullptr;  // the batched x images (n_seq > 1)
  int nsg = 0;
  // tensor-parallel batch: the row-split projections' outputs of every
  // sequence, contiguous ([n_seq][n_embd]) for one all-reduce, and the
  // sequences' LM-head argmax keys
  float *tpbuf = nullptr;
  unsigned long long *tpkeys = nullptr;
  // prefill (unltd_qwen35_prefill): kPrefillLanes activation lanes (a
  // chunk's tokens), made on first use; the state stays the session's
  struct Prefill {
    size_t ss = 0;
    uint8_t *arena = nullptr;
    float *X = nullptr, *R = nullptr, *T = nullptr, *F = nullptr, *proj = nullptr, *Y = nullptr, *FF = nullptr;
    float *q = nullptr, *scores = nullptr, *logits = nullptr;
    double2 *part = nullptr;
    int *pos = nullptr;
    uint32_t *tok = nullptr;  // the chunk's tokens, contiguous; then the LM head's
    uint8_t *bimg = nullptr;
  } pf;
  std::vector<int> seq_pos;
  // activations
  float *X = nullptr, *R = nullptr, *T = nullptr, *F = nullptr;
  float *proj = nullptr, *Y = nullptr, *FF = nullptr;
  float *q = nullptr, *scores = nullptr, *logits = nullptr;
  double2 *rope = nullptr, *part = nullptr;
  uint8_t *img4 = nullptr, *img6 = nullptr;  // x images written by the fused producer kernels
  unsigned long long *tpkey = nullptr;       // this rank's LM-head argmax key, then the global one
  int nsplit = 0;
  uint32_t *cur_token = nullptr, *hist = nullptr, *feed = nullptr;
  int *counter = nullptr, *pos = nullptr;
  unsigned *span_ctr = nullptr;  // recurrent layers: CTAs done per span of the GDN output
  std::vector<float *> ring, state, kc, vc;
  std::vector<void *> bufs;
  cudaGraphExec_t graph = nullptr;
  bool graph_tried = false;
  int64_t launches_per_step = 0;
};

namespace {

int32_t derive(const unltd_qwen35_config &c, Derived *d) {
  auto bad = [](const std::string &m) { return set_error(UNLTD_ERR_INVALID_ARG, "qwen35 config: " + m); };
  auto unsup = [](const std::string &m) { return set_error(UNLTD_ERR_UNSUPPORTED, "qwen35 config: " + m); };
  // qwen35.rs:174-252
  if (c.n_layer < 1) return bad("block_count = 0");
  if (c.n_embd <= 0 || c.n_ff <= 0) return bad("zero embedding/FFN dims");
  if (c.n_head < 1) return bad("attention.head_count = 0");
  if (c.n_head_kv < 1 || c.n_head % c.n_head_kv) return bad("invalid GQA");
  if (c.n_head * c.head_dim != c.n_embd) return bad("head_count * key_length != n_embd");
  if (c.head_dim != c.head_dim_v) return bad("key_length != value_length");
  if (c.n_rot % 2 || c.n_rot > c.head_dim || c.n_rot < 0) return bad("n_rot must be even and <= head_dim");
  if (!(c.freq_base > 0.0f)) return bad("rope.freq_base <= 0");
  if (!(c.rms_eps > 0.0f)) return bad("layer_norm_rms_epsilon <= 0");
  if (c.conv_kernel < 2) return bad("ssm.conv_kernel < 2");
  if (c.group_count < 1) return bad("ssm.group_count = 0");
  if (c.d_inner <= 0 || c.d_inner % (2 * c.group_count)) return bad("d_inner not a multiple of 2*group_count");
  if (c.time_step_rank < 1) return bad("ssm.time_step_rank = 0");
  const int hd = c.d_inner / (2 * c.group_count);
  if (c.state_size != hd) return bad("state_size != linear head dim");
  if (c.full_attn_interval < 1) return bad("full_attention_interval = 0");
  if (c.vocab < 1) return bad("vocab = 0");
  // what the kernels of this library cover
  if (c.d_inner != c.n_embd) return unsup("d_inner != n_embd (the recurrent output feeds an n_embd x n_embd ssm_out)");
  if (hd != 128) return unsup("linear head dim must be 128");
  if (c.head_dim != 256 && c.head_dim != 128) return unsup("head_dim must be 128 or 256");
  if (c.n_embd % 256 || c.n_ff % 256) return unsup("n_embd and n_ff must be multiples of 256");
  if (c.conv_kernel > 16) return unsup("conv_kernel > 16");
  if (c.n_head / c.n_head_kv > kMaxGroup) return unsup("more than 8 query heads per kv head");
  d->n = c.n_embd;
  d->nff = c.n_ff;
  d->nh = c.n_head;
  d->nkv = c.n_head_kv;
  d->hdv = c.head_dim;
  d->n_rot = c.n_rot;
  d->K = c.conv_kernel;
  d->nqk = c.group_count;
  d->hd = hd;
  d->nv = c.d_inner / hd;
  d->dconv = 2 * c.d_inner;
  d->kvlen = c.n_head_kv * c.head_dim;
  d->vocab = c.vocab;
  d->n_layer = c.n_layer;
  d->interval = c.full_attn_interval;
  d->nrp = (c.n_rot / 2 + 2) / 3;
  d->eps = c.rms_eps;
  d->kq_scale = 1.0f / std::sqrt((float)c.head_dim);
  d->theta_scale = (double)std::pow(c.freq_base, -2.0f / (float)c.n_rot);
  return UNLTD_OK;
}

int32_t derive_tp(Derived *d, int rank, int world);

bool is_attn(const Derived &d, int il) { return (il + 1) % d.interval == 0; }

// Tensor-parallel split of rank `rank` of `world`: gate/up and the q/k/v and
// qkv/z/beta/alpha projections by output rows (heads), down and the output
// projections by input columns (their partial outputs are summed across
// ranks), the LM head by vocab rows; norms, conv and GDN parameters follow
// their heads; the embedding is replicated.
int32_t derive_tp(Derived *d, int rank, int world) {
  auto unsup = [](const std::string &m) { return set_error(UNLTD_ERR_UNSUPPORTED, "qwen35 tensor parallel: " + m); };
  if (world < 1 || rank < 0 || rank >= world) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35: bad rank/world");
  d->rank = rank;
  d->world = world;
  if (d->nv % world) return unsup("v heads not divisible by the GPU count");
  d->nvl = d->nv / world;
  if (d->nvl <= d->nqk) {
    d->nqkl = d->nvl;
  } else {
    if (d->nvl % d->nqk) return unsup("local v heads not a multiple of the qk heads");
    d->nqkl = d->nqk;
  }
  d->vh0 = rank * d->nvl;
  d->dconvl = 2 * d->nqkl * d->hd + d->nvl * d->hd;
  if (world > 1 && (d->nvl * d->hd) % 256) return unsup("local recurrent width not a multiple of 256");
  if (d->nh % world) return unsup("q heads not divisible by the GPU count");
  d->nhl = d->nh / world;
  const int G = d->nh / d->nkv;
  if (d->nhl >= G) {
    if (d->nhl % G) return unsup("local q heads split a kv group");
    d->nkvl = d->nhl / G;
  } else {
    if (G % d->nhl) return unsup("kv group not divisible by the local q heads");
    d->nkvl = 1;
  }
  d->qh0 = rank * d->nhl;
  d->kv0 = d->qh0 / G;
  d->kvlenl = d->nkvl * d->hdv;
  if (world > 1 && (d->nhl * d->hdv) % 256) return unsup("local attention width not a multiple of 256");
  if (d->nff % (256 * world)) return unsup("n_ff not a multiple of 256 x GPU count");
  d->nffl = d->nff / world;
  const int per = (d->vocab + world - 1) / world;
  d->v0 = std::min(d->vocab, rank * per);
  d->v1 = std::min(d->vocab, d->v0 + per);
  if (d->v1 <= d->v0) return unsup("vocab smaller than the GPU count");
  return UNLTD_OK;
}

// The rank's part of a tensor: source row ranges (element ranges for F32
// tensors) concatenated in order, each row restricted to input columns
// [in0, in1).
struct Shard {
  std::vector<std::pair<size_t, size_t>> rows;
  size_t in0 = 0, in1 = 0;
  size_t nrows() const {
    size_t r = 0;
    for (auto &p : rows) r += p.second - p.first;
    return r;
  }
};

Shard shard_of(const Derived &d, const std::string &name, size_t dim_in, size_t dim_out) {
  Shard s;
  s.in0 = 0;
  s.in1 = dim_in;
  const bool f32 = dim_out == 1;  // F32 tensors: "rows" are elements
  const size_t len = f32 ? dim_in : dim_out;
  if (f32) s.in1 = 1;
  const std::string kind = name.compare(0, 4, "blk.") == 0 ? name.substr(name.find('.', 4) + 1) : name;
  const size_t hd = d.hd, hdv = d.hdv;
  auto all = [&]() { s.rows.push_back({0, len}); };
  auto qk_rows = [&](size_t base, size_t unit) {  // rows of the local qk heads, in local order
    for (int j = 0; j < d.nqkl; j++) {
      const size_t gq = (size_t)((d.vh0 + j) % d.nqk);
      s.rows.push_back({base + gq * unit, base + (gq + 1) * unit});
    }
  };
  if (kind == "output.weight") {
    s.rows.push_back({(size_t)d.v0, (size_t)d.v1});
  } else if (kind == "ffn_gate.weight" || kind == "ffn_up.weight") {
    s.rows.push_back({(size_t)d.rank * d.nffl, (size_t)(d.rank + 1) * d.nffl});
  } else if (kind == "ffn_down.weight") {
    all();
    s.in0 = (size_t)d.rank * d.nffl;
    s.in1 = s.in0 + d.nffl;
  } else if (kind == "attn_q.weight") {
    s.rows.push_back({(size_t)d.qh0 * 2 * hdv, (size_t)(d.qh0 + d.nhl) * 2 * hdv});
  } else if (kind == "attn_k.weight" || kind == "attn_v.weight") {
    s.rows.push_back({(size_t)d.kv0 * hdv, (size_t)(d.kv0 + d.nkvl) * hdv});
  } else if (kind == "attn_output.weight") {
    all();
    s.in0 = (size_t)d.qh0 * hdv;
    s.in1 = s.in0 + (size_t)d.nhl * hdv;
  } else if (kind == "attn_qkv.weight") {
    qk_rows(0, hd);
    qk_rows((size_t)d.nqk * hd, hd);
    s.rows.push_back({2 * (size_t)d.nqk * hd + (size_t)d.vh0 * hd, 2 * (size_t)d.nqk * hd + (size_t)(d.vh0 + d.nvl) * hd});
  } else if (kind == "ssm_conv1d.weight") {  // [channel][tau]: channel ranges times K
    const size_t K = d.K;
    for (int j = 0; j < d.nqkl; j++) {
      const size_t gq = (size_t)((d.vh0 + j) % d.nqk);
      s.rows.push_back({gq * hd * K, (gq + 1) * hd * K});
    }
    for (int j = 0; j < d.nqkl; j++) {
      const size_t gq = (size_t)((d.vh0 + j) % d.nqk);
      s.rows.push_back({((size_t)d.nqk + gq) * hd * K, ((size_t)d.nqk + gq + 1) * hd * K});
    }
    s.rows.push_back({(2 * (size_t)d.nqk * hd + (size_t)d.vh0 * hd) * K, (2 * (size_t)d.nqk * hd + (size_t)(d.vh0 + d.nvl) * hd) * K});
  } else if (kind == "attn_gate.weight") {
    s.rows.push_back({(size_t)d.vh0 * hd, (size_t)(d.vh0 + d.nvl) * hd});
  } else if (kind == "ssm_beta.weight" || kind == "ssm_alpha.weight" || kind == "ssm_dt.bias" || kind == "ssm_a") {
    s.rows.push_back({(size_t)d.vh0, (size_t)(d.vh0 + d.nvl)});
  } else if (kind == "ssm_out.weight") {
    all();
    s.in0 = (size_t)d.vh0 * hd;
    s.in1 = s.in0 + (size_t)d.nvl * hd;
  } else {
    all();  // embedding, norms: replicated
  }
  // merge adjacent ranges (one range per tensor on a single GPU)
  std::vector<std::pair<size_t, size_t>> merged;
  for (auto &r : s.rows) {
    if (!merged.empty() && merged.back().second == r.first) merged.back().second = r.second;
    else merged.push_back(r);
  }
  s.rows = merged;
  return s;
}

// Gather the rank's bytes of a host tensor (rows of row_bytes, blocks of
// block_bytes covering block_elems input elements each).
std::vector<uint8_t> gather_shard(const Shard &sh, const uint8_t *host, size_t row_bytes, size_t elem_per_block,
                                  size_t block_bytes) {
  const size_t b0 = sh.in0 / elem_per_block, b1 = sh.in1 / elem_per_block;
  const size_t out_rb = (b1 - b0) * block_bytes;
  std::vector<uint8_t> out(sh.nrows() * out_rb);
  size_t o = 0;
  for (auto &r : sh.rows)
    for (size_t row = r.first; row < r.second; row++, o += out_rb)
      memcpy(out.data() + o, host + row * row_bytes + b0 * block_bytes, out_rb);
  return out;
}

// Expected tensors (qwen35_forward.rs:139-221, min_forward.rs): name -> shape, dtypes.
std::vector<Part> expected(const Derived &d) {
  std::vector<Part> v;
  const std::vector<int> f32{F32}, q4{Q4K}, q46{Q4K, Q6K};
  v.push_back({"token_embd.weight", (size_t)d.n, (size_t)d.vocab, q4});
  v.push_back({"output_norm.weight", (size_t)d.n, 1, f32});
  v.push_back({"output.weight", (size_t)d.n, (size_t)d.vocab, q46});
  for (int il = 0; il < d.n_layer; il++) {
    const std::string p = "blk." + std::to_string(il) + ".";
    v.push_back({p + "attn_norm.weight", (size_t)d.n, 1, f32});
    v.push_back({p + "post_attention_norm.weight", (size_t)d.n, 1, f32});
    v.push_back({p + "ffn_gate.weight", (size_t)d.n, (size_t)d.nff, q4});
    v.push_back({p + "ffn_up.weight", (size_t)d.n, (size_t)d.nff, q4});
    v.push_back({p + "ffn_down.weight", (size_t)d.nff, (size_t)d.n, q46});
    if (is_attn(d, il)) {
      v.push_back({p + "attn_q.weight", (size_t)d.n, (size_t)(2 * d.n), q4});
      v.push_back({p + "attn_q_norm.weight", (size_t)d.hdv, 1, f32});
      v.push_back({p + "attn_k.weight", (size_t)d.n, (size_t)d.kvlen, q4});
      v.push_back({p + "attn_k_norm.weight", (size_t)d.hdv, 1, f32});
      v.push_back({p + "attn_v.weight", (size_t)d.n, (size_t)d.kvlen, q46});
      v.push_back({p + "attn_output.weight", (size_t)d.n, (size_t)d.n, q4});
    } else {
      v.push_back({p + "attn_qkv.weight", (size_t)d.n, (size_t)d.dconv, q46});
      v.push_back({p + "attn_gate.weight", (size_t)d.n, (size_t)d.n, q4});
      v.push_back({p + "ssm_conv1d.weight", (size_t)(d.K * d.dconv), 1, f32});
      v.push_back({p + "ssm_dt.bias", (size_t)d.nv, 1, f32});
      v.push_back({p + "ssm_a", (size_t)d.nv, 1, f32});
      v.push_back({p + "ssm_beta.weight", (size_t)d.n, (size_t)d.nv, q4});
      v.push_back({p + "ssm_alpha.weight", (size_t)d.n, (size_t)d.nv, q4});
      v.push_back({p + "ssm_norm.weight", (size_t)d.hd, 1, f32});
      v.push_back({p + "ssm_out.weight", (size_t)d.n, (size_t)d.n, q4});
    }
  }
  return v;
}

const char *dtype_str(int t) {
  switch (t) {
    case F32: return "F32";
    case Q4K: return "Q4_K";
    case Q6K: return "Q6_K";
    case Q8_0: return "Q8_0";
    default: return "other";
  }
}

// Merge row-concatenated weights of one dtype into one device allocation.
int32_t merge(unltd_ctx ctx, const std::vector<unltd_weight_s *> &parts, unltd_weight_s **out) {
  if (parts.size() == 1) {
    *out = parts[0];
    return UNLTD_OK;
  }
  unltd_weight_s *w = new unltd_weight_s(*parts[0]);
  size_t rows = 0;
  for (auto *p : parts) rows += p->dim_out;
  w->dim_out = rows;
  cudaError_t e = cudaMalloc(&w->dev, std::max<size_t>(rows * w->row_stride, 16));
  if (e != cudaSuccess) {
    delete w;
    return cuda_error(e, "qwen35: merged weight alloc");
  }
  size_t r = 0;
  for (auto *p : parts) {
    e = cudaMemcpyAsync(w->dev + r * w->row_stride, p->dev, p->dim_out * p->row_stride, cudaMemcpyDeviceToDevice,
                        ctx->stream);
    if (e != cudaSuccess) break;
    r += p->dim_out;
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) {
    cudaFree(w->dev);
    delete w;
    return cuda_error(e, "qwen35: merge copy");
  }
  for (auto *p : parts) unltd_weight_free(p);
  *out = w;
  return UNLTD_OK;
}

int32_t build_proj(unltd_qwen35 m, const std::vector<std::string> &names, Proj *pr) {
  std::vector<unltd_weight_s *> run;
  size_t off = 0, run_off = 0;
  auto flush = [&]() -> int32_t {
    if (run.empty()) return UNLTD_OK;
    unltd_weight_s *w = nullptr;
    int32_t rc = merge(m->ctx, run, &w);
    if (rc) return rc;
    pr->w.push_back(w);
    pr->off.push_back(run_off);
    run.clear();
    return UNLTD_OK;
  };
  for (const auto &nm : names) {
    Staged &s = m->staged.at(nm);
    if (!run.empty() && run.back()->dtype != s.w->dtype) {
      if (int32_t rc = flush()) return rc;
    }
    if (run.empty()) run_off = off;
    run.push_back(s.w);
    off += s.w->dim_out;
    s.w = nullptr;
  }
  if (int32_t rc = flush()) return rc;
  pr->rows = off;
  return UNLTD_OK;
}

template <class T>
int32_t dalloc(std::vector<void *> &bufs, T **p, size_t n, const char *what) {
  cudaError_t e = cudaMalloc(reinterpret_cast<void **>(p), std::max<size_t>(n * sizeof(T), 16));
  if (e != cudaSuccess) return cuda_error(e, what);
  bufs.push_back(*p);
  return UNLTD_OK;
}

// GEMV whose x image a fused producer kernel already wrote.
int64_t launch_gemv_img(unltd_qwen35_session s, const unltd_weight_s *w, float *y, int32_t *rc, bool send = false) {
  if (s->nseq > 1) {  // every sequence's GEMV in one pass over w
    BatchGemvArgs b{w};
    b.img = s->bimg;
    b.nsg = s->nsg;
    b.y = y;
    b.ystride = s->tpbuf && y == s->tpbuf ? (size_t)s->m->d.n : s->ss / 4;  // tpbuf: contiguous rows
    b.nseq = s->nseq;
    if (!*rc) *rc = gemv_batch_launch(s->ctx, b);
    return 1;
  }
  GemvArgs g{w, nullptr, send ? nullptr : y, MODE_Q8K, nullptr, nullptr, nullptr};
  g.img = w->dtype == Q4K ? s->img4 : s->img6;
  g.peer_send = send;
  if (!*rc) *rc = gemv_launch(s->ctx, g);
  return 1;
}

// Kernel launch with programmatic stream serialization: the kernel may become
// resident while its predecessor runs; it calls griddepcontrol.wait before
// reading the predecessor's output or writing anything.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

bool any_dtype(const Proj &p, int dt) {
  for (auto *w : p.w)
    if (w->dtype == dt) return true;
  return false;
}

size_t softmax_smem(int ctx_len) {
  return round_up((size_t)ctx_len * 4, 16) + (size_t)((ctx_len + 1) / 2 + (ctx_len + 3) / 4 + 1) * 8;
}

// Enqueue one decode step on the session's stream.
int32_t enqueue_step(unltd_qwen35_session s) {
  unltd_qwen35 m = s->m;
  const Derived &d = m->d;
  cudaStream_t st = s->ctx->stream;
  int32_t rc = UNLTD_OK;
  int64_t nl = 0;
  auto chk = [&](cudaError_t e, const char *what) {
    if (!rc) rc = cuda_error(e, what);
    nl++;
  };
  // partial outputs of the input-split projections: sum over the ranks (NCCL)
  auto allreduce = [&](float *buf, int count) {
    if (d.world == 1) return;
    if (!rc) rc = comm_allreduce(m->ctx, st, buf, (size_t)count, false);
    nl++;
  };
  const bool batch = s->nseq > 1;
  const unsigned nz = (unsigned)s->nseq;
  // a tensor-parallel batch: the row-split outputs go to tpbuf, one
  // all-reduce for all sequences, and the consuming norm reads them there
  const bool tpb = batch && d.world > 1;
  const size_t tpss = (size_t)d.n * 4;
  // the images a producer writes for its consumers: in a batch session the
  // batched image only (the batched GEMV reads it for both formats)
  auto im4 = [&](bool q4) { return !batch && q4 ? s->img4 : nullptr; };
  auto im6 = [&](bool q6) { return !batch && q6 ? s->img6 : nullptr; };
  auto norm = [&](const float *a, const float *b, float *r_out, const float *w, bool q4, bool q6, bool argmax) {
    NormArgs p{a, b, r_out, w, d.n, d.eps, im4(q4), im6(q6),
               argmax && !batch ? s->ctx->argmax_key : nullptr, argmax && !batch ? s->ctx->argmax_done : nullptr};
    p.ss = s->ss;
    if (tpb && b == s->tpbuf) p.bss = tpss;
    p.bimg = s->bimg;
    p.nsg = s->nsg;
    chk(launch_pdl(norm_quant_kernel, dim3(d.n / 256, 1, nz), dim3(256), 0, st, p), "norm");
  };
  // RMSNorm of a (+ b) feeding projection p (outputs at out + p.off[i]): fused
  // into the prologue of p's first tensor-core Q4_K GEMV when it has one,
  // which then also writes the images p's other GEMVs read; else the
  // stand-alone norm kernel followed by the GEMVs.
  // Tensor parallelism with peer memory: a row-split GEMV (ssm_out /
  // attn_output, ffn_down) stores its partial rows into every rank's peer area
  // and the consuming GEMV's fused norm sums them in rank order: no separate
  // all-reduce kernel. The last layer's down keeps the all-reduce (the output
  // norm is a kernel of its own).
  const bool peer_sum = d.world > 1 && s->ctx->peer_ok && (size_t)d.n <= kPeerMaxCount;
  auto proj_fusable = [&](const Proj &p) {
    for (auto *w : p.w)
      if (gemv_norm_fusable(s->ctx, *w, MODE_Q8K)) return true;
    return false;
  };
  auto norm_proj = [&](const float *a, const float *b, float *r_out, const float *w, const Proj &p, float *out,
                       bool recv = false) {
    int fi = -1;
    for (size_t i = 0; i < p.w.size() && fi < 0 && !batch; i++)
      if (gemv_norm_fusable(s->ctx, *p.w[i], MODE_Q8K)) fi = (int)i;
    if (fi < 0) {
      norm(a, b, r_out, w, any_dtype(p, Q4K), any_dtype(p, Q6K), false);
      for (size_t i = 0; i < p.w.size(); i++) nl += launch_gemv_img(s, p.w[i], out + p.off[i], &rc);
      return;
    }
    bool need4 = false, need6 = false;
    for (size_t i = 0; i < p.w.size(); i++) {
      if ((int)i == fi) continue;
      need4 |= p.w[i]->dtype == Q4K;
      need6 |= p.w[i]->dtype == Q6K;
    }
    GemvNorm gn{a, recv ? nullptr : b, r_out, w, d.eps, need4 ? s->img4 : nullptr, need6 ? s->img6 : nullptr};
    gn.peer_recv = recv;
    GemvArgs g{p.w[fi], nullptr, out + p.off[fi], MODE_Q8K, nullptr, nullptr, nullptr};
    g.norm = &gn;
    if (!rc) rc = gemv_launch(s->ctx, g);
    nl++;
    for (size_t i = 0; i < p.w.size(); i++)
      if ((int)i != fi) nl += launch_gemv_img(s, p.w[i], out + p.off[i], &rc);
  };
  chk(launch_pdl(embed_q4k_kernel, dim3(d.n / 256, 1, nz), dim3(256), 0, st, (const uint8_t *)m->embd->dev,
                 m->embd->row_stride, m->embd->nb, (const uint32_t *)s->cur_token, (uint32_t)d.vocab, s->X, d.n,
                 s->ctx->err, s->ss, s->ss),
      "embed");
  bool down_sent = false;  // the previous layer's down GEMV sent its rows to the peers
  for (int il = 0; il < d.n_layer; il++) {
    const Layer &L = m->layers[il];
    const bool out_send = peer_sum && proj_fusable(L.gate_up) && gemv_tc_eligible(s->ctx, *L.out, MODE_Q8K);
    const bool down_send = peer_sum && il + 1 < d.n_layer && proj_fusable(m->layers[il + 1].in) &&
                           gemv_tc_eligible(s->ctx, *L.down, MODE_Q8K);
    // layer input = l_out of the previous layer (residual + ffn), fused into the norm
    if (il == 0) norm_proj(s->X, nullptr, nullptr, L.attn_norm, L.in, s->proj);
    else norm_proj(s->R, tpb ? s->tpbuf : s->F, s->X, L.attn_norm, L.in, s->proj, down_sent);
    if (!L.attn) {
      RecrArgs a;
      a.proj = s->proj;
      a.ring = s->ring[L.slot];
      a.convw = L.convw;
      a.dt_bias = L.dt_bias;
      a.ssm_a = L.ssm_a;
      a.ssm_norm = L.ssm_norm;
      a.state = s->state[L.slot];
      a.y = s->Y;
      a.pos = s->pos;
      a.K = d.K;
      a.nqk = d.nqkl;
      a.nv = d.nvl;
      a.dconv = d.dconvl;
      a.z_off = d.dconvl;
      a.beta_off = d.dconvl + d.nvl * d.hd;
      a.alpha_off = a.beta_off + d.nvl;
      a.eps = d.eps;
      a.span_ctr = s->span_ctr;
      a.img4 = im4(L.out->dtype == Q4K);
      a.img6 = im6(L.out->dtype == Q6K);
      a.ss = s->ss;
      a.bimg = s->bimg;
      a.nsg = s->nsg;
      const dim3 rg(d.nvl, 128 / kGdnCols, nz);
      if (d.K == 4) chk(launch_pdl(recr_mid_kernel<128, 4>, rg, dim3(128), 0, st, a), "recr_mid");
      else chk(launch_pdl(recr_mid_kernel<128, 0>, rg, dim3(128), 0, st, a), "recr_mid");
      nl += launch_gemv_img(s, L.out, tpb ? s->tpbuf : s->T, &rc, out_send);
      if (tpb) allreduce(s->tpbuf, (int)(nz * d.n));
      else if (!out_send) allreduce(s->T, d.n);
    } else {
      AttnArgs a;
      a.qk = s->proj;
      a.v = s->proj + 2 * d.nhl * d.hdv + d.kvlenl;
      a.q_norm = L.q_norm;
      a.k_norm = L.k_norm;
      a.rope = s->rope;
      a.q = s->q;
      a.kcache = s->kc[L.slot];
      a.vcache = s->vc[L.slot];
      a.scores = s->scores;
      a.part = s->part;
      a.img4 = im4(L.out->dtype == Q4K);
      a.img6 = im6(L.out->dtype == Q6K);
      a.pos = s->pos;
      a.nh = d.nhl;
      a.nkv = d.nkvl;
      a.n_rot = d.n_rot;
      a.nrp = d.nrp;
      a.ctx = s->ctx_len;
      a.nsplit = s->nsplit;
      a.eps = d.eps;
      a.kq_scale = d.kq_scale;
      a.ss = s->ss;
      a.kv_ss = s->ss;
      a.bimg = s->bimg;
      a.nsg = s->nsg;
      const dim3 sg(d.nkvl, (s->ctx_len + 31) / 32, nz), vg(d.nkvl, s->nsplit, nz);
      const size_t q_smem = (size_t)(d.nhl / d.nkvl) * d.hdv * 8, v_smem = (size_t)kChunk * d.hdv * 4;
      const size_t sm_smem = softmax_smem(s->ctx_len);
      const dim3 cg(d.nhl * d.hdv / 256, 1, nz), pg(d.nhl + d.nkvl, 1, nz), smg(d.nhl, 1, nz);
      if (d.hdv == 256) {
        chk(launch_pdl(attn_pre_kernel<256>, pg, dim3(256), 0, st, a), "attn_pre");
        chk(launch_pdl(attn_scores_kernel<256>, sg, dim3(256), q_smem, st, a), "attn_scores");
        chk(launch_pdl(attn_softmax_kernel, smg, dim3(256), sm_smem, st, a), "attn_softmax");
        chk(launch_pdl(attn_values_kernel<256>, vg, dim3(256), v_smem, st, a), "attn_values");
        chk(launch_pdl(attn_combine_quant_kernel<256>, cg, dim3(256), 0, st, a), "attn_combine");
      } else {
        chk(launch_pdl(attn_pre_kernel<128>, pg, dim3(128), 0, st, a), "attn_pre");
        chk(launch_pdl(attn_scores_kernel<128>, sg, dim3(256), q_smem, st, a), "attn_scores");
        chk(launch_pdl(attn_softmax_kernel, smg, dim3(256), sm_smem, st, a), "attn_softmax");
        chk(launch_pdl(attn_values_kernel<128>, vg, dim3(128), v_smem, st, a), "attn_values");
        chk(launch_pdl(attn_combine_quant_kernel<128>, cg, dim3(256), 0, st, a), "attn_combine");
      }
      nl += launch_gemv_img(s, L.out, tpb ? s->tpbuf : s->T, &rc, out_send);
      if (tpb) allreduce(s->tpbuf, (int)(nz * d.n));
      else if (!out_send) allreduce(s->T, d.n);
    }
    // residual = x_in + attn_out; rmsnorm(residual, post_attention_norm) -> gate|up image
    norm_proj(s->X, tpb ? s->tpbuf : s->T, s->R, L.post_norm, L.gate_up, s->FF, out_send);
    chk(launch_pdl(swiglu_quant_kernel, dim3(d.nffl / 256, 1, nz), dim3(256), 0, st, (const float *)s->FF,
                   (const float *)(s->FF + d.nffl), im4(L.down->dtype == Q4K), im6(L.down->dtype == Q6K), s->ss,
                   s->bimg, s->nsg),
        "swiglu");
    nl += launch_gemv_img(s, L.down, tpb ? s->tpbuf : s->F, &rc, down_send);
    if (tpb) allreduce(s->tpbuf, (int)(nz * d.n));
    else if (!down_send) allreduce(s->F, d.n);
    down_sent = down_send;
  }
  // l_out of the last layer -> output norm -> LM head + greedy argmax
  norm(s->R, tpb ? s->tpbuf : s->F, s->X, m->out_norm, m->output->dtype == Q4K, m->output->dtype == Q6K, true);
  if (batch) {
    BatchGemvArgs b{m->output};
    b.img = s->bimg;
    b.nsg = s->nsg;
    b.y = s->logits;
    b.ystride = s->ss / 4;
    b.nseq = s->nseq;
    b.key = s->ctx->bkey;
    b.done = s->ctx->bdone;
    b.token = s->cur_token;
    b.tstride = s->ss / 4;
    if (tpb) {  // vocab shards: every sequence's key, MAX across the ranks, then its token
      b.row0 = d.v0;
      b.key_out = s->tpkeys;
    }
    if (!rc) rc = gemv_batch_launch(s->ctx, b);
    nl += 1;
    if (tpb) {
      if (!rc) rc = comm_allreduce(m->ctx, st, s->tpkeys, nz, true);
      nl += 1;
      chk(launch_pdl(key_to_token_kernel, dim3(1, 1, nz), dim3(1), 0, st, (const unsigned long long *)s->tpkeys,
                     s->cur_token, s->ss),
          "key_to_token");
    }
  } else {
    GemvArgs g{m->output, nullptr, s->logits, MODE_Q8K, s->ctx->argmax_key, s->ctx->argmax_done, s->cur_token};
    g.img = m->output->dtype == Q4K ? s->img4 : s->img6;
    g.argmax_row0 = d.v0;
    if (d.world > 1) g.key_out = s->tpkey;
    if (!rc) rc = gemv_launch(s->ctx, g);
    nl += 1;
    if (d.world > 1) {  // vocab shards: MAX of the packed keys, then the token
      if (!rc) rc = comm_allreduce(m->ctx, st, s->tpkey, 1, true);
      nl += 1;
      chk(launch_pdl(key_to_token_kernel, dim3(1), dim3(1), 0, st, (const unsigned long long *)s->tpkey,
                     s->cur_token, (size_t)0),
          "key_to_token");
    }
  }
  chk(launch_pdl(step_end_kernel, dim3(1, 1, nz), dim3(1), 0, st, (const uint32_t *)s->cur_token, s->hist,
                 s->counter, s->pos, s->ss),
      "step_end");
  s->launches_per_step = nl;
  return rc;
}

int32_t run_step(unltd_qwen35_session s) {
  if (!s->graph_tried) {
    s->graph_tried = true;
    const char *env = getenv("UNLTD_NO_GRAPH");
    if (!(env && env[0] == '1')) {
      cudaStream_t st = s->ctx->stream;
      cudaGraph_t g = nullptr;
      cudaError_t e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
      int32_t rc = UNLTD_OK;
      if (e == cudaSuccess) {
        rc = enqueue_step(s);
        e = cudaStreamEndCapture(st, &g);
      }
      if (e == cudaSuccess && rc == UNLTD_OK) e = cudaGraphInstantiate(&s->graph, g, 0);
      if (g) cudaGraphDestroy(g);
      if (e != cudaSuccess || rc != UNLTD_OK) {
        s->graph = nullptr;
        cudaGetLastError();  // capture failure: run uncaptured launches instead
      }
    }
  }
  if (s->graph) {
    s->ctx->launches += s->launches_per_step;
    return cuda_error(cudaGraphLaunch(s->graph, s->ctx->stream), "qwen35: graph launch");
  }
  return enqueue_step(s);
}

constexpr int kPrefillLanes = 32;
static_assert(kPrefillLanes == kChunkTok, "the recurrent chunk kernel holds a chunk's tokens");
constexpr int kPrefillNsg = kPrefillLanes / 8;

// The prefill workspace: the activation buffers of kPrefillLanes tokens.
int32_t prefill_alloc(unltd_qwen35_session s) {
  if (s->pf.arena) return UNLTD_OK;
  unltd_qwen35 m = s->m;
  const Derived &d = m->d;
  auto &P = s->pf;
  struct Slot {
    void **p;
    size_t bytes, off;
  };
  std::vector<Slot> sl;
  size_t off = 0;
  auto add = [&](void **p, size_t bytes) {
    off = round_up(off, 256);
    sl.push_back({p, bytes, off});
    off += std::max<size_t>(bytes, 16);
  };
  const size_t n = (size_t)d.n * 4;
  add((void **)&P.X, n);
  add((void **)&P.R, n);
  add((void **)&P.T, n);
  add((void **)&P.F, n);
  add((void **)&P.proj, m->proj_rows * 4);
  add((void **)&P.Y, n);
  add((void **)&P.FF, 2 * (size_t)d.nffl * 4);
  add((void **)&P.q, (size_t)d.nhl * d.hdv * 4);
  add((void **)&P.scores, (size_t)d.nhl * s->ctx_len * 4);
  add((void **)&P.part, (size_t)d.nhl * s->nsplit * d.hdv * sizeof(double2));
  add((void **)&P.logits, (size_t)(d.v1 - d.v0) * 4);
  add((void **)&P.pos, 4);
  P.ss = round_up(off, 4096);
  const size_t spans = (size_t)std::max(d.n, d.nff) / 256;
  const size_t img_bytes = spans * kPrefillNsg * kBImgBlock;
  const size_t extra = kPrefillLanes * 4 + img_bytes;
  cudaError_t e = cudaMalloc(&P.arena, P.ss * kPrefillLanes + extra);
  if (e == cudaSuccess) e = cudaMemset(P.arena, 0, P.ss * kPrefillLanes + extra);
  if (e != cudaSuccess) {
    if (P.arena) cudaFree(P.arena);
    P.arena = nullptr;
    return cuda_error(e, "qwen35_prefill: workspace");
  }
  for (auto &x : sl) *x.p = P.arena + x.off;
  P.tok = reinterpret_cast<uint32_t *>(P.arena + P.ss * kPrefillLanes);
  P.bimg = P.arena + P.ss * kPrefillLanes + kPrefillLanes * 4;
  s->bufs.push_back(P.arena);
  // the batched GEMV's operands of the Q6_K projections, its kernels' attributes
  std::vector<unltd_weight_s *> ws{m->output};
  for (const Layer &L : m->layers) {
    ws.insert(ws.end(), L.in.w.begin(), L.in.w.end());
    ws.insert(ws.end(), L.gate_up.w.begin(), L.gate_up.w.end());
    ws.push_back(L.out);
    ws.push_back(L.down);
  }
  int32_t rc = cuda_error(gemv_batch_prewarm(m->ctx->device), "batched GEMV attributes");
  if (!rc)
    for (auto fn : {recr_chunk_kernel<128, 4>, recr_chunk_kernel<128, 0>})
      if (!rc)
        rc = cuda_error(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)sizeof(RecrChunkSmem<128>)),
                        "prefill recurrence attributes");
  for (auto *w : ws)
    if (!rc) rc = gemv_batch_prepare(m->ctx, w);
  return rc;
}

// Enqueue one prefill chunk of T tokens (already in pf.tok): the tokens'
// projections as batched GEMVs (one pass over every weight for the chunk),
// the norms, SwiGLU and attention batched over the tokens (attention shares
// the session's cache: token t attends to positions <= its own, whose K/V
// rows the chunk's attn_pre wrote first), the recurrent kernel token by token
// on the session's state. Every token's arithmetic is that of a decode step,
// so the state after the chunk, and with `head` the greedy token after it,
// are the bits the one-token steps give. Without `head` the LM head is
// skipped (a prompt's earlier chunks need no logits).
int32_t enqueue_prefill(unltd_qwen35_session s, int T, bool head) {
  unltd_qwen35 m = s->m;
  const Derived &d = m->d;
  auto &P = s->pf;
  cudaStream_t st = s->ctx->stream;
  int32_t rc = UNLTD_OK;
  const unsigned nz = (unsigned)T;
  const size_t pss = P.ss;
  auto chk = [&](cudaError_t e, const char *what) {
    if (!rc) rc = cuda_error(e, what);
  };
  auto lane = [&](auto *p, int t) {
    return reinterpret_cast<decltype(p)>(reinterpret_cast<uint8_t *>(p) + (size_t)t * pss);
  };
  auto norm = [&](const float *a, const float *b, float *r_out, const float *w) {
    NormArgs p{a, b, r_out, w, d.n, d.eps, nullptr, nullptr, nullptr, nullptr};
    p.ss = pss;
    p.bimg = P.bimg;
    p.nsg = kPrefillNsg;
    chk(launch_pdl(norm_quant_kernel, dim3(d.n / 256, 1, nz), dim3(256), 0, st, p), "prefill norm");
  };
  auto gemv = [&](const unltd_weight_s *w, float *y) {
    BatchGemvArgs b{w};
    b.img = P.bimg;
    b.nsg = kPrefillNsg;
    b.y = y;
    b.ystride = pss / 4;
    b.nseq = T;
    if (!rc) rc = gemv_batch_launch(s->ctx, b);
  };
  auto norm_proj = [&](const float *a, const float *b, float *r_out, const float *w, const Proj &p, float *out) {
    norm(a, b, r_out, w);
    for (size_t i = 0; i < p.w.size(); i++) gemv(p.w[i], out + p.off[i]);
  };
  chk(launch_pdl(prefill_begin_kernel, dim3(1), dim3(32), 0, st, (const int *)s->pos, P.pos, pss, T), "prefill");
  chk(launch_pdl(embed_q4k_kernel, dim3(d.n / 256, 1, nz), dim3(256), 0, st, (const uint8_t *)m->embd->dev,
                 m->embd->row_stride, m->embd->nb, (const uint32_t *)P.tok, (uint32_t)d.vocab, P.X, d.n,
                 s->ctx->err, pss, (size_t)4),
      "prefill embed");
  for (int il = 0; il < d.n_layer; il++) {
    const Layer &L = m->layers[il];
    if (il == 0) norm_proj(P.X, nullptr, nullptr, L.attn_norm, L.in, P.proj);
    else norm_proj(P.R, P.F, P.X, L.attn_norm, L.in, P.proj);
    if (!L.attn) {
      // the recurrence: the chunk's tokens in order inside one launch, on the session's state
      RecrChunkArgs c;
      RecrArgs &a = c.r;
      a.proj = P.proj;
      a.ring = s->ring[L.slot];
      a.convw = L.convw;
      a.dt_bias = L.dt_bias;
      a.ssm_a = L.ssm_a;
      a.ssm_norm = L.ssm_norm;
      a.state = s->state[L.slot];
      a.y = P.Y;
      a.pos = s->pos;
      a.K = d.K;
      a.nqk = d.nqkl;
      a.nv = d.nvl;
      a.dconv = d.dconvl;
      a.z_off = d.dconvl;
      a.beta_off = d.dconvl + d.nvl * d.hd;
      a.alpha_off = a.beta_off + d.nvl;
      a.eps = d.eps;
      a.span_ctr = nullptr;
      a.img4 = nullptr;
      a.img6 = nullptr;
      a.ss = 0;
      a.bimg = P.bimg;
      a.nsg = kPrefillNsg;
      c.pss = pss;
      c.T = T;
      chk(launch_pdl(d.K == 4 ? recr_chunk_kernel<128, 4> : recr_chunk_kernel<128, 0>, dim3(d.nvl, 128 / kGdnCols),
                     dim3(128), sizeof(RecrChunkSmem<128>), st, c),
          "prefill recurrence");
      chk(launch_pdl(prefill_gnorm_kernel<128>, dim3(d.nvl * d.hd / 256, T), dim3(128), 0, st, (const float *)P.Y,
                     (const float *)P.proj, pss, d.dconvl, (const float *)L.ssm_norm, d.eps, P.bimg, kPrefillNsg),
          "prefill gated norm");
      const int nring = std::min(T, d.K) * d.dconvl;
      chk(launch_pdl(prefill_ring_kernel, dim3((nring + 255) / 256), dim3(256), 0, st, (const float *)P.proj, pss, T,
                     s->ring[L.slot], d.dconvl, d.K, (const int *)s->pos),
          "prefill ring");
    } else {
      AttnArgs a;
      a.qk = P.proj;
      a.v = P.proj + 2 * d.nhl * d.hdv + d.kvlenl;
      a.q_norm = L.q_norm;
      a.k_norm = L.k_norm;
      a.rope = s->rope;
      a.q = P.q;
      a.kcache = s->kc[L.slot];
      a.vcache = s->vc[L.slot];
      a.scores = P.scores;
      a.part = P.part;
      a.img4 = nullptr;
      a.img6 = nullptr;
      a.pos = P.pos;
      a.nh = d.nhl;
      a.nkv = d.nkvl;
      a.n_rot = d.n_rot;
      a.nrp = d.nrp;
      a.ctx = s->ctx_len;
      a.nsplit = s->nsplit;
      a.eps = d.eps;
      a.kq_scale = d.kq_scale;
      a.ss = pss;
      a.kv_ss = 0;  // one cache for the chunk's tokens
      a.bimg = P.bimg;
      a.nsg = kPrefillNsg;
      const dim3 sg(d.nkvl, (s->ctx_len + 31) / 32, nz), vg(d.nkvl, s->nsplit, nz);
      const size_t q_smem = (size_t)(d.nhl / d.nkvl) * d.hdv * 8, v_smem = (size_t)kChunk * d.hdv * 4;
      const size_t sm_smem = softmax_smem(s->ctx_len);
      const dim3 cg(d.nhl * d.hdv / 256, 1, nz), pg(d.nhl + d.nkvl, 1, nz), smg(d.nhl, 1, nz);
      if (d.hdv == 256) {
        chk(launch_pdl(attn_pre_kernel<256>, pg, dim3(256), 0, st, a), "attn_pre");
        chk(launch_pdl(attn_scores_kernel<256>, sg, dim3(256), q_smem, st, a), "attn_scores");
        chk(launch_pdl(attn_softmax_kernel, smg, dim3(256), sm_smem, st, a), "attn_softmax");
        chk(launch_pdl(attn_values_kernel<256>, vg, dim3(256), v_smem, st, a), "attn_values");
        chk(launch_pdl(attn_combine_quant_kernel<256>, cg, dim3(256), 0, st, a), "attn_combine");
      } else {
        chk(launch_pdl(attn_pre_kernel<128>, pg, dim3(128), 0, st, a), "attn_pre");
        chk(launch_pdl(attn_scores_kernel<128>, sg, dim3(256), q_smem, st, a), "attn_scores");
        chk(launch_pdl(attn_softmax_kernel, smg, dim3(256), sm_smem, st, a), "attn_softmax");
        chk(launch_pdl(attn_values_kernel<128>, vg, dim3(128), v_smem, st, a), "attn_values");
        chk(launch_pdl(attn_combine_quant_kernel<128>, cg, dim3(256), 0, st, a), "attn_combine");
      }
    }
    gemv(L.out, P.T);
    norm_proj(P.X, P.T, P.R, L.post_norm, L.gate_up, P.FF);
    chk(launch_pdl(swiglu_quant_kernel, dim3(d.nffl / 256, 1, nz), dim3(256), 0, st, (const float *)P.FF,
                   (const float *)(P.FF + d.nffl), (uint8_t *)nullptr, (uint8_t *)nullptr, pss, P.bimg,
                   kPrefillNsg),
        "prefill swiglu");
    gemv(L.down, P.F);
  }
  const uint32_t *last = nullptr;
  if (head) {
    // l_out -> output norm -> LM head + greedy argmax of every token (the last one's is kept)
    norm(P.R, P.F, P.X, m->out_norm);
    BatchGemvArgs b{m->output};
    b.img = P.bimg;
    b.nsg = kPrefillNsg;
    b.y = P.logits;
    b.ystride = pss / 4;
    b.nseq = T;
    b.key = s->ctx->bkey;
    b.done = s->ctx->bdone;
    b.token = P.tok;
    b.tstride = 1;
    if (!rc) rc = gemv_batch_launch(s->ctx, b);
    last = P.tok + (T - 1);
    // the last token's hidden state and logits where session_read finds them
    chk(cudaMemcpyAsync(s->X, lane(P.X, T - 1), (size_t)d.n * 4, cudaMemcpyDeviceToDevice, st), "prefill");
    chk(cudaMemcpyAsync(s->logits, lane(P.logits, T - 1), (size_t)(d.v1 - d.v0) * 4, cudaMemcpyDeviceToDevice, st),
        "prefill");
  }
  chk(launch_pdl(prefill_end_kernel, dim3(1), dim3(1), 0, st, s->pos, T, s->cur_token, last), "prefill end");
  return rc;
}

}  // namespace

namespace {
// Per-sequence buffers of a session laid out in one arena: offsets of every
// buffer (256-byte aligned), then one allocation of n_seq arenas.
struct ArenaPlan {
  size_t bytes = 0;
  std::vector<std::pair<void **, size_t>> slots;
  template <class T>
  void add(T **p, size_t n) {
    bytes = round_up(bytes, 256);
    slots.push_back({reinterpret_cast<void **>(p), bytes});
    bytes += std::max<size_t>(n * sizeof(T), 16);
  }
};

// Sequence seq's copy of a per-sequence buffer of s.
template <class T>
T *seq_buf(unltd_qwen35_session s, T *p, int seq) {
  return reinterpret_cast<T *>(reinterpret_cast<uint8_t *>(p) + (size_t)seq * s->ss);
}

}  // namespace

extern "C" {

int32_t unltd_qwen35_create_tp(unltd_ctx ctx, const unltd_qwen35_config *cfg, int32_t rank, int32_t world,
                               unltd_qwen35 *out) {
  if (!ctx || !cfg || !out) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_create: NULL argument");
  *out = nullptr;
  Derived d;
  if (int32_t rc = derive(*cfg, &d)) return rc;
  if (int32_t rc = derive_tp(&d, rank, world)) return rc;
  if (world > 1 && (!ctx->comm || ctx->rank != rank || ctx->world != world))
    return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_create_tp: the context needs a communicator of this rank/world "
                                            "(unltd_comm_init)");
  unltd_qwen35 m = new unltd_qwen35_s();
  m->ctx = ctx;
  m->cfg = *cfg;
  m->d = d;
  *out = m;
  return UNLTD_OK;
}

int32_t unltd_qwen35_create(unltd_ctx ctx, const unltd_qwen35_config *cfg, unltd_qwen35 *out) {
  return unltd_qwen35_create_tp(ctx, cfg, 0, 1, out);
}

int32_t unltd_qwen35_shard(const unltd_qwen35_config *cfg, int32_t rank, int32_t world, const char *name,
                           int64_t *ranges, int32_t max_ranges, int32_t *n_ranges, int64_t *in_begin,
                           int64_t *in_end) {
  if (!cfg || !name || !n_ranges || !in_begin || !in_end || (max_ranges > 0 && !ranges))
    return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_shard: NULL argument");
  Derived d;
  if (int32_t rc = derive(*cfg, &d)) return rc;
  if (int32_t rc = derive_tp(&d, rank, world)) return rc;
  for (const auto &p : expected(d)) {
    if (p.name != name) continue;
    const Shard sh = shard_of(d, p.name, p.dim_in, p.dim_out);
    *n_ranges = (int32_t)sh.rows.size();
    if ((int32_t)sh.rows.size() > max_ranges) return set_error(UNLTD_ERR_LENGTH, "qwen35_shard: too many ranges");
    for (size_t i = 0; i < sh.rows.size(); i++) {
      ranges[2 * i] = (int64_t)sh.rows[i].first;
      ranges[2 * i + 1] = (int64_t)sh.rows[i].second;
    }
    *in_begin = (int64_t)sh.in0;
    *in_end = (int64_t)sh.in1;
    return UNLTD_OK;
  }
  return set_error(UNLTD_ERR_INVALID_ARG, std::string("qwen35_shard: unexpected tensor '") + name + "'");
}

int32_t unltd_qwen35_set_tensor(unltd_qwen35 m, const char *name, const void *host, size_t nbytes, int32_t dtype) {
  if (!m || !name || !host) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_set_tensor: NULL argument");
  if (m->finalized) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_set_tensor: model already finalized");
  const std::vector<Part> parts = expected(m->d);
  const Part *pt = nullptr;
  for (const auto &p : parts)
    if (p.name == name) pt = &p;
  if (!pt) return set_error(UNLTD_ERR_INVALID_ARG, std::string("qwen35_set_tensor: unexpected tensor '") + name + "'");
  bool ok = false;
  for (int t : pt->dtypes) ok |= t == dtype;
  if (!ok)
    return set_error(UNLTD_ERR_UNSUPPORTED,
                     std::string("tensor '") + name + "': dtype " + dtype_str(dtype) + " not accepted");
  const size_t want = gguf_row_bytes(dtype, pt->dim_in) * pt->dim_out;
  if (nbytes != want)
    return set_error(UNLTD_ERR_LENGTH, std::string("tensor '") + name + "': " + std::to_string(nbytes) +
                                           " bytes, expected " + std::to_string(want));
  CtxGuard g(m->ctx->device);
  Staged s;
  s.dtype = dtype;
  auto it = m->staged.find(name);
  if (it != m->staged.end()) {
    if (it->second.w) unltd_weight_free(it->second.w);
    if (it->second.f) cudaFree(it->second.f);
    m->staged.erase(it);
  }
  const Shard sh = shard_of(m->d, pt->name, pt->dim_in, pt->dim_out);
  const uint8_t *src = static_cast<const uint8_t *>(host);
  if (dtype == F32) {
    const std::vector<uint8_t> loc = gather_shard(sh, src, 4, 1, 4);
    cudaError_t e = cudaMalloc(&s.f, std::max<size_t>(loc.size(), 16));
    if (e == cudaSuccess) e = cudaMemcpy(s.f, loc.data(), loc.size(), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_error(e, "qwen35_set_tensor");
  } else if (m->d.world == 1) {
    int32_t rc = unltd_weight_upload(m->ctx, host, nbytes, dtype, pt->dim_in, pt->dim_out, &s.w);
    if (rc) return rc;
  } else {
    const size_t epb = dtype == Q8_0 ? kQ80Elems : kQK;
    const size_t bb = gguf_row_bytes(dtype, epb);
    const std::vector<uint8_t> loc = gather_shard(sh, src, gguf_row_bytes(dtype, pt->dim_in), epb, bb);
    int32_t rc = unltd_weight_upload(m->ctx, loc.data(), loc.size(), dtype, sh.in1 - sh.in0, sh.nrows(), &s.w);
    if (rc) return rc;
  }
  m->staged[name] = s;
  return UNLTD_OK;
}

// Every tensor Qwen35Forward::open checks (qwen35_forward.rs:139-232), taken
// from the GGUF mapping: a weight must be 2-D with ne = [dim_in, dim_out], a
// vector (norms, conv taps, dt bias, A) must hold dim_in elements; dtype and
// byte count are checked again by set_tensor.
int32_t unltd_qwen35_load_gguf(unltd_qwen35 m, unltd_gguf g) {
  if (!m || !g) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_load_gguf: NULL argument");
  if (m->finalized) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_load_gguf: model already finalized");
  for (const Part &p : expected(m->d)) {
    GgufTensorView t;
    if (!gguf_tensor(g, p.name, &t)) return set_error(UNLTD_ERR_INVALID_ARG, "gguf: missing tensor '" + p.name + "'");
    if (!t.data)
      return set_error(UNLTD_ERR_UNSUPPORTED, "gguf: tensor '" + p.name + "' has a type this path does not read");
    const int64_t nel = t.ne[0] * t.ne[1] * t.ne[2] * t.ne[3];
    const bool shape_ok = p.dim_out > 1 ? (t.ndims == 2 && t.ne[0] == (int64_t)p.dim_in && t.ne[1] == (int64_t)p.dim_out)
                                        : nel == (int64_t)p.dim_in;
    if (!shape_ok) return set_error(UNLTD_ERR_LENGTH, "gguf: tensor '" + p.name + "' has the wrong shape");
    if (int32_t rc = unltd_qwen35_set_tensor(m, p.name.c_str(), t.data, t.nbytes, t.dtype)) return rc;
  }
  return unltd_qwen35_finalize(m);
}

int32_t unltd_qwen35_finalize(unltd_qwen35 m) {
  if (!m) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_finalize: NULL model");
  if (m->finalized) return UNLTD_OK;
  const Derived &d = m->d;
  for (const auto &p : expected(d))
    if (!m->staged.count(p.name)) return set_error(UNLTD_ERR_INVALID_ARG, "missing tensor '" + p.name + "'");
  CtxGuard g(m->ctx->device);
  auto take_f = [&](const std::string &nm) {
    float *f = m->staged.at(nm).f;
    m->staged.at(nm).f = nullptr;
    m->f32_bufs.push_back(f);
    return f;
  };
  auto take_w = [&](const std::string &nm) {
    unltd_weight_s *w = m->staged.at(nm).w;
    m->staged.at(nm).w = nullptr;
    return w;
  };
  m->embd = take_w("token_embd.weight");
  m->output = take_w("output.weight");
  m->out_norm = take_f("output_norm.weight");
  m->layers.resize(d.n_layer);
  size_t proj_rows = 0;
  for (int il = 0; il < d.n_layer; il++) {
    Layer &L = m->layers[il];
    const std::string p = "blk." + std::to_string(il) + ".";
    L.attn = is_attn(d, il);
    L.slot = L.attn ? m->n_attn++ : m->n_recr++;
    L.attn_norm = take_f(p + "attn_norm.weight");
    L.post_norm = take_f(p + "post_attention_norm.weight");
    int32_t rc;
    if (L.attn) {
      rc = build_proj(m, {p + "attn_q.weight", p + "attn_k.weight", p + "attn_v.weight"}, &L.in);
      L.q_norm = take_f(p + "attn_q_norm.weight");
      L.k_norm = take_f(p + "attn_k_norm.weight");
      L.out = take_w(p + "attn_output.weight");
    } else {
      rc = build_proj(m, {p + "attn_qkv.weight", p + "attn_gate.weight", p + "ssm_beta.weight", p + "ssm_alpha.weight"},
                      &L.in);
      L.convw = take_f(p + "ssm_conv1d.weight");
      L.dt_bias = take_f(p + "ssm_dt.bias");
      L.ssm_a = take_f(p + "ssm_a");
      L.ssm_norm = take_f(p + "ssm_norm.weight");
      L.out = take_w(p + "ssm_out.weight");
    }
    if (rc) return rc;
    if ((rc = build_proj(m, {p + "ffn_gate.weight", p + "ffn_up.weight"}, &L.gate_up))) return rc;
    L.down = take_w(p + "ffn_down.weight");
    proj_rows = std::max(proj_rows, L.in.rows);
  }
  m->proj_rows = proj_rows;
  m->staged.clear();
  m->finalized = true;
  return UNLTD_OK;
}

int32_t unltd_qwen35_destroy(unltd_qwen35 m) {
  if (!m) return UNLTD_OK;
  CtxGuard g(m->ctx->device);
  cudaStreamSynchronize(m->ctx->stream);
  for (auto &kv : m->staged) {
    if (kv.second.w) unltd_weight_free(kv.second.w);
    if (kv.second.f) cudaFree(kv.second.f);
  }
  for (auto &L : m->layers) {
    for (auto *w : L.in.w) unltd_weight_free(w);
    for (auto *w : L.gate_up.w) unltd_weight_free(w);
    unltd_weight_free(L.out);
    unltd_weight_free(L.down);
  }
  unltd_weight_free(m->embd);
  unltd_weight_free(m->output);
  for (void *p : m->f32_bufs) cudaFree(p);
  delete m;
  return UNLTD_OK;
}

int32_t unltd_qwen35_session_destroy(unltd_qwen35_session s);


int32_t unltd_qwen35_session_create_batch(unltd_qwen35 m, int32_t ctx_len, int32_t n_seq,
                                          unltd_qwen35_session *out) {
  if (!m || !out) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_session_create: NULL argument");
  *out = nullptr;
  if (!m->finalized) {
    if (int32_t rc = unltd_qwen35_finalize(m)) return rc;
  }
  if (ctx_len < 1 || ctx_len > 16384)
    return set_error(UNLTD_ERR_UNSUPPORTED, "qwen35_session_create: ctx must be in [1, 16384]");
  if (n_seq < 1 || n_seq > kMaxBatch)
    return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_session_create: n_seq must be in [1, 32]");
  const Derived &d = m->d;
  if (n_seq > 1 && d.world > 1 && (size_t)n_seq * d.n > kPeerMaxCount)
    return set_error(UNLTD_ERR_UNSUPPORTED, "qwen35_session_create: batch too large for the tensor-parallel sum");
  if (n_seq > 1) {  // every projection must have a batched GEMV
    auto ok = [&](const unltd_weight_s *w) { return gemv_batch_supported(m->ctx->device, *w); };
    bool all = ok(m->output);
    for (const Layer &L : m->layers) {
      for (auto *w : L.in.w) all &= ok(w);
      for (auto *w : L.gate_up.w) all &= ok(w);
      all &= ok(L.out) && ok(L.down);
    }
    if (!all) return set_error(UNLTD_ERR_UNSUPPORTED, "qwen35_session_create: a projection has no batched GEMV");
  }
  unltd_qwen35_session s = new unltd_qwen35_session_s();
  s->m = m;
  s->ctx_len = ctx_len;
  s->nseq = n_seq;
  s->seq_pos.assign(n_seq, 0);
  int32_t rc = unltd_ctx_create(m->ctx->device, &s->ctx);
  if (rc) {
    delete s;
    return rc;
  }
  CtxGuard g(m->ctx->device);
  auto &B = s->bufs;
  const size_t n = d.n;
  s->nsplit = (ctx_len + kChunk - 1) / kChunk;
  const size_t spans = (size_t)std::max(d.n, d.nff) / 256;
  ArenaPlan A;
  A.add(&s->X, n);
  A.add(&s->R, n);
  A.add(&s->T, n);
  A.add(&s->F, n);
  A.add(&s->proj, m->proj_rows);
  A.add(&s->Y, n);
  A.add(&s->FF, 2 * (size_t)d.nffl);
  A.add(&s->q, (size_t)d.nhl * d.hdv);
  A.add(&s->scores, (size_t)d.nhl * ctx_len);
  A.add(&s->part, (size_t)d.nhl * s->nsplit * d.hdv);
  A.add(&s->tpkey, 1);
  A.add(&s->img4, spans * kImgQ8K4);
  A.add(&s->img6, spans * kImgQ8K6);
  A.add(&s->logits, (size_t)(d.v1 - d.v0));
  A.add(&s->cur_token, 1);
  A.add(&s->hist, (size_t)ctx_len + 1);
  A.add(&s->feed, (size_t)ctx_len + 1);
  A.add(&s->counter, 1);
  A.add(&s->pos, 1);
  A.add(&s->span_ctr, (size_t)d.nvl * d.hd / 256 + 1);
  s->ring.assign(m->n_recr, nullptr);
  s->state.assign(m->n_recr, nullptr);
  s->kc.assign(m->n_attn, nullptr);
  s->vc.assign(m->n_attn, nullptr);
  for (int i = 0; i < m->n_recr; i++) {
    A.add(&s->ring[i], (size_t)d.K * d.dconvl);
    A.add(&s->state[i], (size_t)d.nvl * d.hd * d.hd);
  }
  for (int i = 0; i < m->n_attn; i++) {
    A.add(&s->kc[i], (size_t)ctx_len * d.kvlenl);
    A.add(&s->vc[i], (size_t)ctx_len * d.kvlenl);
  }
  s->ss = round_up(A.bytes, 4096);
  // everything starts at zero: token, step counter, position, span counters,
  // conv windows, GDN states and caches
  rc = dalloc(B, &s->arena, s->ss * (size_t)n_seq, "session arena");
  if (!rc) rc = cuda_error(cudaMemset(s->arena, 0, s->ss * (size_t)n_seq), "session init");
  if (!rc)
    for (auto &sl : A.slots) *sl.first = s->arena + sl.second;
  if (!rc) rc = dalloc(B, &s->rope, (size_t)ctx_len * std::max(d.nrp, 1), "session");
  if (!rc && n_seq > 1) {
    s->nsg = (n_seq + 7) / 8;
    rc = dalloc(B, &s->bimg, spans * s->nsg * kBImgBlock, "session batched images");
  }
  if (!rc && n_seq > 1 && d.world > 1) {
    rc = dalloc(B, &s->tpbuf, (size_t)n_seq * d.n, "session tensor-parallel sums");
    if (!rc) rc = dalloc(B, &s->tpkeys, (size_t)n_seq, "session tensor-parallel keys");
    if (!rc) rc = cuda_error(cudaMemset(s->tpbuf, 0, (size_t)n_seq * d.n * 4), "session init");
  }
  // IMROPE angles (kernels.rs:381-400): angle = pos * theta^ic by repeated
  // multiplication; (cos, sin) of the rotated pairs ic % 3 == 0, from libm.
  if (!rc && d.nrp > 0) {
    std::vector<double2> tab((size_t)ctx_len * d.nrp);
    for (int p = 0; p < ctx_len; p++) {
      double angle = (double)p;
      for (int ic = 0; ic < d.n_rot / 2; ic++) {
        if (ic % 3 == 0) tab[(size_t)p * d.nrp + ic / 3] = make_double2(std::cos(angle), std::sin(angle));
        angle *= d.theta_scale;
      }
    }
    rc = cuda_error(cudaMemcpy(s->rope, tab.data(), tab.size() * sizeof(double2), cudaMemcpyHostToDevice), "rope table");
  }
  // GEMV scratch (the projections that still run a prep kernel) sized before
  // any graph capture
  if (!rc) {
    const int sm_smem = (int)softmax_smem(ctx_len);
    cudaError_t e = cudaFuncSetAttribute(attn_softmax_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sm_smem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attn_values_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, kChunk * 256 * 4);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attn_values_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, kChunk * 128 * 4);
    rc = cuda_error(e, "attention smem");
  }
  if (!rc && n_seq > 1) rc = cuda_error(gemv_batch_prewarm(m->ctx->device), "batched GEMV attributes");
  if (!rc && n_seq > 1) {  // the batched GEMV's operands of the Q6_K projections
    std::vector<unltd_weight_s *> ws{m->output};
    for (const Layer &L : m->layers) {
      ws.insert(ws.end(), L.in.w.begin(), L.in.w.end());
      ws.insert(ws.end(), L.gate_up.w.begin(), L.gate_up.w.end());
      ws.push_back(L.out);
      ws.push_back(L.down);
    }
    for (auto *w : ws)
      if (!rc) rc = gemv_batch_prepare(m->ctx, w);
  }
  if (!rc) rc = cuda_error(cudaDeviceSynchronize(), "session init");
  if (!rc && d.world > 1) {
    // set up NCCL's connections for both collectives of a step before any
    // graph capture (its lazy set-up allocates)
    rc = cuda_error(cudaMemset(s->T, 0, (size_t)d.n * 4), "session init");
    if (!rc) rc = cuda_error(cudaMemset(s->tpkey, 0, 8), "session init");
    if (!rc) rc = comm_allreduce(m->ctx, s->ctx->stream, s->T, (size_t)d.n, false);
    if (!rc) rc = comm_allreduce(m->ctx, s->ctx->stream, s->tpkey, 1, true);
    if (!rc && n_seq > 1) {  // a batch's collectives too
      rc = comm_allreduce(m->ctx, s->ctx->stream, s->tpbuf, (size_t)n_seq * d.n, false);
      if (!rc) rc = cuda_error(cudaMemset(s->tpkeys, 0, (size_t)n_seq * 8), "session init");
      if (!rc) rc = comm_allreduce(m->ctx, s->ctx->stream, s->tpkeys, (size_t)n_seq, true);
    }
    if (!rc) rc = cuda_error(cudaStreamSynchronize(s->ctx->stream), "session init");
  }
  if (rc) {
    unltd_qwen35_session_destroy(s);
    return rc;
  }
  *out = s;
  return UNLTD_OK;
}

int32_t unltd_qwen35_session_create(unltd_qwen35 m, int32_t ctx_len, unltd_qwen35_session *out) {
  return unltd_qwen35_session_create_batch(m, ctx_len, 1, out);
}

int32_t unltd_qwen35_session_destroy(unltd_qwen35_session s) {
  if (!s) return UNLTD_OK;
  CtxGuard g(s->m->ctx->device);
  if (s->ctx) cudaStreamSynchronize(s->ctx->stream);
  if (s->graph) cudaGraphExecDestroy(s->graph);
  for (void *p : s->bufs) cudaFree(p);
  if (s->ctx) unltd_ctx_destroy(s->ctx);
  delete s;
  return UNLTD_OK;
}

// The rank's conv channels, in its local order: [q of the local qk heads |
// k of the local qk heads | v of the local v heads] (the sharded qkv rows).
std::vector<std::pair<size_t, size_t>> conv_channel_ranges(const Derived &d) {
  std::vector<std::pair<size_t, size_t>> r;
  const size_t hd = d.hd;
  for (int part = 0; part < 2; part++)
    for (int j = 0; j < d.nqkl; j++) {
      const size_t gq = (size_t)((d.vh0 + j) % d.nqk) + (size_t)part * d.nqk;
      r.push_back({gq * hd, (gq + 1) * hd});
    }
  r.push_back({2 * (size_t)d.nqk * hd + (size_t)d.vh0 * hd, 2 * (size_t)d.nqk * hd + (size_t)(d.vh0 + d.nvl) * hd});
  return r;
}

int32_t unltd_qwen35_batch_set_state(unltd_qwen35_session s, int32_t seq, int32_t position, const float *const *conv,
                                     const float *const *gdn, const float *const *kcache,
                                     const float *const *vcache) {
  if (!s) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_set_state: NULL session");
  if (seq < 0 || seq >= s->nseq) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_set_state: sequence out of range");
  if (position < 0 || position >= s->ctx_len)
    return set_error(UNLTD_ERR_LENGTH, "qwen35_set_state: position outside the context");
  const Derived &d = s->m->d;
  auto ring = [&](int i) { return seq_buf(s, s->ring[i], seq); };
  auto state = [&](int i) { return seq_buf(s, s->state[i], seq); };
  auto kc = [&](int i) { return seq_buf(s, s->kc[i], seq); };
  auto vc = [&](int i) { return seq_buf(s, s->vc[i], seq); };
  CtxGuard g(s->m->ctx->device);
  cudaStream_t st = s->ctx->stream;
  cudaError_t e = cudaStreamSynchronize(st);
  const auto chans = conv_channel_ranges(d);
  std::vector<float> row((size_t)d.dconvl);
  for (int i = 0; e == cudaSuccess && i < s->m->n_recr; i++) {
    e = cudaMemset(ring(i), 0, (size_t)d.K * d.dconvl * 4);
    // row tau of the window (oldest first) lives in slot (position + tau) % K
    for (int tau = 0; e == cudaSuccess && conv && conv[i] && tau < d.K - 1; tau++) {
      size_t o = 0;
      for (auto &c : chans)
        for (size_t ch = c.first; ch < c.second; ch++) row[o++] = conv[i][(size_t)tau * d.dconv + ch];
      e = cudaMemcpy(ring(i) + (size_t)((position + tau) % d.K) * d.dconvl, row.data(), (size_t)d.dconvl * 4,
                     cudaMemcpyHostToDevice);
    }
    const size_t hh = (size_t)d.hd * d.hd;
    if (e == cudaSuccess) {
      if (gdn && gdn[i]) e = cudaMemcpy(state(i), gdn[i] + (size_t)d.vh0 * hh, (size_t)d.nvl * hh * 4, cudaMemcpyHostToDevice);
      else e = cudaMemset(state(i), 0, (size_t)d.nvl * hh * 4);
    }
  }
  for (int i = 0; e == cudaSuccess && i < s->m->n_attn; i++) {
    const size_t full = (size_t)s->ctx_len * d.kvlenl * 4;
    e = cudaMemset(kc(i), 0, full);
    if (e == cudaSuccess) e = cudaMemset(vc(i), 0, full);
    const size_t col0 = (size_t)d.kv0 * d.hdv;  // the local kv heads' columns of each full row
    if (e == cudaSuccess && position && kcache && kcache[i])
      e = cudaMemcpy2D(kc(i), (size_t)d.kvlenl * 4, kcache[i] + col0, (size_t)d.kvlen * 4, (size_t)d.kvlenl * 4,
                       (size_t)position, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && position && vcache && vcache[i])
      e = cudaMemcpy2D(vc(i), (size_t)d.kvlenl * 4, vcache[i] + col0, (size_t)d.kvlen * 4, (size_t)d.kvlenl * 4,
                       (size_t)position, cudaMemcpyHostToDevice);
  }
  if (e == cudaSuccess) e = cudaMemcpy(seq_buf(s, s->pos, seq), &position, 4, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_error(e, "qwen35_set_state");
  s->seq_pos[seq] = position;
  if (seq == 0) s->host_pos = position;
  return UNLTD_OK;
}

int32_t unltd_qwen35_session_set_state(unltd_qwen35_session s, int32_t position, const float *const *conv,
                                       const float *const *gdn, const float *const *kcache,
                                       const float *const *vcache) {
  return unltd_qwen35_batch_set_state(s, 0, position, conv, gdn, kcache, vcache);
}

// Copy the session state out at the current position: per recurrent layer
// the conv window ((K-1) x local channels, oldest row first) and the local
// GDN matrices, per attention layer `position` rows of the local K and V
// columns. With one GPU this is exactly the layout set_state takes.
int32_t unltd_qwen35_batch_get_state(unltd_qwen35_session s, int32_t seq, float *const *conv, float *const *gdn,
                                     float *const *kcache, float *const *vcache) {
  if (!s) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_get_state: NULL session");
  if (seq < 0 || seq >= s->nseq) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_get_state: sequence out of range");
  const Derived &d = s->m->d;
  CtxGuard g(s->m->ctx->device);
  cudaError_t e = cudaStreamSynchronize(s->ctx->stream);
  const int position = s->seq_pos[seq];
  for (int i = 0; e == cudaSuccess && i < s->m->n_recr; i++) {
    const float *ring = seq_buf(s, s->ring[i], seq);
    for (int tau = 0; e == cudaSuccess && conv && conv[i] && tau < d.K - 1; tau++)
      e = cudaMemcpy(conv[i] + (size_t)tau * d.dconvl, ring + (size_t)((position + tau) % d.K) * d.dconvl,
                     (size_t)d.dconvl * 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && gdn && gdn[i])
      e = cudaMemcpy(gdn[i], seq_buf(s, s->state[i], seq), (size_t)d.nvl * d.hd * d.hd * 4, cudaMemcpyDeviceToHost);
  }
  for (int i = 0; e == cudaSuccess && i < s->m->n_attn; i++) {
    const size_t part = (size_t)position * d.kvlenl * 4;
    if (part && kcache && kcache[i]) e = cudaMemcpy(kcache[i], seq_buf(s, s->kc[i], seq), part, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && part && vcache && vcache[i])
      e = cudaMemcpy(vcache[i], seq_buf(s, s->vc[i], seq), part, cudaMemcpyDeviceToHost);
  }
  return cuda_error(e, "qwen35_get_state");
}

int32_t unltd_qwen35_session_get_state(unltd_qwen35_session s, float *const *conv, float *const *gdn,
                                       float *const *kcache, float *const *vcache) {
  return unltd_qwen35_batch_get_state(s, 0, conv, gdn, kcache, vcache);
}

// Element counts of the rank's state pieces and its vocab rows.
int32_t unltd_qwen35_session_shape(unltd_qwen35_session s, int64_t *conv_row, int64_t *gdn_heads,
                                   int64_t *kv_row, int64_t *vocab_begin, int64_t *vocab_end) {
  if (!s) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_session_shape: NULL session");
  const Derived &d = s->m->d;
  if (conv_row) *conv_row = d.dconvl;
  if (gdn_heads) *gdn_heads = d.nvl;
  if (kv_row) *kv_row = d.kvlenl;
  if (vocab_begin) *vocab_begin = d.v0;
  if (vocab_end) *vocab_end = d.v1;
  return UNLTD_OK;
}

// Teacher-forced steps over `tokens` (a prompt); then *next_token = the
// greedy token after the last one (may be NULL).
int32_t unltd_qwen35_feed(unltd_qwen35_session s, const uint32_t *tokens, int32_t n, uint32_t *next_token) {
  if (!s || (!tokens && n > 0)) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_feed: NULL argument");
  if (s->nseq != 1) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_feed: a batch session (use qwen35_batch_decode)");
  if (n < 0 || n > s->ctx_len - s->host_pos)
    return set_error(UNLTD_ERR_LENGTH, "qwen35_feed: context full (" + std::to_string(s->host_pos) + " of " +
                                           std::to_string(s->ctx_len) + " positions used)");
  for (int i = 0; i < n; i++)
    if (tokens[i] >= (uint32_t)s->m->d.vocab)
      return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_feed: token " + std::to_string(tokens[i]) + " outside the vocab");
  CtxGuard g(s->m->ctx->device);
  cudaStream_t st = s->ctx->stream;
  cudaError_t e = cudaSuccess;
  if (n > 0) e = cudaMemcpyAsync(s->feed, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(s->counter, 0, 4, st);
  int32_t rc = cuda_error(e, "qwen35_feed");
  for (int i = 0; !rc && i < n; i++) {
    rc = cuda_error(cudaMemcpyAsync(s->cur_token, s->feed + i, 4, cudaMemcpyDeviceToDevice, st), "qwen35_feed");
    if (!rc) rc = run_step(s);
  }
  if (!rc && next_token && n > 0) rc = cuda_error(cudaMemcpyAsync(next_token, s->cur_token, 4, cudaMemcpyDeviceToHost, st), "qwen35_feed");
  if (!rc) rc = sync_and_check(s->ctx, st, "qwen35_feed");
  if (!rc) {
    s->host_pos += n;
    s->seq_pos[0] = s->host_pos;
  }
  return rc;
}

// A prompt in chunks of up to 32 tokens (enqueue_prefill): the same state,
// logits, hidden state and next token as unltd_qwen35_feed, with every weight
// read once per chunk.
int32_t unltd_qwen35_prefill(unltd_qwen35_session s, const uint32_t *tokens, int32_t n, uint32_t *next_token) {
  if (!s || (!tokens && n > 0)) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_prefill: NULL argument");
  if (s->nseq != 1) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_prefill: a batch session");
  if (s->m->d.world != 1) return set_error(UNLTD_ERR_UNSUPPORTED, "qwen35_prefill: one GPU (use qwen35_feed)");
  if (n < 0 || n > s->ctx_len - s->host_pos)
    return set_error(UNLTD_ERR_LENGTH, "qwen35_prefill: context full (" + std::to_string(s->host_pos) + " of " +
                                           std::to_string(s->ctx_len) + " positions used)");
  for (int i = 0; i < n; i++)
    if (tokens[i] >= (uint32_t)s->m->d.vocab)
      return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_prefill: token " + std::to_string(tokens[i]) + " outside the vocab");
  if (n == 0) return UNLTD_OK;
  CtxGuard g(s->m->ctx->device);
  int32_t rc = prefill_alloc(s);
  cudaStream_t st = s->ctx->stream;
  for (int i0 = 0; !rc && i0 < n; i0 += kPrefillLanes) {
    const int T = std::min(kPrefillLanes, n - i0);
    rc = cuda_error(cudaMemcpyAsync(s->pf.tok, tokens + i0, (size_t)T * 4, cudaMemcpyHostToDevice, st),
                    "qwen35_prefill");
    if (!rc) rc = enqueue_prefill(s, T, i0 + T == n);  // the next chunk's copy is ordered after it
  }
  if (!rc && next_token) rc = cuda_error(cudaMemcpyAsync(next_token, s->cur_token, 4, cudaMemcpyDeviceToHost, st),
                                         "qwen35_prefill");
  if (!rc) rc = sync_and_check(s->ctx, st, "qwen35_prefill");
  if (!rc) {
    s->host_pos += n;
    s->seq_pos[0] = s->host_pos;
  }
  return rc;
}

// Greedy decode: step 0 consumes `token`; step i > 0 consumes the token step
// i-1 produced. tokens_out[i] = the greedy token of step i.
int32_t unltd_qwen35_decode(unltd_qwen35_session s, uint32_t token, int32_t n_steps, uint32_t *tokens_out) {
  if (!s || (!tokens_out && n_steps > 0)) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_decode: NULL argument");
  if (s->nseq != 1) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_decode: a batch session (use qwen35_batch_decode)");
  if (n_steps < 0 || n_steps > s->ctx_len - s->host_pos)
    return set_error(UNLTD_ERR_LENGTH, "qwen35_decode: context full (" + std::to_string(s->host_pos) + " of " +
                                           std::to_string(s->ctx_len) + " positions used)");
  if (token >= (uint32_t)s->m->d.vocab)
    return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_decode: token " + std::to_string(token) + " outside the vocab");
  CtxGuard g(s->m->ctx->device);
  cudaStream_t st = s->ctx->stream;
  cudaError_t e = cudaMemcpyAsync(s->cur_token, &token, 4, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(s->counter, 0, 4, st);
  int32_t rc = cuda_error(e, "qwen35_decode");
  for (int i = 0; !rc && i < n_steps; i++) rc = run_step(s);
  if (!rc && n_steps > 0)
    rc = cuda_error(cudaMemcpyAsync(tokens_out, s->hist, (size_t)n_steps * 4, cudaMemcpyDeviceToHost, st), "qwen35_decode");
  if (!rc) rc = sync_and_check(s->ctx, st, "qwen35_decode");
  if (!rc) {
    s->host_pos += n_steps;
    s->seq_pos[0] = s->host_pos;
  }
  return rc;
}

// Greedy decode of every sequence of a batch session: step 0 of sequence z
// consumes tokens[z]; tokens_out[z * n_steps + i] = its greedy token of step i.
int32_t unltd_qwen35_batch_decode(unltd_qwen35_session s, const uint32_t *tokens, int32_t n_steps,
                                  uint32_t *tokens_out) {
  if (!s || !tokens || (!tokens_out && n_steps > 0))
    return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_batch_decode: NULL argument");
  int maxpos = 0;
  for (int z = 0; z < s->nseq; z++) maxpos = std::max(maxpos, s->seq_pos[z]);
  if (n_steps < 0 || n_steps > s->ctx_len - maxpos)
    return set_error(UNLTD_ERR_LENGTH, "qwen35_batch_decode: context full (" + std::to_string(maxpos) + " of " +
                                           std::to_string(s->ctx_len) + " positions used)");
  for (int z = 0; z < s->nseq; z++)
    if (tokens[z] >= (uint32_t)s->m->d.vocab)
      return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_batch_decode: token " + std::to_string(tokens[z]) +
                                                  " outside the vocab");
  CtxGuard g(s->m->ctx->device);
  cudaStream_t st = s->ctx->stream;
  cudaError_t e = cudaSuccess;
  for (int z = 0; e == cudaSuccess && z < s->nseq; z++) {
    e = cudaMemcpyAsync(seq_buf(s, s->cur_token, z), tokens + z, 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(seq_buf(s, s->counter, z), 0, 4, st);
  }
  int32_t rc = cuda_error(e, "qwen35_batch_decode");
  for (int i = 0; !rc && i < n_steps; i++) rc = run_step(s);
  for (int z = 0; !rc && n_steps > 0 && z < s->nseq; z++)
    rc = cuda_error(cudaMemcpyAsync(tokens_out + (size_t)z * n_steps, seq_buf(s, s->hist, z), (size_t)n_steps * 4,
                                    cudaMemcpyDeviceToHost, st),
                    "qwen35_batch_decode");
  if (!rc) rc = sync_and_check(s->ctx, st, "qwen35_batch_decode");
  if (!rc) {
    for (int z = 0; z < s->nseq; z++) s->seq_pos[z] += n_steps;
    s->host_pos = s->seq_pos[0];
  }
  return rc;
}

int32_t unltd_qwen35_session_info(unltd_qwen35_session s, int32_t *position, void **stream, int64_t *launches_per_step) {
  if (!s) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_session_info: NULL session");
  if (position) *position = s->host_pos;
  if (stream) *stream = s->ctx->stream;
  if (launches_per_step) *launches_per_step = s->launches_per_step;
  return UNLTD_OK;
}

// Copy the last step's logits (vocab floats) and/or hidden state (l_out of
// the last layer, n_embd floats) to host buffers (NULL skips).
int32_t unltd_qwen35_batch_read(unltd_qwen35_session s, int32_t seq, float *logits, float *hidden) {
  if (!s) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_session_read: NULL session");
  if (seq < 0 || seq >= s->nseq) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_session_read: sequence out of range");
  CtxGuard g(s->m->ctx->device);
  cudaStream_t st = s->ctx->stream;
  cudaError_t e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && logits)
    e = cudaMemcpy(logits, seq_buf(s, s->logits, seq), (size_t)(s->m->d.v1 - s->m->d.v0) * 4, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && hidden)
    e = cudaMemcpy(hidden, seq_buf(s, s->X, seq), (size_t)s->m->d.n * 4, cudaMemcpyDeviceToHost);
  return cuda_error(e, "qwen35_session_read");
}

int32_t unltd_qwen35_session_read(unltd_qwen35_session s, float *logits, float *hidden) {
  return unltd_qwen35_batch_read(s, 0, logits, hidden);
}

int32_t unltd_qwen35_batch_info(unltd_qwen35_session s, int32_t *n_seq, int32_t *positions) {
  if (!s) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_batch_info: NULL session");
  if (n_seq) *n_seq = s->nseq;
  for (int z = 0; positions && z < s->nseq; z++) positions[z] = s->seq_pos[z];
  return UNLTD_OK;
}

}  // extern "C"
