// Exact quantize_q8_k (crates/unltd-tensor/src/quants.rs:250-290) of one
// 256-element span held one element per thread by a 256-thread CTA, written
// into the GEMV x images (layouts in unltd_internal.cuh). Shared by the GEMV
// prep kernel and the fused producer kernels of the decode step.
#pragma once

#include "unltd_internal.cuh"

namespace unltd {

struct Q8KSpanSmem {
  float a[8];
  float v[8];
  int i[8];
  int hsum[16];
};

// v = element t (threadIdx.x) of the span. im4 / im6 (either may be null):
// this span's Q4_K / Q6_K image; imb (may be null): the span's batched image
// (kBImgBlock, unltd_internal.cuh) of this sequence's group, sl = the
// sequence's index in it. All 256 threads must call.
__device__ __forceinline__ void q8k_span_write(float v, uint8_t *im4, uint8_t *im6, Q8KSpanSmem &s,
                                               uint8_t *imb = nullptr, int sl = 0) {
  const int t = threadIdx.x;
  if (t < 16) s.hsum[t] = 0;
  // first strict argmax of |x|; NaN never wins (the reference's `ax > amax`)
  float a = fabsf(v);
  if (isnan(a)) a = -1.0f;
  int idx = t;
  float val = v;
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float oa = __shfl_xor_sync(0xffffffffu, a, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    const float ov = __shfl_xor_sync(0xffffffffu, val, o);
    if (oa > a || (oa == a && oi < idx)) {
      a = oa;
      idx = oi;
      val = ov;
    }
  }
  if ((t & 31) == 0) {
    s.a[t >> 5] = a;
    s.i[t >> 5] = idx;
    s.v[t >> 5] = val;
  }
  __syncthreads();
  float amax = s.a[0], mx = s.v[0];
  int imax = s.i[0];
#pragma unroll
  for (int w = 1; w < 8; w++) {
    if (s.a[w] > amax || (s.a[w] == amax && s.i[w] < imax)) {
      amax = s.a[w];
      imax = s.i[w];
      mx = s.v[w];
    }
  }
  int q = 0;
  float d = 0.0f;
  if (amax > 0.0f) {
    const float iscale = __fdiv_rn(-127.0f, mx);
    const float prod = __fmul_rn(iscale, v);
    const int ni = (__float_as_int(__fadd_rn(prod, 12582912.0f)) & 0x007fffff) - 0x00400000;
    q = ni < 127 ? ni : 127;
    d = __fdiv_rn(1.0f, iscale);
  }
  if (im4) im4[q4k_q8k_xpos(t)] = (uint8_t)(int8_t)q;  // class-major (q4k_q8k_xpos)
  if (imb) imb[bimg_q8(t, sl)] = (uint8_t)(int8_t)q;
  if (im4 || imb) atomicAdd(&s.hsum[t >> 5], q);      // hsum[g] = sum of group g's q8 values
  if (im6) {
    // element -> (lane j, half hh, run position ipos); word w = (ipos%8)/2 holds
    // run positions (2w, 2w+8 | 2w+1, 2w+9); masked copies A (bytes 0,1) and
    // B (bytes 2,3): each element writes its byte into one copy and a zero
    // into the same byte of the other, so every byte is written once.
    const int h = t >> 7, pos = t & 127, hh = pos >> 6, c = pos & 63, u = c >> 4, ipos = c & 15;
    const int j = 4 * h + u;
    const int pic = q6_pic(ipos);
    const int w = pic >> 2, bpos = pic & 3;
    const int own = bpos < 2 ? 0 : 1;
    im6[q6_q8k_byte(j, hh, w, own, bpos)] = (uint8_t)(int8_t)q;
    im6[q6_q8k_byte(j, hh, w, 1 - own, bpos)] = 0;
    if (t == 0) *reinterpret_cast<float *>(im6 + kImgQ8K6_D) = d;
  }
  __syncthreads();
  if (im4 || imb) {
    if (t == 0 && im4) *reinterpret_cast<float *>(im4 + kImgQ8K4_D) = d;
    if (t == 0 && imb) *reinterpret_cast<float *>(imb + bimg_d(sl)) = d;
    if (t < 16 && im4) reinterpret_cast<int *>(im4 + kImgQ8K4_BS)[t] = s.hsum[t];
    if (t < 4) {  // the min term's B operand words (kImgQ8K4_BM)
      const int c = t >> 1, tg = t & 1;
      uint32_t bm = 0u;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int g = s.hsum[4 * tg + i];
        const int lo = ((g + 128) & 255) - 128, hi = (g - lo) >> 8;
        bm |= (uint32_t)((c == 0 ? lo : hi) & 0xFF) << (8 * i);
      }
      if (im4) reinterpret_cast<uint32_t *>(im4 + kImgQ8K4_BM)[t] = bm;
      if (imb) *reinterpret_cast<uint32_t *>(imb + bimg_bm(sl, tg, c)) = bm;
    }
  }
}

// The same quantize_q8_k of one span held by ONE warp: lane l holds elements
// 8l .. 8l+7 in v[0..7]. Warp shuffles only, no block barrier, so the warps
// of a CTA quantize their spans concurrently. imb / sl as q8k_span_write.
__device__ __forceinline__ void q8k_span_write_warp(const float (&v)[8], int lane, uint8_t *im4, uint8_t *im6,
                                                    uint8_t *imb = nullptr, int sl = 0) {
  // first strict argmax of |x| (ties: lowest index); NaN never wins
  float a = -1.0f, val = 0.0f;
  int idx = 8 * lane;
#pragma unroll
  for (int k = 0; k < 8; k++) {
    float ak = fabsf(v[k]);
    if (isnan(ak)) ak = -1.0f;
    if (ak > a) {
      a = ak;
      idx = 8 * lane + k;
      val = v[k];
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float oa = __shfl_xor_sync(0xffffffffu, a, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    const float ov = __shfl_xor_sync(0xffffffffu, val, o);
    if (oa > a || (oa == a && oi < idx)) {
      a = oa;
      idx = oi;
      val = ov;
    }
  }
  int q[8];
  float d = 0.0f;
  if (a > 0.0f) {
    const float iscale = __fdiv_rn(-127.0f, val);
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const float prod = __fmul_rn(iscale, v[k]);
      const int ni = (__float_as_int(__fadd_rn(prod, 12582912.0f)) & 0x007fffff) - 0x00400000;
      q[k] = ni < 127 ? ni : 127;
    }
    d = __fdiv_rn(1.0f, iscale);
  } else {
#pragma unroll
    for (int k = 0; k < 8; k++) q[k] = 0;
  }
  if (im4 || imb) {
    // class-major (q4k_q8k_xpos of e = 8 lane + k); group g = lane / 4
    const int g = lane >> 2;
    const int base = 128 * (g >> 2) + 4 * (g & 3) + (lane & 3);
    int hs = 0;
#pragma unroll
    for (int k = 0; k < 8; k++) {
      if (im4) im4[base + 16 * k] = (uint8_t)(int8_t)q[k];
      if (imb) imb[bimg_q8(8 * lane + k, sl)] = (uint8_t)(int8_t)q[k];
      hs += q[k];
    }
    hs += __shfl_xor_sync(0xffffffffu, hs, 1);
    hs += __shfl_xor_sync(0xffffffffu, hs, 2);
    if (im4) {
      int *bs = reinterpret_cast<int *>(im4 + kImgQ8K4_BS);
      if ((lane & 3) == 0) bs[g] = hs;
      if (lane < 8) bs[8 + lane] = 0;
      if (lane == 0) *reinterpret_cast<float *>(im4 + kImgQ8K4_D) = d;
    }
    if (imb && lane == 0) *reinterpret_cast<float *>(imb + bimg_d(sl)) = d;
    // the min term's B operand words (kImgQ8K4_BM): lane 2c + t packs the
    // low (c = 0) or high (c = 1) bytes of group sums 4t .. 4t + 3
    uint32_t bm = 0u;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int gs = __shfl_sync(0xffffffffu, hs, 16 * (lane & 1) + 4 * i);
      const int lo = ((gs + 128) & 255) - 128, hi = (gs - lo) >> 8;
      bm |= (uint32_t)(((lane >> 1) & 1 ? hi : lo) & 0xFF) << (8 * i);
    }
    if (lane < 4 && im4) reinterpret_cast<uint32_t *>(im4 + kImgQ8K4_BM)[lane] = bm;
    if (lane < 4 && imb) *reinterpret_cast<uint32_t *>(imb + bimg_bm(sl, lane & 1, (lane >> 1) & 1)) = bm;
  }
  if (im6) {
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int t = 8 * lane + k;
      const int h = t >> 7, pos = t & 127, hh = pos >> 6, c = pos & 63, u = c >> 4, ipos = c & 15;
      const int j = 4 * h + u;
      const int pic = q6_pic(ipos);
      const int w = pic >> 2, bpos = pic & 3;
      const int own = bpos < 2 ? 0 : 1;
      im6[q6_q8k_byte(j, hh, w, own, bpos)] = (uint8_t)(int8_t)q[k];
      im6[q6_q8k_byte(j, hh, w, 1 - own, bpos)] = 0;
    }
    if (lane == 0) *reinterpret_cast<float *>(im6 + kImgQ8K6_D) = d;
  }
}

}  // namespace unltd
