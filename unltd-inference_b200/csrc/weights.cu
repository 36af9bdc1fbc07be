// Weight repack (GGUF bytes -> row planes) and bit-exact dequantization.
//
// The repack is a pure byte permutation (see unltd_internal.cuh), so the
// dequantized values are those of the GGUF bytes, computed with the
// reference's f32 formulas:
//   Q4_K  d1 = d*sc, m1 = dmin*m, y = d1*q - m1        (quants.rs:534-567)
//   Q6_K  y = d*(sc*q), exact in f32                    (quants.rs:171-200)
//   Q8_0  y = d*q, exact in f32                         (format restated)
#include "unltd_host.h"
#include "unltd_internal.cuh"

namespace unltd {
namespace {

// One thread per (row, block): copy the block's bytes into its planes.
__global__ void repack_q4k(const uint8_t *__restrict__ raw, uint8_t *__restrict__ dev, size_t rows,
                           size_t nb, size_t row_bytes, size_t stride) {
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= rows * nb) return;
  size_t r = t / nb, b = t % nb;
  const uint8_t *src = raw + r * row_bytes + b * kQ4Bytes;
  uint8_t *hdr = dev + r * stride + b * 16;
  uint8_t *qs = dev + r * stride + nb * 16 + b * 128;
  for (int i = 0; i < 16; i++) hdr[i] = src[i];
  for (int o = 0; o < 128; o++) {
    int p = o >> 5, rr = o & 31;
    qs[32 * p + 4 * (rr & 7) + (rr >> 3)] = src[16 + o];
  }
}

__global__ void repack_q6k(const uint8_t *__restrict__ raw, uint8_t *__restrict__ dev, size_t rows,
                           size_t nb, size_t row_bytes, size_t stride) {
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= rows * nb) return;
  size_t r = t / nb, b = t % nb;
  const uint8_t *src = raw + r * row_bytes + b * kQ6Bytes;
  size_t off;
  int nbl, bl;
  q6_locate(nb, b, off, nbl, bl);
  uint8_t *row = dev + r * stride + off;
  uint8_t *ql = row + bl * 128, *qh = row + nbl * 128 + bl * 64;
  uint8_t *sc = row + nbl * 192 + bl * 16, *d = row + nbl * 208 + bl * 2;
  for (int o = 0; o < 128; o++) ql[16 * (o >> 4) + q6_pic(o & 15)] = src[o];
  // the top bit of every 2-bit field flipped: the GEMVs' 4*(q - 32) operand
  // words then need no sign flip of their own (q6_a4_lo / q6_a4_hi)
  for (int o = 0; o < 64; o++) qh[16 * (o >> 4) + q6_pic(o & 15)] = src[128 + o] ^ 0xAAu;
  for (int i = 0; i < 16; i++) sc[i] = src[192 + i];
  d[0] = src[208];
  d[1] = src[209];
}

__global__ void repack_q80(const uint8_t *__restrict__ raw, uint8_t *__restrict__ dev, size_t rows,
                           size_t nb, size_t row_bytes, size_t stride) {
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= rows * nb) return;
  size_t r = t / nb, b = t % nb;
  const uint8_t *src = raw + r * row_bytes + b * kQ80Bytes;
  uint8_t *row = dev + r * stride;
  for (int i = 0; i < 32; i++) row[b * 32 + i] = src[2 + i];
  row[nb * 32 + b * 2] = src[0];
  row[nb * 32 + b * 2 + 1] = src[1];
}

__global__ void copy_f32_rows(const uint8_t *__restrict__ raw, uint8_t *__restrict__ dev, size_t rows,
                              size_t row_bytes, size_t stride) {
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= rows * row_bytes) return;
  size_t r = t / row_bytes, o = t % row_bytes;
  dev[r * stride + o] = raw[t];
}

// One thread per output element.
__global__ void dequant_q4k(const uint8_t *__restrict__ dev, float *__restrict__ out, size_t rows,
                            size_t nb, size_t stride) {
  size_t n = nb * kQK;
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= rows * n) return;
  size_t r = t / n, e = t % n;
  out[t] = q4k_row_elem(dev + r * stride, nb, e);
}

__global__ void dequant_q6k(const uint8_t *__restrict__ dev, float *__restrict__ out, size_t rows,
                            size_t nb, size_t stride) {
  size_t n = nb * kQK;
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= rows * n) return;
  size_t r = t / n, e = t % n;
  size_t off;
  int nbl, b;
  q6_locate(nb, e / kQK, off, nbl, b);
  int el = (int)(e % kQK);
  const uint8_t *row = dev + r * stride + off;
  int h = el >> 7, pos = el & 127;
  int qlo = 64 * h + (pos & 63);
  int qho = 32 * h + (pos & 31);
  uint8_t lb = row[b * 128 + 16 * (qlo >> 4) + q6_pic(qlo & 15)];
  uint8_t hb = row[nbl * 128 + b * 64 + 16 * (qho >> 4) + q6_pic(qho & 15)] ^ 0xAAu;  // stored flipped
  int nib = pos < 64 ? (lb & 0xF) : (lb >> 4);
  int hi2 = (hb >> (2 * (pos >> 5))) & 3;
  int q = (nib | (hi2 << 4)) - 32;
  int sc = (int8_t)row[nbl * 192 + b * 16 + (el >> 4)];
  const uint8_t *dp = row + nbl * 208 + b * 2;
  float d = h2f_bits(dp[0] | (dp[1] << 8));
  // f32 product, not an integer one: keeps the sign of a zero weight
  // (a negative scale times q = 0 is -0.0 in the reference's f64 decode).
  out[t] = __fmul_rn(d, __fmul_rn((float)sc, (float)q));
}

__global__ void dequant_q80(const uint8_t *__restrict__ dev, float *__restrict__ out, size_t rows,
                            size_t nb, size_t stride) {
  size_t n = nb * kQ80Elems;
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= rows * n) return;
  size_t r = t / n, e = t % n, b = e / kQ80Elems;
  const uint8_t *row = dev + r * stride;
  int q = (int8_t)row[b * 32 + (e % kQ80Elems)];
  const uint8_t *dp = row + nb * 32 + b * 2;
  float d = h2f_bits(dp[0] | (dp[1] << 8));
  out[t] = __fmul_rn(d, (float)q);
}

__global__ void dequant_f32(const uint8_t *__restrict__ dev, float *__restrict__ out, size_t rows,
                            size_t n, size_t stride) {
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= rows * n) return;
  size_t r = t / n, e = t % n;
  out[t] = reinterpret_cast<const float *>(dev + r * stride)[e];
}

inline unsigned grid_for(size_t n, int threads) { return (unsigned)((n + threads - 1) / threads); }

}  // namespace

cudaError_t launch_repack(const unltd_weight_s &w, const uint8_t *raw_dev, size_t row0_local,
                          size_t rows, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  uint8_t *dst = w.dev + row0_local * w.row_stride;
  const int T = 256;
  switch (w.dtype) {
    case Q4K:
      repack_q4k<<<grid_for(rows * w.nb, T), T, 0, s>>>(raw_dev, dst, rows, w.nb, w.row_bytes, w.row_stride);
      break;
    case Q6K:
      repack_q6k<<<grid_for(rows * w.nb, T), T, 0, s>>>(raw_dev, dst, rows, w.nb, w.row_bytes, w.row_stride);
      break;
    case Q8_0:
      repack_q80<<<grid_for(rows * w.nb, T), T, 0, s>>>(raw_dev, dst, rows, w.nb, w.row_bytes, w.row_stride);
      break;
    default:
      copy_f32_rows<<<grid_for(rows * w.row_bytes, T), T, 0, s>>>(raw_dev, dst, rows, w.row_bytes, w.row_stride);
      break;
  }
  return cudaGetLastError();
}

cudaError_t launch_dequant(const unltd_weight_s &w, float *out, cudaStream_t s) {
  const int T = 256;
  size_t n = w.dim_out * w.dim_in;
  if (n == 0) return cudaSuccess;
  switch (w.dtype) {
    case Q4K: dequant_q4k<<<grid_for(n, T), T, 0, s>>>(w.dev, out, w.dim_out, w.nb, w.row_stride); break;
    case Q6K: dequant_q6k<<<grid_for(n, T), T, 0, s>>>(w.dev, out, w.dim_out, w.nb, w.row_stride); break;
    case Q8_0: dequant_q80<<<grid_for(n, T), T, 0, s>>>(w.dev, out, w.dim_out, w.nb, w.row_stride); break;
    default: dequant_f32<<<grid_for(n, T), T, 0, s>>>(w.dev, out, w.dim_out, w.dim_in, w.row_stride); break;
  }
  return cudaGetLastError();
}

}  // namespace unltd
