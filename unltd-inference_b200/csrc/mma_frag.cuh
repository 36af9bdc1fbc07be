// Fragment helpers shared by the quantized GEMV kernels (gemv.cu,
// gemv_batch.cu): int8 mma.sync wrappers, byte extraction, the Q6_K A-operand
// words and the Q6_K x-image B operands, and the argmax key.
#pragma once

#include "unltd_internal.cuh"

namespace unltd {
namespace {

__device__ __forceinline__ uint4 lds128(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }
__device__ __forceinline__ uint2 lds64(const uint8_t *p) { return *reinterpret_cast<const uint2 *>(p); }

// D = A(16x32 s8, row) * B(32x8 s8, col), exact int32 (tensor cores)
__device__ __forceinline__ void mma_s8(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1,
                                       int &d0, int &d1, int &d2, int &d3) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// byte k (0..3) of w as an int
__device__ __forceinline__ int byte_of(uint32_t w, int k) { return (int)__byte_perm(w, 0u, 0x4440u | (uint32_t)k); }

// A(16x32 u8, row) * B(32x8 s8, col), exact int32: the high nibbles of the
// Q4_K words taken in place (w & 0xF0F0F0F0, i.e. 16 x nibble)
__device__ __forceinline__ void mma_u8s8(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1,
                                         int &d0, int &d1, int &d2, int &d3) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// D = A(16x16 s8, row) * B(16x8 s8, col), exact int32 (tensor cores)
__device__ __forceinline__ void mma_s8_k16(uint32_t a0, uint32_t a1, uint32_t b0, int &d0, int &d1, int &d2, int &d3) {
  asm("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};"
      : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
      : "r"(a0), "r"(a1), "r"(b0), "r"(0));
}

// Q6_K: a word of 4*(raw6 - 32) as s8 from ql/qh words (2-bit field of qh at
// shift sl for the low-nibble half, sl + 4 for the high half). The device
// layout stores qh with the top bit of every field flipped (repack_q6k), so
// the field lands in bits 6-7 already as the sign-flipped high bits of
// 4*raw6 - 128.
__device__ __forceinline__ uint32_t q6_a4_lo(uint32_t ql, uint32_t qh, int sl) {
  return ((ql << 2) & 0x3C3C3C3Cu) | ((qh << (6 - sl)) & 0xC0C0C0C0u);
}
__device__ __forceinline__ uint32_t q6_a4_hi(uint32_t ql, uint32_t qh, int sl) {
  return ((ql >> 2) & 0x3C3C3C3Cu) | ((qh << (2 - sl)) & 0xC0C0C0C0u);
}

// signed byte k (0..3) of w: prmt with the sign-replicate selector bit (the
// __byte_perm intrinsic ignores that bit)
__device__ __forceinline__ int sbyte_of(uint32_t w, int k) {
  int r;
  asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(w), "r"(0x8880u | (0x1111u * (uint32_t)k)));
  return r;
}

// One block of the Q6_K Q8_K x image as MMA B operands of this lane: for
// ql chunk j and half hh (the 16-element sub-blocks 8h + u and 8h + 4 + u,
// j = 4h + u), the k-quad tig of the chunk's words holds run positions
// (2 tig, 2 tig + 8, 2 tig + 1, 2 tig + 9), i.e. classes 2 tig (bytes 0, 1)
// and 2 tig + 1 (bytes 2, 3); column gid of B keeps only its class: the
// image's masked copy A when gid = 2 tig, copy B when gid = 2 tig + 1.
struct XBlock6 {
  uint32_t b[16];  // [2 j + hh]
  float xd;
};

// Block b of a Q6_K row in shared memory: moves row to the planes holding
// it (its 16-block chunk when the row is chunked) and returns b's index
// there, with the block count those planes are laid out for in nbl.
__device__ __forceinline__ int q6_planes(const uint8_t *&row, int nb, int b, int &nbl) {
  if (q6_chunked((size_t)nb)) {
    row += (b / kQ6Chunk) * (kQ6Chunk * 210);
    nbl = kQ6Chunk;
    return b % kQ6Chunk;
  }
  nbl = nb;
  return b;
}

__device__ __forceinline__ void load_xblock6(const uint8_t *im, XBlock6 &x) {
  const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
  const bool own = (gid >> 1) == tig;
  const int ab = gid & 1;
#pragma unroll
  for (int j = 0; j < 8; j++)
#pragma unroll
    for (int hh = 0; hh < 2; hh++)
      x.b[2 * j + hh] =
          own ? *reinterpret_cast<const uint32_t *>(im + q6_q8k_byte(j, hh, tig, ab, 0)) : 0u;
  x.xd = *reinterpret_cast<const float *>(im + kImgQ8K6_D);
}

__device__ __forceinline__ unsigned long long argmax_key(float v, int row) {
  if (isnan(v)) return row == 0 ? ~0ull : 0ull;
  return ((unsigned long long)orderable(v) << 32) | (0xffffffffu - (uint32_t)row);
}

}  // namespace
}  // namespace unltd
