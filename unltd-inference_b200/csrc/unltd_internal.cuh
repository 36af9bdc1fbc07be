// Internal definitions shared by the CUDA translation units of libunltd_gpu.
//
// Device weight layout ("row planes"). Every uploaded row keeps its GGUF byte
// count (row_bytes, min_forward.rs:52-80); rows are padded to a 16-byte
// stride so each lane can use 128-bit loads. Inside a row the bytes of each
// block are regrouped into planes and permuted *within* a block, losslessly:
//
//   Q4_K  [hdr  nb x 16 B: d f16 | dmin f16 | scales[12] (unchanged)]
//         [qs   nb x 128 B, permuted: old qs[32p + k + 8i] -> new 32p + 4k + i]
//   Q6_K  [ql   nb x 128 B, permuted within each 16-byte chunk by PIC6]
//         [qh   nb x 64 B,  permuted within each 16-byte chunk by PIC6, every
//                           2-bit field's top bit flipped (byte ^ 0xAA)]
//         [sc   nb x 16 B  (int8 scales, unchanged)]
//         [d    nb x 2 B   (f16)]
//   Q8_0  [qs   nb x 32 B][d nb x 2 B]          (nb = dim_in / 32 here)
//
// The permutations put, into each 32-bit word a lane loads, four elements
// that share both their scale group and their Q8_K lane class e % 8 (Q4_K)
// or two pairs of such elements (Q6_K). That is what lets one DP4A produce a
// term of the reference's per-lane integer sums exactly
// (quants.rs:337-342, 390-401) and, in F32X mode, a chain of DP4As share one
// scale.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace unltd {

constexpr int kQK = 256;          // K-quant super-block
constexpr int kQ4Bytes = 144;
constexpr int kQ6Bytes = 210;
constexpr int kQ80Bytes = 34;
constexpr int kQ80Elems = 32;

enum Dtype : int { F32 = 0, F16 = 1, BF16 = 2, I8 = 3, U8 = 4, Q4K = 5, Q6K = 6, Q8_0 = 7 };
enum Mode : int { MODE_F32X = 0, MODE_Q8K = 1 };

// ---- x images: per 256-element span, what one GEMV call prepares once ----
// F32X (all formats): limb planes hi (s8) | mid (u8) | lo (u8), 256 B each,
// element order = the format's lane order; then xs (f32 scale 2^(e-22)),
// then 16 f32 lane-half sums (Q4_K min term).
constexpr int kImgF32X = 848;
constexpr int kImgF32X_XS = 768;
constexpr int kImgF32X_XSUM = 784;
// Q8K for Q4_K: q8 (256 B, class-major: q4k_q8k_xpos) | d f32 | pad | 8 x i32
// group sums (then 8 zero words) | the min term's MMA B operand: 4 words,
// word 2c + t = the balanced low (c = 0) or high (c = 1) bytes of the group
// sums 4t .. 4t + 3 (low = ((s + 128) & 255) - 128, high = (s - low) / 256)
constexpr int kImgQ8K4 = 352;
constexpr int kImgQ8K4_D = 256;
constexpr int kImgQ8K4_BS = 272;
constexpr int kImgQ8K4_BM = 336;
// Q8K for Q6_K: for lane j, half h, word t: two masked q8 words (A: bytes
// 0,1; B: bytes 2,3) -> 8*2*4*2 words = 512 B | d f32 | pad
constexpr int kImgQ8K6 = 528;
constexpr int kImgQ8K6_D = 512;

__host__ __device__ inline int img_stride(int dtype, int mode) {
  return mode == MODE_F32X ? kImgF32X : (dtype == Q4K ? kImgQ8K4 : kImgQ8K6);
}

// Element e (0..255) of a span -> byte index in a lane-ordered 256-byte
// plane of an x image. Lane j of an 8-lane subgroup reads its low-nibble
// (or first-half) words at 16j and its high-nibble words at 128 + 16j, so
// the eight lanes of a quarter-warp touch 128 contiguous bytes (no bank
// conflicts). The same in-word order as the weights' permutation:
//  Q4_K: p = e/64 (qs segment), half = (e%64)/32 (low/high nibble group),
//        r = e%32, k = r%8, i = r/8, lane j = 2p + k/4
//        -> 128*half + 32p + 4k + i
__host__ __device__ inline int q4_xpos(int e) {
  int p = e >> 6, half = (e >> 5) & 1, r = e & 31;
  return 128 * half + 32 * p + 4 * (r & 7) + (r >> 3);
}
// Q8K image of a Q4_K span: element e = 32g + 8i + k (group g, class k = e % 8)
// at 128*(g/4) + 16k + 4*(g%4) + i, so lane k reads its class's q8 words for
// groups 0..3 at 16k and 4..7 at 128 + 16k (eight lanes: 128 contiguous bytes).
__host__ __device__ inline int q4k_q8k_xpos(int e) {
  const int g = e >> 5;
  return 128 * (g >> 2) + 16 * (e & 7) + 4 * (g & 3) + ((e >> 3) & 3);
}

// In-chunk position of run position ipos (0..15) for Q6_K: word t holds run
// positions (2t, 2t+8, 2t+1, 2t+9), i.e. Q8_K lane classes 2t and 2t+1.
__host__ __device__ inline int q6_pic(int ipos) {
  return 4 * ((ipos & 7) >> 1) + 2 * (ipos & 1) + (ipos >> 3);
}
//  Q6_K: h = e/128, pos = e%128, hi = pos/64, c = pos%64, u = c/16,
//        lane j = 4h + u  ->  128*hi + 16j + pic(c%16)
__host__ __device__ inline int q6_xpos(int e) {
  int h = e >> 7, pos = e & 127, hi = pos >> 6, c = pos & 63, u = c >> 4;
  return 128 * hi + 16 * (4 * h + u) + q6_pic(c & 15);
}
//  Q8_0 (a span is 8 blocks of 32): lane j = e/32 owns block j; its first 16
//  elements at 16j, the next 16 at 128 + 16j.
__host__ __device__ inline int q80_xpos(int e) {
  return 128 * ((e >> 4) & 1) + 16 * (e >> 5) + (e & 15);
}
// Q8K image of Q6_K: lane j's four 16-byte chunks q = 0..3 at 128q + 16j.
// Chunk q = 2*hh + (w >> 1) holds, for half hh and words w, w+1 of the lane,
// the masked q8 words (A: run positions 2w, 2w+8 in bytes 0,1; B: 2w+1,
// 2w+9 in bytes 2,3) as A_w, B_w, A_{w+1}, B_{w+1}.
__host__ __device__ inline int q6_q8k_byte(int j, int hh, int w, int ab, int bpos) {
  return 128 * (2 * hh + (w >> 1)) + 16 * j + 4 * (2 * (w & 1) + ab) + bpos;
}

// Batched x images (batch decode): one image per (span, group of 8
// sequences), kBImgBlock bytes, the Q8_K values laid out as the batched
// GEMV's MMA B fragments so a lane's operand is one coalesced 8-byte load:
//   [0, 2048)    class k at 256 k; lane (sl, t) = 4 sl + t at 8 lane: the
//                q8 words of groups 2t and 2t + 1 (byte i: element 32 g +
//                8 i + k) of sequence sl of the group;
//   [2048, 2304) lane 4 sl + t (t < 2): the balanced low / high bytes of the
//                group sums 4t .. 4t + 3 of sequence sl (the Q4_K min term);
//   [2304, 2336) the eight sequences' d.
constexpr int kBImgBlock = 2368;
__host__ __device__ inline size_t bimg_block(size_t span, int sg, int nsg) {
  return (span * (size_t)nsg + (size_t)sg) * kBImgBlock;
}
__host__ __device__ inline int bimg_q8(int e, int sl) {
  return (e & 7) * 256 + (sl * 4 + (e >> 6)) * 8 + ((e >> 5) & 1) * 4 + ((e >> 3) & 3);
}
__host__ __device__ inline int bimg_bm(int sl, int t, int c) { return 2048 + (sl * 4 + t) * 8 + c * 4; }
__host__ __device__ inline int bimg_d(int sl) { return 2304 + 4 * sl; }

// Q6_K rows of more than 16 blocks (a multiple of 16) are stored as chunks of
// 16 blocks, each laid out like a 16-block row ([ql][qh][scales][d]), so a
// 16-block slice of a long row is one contiguous 3360-byte range (the
// tensor-core GEMV streams rows of 12288 inputs as three such chunks). Other
// rows keep the planes of the whole row.
constexpr int kQ6Chunk = 16;
__host__ __device__ inline bool q6_chunked(size_t nb) { return nb > (size_t)kQ6Chunk && nb % kQ6Chunk == 0; }
// Block b of a Q6_K row: byte offset of the planes holding it (its chunk, or
// the row), the block count those planes are laid out for, and b's index there.
__host__ __device__ inline void q6_locate(size_t nb, size_t b, size_t &off, int &nbl, int &bl) {
  if (q6_chunked(nb)) {
    off = (b / kQ6Chunk) * (size_t)(kQ6Chunk * 210);
    nbl = kQ6Chunk;
    bl = (int)(b % kQ6Chunk);
  } else {
    off = 0;
    nbl = (int)nb;
    bl = (int)b;
  }
}

__host__ __device__ inline size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// GGUF bytes of one row (min_forward.rs:52-80); 0 when not a whole number of blocks.
__host__ __device__ inline size_t gguf_row_bytes(int dtype, size_t dim_in) {
  switch (dtype) {
    case F32: return dim_in * 4;
    case Q4K: return dim_in % kQK ? 0 : dim_in / kQK * kQ4Bytes;
    case Q6K: return dim_in % kQK ? 0 : dim_in / kQK * kQ6Bytes;
    case Q8_0: return dim_in % kQ80Elems ? 0 : dim_in / kQ80Elems * kQ80Bytes;
    default: return 0;
  }
}

// ---- small device helpers ---------------------------------------------
__device__ __forceinline__ int dp4a_uu(unsigned a, unsigned b, int c) {
  int r;
  asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}
__device__ __forceinline__ int dp4a_us(unsigned a, unsigned b, int c) {  // a unsigned, b signed
  int r;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}
__device__ __forceinline__ int dp4a_ss(unsigned a, unsigned b, int c) {
  int r;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}
__device__ __forceinline__ int dp4a_su(unsigned a, unsigned b, int c) {  // a signed, b unsigned
  int r;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

__device__ __forceinline__ uint4 ldg_stream(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ float h2f_bits(uint32_t bits16) {
  return __half2float(__ushort_as_half((unsigned short)bits16));
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

// ---- mbarrier + bulk-copy (TMA, non-tensor) helpers ----------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// The same test, but a thread whose phase is not complete yet is suspended
// in hardware until it completes or about `hint_ns` pass (no issue slots
// spent spinning while other warps of the SM compute).
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t *bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Wait for the phase of `parity` to complete, for at most ~2 s of wall time;
// on timeout record code 1 in *err and return false (never spins forever).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, int *err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_hint(bar, parity, 1000u)) return true;
    if ((it & 255u) == 0 && global_ns() - t0 > 2000000000ull) {
      atomicExch(err, 1);
      return false;
    }
  }
}
// 1-D bulk copy global -> shared, completing `bytes` of transaction on `bar`.
// Addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// bar.red.and over a named barrier: true iff `pred` holds in every participant.
__device__ __forceinline__ bool named_bar_red_and(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// f32 -> order-preserving u32 (larger float -> larger key).
__device__ __forceinline__ uint32_t orderable(float v) {
  uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Element e of a repacked Q4_K row with nb blocks, with the f32 operations
// of dequantize_q4_k (quants.rs:534-567): d1 = d*sc, m1 = dmin*m, y = d1*q - m1.
__device__ __forceinline__ float q4k_row_elem(const uint8_t *row, size_t nb, size_t e) {
  size_t b = e / kQK;
  int el = (int)(e % kQK), g = el >> 5;
  const uint8_t *hdr = row + b * 16;
  const uint8_t *s = hdr + 4;
  int sc, m;
  if (g < 4) {
    sc = s[g] & 63;
    m = s[g + 4] & 63;
  } else {
    sc = (s[g + 4] & 0xF) | ((s[g - 4] >> 6) << 4);
    m = (s[g + 4] >> 4) | ((s[g] >> 6) << 4);
  }
  float d = h2f_bits(hdr[0] | (hdr[1] << 8));
  float dmin = h2f_bits(hdr[2] | (hdr[3] << 8));
  int rr = el & 31, p = g >> 1;
  uint8_t byte = row[nb * 16 + b * 128 + 32 * p + 4 * (rr & 7) + (rr >> 3)];
  int q = (g & 1) ? (byte >> 4) : (byte & 0xF);
  float d1 = __fmul_rn(d, (float)sc);
  float m1 = __fmul_rn(dmin, (float)m);
  return __fsub_rn(__fmul_rn(d1, (float)q), m1);
}

// f(seq) for the reference's left-to-right f64 sum `seq` of n terms, given
// the parallel sum S of the same terms and their absolute sum A, with f a
// monotone non-decreasing map to f32. True when the bound decides it.
template <class F>
__device__ __forceinline__ bool resolve_sum(double S, double A, int n, F f, float *out) {
  const double B = (double)(n + 8) * 0x1p-51 * A;
  const float lo = f(S - B), hi = f(S + B);
  *out = lo;
  return lo == hi;
}

struct MeanOf {
  int n;
  __device__ float operator()(double s) const { return (float)(s / (double)n); }
};
struct ToF32 {
  __device__ float operator()(double s) const { return (float)s; }
};

}  // namespace unltd
