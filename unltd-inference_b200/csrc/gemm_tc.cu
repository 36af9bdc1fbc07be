// Batched prefill GEMM over Q4_K weights on the 5th-generation tensor cores:
// Y[m][n] = sum_k X[m][k] * W[n][k]  (Y = X . W^T, the reference's
// gemv_quant applied to every token at once; the reference itself runs
// prefill token by token, qwen35_forward.rs:8-12).
//
// Design (one CTA per SM, persistent over 256-token x 192-row output tiles):
//  * X is converted once per call to fp16, with the columns of every
//    64-element segment permuted to the K order in which the dequant writes
//    the weight tile, so A and B agree without any byte transpose.
//  * warps 0 and 2 (one thread each): TMA producers. Per 64-wide K step they load the two
//    128x64 fp16 A tiles (SWIZZLE_128B tensor map) and, for the 192 weight
//    rows of the tile, the 32-byte quant segment and 16-byte block header
//    (2-D tensor maps over the repacked rows). Three rings decouple the
//    latencies: packed weights (8 small stages, freed by the dequant, so they
//    stream far ahead from HBM), X tiles (3 stages) and fp16 weight tiles (2
//    stages), both freed by the MMAs' tcgen05.commit.
//  * warps 3-14 (384 threads, two per weight row, one per nibble group):
//    dequantize to fp16 — nibble -> exact fp16 (the 1024 + q bias trick),
//    then q * fp16(d*sc) - fp16(dmin*m) in one fp16 FMA — and store into the
//    B tile in the canonical K-major SWIZZLE_128B layout.
//  * warp 1 (one thread): issues tcgen05.mma kind::f16 (fp16 x fp16 -> f32),
//    M=128 N=192 K=16, for both 128-token halves, accumulating in TMEM
//    (columns [0,192) and [256,448)); tcgen05.commit frees each stage and,
//    after the last step, signals the epilogue.
//  * warps 15-18: tcgen05.ld the accumulators (32x32b) and store Y in f32.
// Every mbarrier wait is bounded (2 s) and records a timeout in the context
// error word; on any timeout all roles leave their loops, in-flight copies and
// MMAs are waited for (bounded), and TMEM is freed before the CTA exits.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include "unltd_host.h"
#include "unltd_internal.cuh"

namespace unltd {
namespace {

constexpr int kTileM = 256;   // tokens per tile (two MMAs of M = 128)
constexpr int kTileN = 192;   // weight rows per tile (MMA N)
constexpr int kStepK = 64;    // K per stage: one Q4_K quant segment
constexpr int kStagesA = 3;   // X tiles, released by the MMAs
constexpr int kStagesB = 3;   // dequantized weight tiles, released by the MMAs
constexpr int kStagesW = 5;   // packed weight segments, released by the dequant
constexpr int kDequantWarps = 12;  // warps 3..14: two threads per weight row
constexpr int kThreadsG = (3 + kDequantWarps + 4) * 32;  // + 2 producers, MMA, 4 epilogue warps
constexpr uint32_t kABytes = 2 * 128 * kStepK * 2;          // 32 KB
constexpr uint32_t kBBytes = kTileN * kStepK * 2;            // 24 KB
constexpr uint32_t kWqBytes = kTileN * 32;                   // 6 KB
constexpr uint32_t kWhBytes = kTileN * 16;                   // 3 KB
constexpr uint32_t kWBytes = kWqBytes + kWhBytes;            // 9 KB
constexpr uint32_t kTmemCols = 512;
constexpr int kSmemBytes =
    kStagesA * kABytes + kStagesB * kBBytes + kStagesW * kWBytes + 1024 /*align*/ + 256 /*barriers*/;

// ---- tcgen05 / TMA wrappers (inline PTX, sm_100a) --------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// UMMA shared-memory descriptor: K-major, SWIZZLE_128B, 8-row atoms of
// 128 B (SBO = 1024 B), sm100 descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;           // LBO (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32; // SBO
  d |= (uint64_t)1 << 46;           // version
  d |= (uint64_t)2 << 61;           // SWIZZLE_128B
  return d;
}

// Instruction descriptor: D f32, A/B f16, both K-major, M=128, N=kTileN.
constexpr uint32_t kIdesc = (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(kTileN >> 3) << 17) |
                            ((uint32_t)(128 >> 4) << 24);

struct GemmParams {
  int M, N, K, nb;
  float *Y;
  int *err;
  int tiles_n, ntiles;
};

__global__ void __launch_bounds__(kThreadsG, 1)
    gemm_q4k_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmWq,
                const __grid_constant__ CUtensorMap tmWh, GemmParams P) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t pad = ((raw + 1023u) & ~1023u) - raw;
  uint8_t *base = smem_raw + pad;
  uint8_t *ringA = base;
  uint8_t *ringB = ringA + kStagesA * kABytes;
  uint8_t *ringW = ringB + kStagesB * kBBytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(ringW + kStagesW * kWBytes);
  uint64_t *afull = bars, *aempty = afull + kStagesA;
  uint64_t *bfull = aempty + kStagesA, *bempty = bfull + kStagesB;
  uint64_t *wfull = bempty + kStagesB, *wempty = wfull + kStagesW;
  uint64_t *acc_full = wempty + kStagesW, *acc_empty = acc_full + 1;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ksteps = P.K / kStepK;
  constexpr int kDequantThreads = kDequantWarps * 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesA; s++) {
      mbar_init(&afull[s], 1);
      mbar_init(&aempty[s], 1);
    }
    for (int s = 0; s < kStagesB; s++) {
      mbar_init(&bfull[s], kDequantThreads);
      mbar_init(&bempty[s], 1);
    }
    for (int s = 0; s < kStagesW; s++) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], kDequantThreads);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 4);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0 || warp == 2) {
    // ---------------- TMA producers: warp 0 the X tiles, warp 2 the weight segments ----
    if (lane == 0) {
      const bool isA = warp == 0;
      const int S = isA ? kStagesA : kStagesW;
      uint64_t *fullb = isA ? afull : wfull;
      uint64_t *emptyb = isA ? aempty : wempty;
      long g = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < P.ntiles && ok; t += gridDim.x) {
        const int tm = t / P.tiles_n, tn = t % P.tiles_n;
        for (int ks = 0; ks < ksteps && ok; ks++, g++) {
          const int s = (int)(g % S);
          const long round = g / S;
          if (round > 0) ok = mbar_wait_bounded(&emptyb[s], (uint32_t)((round - 1) & 1), P.err);
          if (!ok) break;
          if (isA) {
            uint8_t *dst = ringA + (size_t)s * kABytes;
            mbar_expect_tx(&fullb[s], kABytes);
            tma_load_2d(dst, &tmA, ks * kStepK, tm * kTileM, &fullb[s]);
            tma_load_2d(dst + kABytes / 2, &tmA, ks * kStepK, tm * kTileM + 128, &fullb[s]);
          } else {
            uint8_t *dst = ringW + (size_t)s * kWBytes;
            const int b = ks >> 2, p = ks & 3;
            mbar_expect_tx(&fullb[s], kWBytes);
            tma_load_2d(dst, &tmWq, P.nb * 16 + b * 128 + 32 * p, tn * kTileN, &fullb[s]);
            tma_load_2d(dst + kWqBytes, &tmWh, b * 16, tn * kTileN, &fullb[s]);
          }
        }
      }
      // leave no copy in flight: wait for the last fill of every stage
      for (long i = g - S < 0 ? 0 : g - S; i < g; i++) mbar_wait_bounded(&fullb[i % S], (uint32_t)((i / S) & 1), P.err);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      long g = 0;
      int it = 0;
      bool ok = true;
      uint64_t *last = nullptr;
      uint32_t last_par = 0;
      for (int t = blockIdx.x; t < P.ntiles && ok; t += gridDim.x, it++) {
        if (it > 0) ok = mbar_wait_bounded(acc_empty, (uint32_t)((it - 1) & 1), P.err);
        if (!ok) break;
        tc_fence_after();
        for (int ks = 0; ks < ksteps && ok; ks++, g++) {
          const int sa = (int)(g % kStagesA), sb = (int)(g % kStagesB);
          ok = mbar_wait_bounded(&afull[sa], (uint32_t)((g / kStagesA) & 1), P.err) &&
               mbar_wait_bounded(&bfull[sb], (uint32_t)((g / kStagesB) & 1), P.err);
          if (!ok) break;
          tc_fence_after();
          const uint32_t a0 = smem_u32(ringA + (size_t)sa * kABytes), b0 = smem_u32(ringB + (size_t)sb * kBBytes);
#pragma unroll
          for (int h = 0; h < 2; h++)
#pragma unroll
            for (int kk = 0; kk < kStepK / 16; kk++)
              umma_f16(tbase + (uint32_t)(h * 256), sw128_desc(a0 + h * (kABytes / 2) + kk * 32),
                       sw128_desc(b0 + kk * 32), kIdesc, (ks > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&aempty[sa]);
          umma_commit(&bempty[sb]);
          last = &bempty[sb];
          last_par = (uint32_t)((g / kStagesB) & 1);
        }
        if (ok) {
          umma_commit(acc_full);
          last = acc_full;
          last_par = (uint32_t)(it & 1);
        }
      }
      if (last) mbar_wait_bounded(last, last_par, P.err);  // MMAs retired before TMEM is freed
    }
  } else if (warp < 3 + kDequantWarps) {
    // ---------------- dequantize Q4_K -> fp16 B tile ----------------
    // Thread (r, hf): weight row r of the tile, nibble half hf (group 2p or
    // 2p+1 of the current 64-element segment p).
    const int dt = threadIdx.x - 96;
    const int r = dt % kTileN, hf = dt / kTileN;
    long g = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < P.ntiles && ok; t += gridDim.x) {
      for (int ks = 0; ks < ksteps && ok; ks++, g++) {
        const int sw = (int)(g % kStagesW), sb = (int)(g % kStagesB);
        ok = mbar_wait_bounded(&wfull[sw], (uint32_t)((g / kStagesW) & 1), P.err);
        if (ok && g >= kStagesB) ok = mbar_wait_bounded(&bempty[sb], (uint32_t)((g / kStagesB - 1) & 1), P.err);
        if (!ok) break;
        const uint8_t *wst = ringW + (size_t)sw * kWBytes;
        const uint4 hq = *reinterpret_cast<const uint4 *>(wst + kWqBytes + r * 16);
        // the two 16-byte halves of the row's 32 quant bytes, read in an
        // order that keeps the 8 lanes of each quarter-warp on distinct banks
        const int f = (r >> 2) & 1;
        const uint4 qa = *reinterpret_cast<const uint4 *>(wst + r * 32 + 16 * f);
        const uint4 qb = *reinterpret_cast<const uint4 *>(wst + r * 32 + 16 * (1 - f));
        mbar_arrive(&wempty[sw]);  // the weight stage is in registers now
        const uint4 q0 = f ? qb : qa, q1 = f ? qa : qb;
        const int p = ks & 3;
        uint32_t SC, MM;
        if (p < 2) {
          SC = hq.y & 0x3F3F3F3Fu;
          MM = hq.z & 0x3F3F3F3Fu;
        } else {
          SC = (hq.w & 0x0F0F0F0Fu) | ((hq.y >> 2) & 0x30303030u);
          MM = ((hq.w >> 4) & 0x0F0F0F0Fu) | ((hq.z >> 2) & 0x30303030u);
        }
        const int sh = (p & 1) * 16 + hf * 8;
        const float d = h2f_bits(hq.x & 0xFFFFu), dmin = h2f_bits(hq.x >> 16);
        const __half2 d1 = __float2half2_rn(__fmul_rn(d, (float)((SC >> sh) & 0xFF)));
        const __half2 nm1 = __float2half2_rn(-__fmul_rn(dmin, (float)((MM >> sh) & 0xFF)));
        const __half2 k1024 = __float2half2_rn(1024.0f);
        const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        uint8_t *brow = ringB + (size_t)sb * kBBytes + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
        for (int c = 0; c < 4; c++) {
          uint32_t outw[4];
#pragma unroll
          for (int ww = 0; ww < 2; ww++) {
            const uint32_t nib = hf ? ((w[2 * c + ww] >> 4) & 0x0F0F0F0Fu) : (w[2 * c + ww] & 0x0F0F0F0Fu);
            // bytes (0,2) and (1,3) as fp16 pairs 1024 + q, exact
            uint32_t a = (nib & 0x000F000Fu) | 0x64006400u;
            uint32_t b = ((nib >> 8) & 0x000F000Fu) | 0x64006400u;
            __half2 qa2 = __hsub2(*reinterpret_cast<__half2 *>(&a), k1024);
            __half2 qb2 = __hsub2(*reinterpret_cast<__half2 *>(&b), k1024);
            __half2 va = __hfma2(qa2, d1, nm1), vb = __hfma2(qb2, d1, nm1);
            outw[2 * ww] = *reinterpret_cast<uint32_t *>(&va);
            outw[2 * ww + 1] = *reinterpret_cast<uint32_t *>(&vb);
          }
          const int chunk = 4 * hf + c;
          *reinterpret_cast<uint4 *>(brow + ((chunk ^ (r & 7)) << 4)) = make_uint4(outw[0], outw[1], outw[2], outw[3]);
        }
        fence_proxy_async();  // generic-proxy stores -> visible to the tensor core
        mbar_arrive(&bfull[sb]);
      }
    }
  } else {
    // ---------------- epilogue: TMEM -> Y ----------------
    const int q = warp & 3;  // TMEM lane quarter of this warp
    int it = 0;
    for (int t = blockIdx.x; t < P.ntiles; t += gridDim.x, it++) {
      if (!mbar_wait_bounded(acc_full, (uint32_t)(it & 1), P.err)) break;
      tc_fence_after();
      const int tm = t / P.tiles_n, tn = t % P.tiles_n;
#pragma unroll 1
      for (int h = 0; h < 2; h++) {
        const int m = tm * kTileM + h * 128 + q * 32 + lane;
#pragma unroll 1
        for (int c = 0; c < kTileN / 32; c++) {
          uint32_t v[32];
          tmem_ld32(tbase + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * 256 + c * 32), v);
          tmem_ld_wait();
          const int n0 = tn * kTileN + c * 32;
          if (m < P.M) {
            float *yr = P.Y + (size_t)m * P.N + n0;
            if (n0 + 32 <= P.N && ((P.N & 3) == 0)) {
#pragma unroll
              for (int i = 0; i < 32; i += 4)
                *reinterpret_cast<float4 *>(yr + i) = make_float4(__uint_as_float(v[i]), __uint_as_float(v[i + 1]),
                                                                  __uint_as_float(v[i + 2]), __uint_as_float(v[i + 3]));
            } else {
              for (int i = 0; i < 32; i++)
                if (n0 + i < P.N) yr[i] = __uint_as_float(v[i]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

// X f32 [M][K] -> fp16 with each 64-element segment's columns permuted to the
// K order in which the dequant warps write the weight tile.
__global__ void x_to_f16_q4perm(const float *__restrict__ X, __half *__restrict__ Xb, size_t M, int K) {
  const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= M * (size_t)K) return;
  const size_t m = i / K;
  const int k = (int)(i % K);
  const int seg = k >> 6, half = (k >> 5) & 1, r = k & 31;
  // element r of the half sits in repacked quant word r%8, byte r/8; the
  // dequant writes each word's bytes in the order (0, 2, 1, 3)
  const int byte = r >> 3;
  const int kp = (seg << 6) + 32 * half + 4 * (r & 7) + ((byte & 1) << 1) + (byte >> 1);
  Xb[m * K + kp] = __float2half_rn(X[i]);
}

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

bool make_map_2d(CUtensorMap *map, CUtensorMapDataType dt, void *gaddr, uint64_t dim0, uint64_t dim1,
                 uint64_t stride1_bytes, uint32_t box0, uint32_t box1, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {dim0, dim1};
  cuuint64_t strides[1] = {stride1_bytes};
  cuuint32_t box[2] = {box0, box1};
  cuuint32_t es[2] = {1, 1};
  return fn(map, dt, 2, gaddr, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

int32_t gemm_launch(unltd_ctx ctx, const unltd_weight_s &w, const float *X, float *Y, size_t M) {
  if (w.dtype != Q4K)
    return set_error(UNLTD_ERR_UNSUPPORTED, "gemm: only Q4_K weights have a tensor-core GEMM so far");
  if (M == 0 || w.dim_out == 0) return UNLTD_OK;
  const int K = (int)w.dim_in;
  cudaStream_t st = ctx->stream;
  // fp16 copy of X with the permuted segment columns
  const size_t xb_bytes = M * (size_t)K * 2;
  if (ctx->gemm_scratch_bytes < xb_bytes) {
    if (ctx->gemm_scratch) cudaFree(ctx->gemm_scratch);
    ctx->gemm_scratch = nullptr;
    ctx->gemm_scratch_bytes = 0;
    cudaError_t e = cudaMalloc(&ctx->gemm_scratch, xb_bytes);
    if (e != cudaSuccess) return cuda_error(e, "gemm scratch");
    ctx->gemm_scratch_bytes = xb_bytes;
  }
  __half *Xb = reinterpret_cast<__half *>(ctx->gemm_scratch);
  {
    const size_t n = M * (size_t)K;
    x_to_f16_q4perm<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(X, Xb, M, K);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, "gemm x convert");
    ctx->launches += 1;
  }
  CUtensorMap tmA, tmWq, tmWh;
  if (!make_map_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, Xb, (uint64_t)K, M, (uint64_t)K * 2, kStepK, 128,
                   CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_2d(&tmWq, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.dev, w.row_stride, w.dim_out, w.row_stride, 32, kTileN,
                   CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_map_2d(&tmWh, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.dev, w.row_stride, w.dim_out, w.row_stride, 16, kTileN,
                   CU_TENSOR_MAP_SWIZZLE_NONE))
    return set_error(UNLTD_ERR_CUDA, "gemm: cuTensorMapEncodeTiled failed");

  GemmParams P;
  P.M = (int)M;
  P.N = (int)w.dim_out;
  P.K = K;
  P.nb = (int)w.nb;
  P.Y = Y;
  P.err = ctx->err;
  P.tiles_n = (P.N + kTileN - 1) / kTileN;
  P.ntiles = ((P.M + kTileM - 1) / kTileM) * P.tiles_n;
  {
    // the attribute belongs to the current device's context: set it once per device
    static std::mutex mu;
    static std::vector<int> done;
    std::lock_guard<std::mutex> lk(mu);
    if (std::find(done.begin(), done.end(), ctx->device) == done.end()) {
      cudaError_t e = cudaFuncSetAttribute(gemm_q4k_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
      if (e != cudaSuccess) return cuda_error(e, "gemm: shared-memory attribute");
      done.push_back(ctx->device);
    }
  }
  const int grid = std::min(P.ntiles, ctx->num_sms);
  gemm_q4k_tc<<<grid, kThreadsG, kSmemBytes, st>>>(tmA, tmWq, tmWh, P);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "gemm launch");
  ctx->launches += 1;
  return UNLTD_OK;
}

}  // namespace unltd
