// NCCL communicators of libunltd_gpu: tensor-parallel decode across the GPUs
// of one box (one process per GPU). NCCL is opened at run time with dlopen,
// so the library binds to the libnccl.so.2 the host process already loaded
// (e.g. PyTorch's) instead of linking a second copy.
#include <dlfcn.h>
#include <algorithm>
#include <nccl.h>

#include <mutex>
#include <string>

#include "unltd_host.h"

namespace unltd {
namespace {

struct NcclApi {
  bool ok = false;
  std::string err;
  ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char *(*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi &nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      api.err = std::string("cannot load libnccl.so.2: ") + dlerror();
      return;
    }
    api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
    api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
    api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
    api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(dlsym(h, "ncclAllReduce"));
    api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.AllReduce && api.GetErrorString;
    if (!api.ok) api.err = "libnccl.so.2 lacks an expected symbol";
  });
  return api;
}

int32_t nccl_error(ncclResult_t r, const char *what) {
  if (r == ncclSuccess) return UNLTD_OK;
  return set_error(UNLTD_ERR_NCCL, std::string(what) + ": " + nccl().GetErrorString(r));
}

}  // namespace

// ---- peer all-reduce: one kernel over NVLink peer memory ------------------
// The receive area layout (kPeer* in unltd_host.h): flags, then two
// parities of per-source slots.

struct PeerArgs {
  uint8_t *map[kPeerMaxRanks];  // every rank's area as mapped here
  unsigned *ctr;                // all-reduces issued so far (this device)
  unsigned *done;               // [2]: CTAs that finished writing / summing (reset by the last)
  int rank, world;
  int *err;
};

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t peer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Grid of G CTAs, CTA b on elements [b count / G, (b + 1) count / G): (1)
// this rank's buf into slot [parity][rank] of every rank's area (peer stores
// over NVLink), (2) after a system fence, the last CTA to finish writing
// raises this rank's flag in every area, (3) every CTA waits (bounded, ~2 s)
// for every rank's flag here, (4) the sum (or max) of its elements of the
// slots in rank order 0, 1, ..., so every rank computes the same bits; the
// last CTA to finish advances the counter. Parities alternate: a rank can
// only reuse a parity after all ranks flagged the following all-reduce, i.e.
// finished reading this one.
template <typename T, bool MAXOP>
__global__ void __launch_bounds__(1024) peer_allreduce_kernel(T *buf, int count, PeerArgs a) {
  __shared__ unsigned s_ep;
  __shared__ int s_ok, s_last;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x == 0) {
    s_ep = *a.ctr + 1u;
    s_ok = 1;
  }
  __syncthreads();
  const unsigned ep = s_ep;
  const int G = gridDim.x;
  const int i0 = (int)((long long)count * blockIdx.x / G), i1 = (int)((long long)count * (blockIdx.x + 1) / G);
  const size_t slot0 = kPeerFlagBytes + (size_t)(ep & 1u) * kPeerMaxRanks * kPeerSlotBytes;
  for (int r = 0; r < a.world; r++) {
    T *dst = reinterpret_cast<T *>(a.map[r] + slot0 + (size_t)a.rank * kPeerSlotBytes);
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) dst[i] = buf[i];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&a.done[0], 1u) == (unsigned)G - 1;
  __syncthreads();
  if (s_last) {  // every CTA's stores are visible: raise the flags
    __threadfence_system();
    if (threadIdx.x < a.world)
      st_release_sys(reinterpret_cast<unsigned *>(a.map[threadIdx.x]) + a.rank, ep);
    if (threadIdx.x == 0) a.done[0] = 0u;
  }
  if (threadIdx.x < a.world) {
    const unsigned *flag = reinterpret_cast<const unsigned *>(a.map[a.rank]) + threadIdx.x;
    if (ld_acquire_sys(flag) - ep > 0x7fffffffu) {  // flag < ep (wrap-safe)
      const uint64_t t0 = peer_ns();
      for (uint32_t it = 1;; ++it) {
        if (ld_acquire_sys(flag) - ep <= 0x7fffffffu) break;
        if ((it & 255u) == 0 && peer_ns() - t0 > 2000000000ull) {
          s_ok = 0;
          atomicExch(a.err, kErrPeer);
          break;
        }
      }
    }
  }
  __syncthreads();
  if (s_ok) {
    const uint8_t *mine = a.map[a.rank] + slot0;
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
      T v = __ldcv(reinterpret_cast<const T *>(mine) + i);
      for (int r = 1; r < a.world; r++) {
        const T o = __ldcv(reinterpret_cast<const T *>(mine + (size_t)r * kPeerSlotBytes) + i);
        if constexpr (MAXOP) v = o > v ? o : v;
        else v = __fadd_rn(v, o);
      }
      buf[i] = v;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(&a.done[1], 1u) == (unsigned)G - 1) {  // every CTA has read ep
    a.done[1] = 0u;
    *a.ctr = ep;
  }
}

int32_t peer_allreduce(unltd_ctx c, cudaStream_t st, void *buf, size_t count, bool max_u64) {
  PeerArgs a;
  for (int r = 0; r < kPeerMaxRanks; r++) a.map[r] = static_cast<uint8_t *>(c->peer_map[r]);
  a.ctr = c->peer_ctr;
  a.done = c->peer_ctr + 2;
  a.rank = c->rank;
  a.world = c->world;
  a.err = c->err;
  cudaLaunchConfig_t cfg = {};
  // one CTA for a decode step's vector (latency), more for a batch's
  cfg.gridDim = dim3((unsigned)std::min<size_t>(64, std::max<size_t>(1, count / 4096)));
  cfg.blockDim = dim3(1024);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaError_t e = max_u64 ? cudaLaunchKernelEx(&cfg, peer_allreduce_kernel<unsigned long long, true>,
                                               static_cast<unsigned long long *>(buf), (int)count, a)
                          : cudaLaunchKernelEx(&cfg, peer_allreduce_kernel<float, false>, static_cast<float *>(buf),
                                               (int)count, a);
  c->launches += 1;
  return cuda_error(e, "peer all-reduce");
}

void peer_close(unltd_ctx c) {
  for (int r = 0; r < kPeerMaxRanks; r++) {
    if (c->peer_map[r] && c->peer_map[r] != c->peer_area) cudaIpcCloseMemHandle(c->peer_map[r]);
    c->peer_map[r] = nullptr;
  }
  if (c->peer_area) cudaFree(c->peer_area);
  if (c->peer_ctr) cudaFree(c->peer_ctr);
  c->peer_area = nullptr;
  c->peer_ctr = nullptr;
  c->peer_done = nullptr;
  c->peer_ok = false;
}

int32_t comm_allreduce(unltd_ctx c, cudaStream_t st, void *buf, size_t count, bool max_u64) {
  if (!c->comm) return set_error(UNLTD_ERR_INVALID_ARG, "allreduce: the context has no communicator");
  if (c->peer_ok && count <= kPeerMaxCount) return peer_allreduce(c, st, buf, count, max_u64);
  NcclApi &n = nccl();
  return nccl_error(n.AllReduce(buf, buf, count, max_u64 ? ncclUint64 : ncclFloat32, max_u64 ? ncclMax : ncclSum,
                                static_cast<ncclComm_t>(c->comm), st),
                    "ncclAllReduce");
}

void comm_destroy(unltd_ctx c) {
  peer_close(c);
  if (c->comm && nccl().ok) nccl().CommDestroy(static_cast<ncclComm_t>(c->comm));
  c->comm = nullptr;
}

}  // namespace unltd

using namespace unltd;

extern "C" {

int32_t unltd_comm_unique_id(void *id_out, size_t id_bytes) {
  if (!id_out || id_bytes < NCCL_UNIQUE_ID_BYTES)
    return set_error(UNLTD_ERR_INVALID_ARG, "comm_unique_id: need a buffer of 128 bytes");
  NcclApi &n = nccl();
  if (!n.ok) return set_error(UNLTD_ERR_NCCL, n.err);
  ncclUniqueId id;
  if (int32_t rc = nccl_error(n.GetUniqueId(&id), "ncclGetUniqueId")) return rc;
  memcpy(id_out, id.internal, NCCL_UNIQUE_ID_BYTES);
  return UNLTD_OK;
}

int32_t unltd_comm_init(unltd_ctx c, int32_t rank, int32_t world, const void *id, size_t id_bytes) {
  if (!c || !id || id_bytes < NCCL_UNIQUE_ID_BYTES)
    return set_error(UNLTD_ERR_INVALID_ARG, "comm_init: NULL context or short unique id");
  if (world < 1 || rank < 0 || rank >= world) return set_error(UNLTD_ERR_INVALID_ARG, "comm_init: bad rank/world");
  if (c->comm) return set_error(UNLTD_ERR_INVALID_ARG, "comm_init: the context already has a communicator");
  NcclApi &n = nccl();
  if (!n.ok) return set_error(UNLTD_ERR_NCCL, n.err);
  CtxGuard g(c->device);
  ncclUniqueId uid;
  memcpy(uid.internal, id, NCCL_UNIQUE_ID_BYTES);
  ncclComm_t comm = nullptr;
  if (int32_t rc = nccl_error(n.CommInitRank(&comm, world, uid, rank), "ncclCommInitRank")) return rc;
  c->comm = comm;
  c->rank = rank;
  c->world = world;
  return UNLTD_OK;
}

int32_t unltd_peer_export(unltd_ctx c, void *handle_out, size_t handle_bytes) {
  if (!c || !handle_out || handle_bytes < sizeof(cudaIpcMemHandle_t))
    return set_error(UNLTD_ERR_INVALID_ARG, "peer_export: NULL context or a handle buffer under 64 bytes");
  if (!c->comm) return set_error(UNLTD_ERR_INVALID_ARG, "peer_export: call comm_init first");
  if (c->world > kPeerMaxRanks) return set_error(UNLTD_ERR_UNSUPPORTED, "peer_export: more than 8 ranks");
  CtxGuard g(c->device);
  if (!c->peer_area) {
    cudaError_t e = cudaMalloc(&c->peer_area, kPeerAreaBytes);
    if (e == cudaSuccess) e = cudaMemset(c->peer_area, 0, kPeerAreaBytes);
    // [0] all-reduces issued, [1] the fused GEMV send path's CTA count, [2..3]
    // the all-reduce kernel's CTA counts
    if (e == cudaSuccess) e = cudaMalloc(&c->peer_ctr, 4 * sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(c->peer_ctr, 0, 4 * sizeof(unsigned));
    c->peer_done = c->peer_ctr + 1;
    if (e != cudaSuccess) {
      peer_close(c);
      return cuda_error(e, "peer_export: area");
    }
  }
  cudaIpcMemHandle_t h;
  if (cudaError_t e = cudaIpcGetMemHandle(&h, c->peer_area)) return cuda_error(e, "cudaIpcGetMemHandle");
  memcpy(handle_out, &h, sizeof(h));
  return UNLTD_OK;
}

int32_t unltd_peer_import(unltd_ctx c, const void *handles, size_t handle_bytes) {
  if (!c || !handles || !c->peer_area)
    return set_error(UNLTD_ERR_INVALID_ARG, "peer_import: NULL argument or peer_export not called");
  if (handle_bytes < sizeof(cudaIpcMemHandle_t) * (size_t)c->world)
    return set_error(UNLTD_ERR_INVALID_ARG, "peer_import: need world x 64 bytes of handles");
  CtxGuard g(c->device);
  for (int r = 0; r < c->world; r++) {
    if (r == c->rank) {
      c->peer_map[r] = c->peer_area;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const uint8_t *>(handles) + r * sizeof(h), sizeof(h));
    void *p = nullptr;
    if (cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess)) {
      peer_close(c);
      return cuda_error(e, "cudaIpcOpenMemHandle");
    }
    c->peer_map[r] = p;
  }
  c->peer_ok = true;
  return UNLTD_OK;
}

int32_t unltd_allreduce_sum_f32(unltd_ctx c, float *buf_dev, size_t count) {
  if (!c || !buf_dev) return set_error(UNLTD_ERR_INVALID_ARG, "allreduce_sum_f32: NULL argument");
  CtxGuard g(c->device);
  return comm_allreduce(c, c->stream, buf_dev, count, false);
}

int32_t unltd_allreduce_max_u64(unltd_ctx c, uint64_t *buf_dev, size_t count) {
  if (!c || !buf_dev) return set_error(UNLTD_ERR_INVALID_ARG, "allreduce_max_u64: NULL argument");
  CtxGuard g(c->device);
  return comm_allreduce(c, c->stream, buf_dev, count, true);
}

}  // extern "C"
