// NCCL communicators of libunltd_gpu: tensor-parallel decode across the GPUs
// of one box (one process per GPU). NCCL is opened at run time with dlopen,
// so the library binds to the libnccl.so.2 the host process already loaded
// (e.g. PyTorch's) instead of linking a second copy.
#include <dlfcn.h>
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

int32_t comm_allreduce(unltd_ctx c, cudaStream_t st, void *buf, size_t count, bool max_u64) {
  if (!c->comm) return set_error(UNLTD_ERR_INVALID_ARG, "allreduce: the context has no communicator");
  NcclApi &n = nccl();
  return nccl_error(n.AllReduce(buf, buf, count, max_u64 ? ncclUint64 : ncclFloat32, max_u64 ? ncclMax : ncclSum,
                                static_cast<ncclComm_t>(c->comm), st),
                    "ncclAllReduce");
}

void comm_destroy(unltd_ctx c) {
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
