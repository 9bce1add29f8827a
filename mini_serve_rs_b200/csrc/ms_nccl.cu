// NCCL binding resolved at run time (dlsym), so libms_engine.so has no link
// dependency on a particular libnccl: in a process that already loaded NCCL
// (torch, or a Rust host linking it) the loaded copy is used; otherwise
// libnccl.so.2 is opened.  Used only for the tensor-parallel configuration
// (the all-reduce after o_proj and down_proj, sharded by KV head).
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "ms_internal.h"

namespace ms {
namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*async_error)(ncclComm_t, ncclResult_t *) = nullptr;
  ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  bool ok = false;
};

const NcclApi &api() {
  static NcclApi a;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = RTLD_DEFAULT;
    if (!dlsym(h, "ncclAllReduce")) {
      h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
      if (!h) return;
    }
    a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    a.comm_abort = reinterpret_cast<decltype(a.comm_abort)>(dlsym(h, "ncclCommAbort"));
    a.async_error = reinterpret_cast<decltype(a.async_error)>(dlsym(h, "ncclCommGetAsyncError"));
    a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(h, "ncclAllReduce"));
    a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
    a.ok = a.get_unique_id && a.comm_init_rank && a.comm_destroy && a.comm_abort && a.async_error && a.all_reduce &&
           a.all_gather;
  });
  return a;
}

}  // namespace

bool nccl_available() { return api().ok; }

// Sum-all-reduce of `count` elements in place on `stream`.
int nccl_allreduce_sum(void *buf, size_t count, int dtype, void *comm, cudaStream_t stream) {
  if (!api().ok) return -1;
  const ncclDataType_t t = dtype == MS_DTYPE_F32 ? ncclFloat32 : dtype == MS_DTYPE_BF16 ? ncclBfloat16 : ncclFloat16;
  return int(api().all_reduce(buf, buf, count, t, ncclSum, static_cast<ncclComm_t>(comm), stream));
}

// In-place all-gather of `bytes` per rank: rank r's part sits at buf + r * bytes.
int nccl_allgather_bytes(void *buf, size_t bytes, int rank, void *comm, cudaStream_t stream) {
  if (!api().ok) return -1;
  return int(api().all_gather(static_cast<char *>(buf) + size_t(rank) * bytes, buf, bytes, ncclUint8,
                              static_cast<ncclComm_t>(comm), stream));
}

// Minimum over ranks of one int32 in device memory, in place.
int nccl_allreduce_min_i32(int32_t *buf, void *comm, cudaStream_t stream) {
  if (!api().ok) return -1;
  return int(api().all_reduce(buf, buf, 1, ncclInt32, ncclMin, static_cast<ncclComm_t>(comm), stream));
}

// 0 = healthy, otherwise the communicator's asynchronous error code.
int nccl_async_error(void *comm) {
  if (!api().ok || !comm) return -1;
  ncclResult_t r = ncclSuccess;
  if (api().async_error(static_cast<ncclComm_t>(comm), &r) != ncclSuccess) return -1;
  return int(r);
}

void nccl_abort(void *comm) {
  if (api().ok && comm) api().comm_abort(static_cast<ncclComm_t>(comm));
}

}  // namespace ms

extern "C" int ms_nccl_get_unique_id(uint8_t *out, int32_t len) {
  if (!out || len < NCCL_UNIQUE_ID_BYTES) return MS_E_INVALID;
  if (!ms::api().ok) return MS_E_DEVICE;
  ncclUniqueId id;
  if (ms::api().get_unique_id(&id) != ncclSuccess) return MS_E_DEVICE;
  std::memcpy(out, id.internal, NCCL_UNIQUE_ID_BYTES);
  return MS_OK;
}

extern "C" int ms_nccl_comm_init(void **comm_out, int32_t nranks, const uint8_t *unique_id, int32_t rank,
                                 int32_t device) {
  if (!comm_out || !unique_id || nranks <= 0 || rank < 0 || rank >= nranks) return MS_E_INVALID;
  if (!ms::api().ok) return MS_E_DEVICE;
  if (cudaSetDevice(device) != cudaSuccess) return MS_E_DEVICE;
  ncclUniqueId id;
  std::memcpy(id.internal, unique_id, NCCL_UNIQUE_ID_BYTES);
  ncclComm_t c = nullptr;
  if (ms::api().comm_init_rank(&c, nranks, id, rank) != ncclSuccess) return MS_E_DEVICE;
  *comm_out = c;
  return MS_OK;
}

extern "C" int ms_nccl_comm_destroy(void *comm) {
  if (!comm) return MS_OK;
  if (!ms::api().ok) return MS_E_DEVICE;
  return ms::api().comm_destroy(static_cast<ncclComm_t>(comm)) == ncclSuccess ? MS_OK : MS_E_DEVICE;
}
