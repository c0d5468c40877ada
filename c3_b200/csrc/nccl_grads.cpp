// Gradient all-reduce through NCCL for hosts that own an NCCL communicator.
//
// This is the exchange step of the data-parallel captured backward (sum of [dW || db] over
// the ranks). The reference has no collective; the C ABI here is the one a C++ host of the
// C3 API calls after c3cu_gemm_dw / c3cu_relu_mask_db. NCCL is resolved at run time
// (dlopen "libnccl.so.2"): a process that already loaded NCCL (e.g. through torch) shares that
// copy, and the library still loads where NCCL is absent (the calls then report
// C3CU_ERR_UNSUPPORTED). Only the public nccl.h types are used.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "c3cu.h"
#include "host_util.h"

namespace {

struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) comm_init_rank = nullptr;
  decltype(&ncclCommDestroy) comm_destroy = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  decltype(&ncclGetVersion) get_version = nullptr;
  bool ok = false;
  char why[256] = {0};
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* names[] = {"libnccl.so.2", "libnccl.so"};
    void* h = nullptr;
    for (const char* n : names) {
      h = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
      if (h) break;
    }
    if (!h) {
      snprintf(api.why, sizeof(api.why), "NCCL not found: %s", dlerror());
      return;
    }
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    api.get_version = reinterpret_cast<decltype(api.get_version)>(dlsym(h, "ncclGetVersion"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_reduce &&
             api.error_string && api.get_version;
    if (!api.ok) snprintf(api.why, sizeof(api.why), "NCCL library lacks a required entry point");
  });
  return api;
}

int nccl_status(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return C3CU_OK;
  c3cu::set_error("%s: NCCL error %d (%s)", what, static_cast<int>(r), nccl().error_string(r));
  return C3CU_ERR_CUDA;
}

int require_nccl() {
  if (nccl().ok) return C3CU_OK;
  c3cu::set_error("%s", nccl().why);
  return C3CU_ERR_UNSUPPORTED;
}

}  // namespace

extern "C" int c3cu_nccl_version(int* version) {
  int rc = require_nccl();
  if (rc != C3CU_OK) return rc;
  if (!version) {
    c3cu::set_error("nccl_version: null pointer");
    return C3CU_ERR_INVALID;
  }
  return nccl_status(nccl().get_version(version), "nccl_version");
}

extern "C" int c3cu_nccl_unique_id(void* id_out) {
  int rc = require_nccl();
  if (rc != C3CU_OK) return rc;
  if (!id_out) {
    c3cu::set_error("nccl_unique_id: null pointer");
    return C3CU_ERR_INVALID;
  }
  ncclUniqueId id;
  rc = nccl_status(nccl().get_unique_id(&id), "nccl_unique_id");
  if (rc == C3CU_OK) std::memcpy(id_out, &id, sizeof(id));
  return rc;
}

extern "C" int c3cu_nccl_comm_init(void** comm_out, const void* id, int world, int rank) {
  int rc = require_nccl();
  if (rc != C3CU_OK) return rc;
  if (!comm_out || !id || world < 1 || rank < 0 || rank >= world) {
    c3cu::set_error("nccl_comm_init: bad arguments (world %d, rank %d)", world, rank);
    return C3CU_ERR_INVALID;
  }
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclComm_t comm = nullptr;
  rc = nccl_status(nccl().comm_init_rank(&comm, world, uid, rank), "nccl_comm_init");
  *comm_out = rc == C3CU_OK ? static_cast<void*>(comm) : nullptr;
  return rc;
}

extern "C" int c3cu_nccl_comm_destroy(void* comm) {
  int rc = require_nccl();
  if (rc != C3CU_OK) return rc;
  if (!comm) return C3CU_OK;
  return nccl_status(nccl().comm_destroy(static_cast<ncclComm_t>(comm)), "nccl_comm_destroy");
}

extern "C" int c3cu_allreduce_grads(void* grads, int64_t count, int dtype, void* comm,
                                    c3cu_stream_t stream) {
  int rc = require_nccl();
  if (rc != C3CU_OK) return rc;
  if (count < 0 || !comm || (count > 0 && !grads) ||
      (dtype != C3CU_DTYPE_F32 && dtype != C3CU_DTYPE_BF16)) {
    c3cu::set_error("allreduce_grads: bad arguments (count %lld, dtype %d)",
                    static_cast<long long>(count), dtype);
    return C3CU_ERR_INVALID;
  }
  if (count == 0) return C3CU_OK;
  const ncclDataType_t t = dtype == C3CU_DTYPE_F32 ? ncclFloat32 : ncclBfloat16;
  return nccl_status(nccl().all_reduce(grads, grads, static_cast<size_t>(count), t, ncclSum,
                                       static_cast<ncclComm_t>(comm), static_cast<cudaStream_t>(stream)),
                     "allreduce_grads");
}
