// NCCL for the batch-1 split-KV step (the long-context case across GPUs): the few entry points this library uses,
// resolved at run time from the process's libnccl.so.2 (the one torch.distributed loads, or the system's), so that
// the library links no NCCL of its own and single-GPU use needs none.
#pragma once

#include <dlfcn.h>
#include <nccl.h>

#include <string>

#include "common.cuh"

namespace xtg {

struct NcclApi {
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

inline const NcclApi& nccl_api() {
  static NcclApi api;
  static bool loaded = false;
  if (loaded) return api;
  void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!lib) throw CudaError(std::string("split-KV: libnccl.so.2 not found: ") + dlerror());
  auto sym = [&](const char* name) {
    void* p = dlsym(lib, name);
    if (!p) throw CudaError(std::string("split-KV: libnccl.so.2 lacks ") + name);
    return p;
  };
  api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
  api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
  api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
  api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
  loaded = true;
  return api;
}

inline void nccl_check(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) throw CudaError(std::string("split-KV: ") + what + ": " + nccl_api().error_string(r));
}

}  // namespace xtg
