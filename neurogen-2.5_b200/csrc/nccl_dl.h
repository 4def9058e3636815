// NCCL resolved at run time (dlopen of libnccl.so.2): the library has no
// link-time NCCL dependency and shares the copy a host process (e.g. torch)
// has already loaded.
#pragma once
#include <cuda_runtime.h>
#include <nccl.h>

namespace ngb {
struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId *);
  ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  const char *(*GetErrorString)(ncclResult_t);
};
// Throws when NCCL cannot be loaded.
const NcclApi &nccl();
void nccl_check(ncclResult_t r, const char *what);
} // namespace ngb
