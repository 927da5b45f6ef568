// The NCCL calls of tensor parallelism, bound when first needed (dlopen of
// libnccl.so.2): a process that never splits a model does not load NCCL,
// and one that already holds it (PyTorch's copy) shares that copy.
#pragma once

#include <nccl.h>

namespace trit {

struct Nccl {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*);
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
  const char* (*GetErrorString)(ncclResult_t);
};

// Throws Error when libnccl.so.2 or one of its functions is missing.
const Nccl& nccl();
void nccl_check(ncclResult_t r, const char* what);

}  // namespace trit
