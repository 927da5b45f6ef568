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
  ncclResult_t (*CommAbort)(ncclComm_t);
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*);
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
  const char* (*GetErrorString)(ncclResult_t);
};

// Throws Error when libnccl.so.2 or one of its functions is missing.
const Nccl& nccl();
void nccl_check(ncclResult_t r, const char* what);

// Joins the group of `size` ranks as `rank` on `device`. A group that has
// not formed within `seconds` (a rank failed, or was never started) is an
// error, not a hang: the join runs on a helper thread that is left behind.
ncclComm_t nccl_join(const ncclUniqueId& id, int size, int rank, int device, double seconds);

}  // namespace trit
