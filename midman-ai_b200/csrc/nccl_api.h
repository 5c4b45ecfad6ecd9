// NCCL entry points resolved at first use with dlopen/dlsym, so loading the
// library does not load NCCL. A process that already has NCCL (for example
// through PyTorch) gets that copy (dlopen by soname returns the loaded one);
// otherwise the system libnccl.so.2 is loaded on the first data-parallel call.
#pragma once
#include <nccl.h>

namespace mm {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*);
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*Reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*Broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*GroupStart)();
  ncclResult_t (*GroupEnd)();
  const char* (*GetErrorString)(ncclResult_t);
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*);
  ncclResult_t (*CommAbort)(ncclComm_t);
};

// Throws std::runtime_error when NCCL cannot be loaded.
const NcclApi& nccl();

}  // namespace mm
