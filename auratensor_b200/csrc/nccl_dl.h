// NCCL entry points resolved at run time (dlopen of libnccl.so.2), so the
// library loads without NCCL and shares the process's already-loaded NCCL
// (for example the one PyTorch brought in) instead of pinning a second copy.
#pragma once

#include <nccl.h>

namespace at {

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

// Loads NCCL once; throws Error(AT_ERR_NCCL) when it is unavailable.
const NcclApi& nccl();
void nccl_check(ncclResult_t r, const char* what);

}  // namespace at
