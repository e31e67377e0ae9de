// NCCL entry points resolved at run time (dlopen of libnccl.so.2) the first
// time tensor parallelism is used. The library has no link-time NCCL
// dependency, so a process that already loaded an NCCL (PyTorch ships its
// own) keeps using that one, and single-GPU users need none at all.
#pragma once
#include <nccl.h>

namespace q4k {

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;  // optional: a failed peer's communicator
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

// Loads NCCL on first use; throws q4k::Error when it is not available.
const NcclApi& nccl();

}  // namespace q4k
