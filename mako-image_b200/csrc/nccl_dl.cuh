// NCCL, loaded at run time. Only the sequence-parallel DiT step uses it, so the library itself does not depend on
// libnccl: the first sequence-parallel call binds the symbols from an already-loaded libnccl.so.2 (PyTorch's, in a
// Python process) or loads the system one.
#pragma once

#include <nccl.h>

#include <string>

namespace mkb {

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

// The bound API, or null with *err set.
const NcclApi* nccl_api(std::string* err);

}  // namespace mkb
