/* A stand-in for libnccl.so.2 whose communicator set-up always fails: the failure-injection tests bind it through
 * MKB_NCCL_LIB to check that mkb_dit_set_sequence_parallel reports the error and leaves the handle usable. It has
 * the nine entry points the library binds, with NCCL's published signatures (nccl.h: ncclResult_t is an int-sized
 * enum, ncclUniqueId a 128-byte struct passed by value). Test infrastructure only. */
#include <stddef.h>
#include <string.h>

typedef struct {
    char internal[128];
} ncclUniqueId;
typedef void* ncclComm_t;
typedef int ncclResult_t;

enum { kSuccess = 0, kSystemError = 2 };

ncclResult_t ncclGetUniqueId(ncclUniqueId* id)
{
    memset(id, 0, sizeof(*id));
    return kSuccess;
}

ncclResult_t ncclCommInitRank(ncclComm_t* comm, int nranks, ncclUniqueId id, int rank)
{
    (void)nranks;
    (void)id;
    (void)rank;
    *comm = NULL;
    return kSystemError;
}

ncclResult_t ncclAllGather(const void* send, void* recv, size_t count, int dtype, ncclComm_t comm, void* stream)
{
    (void)send;
    (void)recv;
    (void)count;
    (void)dtype;
    (void)comm;
    (void)stream;
    return kSystemError;
}

#ifndef FAKE_NCCL_NO_P2P /* built without them: a library the binding must refuse */
ncclResult_t ncclSend(const void* send, size_t count, int dtype, int peer, ncclComm_t comm, void* stream)
{
    (void)send;
    (void)count;
    (void)dtype;
    (void)peer;
    (void)comm;
    (void)stream;
    return kSystemError;
}

ncclResult_t ncclRecv(void* recv, size_t count, int dtype, int peer, ncclComm_t comm, void* stream)
{
    (void)recv;
    (void)count;
    (void)dtype;
    (void)peer;
    (void)comm;
    (void)stream;
    return kSystemError;
}

ncclResult_t ncclGroupStart(void)
{
    return kSuccess;
}

ncclResult_t ncclGroupEnd(void)
{
    return kSuccess;
}
#endif

ncclResult_t ncclCommDestroy(ncclComm_t comm)
{
    (void)comm;
    return kSuccess;
}

const char* ncclGetErrorString(ncclResult_t r)
{
    return r == kSuccess ? "no error" : "injected failure (fake NCCL)";
}
