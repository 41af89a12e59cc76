// nccl_dl.h -- NCCL entry points resolved at run time.
//
// A single-GPU handle needs no NCCL, and a process may already hold a
// different libnccl.so.2 (PyTorch bundles its own); linking one at build time
// would make whichever loads second bind to the wrong one.  The library
// therefore opens NCCL on first use by a multi-rank handle, reusing the copy
// already loaded in the process when there is one.
#pragma once

#include <nccl.h>

namespace ttl {

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId *);
    ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *);
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *);
    ncclResult_t (*CommFinalize)(ncclComm_t);
    ncclResult_t (*CommAbort)(ncclComm_t);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*GroupStart)();
    ncclResult_t (*GroupEnd)();
    const char *(*GetErrorString)(ncclResult_t);
};

// The resolved API, or nullptr (with *why set) when NCCL cannot be loaded.
const NcclApi *nccl(const char **why);

} // namespace ttl
