// NCCL entry points loaded at run time (dlopen), so that the library loads
// without NCCL and only tensor-parallel decoding requires it.  The library
// looked for is AXQ8_NCCL_LIB if set, else the NCCL found at build time
// (the one PyTorch ships), else libnccl.so.2 from the loader's search path.
#pragma once

#include <nccl.h>

namespace axq8 {

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*);
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t);
    const char* (*GetErrorString)(ncclResult_t);
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    // failure handling: the communicator's asynchronous error, and abort
    // (ends pending NCCL work so that a rank whose peer died can exit)
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*);
    ncclResult_t (*CommAbort)(ncclComm_t);
};

// The loaded API, or nullptr (with the error recorded for axq8_last_error).
const NcclApi* nccl_api();

}  // namespace axq8
