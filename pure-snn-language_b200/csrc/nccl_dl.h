// NCCL entry points used by column sharding, resolved at run time.
//
// The library does not link NCCL: it is opened (dlopen of libnccl.so.2) the
// first time a network is sharded or a unique id is made.  A process that
// never shards then loads no NCCL at all, and a process that has loaded an
// NCCL build already (PyTorch bundles its own) shares that one instead of
// binding the soname to another version first, which would leave the later
// loader's newer symbols unresolved.
#pragma once
#include <cuda_runtime.h>
#include <nccl.h>

namespace snnb {

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*);
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int);
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    const char* (*GetErrorString)(ncclResult_t);
};

// The resolved entry points; throws snnb::Error(SNN_ERR_UNSUPPORTED) when
// libnccl.so.2 or one of them cannot be found.
const NcclApi& nccl();

}  // namespace snnb
