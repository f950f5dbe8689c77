// nccl_dl.h -- the NCCL entry points the tensor-parallel engine uses,
// resolved at run time from the process's libnccl.so.2 (the one already
// loaded, e.g. by PyTorch, else the first the loader finds), so that the
// library does not link a second NCCL into a process that has one.
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>

namespace rt {

struct NcclApi {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
};

// The resolved entry points, or null with *why set.
const NcclApi* nccl_api(const char** why);

}  // namespace rt
