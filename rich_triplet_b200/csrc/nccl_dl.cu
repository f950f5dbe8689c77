// nccl_dl.cu -- run-time binding of NCCL (nccl_dl.h).
#include <dlfcn.h>

#include <mutex>

#include "nccl_dl.h"

namespace rt {

const NcclApi* nccl_api(const char** why) {
    static std::once_flag once;
    static NcclApi api;
    static const char* err = nullptr;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            err = "libnccl.so.2 not found";
            return;
        }
        auto sym = [&](const char* name) {
            void* p = dlsym(h, name);
            if (!p && !err) err = name;
            return p;
        };
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(sym("ncclAllReduce"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
    });
    if (why) *why = err;
    return err ? nullptr : &api;
}

}  // namespace rt
