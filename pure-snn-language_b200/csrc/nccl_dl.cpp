#include "nccl_dl.h"

#include <dlfcn.h>

#include <mutex>
#include <string>

#include "common.h"

namespace snnb {

const NcclApi& nccl() {
    static NcclApi api{};
    static std::string err;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) {
            const char* e = dlerror();
            err = std::string("cannot open libnccl.so.2: ") + (e ? e : "unknown error");
            return;
        }
        auto sym = [&](const char* name) -> void* {
            void* p = dlsym(h, name);
            if (!p && err.empty()) err = std::string("libnccl.so.2 lacks ") + name;
            return p;
        };
        api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(sym("ncclGetUniqueId"));
        api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(sym("ncclCommInitRank"));
        api.AllGather = reinterpret_cast<decltype(api.AllGather)>(sym("ncclAllGather"));
        api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(sym("ncclCommDestroy"));
        api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(sym("ncclGetErrorString"));
    });
    SNN_REQUIRE(err.empty(), SNN_ERR_UNSUPPORTED, err);
    return api;
}

}  // namespace snnb
