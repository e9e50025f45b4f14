#include "nccl_dl.cuh"

#include <dlfcn.h>

#include <mutex>

namespace mkb {

const NcclApi* nccl_api(std::string* err)
{
    static NcclApi api;
    static std::string load_error;
    static bool ok = false;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h)
            h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) {
            const char* e = dlerror();
            load_error = std::string("libnccl.so.2 not loadable: ") + (e ? e : "?");
            return;
        }
        auto bind = [&](auto& fn, const char* name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            return fn != nullptr;
        };
        if (!bind(api.GetUniqueId, "ncclGetUniqueId") || !bind(api.CommInitRank, "ncclCommInitRank") ||
            !bind(api.AllGather, "ncclAllGather") || !bind(api.CommDestroy, "ncclCommDestroy") ||
            !bind(api.GetErrorString, "ncclGetErrorString")) {
            load_error = "libnccl.so.2 lacks an expected symbol";
            return;
        }
        ok = true;
    });
    if (!ok) {
        if (err)
            *err = load_error;
        return nullptr;
    }
    return &api;
}

}  // namespace mkb
