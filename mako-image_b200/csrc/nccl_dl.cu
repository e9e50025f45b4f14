#include "nccl_dl.cuh"

#include <dlfcn.h>

#include <cstdlib>
#include <mutex>
#include <string>

namespace mkb {

const NcclApi* nccl_api(std::string* err)
{
    static NcclApi api;
    static std::string load_error;
    static bool ok = false;
    static std::once_flag once;
    std::call_once(once, [] {
        // MKB_NCCL_LIB names another NCCL build to bind (a path or soname); by default the process's already
        // loaded libnccl.so.2 (PyTorch's), else the system's.
        const char* over = std::getenv("MKB_NCCL_LIB");
        const std::string lib = over && over[0] ? over : "libnccl.so.2";
        void* h = over && over[0] ? nullptr : dlopen(lib.c_str(), RTLD_NOW | RTLD_NOLOAD);
        if (!h)
            h = dlopen(lib.c_str(), RTLD_NOW | RTLD_LOCAL);
        if (!h) {
            const char* e = dlerror();
            load_error = lib + " not loadable: " + (e ? e : "?");
            return;
        }
        auto bind = [&](auto& fn, const char* name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            return fn != nullptr;
        };
        if (!bind(api.GetUniqueId, "ncclGetUniqueId") || !bind(api.CommInitRank, "ncclCommInitRank") ||
            !bind(api.AllGather, "ncclAllGather") || !bind(api.Send, "ncclSend") || !bind(api.Recv, "ncclRecv") ||
            !bind(api.GroupStart, "ncclGroupStart") || !bind(api.GroupEnd, "ncclGroupEnd") ||
            !bind(api.CommDestroy, "ncclCommDestroy") ||
            !bind(api.GetErrorString, "ncclGetErrorString")) {
            load_error = lib + " lacks an expected symbol";
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
