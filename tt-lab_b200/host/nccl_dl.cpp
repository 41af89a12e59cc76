// nccl_dl.cpp -- run-time binding of the NCCL entry points (see nccl_dl.h).
#include "../csrc/nccl_dl.h"

#include <dlfcn.h>

#include <mutex>

namespace ttl {

const NcclApi *nccl(const char **why) {
    static NcclApi api;
    static const NcclApi *result = nullptr;
    static const char *error = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // already in the process?
        if (!lib) {
            lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        }
        if (!lib) {
            error = "libnccl.so.2 not found";
            return;
        }
        bool ok = true;
        auto get = [&](auto &fn, const char *name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(lib, name));
            ok = ok && fn != nullptr;
        };
        get(api.GetUniqueId, "ncclGetUniqueId");
        get(api.CommInitRankConfig, "ncclCommInitRankConfig");
        get(api.CommGetAsyncError, "ncclCommGetAsyncError");
        get(api.CommFinalize, "ncclCommFinalize");
        get(api.CommAbort, "ncclCommAbort");
        get(api.CommDestroy, "ncclCommDestroy");
        get(api.AllReduce, "ncclAllReduce");
        get(api.AllGather, "ncclAllGather");
        get(api.Send, "ncclSend");
        get(api.Recv, "ncclRecv");
        get(api.GroupStart, "ncclGroupStart");
        get(api.GroupEnd, "ncclGroupEnd");
        get(api.GetErrorString, "ncclGetErrorString");
        if (!ok) {
            error = "libnccl.so.2 lacks an expected entry point";
            return;
        }
        result = &api;
    });
    if (why) {
        *why = error;
    }
    return result;
}

} // namespace ttl
