// NCCL, loaded at run time for the expert-parallel entry points (moe_ep_init / moe_forward_ep).
//
// The library does not link NCCL: a process that only runs single-GPU layers never needs it, and
// a process that already loaded an NCCL build (PyTorch bundles one) keeps using that copy, since
// dlopen of the same soname returns the loaded library.  Types and signatures come from the
// system's nccl.h; only the entry points below are resolved.
#include <dlfcn.h>

#include <mutex>

#include "moe_internal.h"

namespace moe {

const NcclApi* nccl_api(std::string* err) {
    static NcclApi api;
    static std::once_flag once;
    static std::string load_err;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            const char* e = dlerror();
            load_err = std::string("cannot load libnccl.so.2: ") + (e ? e : "unknown error");
            return;
        }
        bool ok = true;
        auto sym = [&](const char* name) {
            void* p = dlsym(h, name);
            if (!p) {
                ok = false;
                load_err = std::string("libnccl lacks ") + name;
            }
            return p;
        };
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
        api.comm_abort = reinterpret_cast<decltype(api.comm_abort)>(sym("ncclCommAbort"));
        api.group_start = reinterpret_cast<decltype(api.group_start)>(sym("ncclGroupStart"));
        api.group_end = reinterpret_cast<decltype(api.group_end)>(sym("ncclGroupEnd"));
        api.send = reinterpret_cast<decltype(api.send)>(sym("ncclSend"));
        api.recv = reinterpret_cast<decltype(api.recv)>(sym("ncclRecv"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(sym("ncclAllReduce"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
        api.ok = ok;
    });
    if (!api.ok) {
        if (err) *err = load_err;
        return nullptr;
    }
    return &api;
}

}  // namespace moe
