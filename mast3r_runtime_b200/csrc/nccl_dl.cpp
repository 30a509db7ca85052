#include "nccl_dl.h"

#include <dlfcn.h>

#include <mutex>

#include "tmap.h"

namespace m3r {

namespace {

NcclApi g_api;
std::string g_load_error;

void load_api() {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
        const char* e = dlerror();
        g_load_error = std::string("cannot load NCCL (libnccl.so.2): ") + (e ? e : "unknown error");
        return;
    }
    auto sym = [&](const char* name) {
        void* p = dlsym(h, name);
        if (!p && g_load_error.empty()) g_load_error = std::string("NCCL symbol missing: ") + name;
        return p;
    };
    g_api.CommInitAll = reinterpret_cast<decltype(g_api.CommInitAll)>(sym("ncclCommInitAll"));
    g_api.CommDestroy = reinterpret_cast<decltype(g_api.CommDestroy)>(sym("ncclCommDestroy"));
    g_api.AllReduce = reinterpret_cast<decltype(g_api.AllReduce)>(sym("ncclAllReduce"));
    g_api.GroupStart = reinterpret_cast<decltype(g_api.GroupStart)>(sym("ncclGroupStart"));
    g_api.GroupEnd = reinterpret_cast<decltype(g_api.GroupEnd)>(sym("ncclGroupEnd"));
    g_api.GetErrorString = reinterpret_cast<decltype(g_api.GetErrorString)>(sym("ncclGetErrorString"));
}

}  // namespace

const NcclApi& nccl() {
    static std::once_flag once;
    std::call_once(once, load_api);
    if (!g_load_error.empty()) throw Error(kErrNccl, g_load_error);
    return g_api;
}

void nccl_check(ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return;
    const char* msg = g_api.GetErrorString ? g_api.GetErrorString(r) : "unknown";
    throw Error(kErrNccl, std::string(what) + ": " + msg);
}

}  // namespace m3r
