// Run-time loading of NCCL (see nccl_dl.h).
#include "nccl_dl.h"

#include <dlfcn.h>
#include <stdio.h>
#include <stdlib.h>

#include <mutex>
#include <string>

#include "axq8_status.h"
#include "runtime.h"

#ifndef AXQ8_NCCL_DIR
#define AXQ8_NCCL_DIR ""
#endif

namespace axq8 {

const NcclApi* nccl_api() {
    static std::once_flag once;
    static NcclApi api;
    static bool ok = false;
    static char why[256] = "";
    std::call_once(once, [] {
        const char* cands[3] = {getenv("AXQ8_NCCL_LIB"), nullptr, "libnccl.so.2"};
        static const std::string dir_lib = std::string(AXQ8_NCCL_DIR) + "/libnccl.so.2";
        if (AXQ8_NCCL_DIR[0]) cands[1] = dir_lib.c_str();
        void* h = nullptr;
        for (const char* c : cands)
            if (c && (h = dlopen(c, RTLD_NOW | RTLD_GLOBAL))) break;
        if (!h) {
            snprintf(why, sizeof(why), "NCCL not found (%s)", dlerror());
            return;
        }
        api.GetUniqueId = (decltype(api.GetUniqueId))dlsym(h, "ncclGetUniqueId");
        api.CommInitRank = (decltype(api.CommInitRank))dlsym(h, "ncclCommInitRank");
        api.CommDestroy = (decltype(api.CommDestroy))dlsym(h, "ncclCommDestroy");
        api.AllReduce = (decltype(api.AllReduce))dlsym(h, "ncclAllReduce");
        api.GetErrorString = (decltype(api.GetErrorString))dlsym(h, "ncclGetErrorString");
        api.AllGather = (decltype(api.AllGather))dlsym(h, "ncclAllGather");
        api.CommGetAsyncError = (decltype(api.CommGetAsyncError))dlsym(h, "ncclCommGetAsyncError");
        api.CommAbort = (decltype(api.CommAbort))dlsym(h, "ncclCommAbort");
        ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.AllReduce &&
             api.GetErrorString && api.AllGather && api.CommGetAsyncError && api.CommAbort;
        if (!ok) snprintf(why, sizeof(why), "NCCL library lacks an entry point");
    });
    if (!ok) {
        fail(AXQ8_ERR_UNSUPPORTED, "%s", why);
        return nullptr;
    }
    return &api;
}

}  // namespace axq8
