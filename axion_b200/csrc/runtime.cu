// Host runtime of the C ABI: error strings, per-device state, workspace and
// the device status word written by bounded waits.
#include "runtime.h"

#include <stdarg.h>
#include <stdio.h>

#include <mutex>
#include <string>
#include <vector>

#include "axq8.h"

namespace axq8 {

// One status word per device that loads this library; kernels record the
// first bounded-wait failure here (see common.cuh).
__device__ int g_status_word;

namespace {
thread_local std::string t_err;
std::mutex g_mu;
std::vector<DeviceState*> g_states;
}  // namespace

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_err = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(AXQ8_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

void clear_error() { t_err.clear(); }
const char* last_error() { return t_err.c_str(); }

DeviceState* device_state() {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        cuda_fail(e, "cudaGetDevice");
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    if ((int)g_states.size() <= dev) g_states.resize(dev + 1, nullptr);
    if (g_states[dev]) return g_states[dev];
    DeviceState* ds = new DeviceState();
    ds->device = dev;
    if ((e = cudaDeviceGetAttribute(&ds->sm_count, cudaDevAttrMultiProcessorCount, dev)) !=
            cudaSuccess ||
        (e = cudaDeviceGetAttribute(&ds->max_smem_optin,
                                    cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) !=
            cudaSuccess) {
        cuda_fail(e, "cudaDeviceGetAttribute");
        delete ds;
        return nullptr;
    }
    void* p = nullptr;
    if ((e = cudaGetSymbolAddress(&p, g_status_word)) != cudaSuccess) {
        cuda_fail(e, "cudaGetSymbolAddress(status)");
        delete ds;
        return nullptr;
    }
    ds->status = static_cast<int*>(p);
    g_states[dev] = ds;
    return ds;
}

bool capture_active(cudaStream_t stream) {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    const cudaError_t e = cudaStreamIsCapturing(stream, &st);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();   // e.g. the legacy stream queried during a global capture
        return true;
    }
    return st != cudaStreamCaptureStatusNone;
}

void* workspace(DeviceState* ds, size_t bytes, cudaStream_t stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (ds->workspace_bytes >= bytes) return ds->workspace;
    if (capture_active(stream)) {
        // a grow synchronizes the device and frees the old buffer, neither of
        // which a stream capture allows
        fail(AXQ8_ERR_STATE,
             "workspace must grow to %zu bytes during a stream capture; make a call of this "
             "size outside capture first",
             bytes);
        return nullptr;
    }
    if (ds->workspace) {
        cudaDeviceSynchronize();   // the old buffer may still be read by queued kernels
        cudaFree(ds->workspace);
        ds->workspace = nullptr;
        ds->workspace_bytes = 0;
    }
    size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, want);
    if (e != cudaSuccess) {
        cuda_fail(e, "cudaMalloc(workspace)");
        return nullptr;
    }
    ds->workspace = p;
    ds->workspace_bytes = want;
    return p;
}

}  // namespace axq8

extern "C" {

const char* axq8_last_error(void) { return axq8::last_error(); }

const char* axq8_version(void) { return "axion_b200 axq8 1.0 (sm_100a)"; }

int axq8_status_read(int* code) {
    if (!code) return axq8::fail(AXQ8_ERR_INVALID, "axq8_status_read: null code");
    AXQ8_CUDA_TRY(cudaDeviceSynchronize(), "axq8_status_read: synchronize");
    AXQ8_CUDA_TRY(cudaMemcpyFromSymbol(code, axq8::g_status_word, sizeof(int)),
                  "axq8_status_read: copy");
    return AXQ8_OK;
}

int axq8_status_clear(void) {
    int zero = 0;
    AXQ8_CUDA_TRY(cudaMemcpyToSymbol(axq8::g_status_word, &zero, sizeof(int)),
                  "axq8_status_clear");
    return AXQ8_OK;
}

}  // extern "C"
