// Host-side runtime shared by the C ABI entry points: thread-local error
// messages, per-device state (SM count, status word, workspace), and a
// launcher that adds the programmatic-dependent-launch attribute.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <utility>

#include "axq8_status.h"

namespace axq8 {

// Record a message for axq8_last_error() and return `code`.
int fail(int code, const char* fmt, ...);
// Record a CUDA failure ("<what>: <cuda error string>") and return AXQ8_ERR_CUDA.
int cuda_fail(cudaError_t e, const char* what);
void clear_error();
const char* last_error();

struct DeviceState {
    int device = -1;
    int sm_count = 0;
    int max_smem_optin = 0;   // bytes of dynamic shared memory a CTA may opt into
    int* status = nullptr;    // device address of this library's status word
    void* workspace = nullptr;
    size_t workspace_bytes = 0;
};

// State of the current CUDA device, created on first use.  Returns nullptr
// (with the error recorded) if the device cannot be queried.
DeviceState* device_state();

// Grow-only per-device workspace for quantized activations and partials.
// Synchronizes the device before replacing a smaller buffer; returns nullptr
// (AXQ8_ERR_STATE recorded) when a grow is needed while `stream` is captured.
void* workspace(DeviceState* ds, size_t bytes, cudaStream_t stream);

// Whether `stream` is being captured into a CUDA graph (an error from the
// query counts as capturing: nothing that needs a synchronization may run).
bool capture_active(cudaStream_t stream);

// Synthetic Q8_0 weight slice in the repacked row layout: rows [row0,
// row0 + N) and columns [col0, col0 + K) of the [*, Kfull] tensor that
// axq8_synth_q8_0(seed, ..., Kfull, ...) generates (q8_linear.cu).
int synth_q8_0_slice(uint64_t seed, int64_t N, int64_t K, int64_t row0, int64_t col0,
                     int64_t Kfull, float mean, float stdv, void* rows, cudaStream_t stream);

#define AXQ8_CUDA_TRY(expr, what)                          \
    do {                                                    \
        cudaError_t _e = (expr);                            \
        if (_e != cudaSuccess) return ::axq8::cuda_fail(_e, what); \
    } while (0)

// Launch `kern` with optional programmatic stream serialization: the grid
// may start while the previous grid in the stream is still running; the
// kernel itself calls griddepcontrol.wait before touching its inputs.
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                     cudaStream_t stream, bool pdl, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace axq8
