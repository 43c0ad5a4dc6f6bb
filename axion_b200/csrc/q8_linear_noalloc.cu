// axq8_linear_noalloc: the A8 linear without any device allocation.
//
// axq8_linear (A8 mode) quantizes the activation into a workspace that the
// library cudaMalloc's on first use and grows on demand.  Some callers cannot
// allow that: code that runs with a fixed, pre-planned device-memory budget
// (an allocator that owns all of HBM, such as a serving runtime's block pool),
// or code that must not synchronize the device, which cudaMalloc/cudaFree may
// do.  This entry point serves them: its scratch is a file-scope static
// device array of fixed size, reserved on every GPU that loads the library
// for as long as the library stays loaded.
//
// Kernels: M <= 8 and M > 64 run the streaming GEMV, 8 < M <= 64 the skinny
// tensor-core product (which combines its K splits on chip).  Up to 64 rows
// these are the kernels axq8_linear picks; above 64 rows axq8_linear runs the
// tcgen05 product, whose split-K partials need global scratch, so this entry
// point keeps the GEMV there (slower at those widths; the result differs from
// axq8_linear's only in the fp32 combination order).
//
// Limits and sharing rules:
//  * at most kNoAllocMaxMK = 1,048,576 activation elements per call (M * K):
//    1 MiB of int8 quants plus 192 KiB of fp32 block scales (1.1875 MiB);
//  * the array is shared by every call on a device and keeps the previous
//    call's contents; the quantizer overwrites every byte a call reads, so
//    nothing needs clearing, but calls that overlap on the GPU (two streams,
//    or two host threads) race on the array and must be serialized by the
//    caller;
//  * the first call on each device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current and keeps it; make that
//    first call before any stream capture, and do not use the library across
//    a cudaDeviceReset (the kept address would be stale).
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "axq8.h"
#include "common.cuh"
#include "q8_mma.h"
#include "runtime.h"

namespace {

constexpr int64_t kNoAllocMaxMK = 1 << 20;
constexpr int64_t kNoAllocScaleOffset = kNoAllocMaxMK;                    // bytes of int8 quants
// fp32 block scales: [M][K/32] for the GEMV (MK/8 bytes), or [K/32][Mp] with
// Mp = M rounded up to 4 for the skinny product (MK/8 + 3K/8 bytes, and
// 3K/8 < 44 KB for the K that M >= 9 allows)
constexpr int64_t kNoAllocScaleBytes = kNoAllocMaxMK / 32 * 4 + (64 << 10);
constexpr int64_t kNoAllocBytes = kNoAllocMaxMK + kNoAllocScaleBytes;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

std::mutex g_mu;
void* g_scratch_dev[64] = {nullptr};   // device address of the array, per device

// Device address of the scratch array on the current device.  The symbol's
// name is only a host-side stand-in: kernels must get this address.
int scratch_address(void** out) {
    int dev = 0;
    AXQ8_CUDA_TRY(cudaGetDevice(&dev), "axq8_linear_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= 64)
        return axq8::fail(AXQ8_ERR_UNSUPPORTED, "axq8_linear_noalloc: device ordinal %d", dev);
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch_dev[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return axq8::cuda_fail(e, "axq8_linear_noalloc: cudaGetSymbolAddress");
        g_scratch_dev[dev] = p;
    }
    *out = g_scratch_dev[dev];
    return AXQ8_OK;
}

}  // namespace

extern "C" int axq8_linear_noalloc(const axq8_weight_t* w, const float* x, int64_t M, float* y,
                                   void* stream) {
    if (!w) return axq8::fail(AXQ8_ERR_INVALID, "axq8_linear_noalloc: null weight");
    if (M < 0) return axq8::fail(AXQ8_ERR_INVALID, "axq8_linear_noalloc: M < 0");
    if (M == 0) return AXQ8_OK;
    if (!x || !y) return axq8::fail(AXQ8_ERR_INVALID, "axq8_linear_noalloc: null pointer");
    if (w->K <= 0 || w->K % axq8::QK)
        return axq8::fail(AXQ8_ERR_INVALID, "axq8_linear_noalloc: bad weight K=%lld",
                          (long long)w->K);
    if (M > kNoAllocMaxMK / w->K)
        return axq8::fail(AXQ8_ERR_INVALID,
                          "axq8_linear_noalloc: M*K = %lld*%lld exceeds the fixed scratch of "
                          "%lld activation elements",
                          (long long)M, (long long)w->K, (long long)kNoAllocMaxMK);
    void* scratch = nullptr;
    int rc = scratch_address(&scratch);
    if (rc) return rc;
    int8_t* xq = static_cast<int8_t*>(scratch);
    float* dx = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + kNoAllocScaleOffset);
    if (axq8::skinny_eligible(w, M)) {
        // the skinny product: scales transposed, [K/32][Mp]
        const int64_t d_bytes = (int64_t)sizeof(float) * (w->K / axq8::QK) * axq8::mma_scale_pitch(M);
        if (d_bytes > kNoAllocScaleBytes)
            return axq8::fail(AXQ8_ERR_INVALID,
                              "axq8_linear_noalloc: %lld bytes of block scales exceed the fixed "
                              "scratch",
                              (long long)d_bytes);
        axq8::DeviceState* ds = axq8::device_state();
        if (!ds) return AXQ8_ERR_CUDA;
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        if ((rc = axq8::mma_quantize(ds, x, M, w->K, xq, dx, s))) return rc;
        return axq8::mmq_linear(ds, w, xq, dx, M, nullptr, y, w->N, s);
    }
    rc = axq8_quantize_act(x, M, w->K, xq, dx, stream);
    if (rc) return rc;
    return axq8_linear_q8act(w, xq, dx, M, nullptr, y, stream);
}
