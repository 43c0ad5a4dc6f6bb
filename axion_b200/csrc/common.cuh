// Shared device helpers for the Q8_0 kernels (sm_100a only).
//
// Inline PTX wrappers for mbarriers, 1-D bulk async copies (TMA engine,
// non-tensor form, no multicast), programmatic dependent launch, and the
// bounded-wait discipline every spin in this library follows: a wait gives up
// after a fixed clock budget, records an error code in the device status word
// and lets the kernel return, so a lost arrival can never hang the GPU.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "axq8_status.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "axion_b200 kernels target sm_100a only"
#endif

namespace axq8 {

constexpr int QK = 32;                 // elements per Q8_0 block
constexpr int Q8_0_BYTES = 34;         // fp16 d + 32 int8 (GGUF on-disk block)

// Device row layout of a repacked Q8_0 weight ("Q8R"): for every output row
// n, K int8 quants, then K/32 fp16 scales, then zero padding to 16 bytes.
// One row is therefore one 16-byte-aligned contiguous span that a single
// bulk copy can move, and the whole [N, K] weight is a 2-D array with a
// 16-byte-multiple row stride (a valid TMA tensor map for the quants).
__host__ __device__ inline int64_t q8r_scale_bytes(int64_t K) {
    return (((K / QK) * 2) + 15) / 16 * 16;
}
__host__ __device__ inline int64_t q8r_row_stride(int64_t K) {
    return K + q8r_scale_bytes(K);
}

// Wall-clock budget of any bounded wait, in SM clock cycles (~1 s at 2 GHz).
constexpr long long WAIT_BUDGET_CYCLES = 2000000000LL;

__device__ inline uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ inline void record_status(int* status, int code) {
    if (status) atomicCAS(status, 0, code);
}

// ---- mbarrier -------------------------------------------------------------

__device__ inline void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ inline void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ inline void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ inline void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ inline bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.  Returns
// false (and records `code`) when the budget runs out.
__device__ inline bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* status,
                                         int code) {
    if (mbar_try_wait(bar, parity)) return true;
    long long t0 = clock64();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (clock64() - t0 > WAIT_BUDGET_CYCLES) {
            record_status(status, code);
            return false;
        }
    }
}

// ---- 1-D bulk copy global -> shared (TMA engine, no tensor map) -----------
// Both addresses 16-byte aligned, size a multiple of 16.  Completion is
// signalled as transaction bytes on `bar`.
__device__ inline void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ---- cp.async (16 bytes global -> shared, no register staging) -------------
__device__ inline void cp_async16(void* smem_dst, const void* gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)),
                 "l"(gmem_src)
                 : "memory");
}
// 16 bytes, or zeros when `valid` is false (src-size 0: nothing is read).
__device__ inline void cp_async16_zfill(void* smem_dst, const void* gmem_src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)),
                 "l"(gmem_src), "r"(valid ? 16 : 0)
                 : "memory");
}
// 8 bytes (both addresses 8-byte aligned), through L1.
__device__ inline void cp_async8(void* smem_dst, const void* gmem_src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src)
                 : "memory");
}
__device__ inline void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ inline void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Wait until at most N of this thread's committed cp.async groups are pending.
template <int N>
__device__ inline void cp_async_wait_group() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---- programmatic dependent launch ----------------------------------------
// wait: block until the preceding grid in the stream has completed and its
// writes are visible (no-op when the launch had no programmatic edge).
__device__ inline void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// launch_dependents: allow the next grid to start launching its CTAs.
__device__ inline void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" :::);
}

// ---- small numeric helpers -------------------------------------------------

__device__ inline float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ inline float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Packed fp32 fused multiply-add (sm_100 fma.rn.f32x2): d = a * b + c per lane
// of the pair, each rounded to nearest like fmaf, at one instruction for both.
// The builtin keeps the pair in a 64-bit register pair for the compiler.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// Loads of data that another kernel of the same stream produced.  Kernels here
// are launched with programmatic dependent launch: a kernel starts while its
// predecessors still run and only griddepcontrol.wait orders it after them.
// The read-only (non-coherent) path that __ldg and `const __restrict__`
// pointers allow assumes the data does not change for the kernel's lifetime,
// which no longer holds, and was measured to return stale values; these
// loads go through L2 (ld.global.cg), which the wait makes coherent.
__device__ __forceinline__ float ld_cg(const float* p) { return __ldcg(p); }
__device__ __forceinline__ int ld_cg(const int* p) { return __ldcg(p); }
__device__ __forceinline__ float2 ld_cg2(const float* p) {
    return __ldcg(reinterpret_cast<const float2*>(p));
}
__device__ __forceinline__ float4 ld_cg4(const float* p) {
    return __ldcg(reinterpret_cast<const float4*>(p));
}

// Round half away from zero and clamp to the symmetric int8 range; the
// activation quantizer's rounding rule (C99 roundf semantics).
__device__ inline int q8_round(float v) {
    float r = roundf(v);
    r = fminf(fmaxf(r, -127.0f), 127.0f);
    return static_cast<int>(r);
}

// A8 quantization of one 32-block held by 4 consecutive lanes, 8 values each
// (lane 4k + i holds elements 8i..8i+7): the 8 quants go to q, the scale to *d
// from the group's first lane.  Bit-identical to quant_block_warp.  Every lane
// of the warp calls it (full-mask shuffles); `valid` only gates the stores.
__device__ __forceinline__ void quant_block_quad(const float (&v)[8], int lane, bool valid,
                                                 int8_t* q, float* d) {
    uint32_t ab = 0;
#pragma unroll
    for (int e = 0; e < 8; e++) ab = max(ab, __float_as_uint(fabsf(v[e])));
    ab = max(ab, __shfl_xor_sync(0xffffffffu, ab, 1));
    ab = max(ab, __shfl_xor_sync(0xffffffffu, ab, 2));
    const float amax = __uint_as_float(ab);
    const float id = amax == 0.0f ? 0.0f : __fdiv_rn(127.0f, amax);
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int e = 0; e < 4; e++) {
        lo |= (uint32_t)(uint8_t)(int8_t)q8_round(__fmul_rn(v[e], id)) << (8 * e);
        hi |= (uint32_t)(uint8_t)(int8_t)q8_round(__fmul_rn(v[e + 4], id)) << (8 * e);
    }
    if (!valid) return;
    *reinterpret_cast<uint2*>(q) = make_uint2(lo, hi);
    if ((lane & 3) == 0) *d = __fdiv_rn(amax, 127.0f);
}

}  // namespace axq8
