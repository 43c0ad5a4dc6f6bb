// Tensor-parallel sum of the hidden state over NVLink peer memory (the
// all-reduce after the row-split O and down projections of a decode step).
//
// Every rank owns three device buffers that the other ranks of the node map
// with CUDA IPC: `part` (its partial [M, H] of the row-split product), `out`
// (its hidden state, the sum) and `flags` ([2][kArMaxRanks] epochs written
// by the peers).  One launch per all-reduce, two phases:
//   1. every CTA announces "partial ready" (this all-reduce's epoch into slot
//      [0][rank] of every rank's flags) and waits until all ranks announced;
//   2. rank r sums slice r of the partials over the ranks in rank order 0,
//      1, ... (peer loads that bypass the caches), writes the sums into every
//      rank's `out`, fences, and the last CTA to finish announces "slice
//      written" ([1][rank]) and waits for every rank's announcement.
// Each slice is summed once, by its owner, so every rank holds bit-identical
// sums.  A rank leaves phase 2 only when all ranks finished reading its
// partial, so the next product may overwrite it.  Every wait is bounded:
// after about two seconds of SM clock it records AXQ8_ERR_WAIT_TIMEOUT in
// the status word and the kernel returns (the sums are then invalid).
// No TMA and no multicast: plain loads and stores to peer addresses.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "axq8.h"
#include "common.cuh"

namespace axq8 {

constexpr int kArMaxRanks = 8;
constexpr int kArThreads = 256;

struct ArPeers {
    float* part[kArMaxRanks];      // every rank's partial buffer, as mapped here
    float* out[kArMaxRanks];       // every rank's output buffer
    unsigned* flags[kArMaxRanks];  // every rank's flags [2][kArMaxRanks]
    unsigned* epoch;               // this rank's all-reduce counter (local)
    int* ctas_done;                // this rank's CTA completion counter (local)
    int* status;
    int rank, world;
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Wait until every rank wrote an epoch >= e into flags[phase][*]; false on timeout.
__device__ __forceinline__ bool ar_wait(const ArPeers& p, int phase, unsigned e) {
    const unsigned* f = p.flags[p.rank] + phase * kArMaxRanks;
    const long long t0 = clock64();
    for (int r = 0; r < p.world; r++) {
        while ((int)(ld_acquire_sys(f + r) - e) < 0) {
            if (clock64() - t0 > 4000000000ll) {   // ~2 s at 1.9 GHz
                record_status(p.status, AXQ8_ERR_WAIT_TIMEOUT);
                return false;
            }
        }
    }
    return true;
}

// n floats (n % 4 == 0) of out = sum over ranks of part.
__global__ void __launch_bounds__(kArThreads) tp_allreduce_kernel(const ArPeers p, int64_t n) {
    pdl_launch_dependents();
    pdl_wait();   // this rank's partial is complete
    const unsigned e = ld_cg(reinterpret_cast<const int*>(p.epoch)) + 1u;
    __shared__ int ok;
    // the partial (the previous grid's, complete after the wait) sits in this
    // GPU's L2, where the peers' loads are served
    if (threadIdx.x < p.world) st_release_sys(p.flags[threadIdx.x] + p.rank, e);   // phase 0, [rank]
    if (threadIdx.x == 0) ok = ar_wait(p, 0, e);
    __syncthreads();
    if (ok) {
        const int64_t n4 = n / 4;
        const int64_t lo = n4 * p.rank / p.world, hi = n4 * (p.rank + 1) / p.world;
        for (int64_t i = lo + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < hi;
             i += (int64_t)gridDim.x * blockDim.x) {
            float4 v[kArMaxRanks];   // all ranks' loads in flight together
#pragma unroll
            for (int r = 0; r < kArMaxRanks; r++)
                if (r < p.world) v[r] = __ldcv(reinterpret_cast<const float4*>(p.part[r]) + i);
            float4 s = v[0];
#pragma unroll
            for (int r = 1; r < kArMaxRanks; r++) {
                if (r >= p.world) break;
                s.x = __fadd_rn(s.x, v[r].x);
                s.y = __fadd_rn(s.y, v[r].y);
                s.z = __fadd_rn(s.z, v[r].z);
                s.w = __fadd_rn(s.w, v[r].w);
            }
#pragma unroll
            for (int r = 0; r < kArMaxRanks; r++)
                if (r < p.world) reinterpret_cast<float4*>(p.out[r])[i] = s;
        }
    }
    __syncthreads();   // the CTA's stores, then one system-scope fence for them
    __shared__ int last;
    if (threadIdx.x == 0) {
        __threadfence_system();
        last = atomicAdd(p.ctas_done, 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    if (threadIdx.x < p.world) __threadfence_system();
    if (threadIdx.x < p.world) st_release_sys(p.flags[threadIdx.x] + kArMaxRanks + p.rank, e);
    if (threadIdx.x == 0) {
        ar_wait(p, 1, e);
        *p.ctas_done = 0;
        *p.epoch = e;
    }
}

}  // namespace axq8
