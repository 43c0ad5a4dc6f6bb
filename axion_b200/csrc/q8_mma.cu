// Host side of the tensor-core Q8_0 x A8 product: TMA tensor maps, tile and
// split-K selection, launch, and its C-ABI entry points.  Kernels in q8_mma.cuh.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdlib.h>

#include <algorithm>
#include <mutex>

#include "q8_mma.cuh"
#include "q8_mma.h"
#include "q8_mmq.cuh"

namespace axq8 {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                             &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

// 2-D tensor map: dim0 (innermost, contiguous) x dim1 rows, row pitch in bytes.
int make_map(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t dim0,
             uint64_t dim1, uint64_t pitch, uint32_t box0, uint32_t box1, CUtensorMapSwizzle sw,
             const char* what) {
    auto fn = encode_fn();
    if (!fn) return fail(AXQ8_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {dim0, dim1};
    cuuint64_t strides[1] = {pitch};
    cuuint32_t box[2] = {box0, box1};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(AXQ8_ERR_CUDA, "cuTensorMapEncodeTiled(%s) failed: %d", what, (int)r);
    return AXQ8_OK;
}

int min_m() {
    static const int v = [] {
        const char* e = getenv("AXQ8_MMA_MIN_M");
        const int x = e ? atoi(e) : kMmaMinM;
        return x >= 32 ? x : kMmaMinM;
    }();
    return v;
}

// Per-device split-K scratch: partial tiles and tile counters (zeroed once,
// returned to zero by every launch).
struct SplitScratch {
    float* part = nullptr;
    size_t part_bytes = 0;
    int* counters = nullptr;
};
constexpr int kMaxDevices = 64;
constexpr int kCounterSlots = 1 << 16;
SplitScratch g_split[kMaxDevices];
std::mutex g_split_mu;

int split_scratch(DeviceState* ds, size_t part_bytes, float** part, int** counters,
                  cudaStream_t stream) {
    std::lock_guard<std::mutex> lk(g_split_mu);
    if (ds->device < 0 || ds->device >= kMaxDevices) return fail(AXQ8_ERR_INVALID, "device id");
    SplitScratch& sc = g_split[ds->device];
    if ((!sc.counters || sc.part_bytes < part_bytes) && capture_active(stream))
        return fail(AXQ8_ERR_STATE,
                    "split-K scratch must grow to %zu bytes during a stream capture; make a call "
                    "of this size outside capture first (or pass caller-owned scratch)",
                    part_bytes);
    if (!sc.counters) {
        AXQ8_CUDA_TRY(cudaMalloc(&sc.counters, sizeof(int) * kCounterSlots), "split counters");
        AXQ8_CUDA_TRY(cudaMemset(sc.counters, 0, sizeof(int) * kCounterSlots), "split counters");
    }
    if (sc.part_bytes < part_bytes) {
        if (sc.part) {
            AXQ8_CUDA_TRY(cudaDeviceSynchronize(), "split scratch resize");
            cudaFree(sc.part);
            sc.part = nullptr;
            sc.part_bytes = 0;
        }
        AXQ8_CUDA_TRY(cudaMalloc(&sc.part, part_bytes), "split partials");
        sc.part_bytes = part_bytes;
    }
    *part = sc.part;
    *counters = sc.counters;
    return AXQ8_OK;
}

template <int BN, bool DOTS>
int launch_bn(DeviceState* ds, const CUtensorMap& tw, const CUtensorMap& tx, const CUtensorMap& td,
              const MmaArgs& a, dim3 grid, cudaStream_t s) {
    auto kern = q8_mma_kernel<BN, DOTS>;
    static int configured[kMaxDevices] = {0};
    const int dev = ds->device < kMaxDevices ? ds->device : kMaxDevices - 1;
    if (!configured[dev]) {
        AXQ8_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           MmaCfg<BN>::SMEM),
                      "cudaFuncSetAttribute(q8_mma)");
        if (MmaCfg<BN>::REG_SPLIT) {
            // the register split must fit the CTA's pool, else setmaxnreg.inc would never return
            cudaFuncAttributes fa;
            AXQ8_CUDA_TRY(cudaFuncGetAttributes(&fa, kern), "cudaFuncGetAttributes(q8_mma)");
            if (fa.numRegs < MmaCfg<BN>::LAUNCH_REGS_MIN)
                return fail(AXQ8_ERR_UNSUPPORTED,
                            "tensor-core linear: kernel built with %d registers, register split needs %d",
                            fa.numRegs, MmaCfg<BN>::LAUNCH_REGS_MIN);
        }
        configured[dev] = 1;
    }
    AXQ8_CUDA_TRY(launch_k(kern, grid, dim3(MmaCfg<BN>::THREADS), MmaCfg<BN>::SMEM, s, true, tw,
                           tx, td, a),
                  "q8_mma launch");
    return AXQ8_OK;
}

}  // namespace

bool skinny_eligible(const axq8_weight_t* w, int64_t M) {
    if (!w || M <= 8 || M > kMmqMaxM || w->K % QK || w->K > (1 << 24)) return false;
    return skinny_preferred(w->N, M) || !mma_eligible(w, M);
}

bool mma_eligible(const axq8_weight_t* w, int64_t M) {
    return w && M >= min_m() && M <= (1 << 24) && w->N >= kMmaBM && w->N <= (1 << 24) &&
           w->K >= kMmaKC && w->K % kMmaKC == 0 && w->K <= (1 << 20);
}

namespace {
// Tile sizes and split count of one call.
struct MmaPlan {
    int BN, splits, per;
    int64_t tiles_n, tiles_m, tiles;
};
MmaPlan mma_plan(DeviceState* ds, int64_t N, int64_t K, int64_t M, bool dots) {
    MmaPlan p;
    p.BN = M >= 128 ? 128 : (M >= 64 ? 64 : 32);
    p.tiles_n = (N + kMmaBM - 1) / kMmaBM;
    p.tiles_m = (M + p.BN - 1) / p.BN;
    p.tiles = p.tiles_n * p.tiles_m;
    const int nst = (int)(K / kMmaKC);
    const int64_t slots = (int64_t)ds->sm_count * (p.BN == 64 ? 2 : 1);
    int splits = 1;
    if (p.tiles < slots && !dots) {
        splits = (int)std::min<int64_t>(slots / p.tiles, std::max(1, nst / 2));
        splits = std::max(splits, 1);
    }
    p.per = (nst + splits - 1) / splits;
    p.splits = (nst + p.per - 1) / p.per;
    return p;
}
}  // namespace

void mma_split_needs(DeviceState* ds, int64_t N, int64_t K, int64_t M, size_t* part_bytes,
                     int64_t* counters) {
    const MmaPlan p = mma_plan(ds, N, K, M, false);
    *part_bytes = p.splits > 1 ? sizeof(float) * (size_t)p.splits * M * N : 0;
    *counters = p.splits > 1 ? p.tiles : 0;
}

int mma_linear(DeviceState* ds, const axq8_weight_t* w, const int8_t* xq, const float* dxT,
               int64_t M, const float* residual, float* y, int64_t ldy, int32_t* dots,
               cudaStream_t stream, const MmaScratch* scratch) {
    if (!w || M < 32 || w->N < kMmaBM || w->K % kMmaKC || !xq || !dxT || !y || ldy < w->N)
        return fail(AXQ8_ERR_INVALID, "tensor-core linear: unsupported arguments");
    if ((reinterpret_cast<uintptr_t>(xq) & 15) || (reinterpret_cast<uintptr_t>(dxT) & 15))
        return fail(AXQ8_ERR_INVALID, "tensor-core linear: xq/dxT not 16-byte aligned");
    const int64_t N = w->N, K = w->K, Mp = mma_scale_pitch(M);
    const MmaPlan plan = mma_plan(ds, N, K, M, dots != nullptr);
    const int BN = plan.BN;
    CUtensorMap tw, tx, td;
    int rc = make_map(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->rows, K, N, w->row_stride, kMmaKC,
                      kMmaBM, CU_TENSOR_MAP_SWIZZLE_128B, "weight quants");
    if (rc) return rc;
    rc = make_map(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT8, xq, K, M, K, kMmaKC, BN,
                  CU_TENSOR_MAP_SWIZZLE_128B, "activation quants");
    if (rc) return rc;
    rc = make_map(&td, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, dxT, Mp, K / QK, Mp * 4, BN, 4,
                  CU_TENSOR_MAP_SWIZZLE_NONE, "activation scales");
    if (rc) return rc;

    const int64_t tiles_n = plan.tiles_n, tiles_m = plan.tiles_m, tiles = plan.tiles;
    const int splits = plan.splits, per = plan.per;
    if (tiles_n > 65535) return fail(AXQ8_ERR_UNSUPPORTED, "tensor-core linear: too many tiles");

    MmaArgs a = {};
    a.rows = static_cast<const uint8_t*>(w->rows);
    a.row_stride = w->row_stride;
    a.N = (int)N;
    a.K = (int)K;
    a.M = (int)M;
    a.stages_per_split = per;
    a.residual = residual;
    a.y = y;
    a.ldy = (int)ldy;
    a.dots = dots;
    a.status = ds->status;
    if (splits > 1) {
        const size_t need = sizeof(float) * (size_t)splits * M * N;
        if (scratch) {
            if (scratch->part_bytes < need || scratch->counter_slots < tiles)
                return fail(AXQ8_ERR_INVALID, "tensor-core linear: caller scratch too small");
            a.part = scratch->part;
            a.counters = scratch->counters;
        } else {
            if (tiles > kCounterSlots)
                return fail(AXQ8_ERR_UNSUPPORTED, "tensor-core linear: too many split tiles");
            rc = split_scratch(ds, need, &a.part, &a.counters, stream);
            if (rc) return rc;
        }
    }
    const dim3 grid((unsigned)tiles_m, (unsigned)tiles_n, (unsigned)splits);
    if (dots) {
        if (BN == 128) return launch_bn<128, true>(ds, tw, tx, td, a, grid, stream);
        if (BN == 64) return launch_bn<64, true>(ds, tw, tx, td, a, grid, stream);
        return launch_bn<32, true>(ds, tw, tx, td, a, grid, stream);
    }
    if (BN == 128) return launch_bn<128, false>(ds, tw, tx, td, a, grid, stream);
    if (BN == 64) return launch_bn<64, false>(ds, tw, tx, td, a, grid, stream);
    return launch_bn<32, false>(ds, tw, tx, td, a, grid, stream);
}

namespace {
struct MmqPlan {
    int splits, per;
    int64_t tiles;
};
// Clusters of s CTAs of q8_mmq_kernel<MT8> that the device runs at once
// (cudaOccupancyMaxActiveClusters: clusters are placed whole within a GPC, so
// this can be below SMs x CTAs per SM / s); 0 when the query fails.  Cached
// per device.
template <int MT8>
int mmq_active_clusters(int dev, int s) {
    static int cached[kMaxDevices][kMmqMaxSplits + 1] = {};
    int& v = cached[dev][s];
    if (v == 0) {
        int n = 0;
        if (cudaFuncSetAttribute(q8_mmq_kernel<MT8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 MmqSmem<MT8>::BYTES) == cudaSuccess) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(1, s, 1);
            cfg.blockDim = dim3(kMmqWarps * 32);
            cfg.dynamicSmemBytes = MmqSmem<MT8>::BYTES;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = 1;
            attr[0].val.clusterDim.y = s;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            if (cudaOccupancyMaxActiveClusters(&n, q8_mmq_kernel<MT8>, &cfg) != cudaSuccess) n = 0;
        }
        (void)cudaGetLastError();
        v = n > 0 ? n : -1;
    }
    return v > 0 ? v : 0;
}
int mmq_active(int dev, int64_t M, int s) {
    if (M <= 8) return mmq_active_clusters<1>(dev, s);
    if (M <= 16) return mmq_active_clusters<2>(dev, s);
    if (M <= 32) return mmq_active_clusters<4>(dev, s);
    return mmq_active_clusters<8>(dev, s);
}

MmqPlan mmq_plan(DeviceState* ds, int64_t N, int64_t K, int64_t M) {
    MmqPlan p;
    p.tiles = (N + kMmqRows - 1) / kMmqRows;
    const int nch = (int)((K / 32 + kMmqChunkKb - 1) / kMmqChunkKb);
    static const bool by_clusters = [] {   // AXQ8_MMQ_PLAN=0: the plain rule below (tuning)
        const char* e = getenv("AXQ8_MMQ_PLAN");
        return !(e && atoi(e) == 0);
    }();
    const int dev = ds->device >= 0 && ds->device < kMaxDevices ? ds->device : 0;
    if (by_clusters && mmq_active(dev, M, 1) > 0) {
        // split count by launch time ~ waves x (chunks per CTA + a fixed two
        // chunks of start-up and combine), waves counted in clusters that fit
        const int smax = std::min(kMmqMaxSplits, std::max(1, nch / 2));
        int64_t best = -1;
        for (int s = 1; s <= smax; s++) {
            const int per = (nch + s - 1) / s;
            const int sp = (nch + per - 1) / per;
            const int act = mmq_active(dev, M, sp);
            if (act <= 0) continue;
            const int64_t waves = (p.tiles + act - 1) / act;
            const int64_t cost = waves * (per + 2);
            if (best < 0 || cost < best) {
                best = cost;
                p.per = per;
            }
        }
        if (best >= 0) {
            p.splits = (nch + p.per - 1) / p.per;
            return p;
        }
    }
    const int64_t want = 2 * (int64_t)ds->sm_count;   // two CTAs per SM
    int splits = (int)std::max<int64_t>(1, (want + p.tiles - 1) / p.tiles);
    splits = std::min(splits, std::max(1, nch / 2));   // >= two chunks per split
    splits = std::min(splits, kMmqMaxSplits);          // one cluster per row tile
    p.per = (nch + splits - 1) / splits;
    p.splits = (nch + p.per - 1) / p.per;
    return p;
}
template <int MT8, bool SILU = false>
int mmq_launch(const MmqArgs& a, dim3 grid, cudaStream_t s) {
    constexpr int smem = MmqSmem<MT8>::BYTES;
    static bool configured[kMaxDevices] = {};
    int dev = 0;
    AXQ8_CUDA_TRY(cudaGetDevice(&dev), "q8_mmq device");
    if (dev < 0 || dev >= kMaxDevices) return fail(AXQ8_ERR_INVALID, "skinny linear: device id");
    if (!configured[dev]) {   // once per device: idempotent, a repeat is harmless
        AXQ8_CUDA_TRY(cudaFuncSetAttribute(q8_mmq_kernel<MT8, SILU>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                      "q8_mmq shared memory attribute");
        configured[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kMmqWarps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = grid.y;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = grid.y > 1 ? 2 : 1;
    AXQ8_CUDA_TRY(cudaLaunchKernelEx(&cfg, q8_mmq_kernel<MT8, SILU>, a), "q8_mmq launch");
    return AXQ8_OK;
}
}  // namespace

int mmq_linear(DeviceState* ds, const axq8_weight_t* w, const int8_t* xq, const float* dxT,
               int64_t M, const float* residual, float* y, int64_t ldy, cudaStream_t stream) {
    if (!w || M < 1 || M > kMmqMaxM || w->K % QK || w->K > (1 << 24) || w->N > (1 << 30) ||
        !xq || !dxT || !y || ldy < w->N)
        return fail(AXQ8_ERR_INVALID, "skinny linear: unsupported arguments");
    const MmqPlan plan = mmq_plan(ds, w->N, w->K, M);
    if (plan.tiles > 0x7fffffff) return fail(AXQ8_ERR_UNSUPPORTED, "skinny linear: N too large");
    MmqArgs a = {};
    a.rows = static_cast<const uint8_t*>(w->rows);
    a.row_stride = w->row_stride;
    a.N = (int)w->N;
    a.K = (int)w->K;
    a.M = (int)M;
    a.xq = xq;
    a.dxT = dxT;
    a.Mp = (int)mma_scale_pitch(M);
    a.chunks_per_split = plan.per;
    a.residual = residual;
    a.y = y;
    a.ldy = (int)ldy;
    const dim3 grid((unsigned)plan.tiles, (unsigned)plan.splits);
    if (M <= 8) return mmq_launch<1>(a, grid, stream);
    if (M <= 16) return mmq_launch<2>(a, grid, stream);
    if (M <= 32) return mmq_launch<4>(a, grid, stream);
    return mmq_launch<8>(a, grid, stream);
}

int mmq_linear_silu(DeviceState* ds, const axq8_weight_t* w, const int8_t* xq, const float* dxT,
                    int64_t M, int8_t* sq, float* sdx, int sdxt, cudaStream_t stream) {
    if (!w || M < 1 || M > kMmqMaxM || w->K % QK || w->K > (1 << 24) || w->N > (1 << 30) ||
        w->N % 64 || !xq || !dxT || !sq || !sdx || sdxt < 0)
        return fail(AXQ8_ERR_INVALID, "skinny linear + SiLU: unsupported arguments");
    const MmqPlan plan = mmq_plan(ds, w->N, w->K, M);
    if (plan.tiles > 0x7fffffff) return fail(AXQ8_ERR_UNSUPPORTED, "skinny linear: N too large");
    MmqArgs a = {};
    a.rows = static_cast<const uint8_t*>(w->rows);
    a.row_stride = w->row_stride;
    a.N = (int)w->N;
    a.K = (int)w->K;
    a.M = (int)M;
    a.xq = xq;
    a.dxT = dxT;
    a.Mp = (int)mma_scale_pitch(M);
    a.chunks_per_split = plan.per;
    a.sq = sq;
    a.sdx = sdx;
    a.sdxt = sdxt;
    const dim3 grid((unsigned)plan.tiles, (unsigned)plan.splits);
    if (M <= 8) return mmq_launch<1, true>(a, grid, stream);
    if (M <= 16) return mmq_launch<2, true>(a, grid, stream);
    if (M <= 32) return mmq_launch<4, true>(a, grid, stream);
    return mmq_launch<8, true>(a, grid, stream);
}

int mma_quantize(DeviceState* ds, const float* x, int64_t M, int64_t K, int8_t* xq, float* dxT,
                 cudaStream_t stream) {
    const int64_t nblocks = M * (K / QK);
    int64_t grid = (nblocks + 7) / 8;
    const int64_t cap = (int64_t)ds->sm_count * 16;
    if (grid > cap) grid = cap;
    AXQ8_CUDA_TRY(launch_k(quantize_act_t_kernel, dim3((unsigned)grid), dim3(256), 0, stream, true, x,
                           (int)M, (int)K, (int)mma_scale_pitch(M), xq, dxT),
                  "quantize_act_t launch");
    return AXQ8_OK;
}

int mma_transpose_scales(DeviceState* ds, const float* dx, int64_t M, int64_t K, float* dxT,
                         cudaStream_t stream) {
    const int64_t total = M * (K / QK);
    int64_t grid = (total + 255) / 256;
    const int64_t cap = (int64_t)ds->sm_count * 8;
    if (grid > cap) grid = cap;
    AXQ8_CUDA_TRY(launch_k(transpose_scales_kernel, dim3((unsigned)grid), dim3(256), 0, stream, true,
                           dx, (int)M, (int)(K / QK), (int)mma_scale_pitch(M), dxT),
                  "transpose_scales launch");
    return AXQ8_OK;
}

}  // namespace axq8

// ---- C ABI ------------------------------------------------------------------------

using namespace axq8;

extern "C" {

int axq8_linear_path(const axq8_weight_t* w, int64_t M, int act_mode) {
    if (!w || M < 0) return fail(AXQ8_ERR_INVALID, "axq8_linear_path: bad argument");
    if (act_mode != AXQ8_ACT_Q8) return AXQ8_PATH_GEMV;
    if (skinny_eligible(w, M)) return AXQ8_PATH_SKINNY;
    return mma_eligible(w, M) ? AXQ8_PATH_TENSOR_CORE : AXQ8_PATH_GEMV;
}

int axq8_linear_q8act_s(const axq8_weight_t* w, const int8_t* xq, const float* dxT, int64_t M,
                        const float* residual, float* y, void* stream) {
    if (!w || !w->rows) return fail(AXQ8_ERR_INVALID, "axq8_linear_q8act_s: null weight");
    if (w->row_stride != q8r_row_stride(w->K) || (reinterpret_cast<uintptr_t>(w->rows) & 15))
        return fail(AXQ8_ERR_INVALID, "axq8_linear_q8act_s: weight not in the repacked layout");
    if (M < 1 || M > kMmqMaxM)
        return fail(AXQ8_ERR_UNSUPPORTED, "axq8_linear_q8act_s: needs 1 <= M <= 64 (M=%lld)",
                    (long long)M);
    if ((reinterpret_cast<uintptr_t>(xq) & 15) || (reinterpret_cast<uintptr_t>(dxT) & 3))
        return fail(AXQ8_ERR_INVALID, "axq8_linear_q8act_s: misaligned xq/dxT");
    DeviceState* ds = device_state();
    if (!ds) return AXQ8_ERR_CUDA;
    return mmq_linear(ds, w, xq, dxT, M, residual, y, w->N, static_cast<cudaStream_t>(stream));
}

int axq8_quantize_act_t(const float* x, int64_t M, int64_t K, int8_t* xq, float* dxT,
                        void* stream) {
    if (M <= 0 || K <= 0 || K % QK || M > (1 << 24) || K > (1 << 20))
        return fail(AXQ8_ERR_INVALID, "axq8_quantize_act_t: bad shape [%lld, %lld]", (long long)M,
                    (long long)K);
    if (!x || !xq || !dxT) return fail(AXQ8_ERR_INVALID, "axq8_quantize_act_t: null pointer");
    DeviceState* ds = device_state();
    if (!ds) return AXQ8_ERR_CUDA;
    return mma_quantize(ds, x, M, K, xq, dxT, static_cast<cudaStream_t>(stream));
}

int axq8_linear_q8act_t(const axq8_weight_t* w, const int8_t* xq, const float* dxT, int64_t M,
                        const float* residual, float* y, void* stream) {
    if (!w || !w->rows) return fail(AXQ8_ERR_INVALID, "axq8_linear_q8act_t: null weight");
    if (w->row_stride != q8r_row_stride(w->K) || (reinterpret_cast<uintptr_t>(w->rows) & 15))
        return fail(AXQ8_ERR_INVALID, "axq8_linear_q8act_t: weight not in the repacked layout");
    if (M < 32 || w->N < kMmaBM || w->K % kMmaKC)
        return fail(AXQ8_ERR_UNSUPPORTED,
                    "axq8_linear_q8act_t: needs M >= 32, N >= 128, K %% 128 == 0 (M=%lld N=%lld K=%lld)",
                    (long long)M, (long long)w->N, (long long)w->K);
    DeviceState* ds = device_state();
    if (!ds) return AXQ8_ERR_CUDA;
    return mma_linear(ds, w, xq, dxT, M, residual, y, w->N, nullptr,
                      static_cast<cudaStream_t>(stream));
}

int axq8_block_dots_tc(const axq8_weight_t* w, const int8_t* xq, const float* dxT, int64_t M,
                       int32_t* dots, float* y, void* stream) {
    if (!w || !w->rows || !dots || !y) return fail(AXQ8_ERR_INVALID, "axq8_block_dots_tc: null argument");
    if (w->row_stride != q8r_row_stride(w->K) || (reinterpret_cast<uintptr_t>(w->rows) & 15))
        return fail(AXQ8_ERR_INVALID, "axq8_block_dots_tc: weight not in the repacked layout");
    if (M < 32 || w->N < kMmaBM || w->K % kMmaKC)
        return fail(AXQ8_ERR_UNSUPPORTED, "axq8_block_dots_tc: needs M >= 32, N >= 128, K %% 128 == 0");
    DeviceState* ds = device_state();
    if (!ds) return AXQ8_ERR_CUDA;
    return mma_linear(ds, w, xq, dxT, M, nullptr, y, w->N, dots, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
