// Llama-architecture decode step on B200 built from the Q8_0 GEMV (C ABI in
// include/axdec.h).
//
// One step processes one position of each of M sequences, in the order of
// StreamingExecutor::decode_layer (streaming_executor.cpp:268-401) and
// ModelRunner::generate (model_runner.cpp:245-317).  In A8 mode (M <= 4) a
// layer is five kernels:
//   GEMV qkv   [prologue rmsnorm->Q8, epilogue NEOX RoPE + KV page append]
//   attention  [split-K flash decode, last CTA merges splits -> Q8]
//   GEMV o     [+ residual, in place]
//   GEMV gu    [prologue rmsnorm->Q8, epilogue silu(gate)*up]
//   GEMV down  [prologue Q8, + residual]
// plus embed at the start and GEMV lm_head [prologue rmsnorm->Q8, epilogue
// argmax + state advance] at the end.  A32 mode and wide batches keep
// RMSNorm and SiLU*up as producer kernels.  Q, K and V share one stacked
// weight (the rows of Q and K permuted per head to (j, j + hd/2) pairs for
// the RoPE epilogue), and so do gate and up (rows interleaved, gate_j then
// up_j, so one GEMV row pair yields one silu(gate_j)*up_j).  All kernels are launched
// with programmatic dependent launch and the whole step is captured once in a
// CUDA graph per batch size; the control state (positions, input tokens, fed
// tokens) lives in device memory so the same graph serves every step.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <cmath>
#include <map>
#include <string>
#include <type_traits>
#include <vector>

#include "axdec.h"
#include "axq8.h"
#include "axtp.h"
#include "common.cuh"
#include "decode_ops.cuh"
#include "nccl_dl.h"
#include "q8_gemv.cuh"
#include "q8_mma.h"
#include "runtime.h"
#include "tp_allreduce.cuh"

using namespace axq8;

namespace {

struct Layer {
    uint8_t* qkv = nullptr;    // [Nq + 2 Nkv, H] Q8R
    uint8_t* o = nullptr;      // [H, Nq]
    uint8_t* gu = nullptr;     // [2F, H], rows gate_0, up_0, gate_1, up_1, ...
    uint8_t* down = nullptr;   // [H, F]
    float* attn_norm = nullptr;
    float* ffn_norm = nullptr;
    void* kc = nullptr;        // [pages][n_kv][B][hd]
    void* vc = nullptr;
};

struct Graph {
    cudaGraphExec_t exec = nullptr;
    int kernels = 0;
};

}  // namespace

struct axdec_model {
    axdec_config_t c{};           // this rank's dimensions (heads, ffn, vocab divided by tp)
    axdec_config_t cf{};          // the whole model's dimensions
    int tp = 1, rank = 0;
    ncclComm_t comm = nullptr;    // tensor-parallel communicator (tp > 1)
    DeviceState* ds = nullptr;
    int Nq = 0, Nkv = 0, Nqkv = 0;
    int64_t rs_h = 0, rs_q = 0, rs_f = 0;
    std::vector<void*> allocs;
    int64_t bytes = 0;
    uint8_t* embd = nullptr;      // [V, H]
    uint8_t* out_w = nullptr;     // [V, H] (== embd when tied)
    bool out_set = false;
    float* out_norm = nullptr;
    std::vector<Layer> L;
    int max_blocks = 0, nsplit = 1, bps = 1;
    // activations
    float* h = nullptr;           // [M, H] residual stream
    int8_t* xq = nullptr;         // [M, maxK]
    float* dx = nullptr;          // [M, maxK/32]
    float* x32 = nullptr;         // [M, maxK] (A32 mode)
    float* qkv = nullptr;         // [M, Nqkv]
    float* gu = nullptr;          // [M, 2F] interleaved gate/up, or [M, F] silu*up (fused GEMV)
    float* part = nullptr;        // attention partials
    float* logits = nullptr;      // [M, V]
    float2* rope = nullptr;       // [max_ctx, hd/2]
    int* block_table = nullptr;   // [max_batch, max_blocks]
    int* tokens = nullptr;        // [M]
    int* pos = nullptr;           // [M]
    int* feed = nullptr;          // [M, max_ctx]
    int* out_tokens = nullptr;    // [M, max_ctx]
    int* argmax = nullptr;        // [M]
    int* ctl = nullptr;           // {n_prompt, feed_len, max_out}
    unsigned long long* amax_key = nullptr;   // [M] argmax epilogue keys
    int* done = nullptr;                      // argmax epilogue completion counter
    int* attn_cnt = nullptr;                  // [M, n_kv] attention split counters
    MmaScratch mma_sc;                        // split-K scratch of the wide-batch products
    cudaStream_t cap_stream = nullptr;
    std::map<int, Graph> graphs;  // per batch size
    // batched prefill (A8): buffers of one prompt chunk, allocated on first use
    int prefill_mode = 1;         // 1: batched where supported, 0: through the decode step
    bool silu_fused = true;       // wide steps: SiLU*up + A8 in the gate|up skinny product
    int pre_cap = 0;              // rows the chunk buffers hold
    float* ph = nullptr;          // [cap, H] residual stream of the chunk
    int8_t* pxq = nullptr;        // [cap, maxK] A8 activations
    float* pdx = nullptr;         // [maxK/32, pitch(cap)] their block scales (transposed)
    float* pqkv = nullptr;        // [cap, Nqkv]
    float* pgu = nullptr;         // [cap, 2F] interleaved gate/up
    int* ptok = nullptr;          // [cap] token ids of the chunk rows
    MmaScratch pre_sc;            // split-K scratch of the chunk products (grown on demand)
    // decode session of axdec_prefill / axdec_decode_step
    int sess_seq = 0, sess_pos = -1;
    // tensor parallelism over NVLink peer memory (tp_allreduce.cuh): the
    // row-split products write their partial into ar_part, the all-reduce
    // sums the ranks' partials into every rank's h
    float* ar_part = nullptr;     // [max_batch, H], mapped by the peers
    unsigned* ar_flags = nullptr; // [2][kArMaxRanks], written by the peers
    unsigned* ar_epoch = nullptr;
    int* ar_ctas = nullptr;
    ArPeers ar{};
    bool ar_on = false;
    std::vector<void*> ar_mapped; // peer mappings to close
};

namespace {

void* dalloc(axdec_model* m, size_t bytes, int* rc) {
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        *rc = cuda_fail(e, "axdec: cudaMalloc");
        return nullptr;
    }
    m->allocs.push_back(p);
    m->bytes += (int64_t)bytes;
    return p;
}

bool parse_layer_name(const char* name, int* layer, std::string* slot) {
    if (strncmp(name, "blk.", 4) != 0) return false;
    char* end = nullptr;
    long l = strtol(name + 4, &end, 10);
    if (end == name + 4 || *end != '.') return false;
    std::string rest(end + 1);
    const std::string suf = ".weight";
    if (rest.size() <= suf.size() || rest.compare(rest.size() - suf.size(), suf.size(), suf) != 0)
        return false;
    *layer = (int)l;
    *slot = rest.substr(0, rest.size() - suf.size());
    return true;
}

const char* kSlots[9] = {"attn_norm", "attn_q", "attn_k", "attn_v", "attn_output",
                         "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"};

int slot_index(const std::string& s) {
    for (int i = 0; i < 9; i++)
        if (s == kSlots[i]) return i;
    return -1;
}

// Destination of a Q8_0 tensor: repacked rows, row offset, and expected shape.
struct Dest {
    uint8_t* rows = nullptr;
    int64_t row0 = 0, N = 0, K = 0;
    float* f32 = nullptr;   // norm weight destination
    int64_t n = 0;
    bool rope_perm = false; // attn_q / attn_k: rows permuted for the RoPE epilogue
    int row_step = 1;       // destination row of source row i: row0 + i * row_step
    // this rank's slice of the whole [src_N, src_K] tensor (rows src_row0..,
    // columns src_col0..); the whole tensor when not split
    int64_t src_row0 = 0, src_col0 = 0, src_N = 0, src_K = 0;
};

int resolve(axdec_model* m, const char* name, Dest* d) {
    const axdec_config_t& c = m->c;
    const int H = c.hidden, F = c.ffn, r = m->rank;
    const int64_t Vf = m->cf.vocab, Nqf = (int64_t)m->cf.n_heads * c.head_dim,
                  Nkvf = (int64_t)m->cf.n_kv_heads * c.head_dim, Ff = m->cf.ffn;
    auto rows_slice = [&](uint8_t* rows, int64_t row0, int64_t n, int64_t src_n, int64_t src_row0) {
        *d = Dest{};
        d->rows = rows;
        d->row0 = row0;
        d->N = n;
        d->K = H;
        d->src_row0 = src_row0;
        d->src_N = src_n;
        d->src_K = H;
    };
    auto cols_slice = [&](uint8_t* rows, int64_t k, int64_t src_k, int64_t src_col0) {
        *d = Dest{};
        d->rows = rows;
        d->N = H;
        d->K = k;
        d->src_col0 = src_col0;
        d->src_N = H;
        d->src_K = src_k;
    };
    if (!strcmp(name, "token_embd.weight")) { rows_slice(m->embd, 0, Vf, Vf, 0); return 0; }
    if (!strcmp(name, "output.weight")) { rows_slice(m->out_w, 0, c.vocab, Vf, (int64_t)r * c.vocab); return 0; }
    if (!strcmp(name, "output_norm.weight")) { *d = Dest{}; d->f32 = m->out_norm; d->n = H; return 0; }
    int layer;
    std::string slot;
    if (!parse_layer_name(name, &layer, &slot) || layer < 0 || layer >= c.n_layers)
        return fail(AXQ8_ERR_INVALID, "axdec: unknown tensor '%s'", name);
    Layer& Ly = m->L[layer];
    const int si = slot_index(slot);
    switch (si) {
        case 0: *d = Dest{}; d->f32 = Ly.attn_norm; d->n = H; return 0;
        case 5: *d = Dest{}; d->f32 = Ly.ffn_norm; d->n = H; return 0;
        case 1: rows_slice(Ly.qkv, 0, m->Nq, Nqf, (int64_t)r * m->Nq); d->rope_perm = true; return 0;
        case 2: rows_slice(Ly.qkv, m->Nq, m->Nkv, Nkvf, (int64_t)r * m->Nkv); d->rope_perm = true; return 0;
        case 3: rows_slice(Ly.qkv, m->Nq + m->Nkv, m->Nkv, Nkvf, (int64_t)r * m->Nkv); return 0;
        case 4: cols_slice(Ly.o, m->Nq, Nqf, (int64_t)r * m->Nq); return 0;
        // gate and up interleaved: gate row j -> row 2j, up row j -> row 2j + 1
        case 6: rows_slice(Ly.gu, 0, F, Ff, (int64_t)r * F); d->row_step = 2; return 0;
        case 7: rows_slice(Ly.gu, 1, F, Ff, (int64_t)r * F); d->row_step = 2; return 0;
        case 8: cols_slice(Ly.down, F, Ff, (int64_t)r * F); return 0;
        default: return fail(AXQ8_ERR_INVALID, "axdec: unknown tensor '%s'", name);
    }
}

int nccl_check(ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return AXQ8_OK;
    const NcclApi* api = nccl_api();
    return fail(AXQ8_ERR_CUDA, "%s: %s", what, api ? api->GetErrorString(r) : "NCCL error");
}

// Where a row-split product (O, down) leaves this rank's partial hidden state:
// the peer-mapped partial buffer for the NVLink all-reduce, else h itself
// (summed in place by NCCL; also the single-GPU case).
float* hidden_partial(axdec_model* m) { return m->ar_on ? m->ar_part : m->h; }

// Sum the ranks' partial [M, H] hidden states into every rank's h.
int allreduce_hidden(axdec_model* m, int M, cudaStream_t s) {
    const int64_t n = (int64_t)M * m->c.hidden;
    if (m->ar_on) {
        const int64_t per = (n / 4 + m->tp - 1) / m->tp;
        const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(64, (per + kArThreads - 1) / kArThreads));
        AXQ8_CUDA_TRY(launch_k(tp_allreduce_kernel, dim3(grid), dim3(kArThreads), 0, s, true, m->ar, n),
                      "axdec: NVLink all-reduce launch");
        return AXQ8_OK;
    }
    const NcclApi* api = nccl_api();
    if (!api) return AXQ8_ERR_UNSUPPORTED;
    return nccl_check(api->AllReduce(m->h, m->h, (size_t)n, ncclFloat, ncclSum, m->comm, s),
                      "axdec: hidden all-reduce");
}

// Map the peers' all-reduce buffers (CUDA IPC handles exchanged with an NCCL
// all-gather) when AXDEC_TP_AR=nvlink asks for the peer-memory all-reduce.
// Every rank must succeed, which an NCCL min-reduction of the outcome
// decides, else all keep NCCL.  NCCL is the default: at two ranks it measured
// 7.33 ms per Llama-3-8B batch-64 step against 7.87 ms for the peer-memory
// kernel (64 all-reduces of 1 MiB per step).
int setup_peer_allreduce(axdec_model* m) {
    const char* env = getenv("AXDEC_TP_AR");
    const bool wanted = m->tp <= kArMaxRanks && env && !strcmp(env, "nvlink");
    const NcclApi* api = nccl_api();
    if (!api) return AXQ8_ERR_UNSUPPORTED;
    for (void* p : m->ar_mapped) cudaIpcCloseMemHandle(p);   // a previous connection's
    m->ar_mapped.clear();
    m->ar_on = false;
    cudaStream_t s = m->cap_stream;
    constexpr int kH = (int)sizeof(cudaIpcMemHandle_t);
    void* bufs[3] = {m->h, m->ar_part, m->ar_flags};
    std::vector<uint8_t> mine(3 * kH, 0), all((size_t)m->tp * 3 * kH, 0);
    int ok = wanted ? 1 : 0;
    for (int i = 0; i < 3 && ok; i++) {
        cudaIpcMemHandle_t h;
        if (cudaIpcGetMemHandle(&h, bufs[i]) != cudaSuccess) {
            (void)cudaGetLastError();
            ok = 0;
        } else {
            memcpy(mine.data() + i * kH, &h, kH);
        }
    }
    uint8_t* dev = nullptr;
    AXQ8_CUDA_TRY(cudaMalloc(&dev, all.size() + 3 * kH + 16), "axdec: handle exchange buffer");
    int* dok = reinterpret_cast<int*>(dev + all.size() + 3 * kH);
    cudaError_t e = cudaMemcpy(dev + all.size(), mine.data(), 3 * kH, cudaMemcpyHostToDevice);
    int rc = e == cudaSuccess ? nccl_check(api->AllGather(dev + all.size(), dev, 3 * kH, ncclUint8,
                                                          m->comm, s),
                                           "axdec: handle all-gather")
                              : cuda_fail(e, "axdec: handle upload");
    if (rc == AXQ8_OK) {
        e = cudaStreamSynchronize(s);
        if (e == cudaSuccess) e = cudaMemcpy(all.data(), dev, all.size(), cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) rc = cuda_fail(e, "axdec: handle exchange");
    }
    ArPeers ar{};
    for (int r = 0; r < m->tp && rc == AXQ8_OK && ok; r++) {
        for (int i = 0; i < 3 && ok; i++) {
            void* ptr = bufs[i];
            if (r != m->rank) {
                cudaIpcMemHandle_t h;
                memcpy(&h, all.data() + ((size_t)r * 3 + i) * kH, kH);
                if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                    (void)cudaGetLastError();
                    ok = 0;
                    break;
                }
                m->ar_mapped.push_back(ptr);
            }
            if (i == 0) ar.out[r] = static_cast<float*>(ptr);
            else if (i == 1) ar.part[r] = static_cast<float*>(ptr);
            else ar.flags[r] = static_cast<unsigned*>(ptr);
        }
    }
    // every rank takes the same decision
    if (rc == AXQ8_OK) {
        e = cudaMemcpy(dok, &ok, sizeof(int), cudaMemcpyHostToDevice);
        rc = e == cudaSuccess ? nccl_check(api->AllReduce(dok, dok, 1, ncclInt32, ncclMin, m->comm, s),
                                           "axdec: all-reduce agreement")
                              : cuda_fail(e, "axdec: agreement upload");
        if (rc == AXQ8_OK) {
            e = cudaStreamSynchronize(s);
            if (e == cudaSuccess) e = cudaMemcpy(&ok, dok, sizeof(int), cudaMemcpyDeviceToHost);
            if (e != cudaSuccess) rc = cuda_fail(e, "axdec: agreement");
        }
    }
    cudaFree(dev);
    if (rc != AXQ8_OK || !ok) {
        for (void* p : m->ar_mapped) cudaIpcCloseMemHandle(p);
        m->ar_mapped.clear();
        m->ar_on = false;
        return rc;
    }
    ar.epoch = m->ar_epoch;
    ar.ctas_done = m->ar_ctas;
    ar.status = m->ds->status;
    ar.rank = m->rank;
    ar.world = m->tp;
    m->ar = ar;
    m->ar_on = true;
    return AXQ8_OK;
}

__global__ void fill_kernel(float* p, int64_t n, float v) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        p[i] = v;
}

// Row permutation of a Q or K weight for the RoPE epilogue: within each head,
// destination row 2j is source dim j and row 2j+1 is source dim j + hd/2, so
// one GEMV row pair yields exactly one NEOX rotation pair.
__global__ void rope_permute_rows_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                         int64_t nrows, int hd, int64_t rs) {
    const int half = hd / 2;
    for (int64_t r = blockIdx.x; r < nrows; r += gridDim.x) {
        const int64_t head = r / hd, pr = r % hd;
        const int64_t srow = head * hd + ((pr & 1) ? half + pr / 2 : pr / 2);
        const uint4* s4 = reinterpret_cast<const uint4*>(src + srow * rs);
        uint4* d4 = reinterpret_cast<uint4*>(dst + r * rs);
        for (int64_t i = threadIdx.x; i < rs / 16; i += blockDim.x) d4[i] = s4[i];
    }
}

// Row i of src to row i * step of dst (rows of rs bytes, rs % 16 == 0).
__global__ void scatter_rows_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                    int64_t nrows, int step, int64_t rs) {
    for (int64_t r = blockIdx.x; r < nrows; r += gridDim.x) {
        const uint4* s4 = reinterpret_cast<const uint4*>(src + r * rs);
        uint4* d4 = reinterpret_cast<uint4*>(dst + r * step * rs);
        for (int64_t i = threadIdx.x; i < rs / 16; i += blockDim.x) d4[i] = s4[i];
    }
}

// Write repacked rows (device, `tmp`) into the destination, permuting Q/K rows
// and interleaving gate/up rows.
int place_rows(axdec_model* m, const Dest& d, const uint8_t* tmp) {
    const int64_t rs = q8r_row_stride(d.K);
    uint8_t* dst = d.rows + d.row0 * rs;
    if (d.rope_perm) {
        rope_permute_rows_kernel<<<256, 128>>>(tmp, dst, d.N, m->c.head_dim, rs);
        AXQ8_CUDA_TRY(cudaGetLastError(), "rope_permute_rows launch");
    } else if (d.row_step != 1) {
        scatter_rows_kernel<<<256, 128>>>(tmp, dst, d.N, d.row_step, rs);
        AXQ8_CUDA_TRY(cudaGetLastError(), "scatter_rows launch");
    } else {
        AXQ8_CUDA_TRY(cudaMemcpy(dst, tmp, (size_t)d.N * rs, cudaMemcpyDeviceToDevice), "place rows");
    }
    AXQ8_CUDA_TRY(cudaDeviceSynchronize(), "place rows");
    return AXQ8_OK;
}

template <typename KV>
int launch_step_kv(axdec_model* m, int M, cudaStream_t s);

int launch_step(axdec_model* m, int M, cudaStream_t s) {
    return m->c.kv_fp32 ? launch_step_kv<float>(m, M, s) : launch_step_kv<__half>(m, M, s);
}

GemvArgs gemv_args(axdec_model* m, const uint8_t* rows, int64_t N, int64_t K, int M,
                   const float* resid, float* y) {
    GemvArgs a = {};
    a.rows = rows;
    a.N = N;
    a.K = K;
    a.row_stride = q8r_row_stride(K);
    a.M = M;
    a.xq = m->xq;
    a.dx = m->dx;
    a.x = m->x32;
    a.residual = resid;
    a.y = y;
    a.ldy = N;
    a.status = m->ds->status;
    a.eps = m->c.rms_eps;
    return a;
}

template <typename KV, int HD>
int launch_attention(axdec_model* m, int M, int layer, cudaStream_t s, int dxt) {
    const axdec_config_t& c = m->c;
    const int G = c.n_heads / c.n_kv_heads;
    if constexpr (std::is_same<KV, __half>::value && HD >= 64) {
      if (M >= 2) {
        // fp16 pages, head dim 64 / 128, batches: the tensor-core kernel (one
        // sequence with short splits keeps the scalar kernel, whose single
        // pass has less set-up per CTA)
        const bool q8 = c.act_mode != AXQ8_ACT_F32;
        // groups of at most 8 heads: tokens as the MMA rows (no padding rows)
        const bool tr = G <= 8;
        const size_t smem = tr ? attn_tct_smem_bytes<HD>(m->bps) : attn_tc_smem_bytes<HD>(m->bps);
        auto kern = tr ? (q8 ? attn_tct_kernel<HD, true> : attn_tct_kernel<HD, false>)
                       : (q8 ? attn_tc_kernel<HD, true> : attn_tc_kernel<HD, false>);
        static int configured[2][2][64] = {{{0}}};
        const int dev = m->ds->device < 64 ? m->ds->device : 63;
        constexpr int kMaxSmem = 200 * 1024;
        if (smem > (size_t)kMaxSmem)
            return fail(AXQ8_ERR_UNSUPPORTED, "attention: %zu B of shared memory", smem);
        if (smem > 48 * 1024 && !configured[tr][q8][dev]) {
            AXQ8_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               kMaxSmem),
                          "attention smem attribute");
            configured[tr][q8][dev] = 1;
        }
        Layer& Ly = m->L[layer];
        const float scale = 1.0f / std::sqrt((float)HD);   // mha.cpp:250
        AXQ8_CUDA_TRY(launch_k(kern, dim3(c.n_kv_heads, M, m->nsplit), dim3(kAttnTcWarps * 32),
                               smem, s, true, (const float*)m->qkv, m->Nqkv, (const int*)m->pos,
                               (const __half*)Ly.kc, (const __half*)Ly.vc,
                               (const int*)m->block_table, m->max_blocks, c.n_heads,
                               c.n_kv_heads, G, m->bps, scale, m->part, m->attn_cnt, m->x32,
                               m->xq, m->dx, dxt),
                      "attention launch");
        return AXQ8_OK;
      }
    }
    // pages per chunk: two chunks of K and V in at most 32 KB
    const int cp = std::max(1, std::min(m->bps, (int)(32768 / (4 * 16 * HD * sizeof(KV)))));
    const size_t smem = attn_smem_bytes<KV, HD>(G, cp, m->bps);
    if (smem > 48 * 1024)
        return fail(AXQ8_ERR_UNSUPPORTED, "attention: %zu B of shared memory", smem);
    const float scale = 1.0f / std::sqrt((float)HD);   // mha.cpp:250
    Layer& Ly = m->L[layer];
    const bool q8 = c.act_mode != AXQ8_ACT_F32;
    auto kern = q8 ? attn_decode_kernel<KV, HD, true> : attn_decode_kernel<KV, HD, false>;
    AXQ8_CUDA_TRY(launch_k(kern, dim3(c.n_kv_heads, M, m->nsplit), dim3(G * 32), smem, s, true,
                           (const float*)m->qkv, m->Nqkv, (const int*)m->pos, (const KV*)Ly.kc,
                           (const KV*)Ly.vc, (const int*)m->block_table, m->max_blocks, c.n_heads,
                           c.n_kv_heads, m->bps, cp, scale, m->part, m->attn_cnt, m->x32, m->xq,
                           m->dx, dxt),
                  "attention launch");
    return AXQ8_OK;
}

int launch_rmsnorm(axdec_model* m, int M, const float* x, const float* w, cudaStream_t s,
                   int dxt = 0) {
    const axdec_config_t& c = m->c;
    const int threads = rmsnorm_threads(c.hidden);   // checked at create
    if (c.act_mode == AXQ8_ACT_F32) {
        AXQ8_CUDA_TRY(launch_k(rmsnorm_kernel<false>, dim3(M), dim3(threads), 0, s, true, x, w,
                               c.hidden, c.rms_eps, m->x32, (int8_t*)nullptr, (float*)nullptr, 0),
                      "rmsnorm launch");
    } else {
        AXQ8_CUDA_TRY(launch_k(rmsnorm_kernel<true>, dim3(M), dim3(threads), 0, s, true, x, w,
                               c.hidden, c.rms_eps, (float*)nullptr, m->xq, m->dx, dxt),
                      "rmsnorm launch");
    }
    return AXQ8_OK;
}

// Grid of silu_mul_kernel for M rows of F (8 elements per thread).
constexpr int kSiluThreads = 256;
inline dim3 silu_grid(int M, int F) {
    const int64_t units = (int64_t)M * (F / 8);
    return dim3((unsigned)((units + kSiluThreads - 1) / kSiluThreads));
}

// Whether a step of M sequences runs wide: A8, M >= kWideMinM (the fused
// GEMV step re-reads its weights every 4 rows beyond that), up to 64 rows on
// the skinny product, beyond on the tcgen05 product when it tiles every linear.
constexpr int kWideMinM = 9;
bool wide_step(const axdec_model* m, int M) {
    // AXDEC_NARROW=1 keeps every batch on the GEMV step (comparison runs)
    static const bool narrow = [] {
        const char* e = getenv("AXDEC_NARROW");
        return e && atoi(e) != 0;
    }();
    if (narrow) return false;
    const axdec_config_t& c = m->c;
    const int64_t H = c.hidden, F = c.ffn;
    if (c.act_mode != AXQ8_ACT_Q8 || M < kWideMinM) return false;
    if (M <= kMmqMaxM) return true;   // skinny product: any shape (K % 32 == 0)
    return mma_shape_ok(m->Nqkv, H, M) && mma_shape_ok(H, m->Nq, M) &&
           mma_shape_ok(2 * F, H, M) && mma_shape_ok(H, F, M) && mma_shape_ok(c.vocab, H, M);
}

// Whether a wide step's linear of [N, K] at M rows takes the skinny product:
// the library's shape rule (skinny_preferred), or AXDEC_SKINNY_M = w (0..64)
// for a plain width threshold (tuning runs).
int skinny_m_override() {
    static const int v = [] {
        const char* e = getenv("AXDEC_SKINNY_M");
        const int x = e ? atoi(e) : -1;
        return x >= 0 && x <= kMmqMaxM ? x : -1;
    }();
    return v;
}

bool use_skinny(int64_t N, int64_t K, int M) {
    if (M > kMmqMaxM) return false;
    if (!mma_shape_ok(N, K, M)) return true;
    const int o = skinny_m_override();
    return o >= 0 ? M <= o : skinny_preferred(N, M);
}

axq8_weight_t wide_weight(axdec_model* m, const uint8_t* rows, int64_t N, int64_t K) {
    axq8_weight_t w = {};
    w.rows = const_cast<uint8_t*>(rows);
    w.N = N;
    w.K = K;
    w.row_stride = q8r_row_stride(K);
    w.device = m->ds->device;
    return w;
}

// y = x.W^T (+ resid) for the A8 activation xq / dxT (transposed scales).
int wide_linear(axdec_model* m, const uint8_t* rows, int64_t N, int64_t K, int M,
                const float* resid, float* y, const int8_t* xq, const float* dxT, cudaStream_t s) {
    axq8_weight_t w = wide_weight(m, rows, N, K);
    if (use_skinny(N, K, M)) return mmq_linear(m->ds, &w, xq, dxT, M, resid, y, N, s);
    return mma_linear(m->ds, &w, xq, dxT, M, resid, y, N, nullptr, s, &m->mma_sc);
}
int wide_linear(axdec_model* m, const uint8_t* rows, int64_t N, int64_t K, int M,
                const float* resid, float* y, cudaStream_t s) {
    return wide_linear(m, rows, N, K, M, resid, y, m->xq, m->dx, s);
}

// Whether a wide step's gate|up product computes SiLU*up and its A8
// quantization itself (the skinny product; the fp32 gate|up is never written).
// One GPU only: measured A/B on one box, Llama-3-8B batch 64, the step took
// 9.51 ms fused against 9.58 ms with the SiLU*up kernel, but with two
// tensor-parallel ranks 7.24-7.27 ms against 6.93 ms.
bool wide_silu_fused(axdec_model* m, int M) {
    const int64_t N = 2 * (int64_t)m->c.ffn;
    return m->silu_fused && m->tp == 1 && N % 64 == 0 && use_skinny(N, m->c.hidden, M);
}

// Wide batches (M >= 9): every linear on the tensor cores (the skinny
// mma.sync product up to 64 rows, tcgen05 kind::i8 beyond) from A8
// activations with transposed block scales, the producers (RMSNorm, SiLU*up, attention) writing that
// layout, RoPE + KV append and the greedy argmax as kernels of their own.
template <typename KV>
int launch_step_wide(axdec_model* m, int M, cudaStream_t s) {
    const axdec_config_t& c = m->c;
    const int H = c.hidden, F = c.ffn, hd = c.head_dim;
    const int dxt = (int)mma_scale_pitch(M);
    DeviceState* ds = m->ds;
    int rc;
    AXQ8_CUDA_TRY(launch_k(embed_kernel, dim3(M), dim3(256), 0, s, true, (const uint8_t*)m->embd,
                           m->rs_h, H, m->cf.vocab, (const int*)m->tokens, m->h, ds->status),
                  "embed launch");
    float* resid = m->rank == 0 ? m->h : nullptr;
    const int heads = c.n_heads + 2 * c.n_kv_heads;
    for (int l = 0; l < c.n_layers; l++) {
        Layer& Ly = m->L[l];
        if ((rc = launch_rmsnorm(m, M, m->h, Ly.attn_norm, s, dxt))) return rc;
        if ((rc = wide_linear(m, Ly.qkv, m->Nqkv, H, M, nullptr, m->qkv, s))) return rc;
        AXQ8_CUDA_TRY(launch_k(rope_kv_rows_kernel<KV>, dim3((M * heads + 7) / 8), dim3(256), 0, s,
                               true, m->qkv, M, c.n_heads, c.n_kv_heads, hd, (const int*)m->pos,
                               0, 0, (const float2*)m->rope, c.max_ctx, (const int*)m->block_table,
                               m->max_blocks, c.kv_block, (KV*)Ly.kc, (KV*)Ly.vc, ds->status),
                      "rope/kv launch");
        if (hd == 32) rc = launch_attention<KV, 32>(m, M, l, s, dxt);
        else if (hd == 64) rc = launch_attention<KV, 64>(m, M, l, s, dxt);
        else rc = launch_attention<KV, 128>(m, M, l, s, dxt);
        if (rc) return rc;
        if ((rc = wide_linear(m, Ly.o, H, m->Nq, M, resid, hidden_partial(m), s))) return rc;
        if (m->tp > 1 && (rc = allreduce_hidden(m, M, s))) return rc;
        if ((rc = launch_rmsnorm(m, M, m->h, Ly.ffn_norm, s, dxt))) return rc;
        if (wide_silu_fused(m, M)) {
            // SiLU*up -> A8 from the gate|up product straight into the gu
            // buffer's storage (it must not alias the product's input xq / dx)
            int8_t* sq = reinterpret_cast<int8_t*>(m->gu);
            float* sdx = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(m->gu) +
                                                  ((size_t)M * F + 255) / 256 * 256);
            const axq8_weight_t wgu = wide_weight(m, Ly.gu, 2 * (int64_t)F, H);
            if ((rc = mmq_linear_silu(ds, &wgu, m->xq, m->dx, M, sq, sdx, dxt, s))) return rc;
            if ((rc = wide_linear(m, Ly.down, H, F, M, resid, hidden_partial(m), sq, sdx, s))) return rc;
        } else {
            if ((rc = wide_linear(m, Ly.gu, 2 * (int64_t)F, H, M, nullptr, m->gu, s))) return rc;
            AXQ8_CUDA_TRY(launch_k(silu_mul_kernel<true>, silu_grid(M, F), dim3(kSiluThreads), 0, s, true,
                                   (const float*)m->gu, F, M, (float*)nullptr, m->xq, m->dx, dxt),
                          "silu launch");
            if ((rc = wide_linear(m, Ly.down, H, F, M, resid, hidden_partial(m), s))) return rc;
        }
        if (m->tp > 1 && (rc = allreduce_hidden(m, M, s))) return rc;
    }
    if ((rc = launch_rmsnorm(m, M, m->h, m->out_norm, s, dxt))) return rc;
    if ((rc = wide_linear(m, m->out_w, c.vocab, H, M, nullptr, m->logits, s))) return rc;
    const int chunks = std::max(1, std::min(64, c.vocab / 4096));
    AXQ8_CUDA_TRY(launch_k(argmax_rows_kernel, dim3(chunks, M), dim3(256), 0, s, true,
                           (const float*)m->logits, c.vocab, m->rank * c.vocab, m->amax_key),
                  "argmax launch");
    if (m->tp > 1) {
        const NcclApi* api = nccl_api();
        if (!api) return AXQ8_ERR_UNSUPPORTED;
        if ((rc = nccl_check(api->AllReduce(m->amax_key, m->amax_key, (size_t)M, ncclUint64, ncclMax,
                                            m->comm, s),
                             "axdec: argmax all-reduce")))
            return rc;
    }
    AXQ8_CUDA_TRY(launch_k(argmax_advance_kernel, dim3((M + 63) / 64), dim3(64), 0, s, true, m->amax_key, M,
                           m->pos, m->tokens, (const int*)m->feed, (const int*)m->ctl,
                           m->out_tokens, m->argmax),
                  "argmax advance launch");
    return AXQ8_OK;
}

template <typename KV>
int launch_step_kv(axdec_model* m, int M, cudaStream_t s) {
    if (wide_step(m, M)) return launch_step_wide<KV>(m, M, s);
    const axdec_config_t& c = m->c;
    const int H = c.hidden, F = c.ffn, hd = c.head_dim;
    const bool a32 = c.act_mode == AXQ8_ACT_F32;
    // fused producers: A8 and the activations of M rows fit in shared memory
    const bool fuse = !a32 && gemv_fused_prologue_fits(PRO_RMS, M, H) &&
                      gemv_fused_prologue_fits(PRO_QNT, M, F);
    const int plain = a32 ? PRO_F32 : PRO_Q8;
    DeviceState* ds = m->ds;
    int rc;
    AXQ8_CUDA_TRY(launch_k(embed_kernel, dim3(M), dim3(256), 0, s, true, (const uint8_t*)m->embd,
                           m->rs_h, H, m->cf.vocab, (const int*)m->tokens, m->h, ds->status),
                  "embed launch");
    // row-split projections: every rank's partial product, the residual added
    // once (rank 0), then summed over the ranks
    float* resid = m->rank == 0 ? m->h : nullptr;
    for (int l = 0; l < c.n_layers; l++) {
        Layer& Ly = m->L[l];
        // Q, K, V (+ RoPE, KV append)
        GemvArgs a = gemv_args(m, Ly.qkv, m->Nqkv, H, M, nullptr, m->qkv);
        a.pos = m->pos;
        a.rope = m->rope;
        a.max_ctx = c.max_ctx;
        a.n_heads = c.n_heads;
        a.n_kv = c.n_kv_heads;
        a.hd = hd;
        a.kc = Ly.kc;
        a.vc = Ly.vc;
        a.block_table = m->block_table;
        a.max_blocks = m->max_blocks;
        a.kv_block = c.kv_block;
        if (fuse) {
            a.src = m->h;
            a.norm_w = Ly.attn_norm;
            rc = gemv_launch_mt<PRO_RMS, EPI_ROPE_KV, KV>(ds, a, s);
        } else {
            if ((rc = launch_rmsnorm(m, M, m->h, Ly.attn_norm, s))) return rc;
            rc = a32 ? gemv_launch_mt<PRO_F32, EPI_ROPE_KV, KV>(ds, a, s)
                     : gemv_launch_mt<PRO_Q8, EPI_ROPE_KV, KV>(ds, a, s);
        }
        if (rc) return rc;
        // attention (+ split merge, + Q8 of its output)
        if (hd == 32) rc = launch_attention<KV, 32>(m, M, l, s, 0);
        else if (hd == 64) rc = launch_attention<KV, 64>(m, M, l, s, 0);
        else rc = launch_attention<KV, 128>(m, M, l, s, 0);
        if (rc) return rc;
        // O projection + residual
        a = gemv_args(m, Ly.o, H, m->Nq, M, resid, hidden_partial(m));
        rc = plain == PRO_F32 ? gemv_launch_mt<PRO_F32, EPI_STORE, float>(ds, a, s)
                              : gemv_launch_mt<PRO_Q8, EPI_STORE, float>(ds, a, s);
        if (rc) return rc;
        if (m->tp > 1 && (rc = allreduce_hidden(m, M, s))) return rc;
        // gate | up (fused: + SiLU*up in the epilogue, rows are (gate_j, up_j) pairs)
        a = gemv_args(m, Ly.gu, 2 * (int64_t)F, H, M, nullptr, m->gu);
        if (fuse) {
            a.src = m->h;
            a.norm_w = Ly.ffn_norm;
            a.ldy = F;
            rc = gemv_launch_mt<PRO_RMS, EPI_SILU, float>(ds, a, s);
        } else {
            if ((rc = launch_rmsnorm(m, M, m->h, Ly.ffn_norm, s))) return rc;
            rc = a32 ? gemv_launch_mt<PRO_F32, EPI_STORE, float>(ds, a, s)
                     : gemv_launch_mt<PRO_Q8, EPI_STORE, float>(ds, a, s);
        }
        if (rc) return rc;
        // down + residual
        a = gemv_args(m, Ly.down, H, F, M, resid, hidden_partial(m));
        if (fuse) {
            a.src = m->gu;   // SiLU*up [M][F], quantized in the prologue
            rc = gemv_launch_mt<PRO_QNT, EPI_STORE, float>(ds, a, s);
        } else {
            if (a32) {
                AXQ8_CUDA_TRY(launch_k(silu_mul_kernel<false>, silu_grid(M, F), dim3(kSiluThreads), 0,
                                       s, true, (const float*)m->gu, F, M, m->x32,
                                       (int8_t*)nullptr, (float*)nullptr, 0),
                              "silu launch");
                rc = gemv_launch_mt<PRO_F32, EPI_STORE, float>(ds, a, s);
            } else {
                AXQ8_CUDA_TRY(launch_k(silu_mul_kernel<true>, silu_grid(M, F), dim3(kSiluThreads), 0,
                                       s, true, (const float*)m->gu, F, M, (float*)nullptr, m->xq,
                                       m->dx, 0),
                              "silu launch");
                rc = gemv_launch_mt<PRO_Q8, EPI_STORE, float>(ds, a, s);
            }
        }
        if (rc) return rc;
        if (m->tp > 1 && (rc = allreduce_hidden(m, M, s))) return rc;
    }
    // final norm + LM head + greedy argmax + advance (this rank's vocabulary
    // slice; with tp > 1 the keys are reduced over the ranks before the advance)
    GemvArgs a = gemv_args(m, m->out_w, c.vocab, H, M, nullptr, m->logits);
    a.idx_offset = m->rank * c.vocab;
    a.no_advance = m->tp > 1;
    a.pos = m->pos;
    a.amax_key = m->amax_key;
    a.done = m->done;
    a.tokens = m->tokens;
    a.feed = m->feed;
    a.ctl = m->ctl;
    a.out_tokens = m->out_tokens;
    a.argmax_out = m->argmax;
    if (fuse) {
        a.src = m->h;
        a.norm_w = m->out_norm;
        rc = gemv_launch_mt<PRO_RMS, EPI_ARGMAX, float>(ds, a, s);
    } else {
        if ((rc = launch_rmsnorm(m, M, m->h, m->out_norm, s))) return rc;
        rc = a32 ? gemv_launch_mt<PRO_F32, EPI_ARGMAX, float>(ds, a, s)
                 : gemv_launch_mt<PRO_Q8, EPI_ARGMAX, float>(ds, a, s);
    }
    if (rc || m->tp == 1) return rc;
    const NcclApi* api = nccl_api();
    if (!api) return AXQ8_ERR_UNSUPPORTED;
    if ((rc = nccl_check(api->AllReduce(m->amax_key, m->amax_key, (size_t)M, ncclUint64, ncclMax,
                                        m->comm, s),
                         "axdec: argmax all-reduce")))
        return rc;
    AXQ8_CUDA_TRY(launch_k(argmax_advance_kernel, dim3((M + 63) / 64), dim3(64), 0, s, true, m->amax_key, M,
                           m->pos, m->tokens, (const int*)m->feed, (const int*)m->ctl,
                           m->out_tokens, m->argmax),
                  "argmax advance launch");
    return AXQ8_OK;
}

// ---- batched prefill -------------------------------------------------------------
// The prompt's positions run through the layers as one wide product per linear
// per chunk (rows = sequences x positions, the tcgen05 product above 64 rows,
// the skinny one up to 64), the chunk's K and V go to the pages, and a causal
// attention kernel reads every earlier page: StreamingExecutor::execute_layer
// (streaming_executor.cpp:110-238) and mha_attention (mha.cpp:167-198) for a
// whole prompt, where ModelRunner::generate feeds the prompt one position at a
// time (model_runner.cpp:291-295).  No logits: the last prompt position goes
// through the decode step, which yields the first generated token.
constexpr int kPrefillRows = 4096;   // rows of one chunk when every linear tiles on tcgen05

bool all_mma_ok(const axdec_model* m, int64_t M) {
    const axdec_config_t& c = m->c;
    const int64_t H = c.hidden, F = c.ffn;
    return mma_shape_ok(m->Nqkv, H, M) && mma_shape_ok(H, m->Nq, M) && mma_shape_ok(2 * F, H, M) &&
           mma_shape_ok(H, F, M);
}

// Whether prompts of n_seq sequences can take the batched prefill.
bool prefill_supported(const axdec_model* m, int n_seq) {
    const axdec_config_t& c = m->c;
    const int G = c.n_heads / c.n_kv_heads;
    if (m->prefill_mode == 0 || c.act_mode != AXQ8_ACT_Q8 || c.kv_fp32) return false;
    if (c.head_dim != 64 && c.head_dim != 128) return false;
    if (G > 8 && G % 8) return false;
    return n_seq <= kMmqMaxM || all_mma_ok(m, kPrefillRows);
}

// Positions of one chunk: as many as fit kPrefillRows rows (64 rows when some
// linear does not tile on tcgen05), at least one.
// AXDEC_PREFILL_ROWS = r (1 .. the cap) sets a smaller chunk (tests of the
// chunk boundaries, tuning runs).
int prefill_chunk_positions(const axdec_model* m, int n_seq, int n_tok) {
    int cap = all_mma_ok(m, kPrefillRows) ? kPrefillRows : kMmqMaxM;
    const char* e = getenv("AXDEC_PREFILL_ROWS");
    const int r = e ? atoi(e) : 0;
    if (r >= 1 && r < cap) cap = r;
    return std::max(1, std::min(n_tok, cap / n_seq));
}

// Chunk buffers for the largest chunk any prompt of this model can form (a
// chunk holds n_seq * T <= the chunk cap rows, or n_seq rows when T = 1).
int prefill_alloc(axdec_model* m) {
    if (m->pre_cap) return AXQ8_OK;
    const axdec_config_t& c = m->c;
    const int cap = all_mma_ok(m, kPrefillRows) ? kPrefillRows : kMmqMaxM;
    const int rows = (int)std::max<int64_t>(std::min<int64_t>(cap, (int64_t)c.max_batch * c.max_ctx),
                                            c.max_batch);
    const int H = c.hidden, F = c.ffn;
    const int maxK = std::max(std::max(H, F), m->Nq);
    int rc = AXQ8_OK;
    m->ph = (float*)dalloc(m, sizeof(float) * (size_t)rows * H, &rc);
    m->pxq = (int8_t*)dalloc(m, (size_t)rows * maxK, &rc);
    m->pdx = (float*)dalloc(m, sizeof(float) * mma_scale_pitch(rows) * (maxK / QK), &rc);
    m->pqkv = (float*)dalloc(m, sizeof(float) * (size_t)rows * m->Nqkv, &rc);
    m->pgu = (float*)dalloc(m, sizeof(float) * (size_t)rows * 2 * F, &rc);
    m->ptok = (int*)dalloc(m, sizeof(int) * rows, &rc);
    if (rc == AXQ8_OK) m->pre_cap = rows;
    return rc;
}

// Split-K scratch for the chunk products at Mc rows (grown outside any capture).
int prefill_scratch(axdec_model* m, int Mc) {
    if (Mc <= kMmqMaxM) return AXQ8_OK;
    const axdec_config_t& c = m->c;
    const int64_t H = c.hidden, F = c.ffn;
    const int64_t shapes[4][2] = {{m->Nqkv, H}, {H, m->Nq}, {2 * F, H}, {H, F}};
    size_t part = 0;
    int64_t cnt = 0;
    for (auto& sh : shapes) {
        size_t pb = 0;
        int64_t cn = 0;
        mma_split_needs(m->ds, sh[0], sh[1], Mc, &pb, &cn);
        part = std::max(part, pb);
        cnt = std::max(cnt, cn);
    }
    MmaScratch& sc = m->pre_sc;
    if (part <= sc.part_bytes && cnt <= sc.counter_slots) return AXQ8_OK;
    AXQ8_CUDA_TRY(cudaDeviceSynchronize(), "axdec: prefill scratch");
    int rc = AXQ8_OK;
    if (part > sc.part_bytes) {
        sc.part = (float*)dalloc(m, part, &rc);
        sc.part_bytes = rc == AXQ8_OK ? part : 0;
    }
    if (rc == AXQ8_OK && cnt > sc.counter_slots) {
        sc.counters = (int*)dalloc(m, sizeof(int) * cnt, &rc);
        sc.counter_slots = rc == AXQ8_OK ? cnt : 0;
        if (rc == AXQ8_OK) AXQ8_CUDA_TRY(cudaMemset(sc.counters, 0, sizeof(int) * cnt), "axdec: counters");
    }
    return rc;
}

int prefill_linear(axdec_model* m, const uint8_t* rows, int64_t N, int64_t K, int Mc,
                   const float* resid, float* y, cudaStream_t s) {
    axq8_weight_t w = {};
    w.rows = const_cast<uint8_t*>(rows);
    w.N = N;
    w.K = K;
    w.row_stride = q8r_row_stride(K);
    w.device = m->ds->device;
    if (Mc <= kMmqMaxM) return mmq_linear(m->ds, &w, m->pxq, m->pdx, Mc, resid, y, N, s);
    return mma_linear(m->ds, &w, m->pxq, m->pdx, Mc, resid, y, N, nullptr, s, &m->pre_sc);
}

template <int HD>
int launch_attn_prefill(axdec_model* m, int layer, int n_seq, int T, int p0, int dxt,
                        cudaStream_t s) {
    const axdec_config_t& c = m->c;
    const int G = c.n_heads / c.n_kv_heads;
    const int Gc = std::min(G, 8), HG = G / Gc;
    const int TQ = 16 * (kPrefWarps / Gc);
    constexpr size_t smem = attn_prefill_smem_bytes<HD>();
    auto kern = attn_prefill_kernel<HD, true>;
    static int configured[64] = {0};
    const int dev = m->ds->device < 64 ? m->ds->device : 63;
    if (smem > 48 * 1024 && !configured[dev]) {
        AXQ8_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                      "prefill attention smem attribute");
        configured[dev] = 1;
    }
    const float scale = 1.0f / std::sqrt((float)HD);   // mha.cpp:131
    Layer& Ly = m->L[layer];
    AXQ8_CUDA_TRY(launch_k(kern, dim3((unsigned)(((T + TQ - 1) / TQ) * HG), c.n_kv_heads, n_seq),
                           dim3(kPrefWarps * 32), smem, s, true, (const float*)m->pqkv, m->Nqkv, T,
                           p0, (const __half*)Ly.kc, (const __half*)Ly.vc,
                           (const int*)m->block_table, m->max_blocks, c.n_kv_heads, G, scale,
                           m->pxq, m->Nq, m->pdx, dxt, (float*)nullptr),
                  "prefill attention launch");
    return AXQ8_OK;
}

// Positions 0 .. n_tok - 1 of sequences 0 .. n_seq - 1, tokens from m->feed
// ([n_seq][feed_len], uploaded by reset_run): KV pages written, no logits.
int prefill_positions(axdec_model* m, int n_seq, int n_tok, int feed_len, cudaStream_t s) {
    const axdec_config_t& c = m->c;
    const int H = c.hidden, F = c.ffn, hd = c.head_dim;
    const int T = prefill_chunk_positions(m, n_seq, n_tok);
    int rc = prefill_alloc(m);
    if (rc) return rc;
    if (n_seq * T > m->pre_cap)
        return fail(AXQ8_ERR_INVALID, "axdec: prefill chunk of %d rows above %d", n_seq * T, m->pre_cap);
    DeviceState* ds = m->ds;
    float* resid = m->rank == 0 ? m->ph : nullptr;
    const int heads = c.n_heads + 2 * c.n_kv_heads;
    const int threads = rmsnorm_threads(H);
    const NcclApi* api = m->tp > 1 ? nccl_api() : nullptr;
    if (m->tp > 1 && !api) return AXQ8_ERR_UNSUPPORTED;
    for (int p0 = 0; p0 < n_tok; p0 += T) {
        const int Tc = std::min(T, n_tok - p0), Mc = n_seq * Tc;
        const int dxt = (int)mma_scale_pitch(Mc);
        if ((rc = prefill_scratch(m, Mc))) return rc;
        AXQ8_CUDA_TRY(launch_k(gather_chunk_tokens_kernel, dim3((Mc + 255) / 256), dim3(256), 0, s,
                               true, (const int*)m->feed, feed_len, n_seq, Tc, p0, m->ptok),
                      "prefill tokens launch");
        AXQ8_CUDA_TRY(launch_k(embed_kernel, dim3(Mc), dim3(256), 0, s, true, (const uint8_t*)m->embd,
                               m->rs_h, H, m->cf.vocab, (const int*)m->ptok, m->ph, ds->status),
                      "prefill embed launch");
        for (int l = 0; l < c.n_layers; l++) {
            Layer& Ly = m->L[l];
            AXQ8_CUDA_TRY(launch_k(rmsnorm_kernel<true>, dim3(Mc), dim3(threads), 0, s, true,
                                   (const float*)m->ph, (const float*)Ly.attn_norm, H, c.rms_eps,
                                   (float*)nullptr, m->pxq, m->pdx, dxt),
                          "prefill rmsnorm launch");
            if ((rc = prefill_linear(m, Ly.qkv, m->Nqkv, H, Mc, nullptr, m->pqkv, s))) return rc;
            AXQ8_CUDA_TRY(launch_k(rope_kv_rows_kernel<__half>, dim3((Mc * heads + 7) / 8), dim3(256), 0,
                                   s, true, m->pqkv, Mc, c.n_heads, c.n_kv_heads, hd,
                                   (const int*)nullptr, Tc, p0, (const float2*)m->rope, c.max_ctx,
                                   (const int*)m->block_table, m->max_blocks, c.kv_block,
                                   (__half*)Ly.kc, (__half*)Ly.vc, ds->status),
                          "prefill rope/kv launch");
            rc = hd == 64 ? launch_attn_prefill<64>(m, l, n_seq, Tc, p0, dxt, s)
                          : launch_attn_prefill<128>(m, l, n_seq, Tc, p0, dxt, s);
            if (rc) return rc;
            if ((rc = prefill_linear(m, Ly.o, H, m->Nq, Mc, resid, m->ph, s))) return rc;
            if (m->tp > 1 &&
                (rc = nccl_check(api->AllReduce(m->ph, m->ph, (size_t)Mc * H, ncclFloat, ncclSum,
                                                m->comm, s),
                                 "axdec: prefill all-reduce")))
                return rc;
            AXQ8_CUDA_TRY(launch_k(rmsnorm_kernel<true>, dim3(Mc), dim3(threads), 0, s, true,
                                   (const float*)m->ph, (const float*)Ly.ffn_norm, H, c.rms_eps,
                                   (float*)nullptr, m->pxq, m->pdx, dxt),
                          "prefill rmsnorm launch");
            if ((rc = prefill_linear(m, Ly.gu, 2 * (int64_t)F, H, Mc, nullptr, m->pgu, s))) return rc;
            AXQ8_CUDA_TRY(launch_k(silu_mul_kernel<true>, silu_grid(Mc, F), dim3(kSiluThreads), 0, s,
                                   true, (const float*)m->pgu, F, Mc, (float*)nullptr, m->pxq, m->pdx,
                                   dxt),
                          "prefill silu launch");
            if ((rc = prefill_linear(m, Ly.down, H, F, Mc, resid, m->ph, s))) return rc;
            if (m->tp > 1 &&
                (rc = nccl_check(api->AllReduce(m->ph, m->ph, (size_t)Mc * H, ncclFloat, ncclSum,
                                                m->comm, s),
                                 "axdec: prefill all-reduce")))
                return rc;
        }
    }
    return AXQ8_OK;
}

// Every sequence at position `p` with input token column `col` of the fed tokens.
int set_positions(axdec_model* m, const int32_t* feed_host, int n_seq, int feed_len, int col, int p,
                  cudaStream_t s) {
    std::vector<int> tok(n_seq), pos(n_seq, p);
    for (int i = 0; i < n_seq; i++) tok[i] = feed_host[(size_t)i * feed_len + col];
    AXQ8_CUDA_TRY(cudaMemcpyAsync(m->tokens, tok.data(), sizeof(int) * n_seq, cudaMemcpyHostToDevice, s),
                  "axdec: tokens upload");
    AXQ8_CUDA_TRY(cudaMemcpyAsync(m->pos, pos.data(), sizeof(int) * n_seq, cudaMemcpyHostToDevice, s),
                  "axdec: positions upload");
    return AXQ8_OK;   // pageable sources: staged before the calls return
}

// Instantiate (once per batch size) the graph of one decode step.  The first
// time, the step runs eagerly once so every kernel is loaded and configured
// before capture; the caller resets the control state afterwards.
int get_graph(axdec_model* m, int M, cudaGraphExec_t* out) {
    auto it = m->graphs.find(M);
    if (it != m->graphs.end()) {
        *out = it->second.exec;
        return AXQ8_OK;
    }
    cudaStream_t s = m->cap_stream;
    // warm-up from position 0 with the prompt/feed state left as is
    AXQ8_CUDA_TRY(cudaMemsetAsync(m->pos, 0, sizeof(int) * m->c.max_batch, s), "axdec: pos reset");
    int rc = launch_step(m, M, s);
    if (rc) return rc;
    AXQ8_CUDA_TRY(cudaStreamSynchronize(s), "axdec: warm-up step");
    cudaGraph_t g = nullptr;
    AXQ8_CUDA_TRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "axdec: begin capture");
    rc = launch_step(m, M, s);
    cudaError_t e = cudaStreamEndCapture(s, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return cuda_fail(e, "axdec: end capture");
    // kernel nodes of the step, reported by axdec_step_kernels
    size_t n_nodes = 0;
    int kernels = 0;
    if (cudaGraphGetNodes(g, nullptr, &n_nodes) == cudaSuccess && n_nodes) {
        std::vector<cudaGraphNode_t> nodes(n_nodes);
        if (cudaGraphGetNodes(g, nodes.data(), &n_nodes) == cudaSuccess)
            for (auto nd : nodes) {
                cudaGraphNodeType t;
                if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel)
                    kernels++;
            }
    }
    cudaGraphExec_t exec = nullptr;
    e = cudaGraphInstantiate(&exec, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return cuda_fail(e, "axdec: graph instantiate");
    m->graphs[M].exec = exec;
    m->graphs[M].kernels = kernels;
    *out = exec;
    return AXQ8_OK;
}

// Reset the control state for a run: positions 0, fed tokens uploaded, first
// input = feed[:, 0].
int reset_run(axdec_model* m, const int32_t* feed_host, int M, int feed_len, int n_prompt,
              int max_out, cudaStream_t s) {
    const int mc = m->c.max_ctx;
    if (feed_len > mc) return fail(AXQ8_ERR_INVALID, "axdec: %d positions > max_ctx %d", feed_len, mc);
    AXQ8_CUDA_TRY(cudaMemcpyAsync(m->feed, feed_host, sizeof(int) * (size_t)M * feed_len,
                                  cudaMemcpyHostToDevice, s), "axdec: feed upload");
    std::vector<int> first(M), zeros(M, 0);
    for (int i = 0; i < M; i++) first[i] = feed_host[(size_t)i * feed_len];
    const int ctl[3] = {n_prompt, feed_len, max_out};
    AXQ8_CUDA_TRY(cudaMemcpyAsync(m->tokens, first.data(), sizeof(int) * M, cudaMemcpyHostToDevice, s),
                  "axdec: tokens upload");
    AXQ8_CUDA_TRY(cudaMemcpyAsync(m->pos, zeros.data(), sizeof(int) * M, cudaMemcpyHostToDevice, s),
                  "axdec: pos reset");
    AXQ8_CUDA_TRY(cudaMemcpyAsync(m->ctl, ctl, sizeof(ctl), cudaMemcpyHostToDevice, s),
                  "axdec: ctl upload");
    // the staging vectors above are pageable host memory: the copies complete
    // before cudaMemcpyAsync returns, so they may go out of scope
    return AXQ8_OK;
}

}  // namespace

extern "C" {

int axdec_tensor_index(const axdec_config_t* c, const char* name) {
    if (!c || !name) return -1;
    if (!strcmp(name, "token_embd.weight")) return 0;
    if (!strcmp(name, "output.weight")) return 1;
    if (!strcmp(name, "output_norm.weight")) return 2;
    int layer;
    std::string slot;
    if (!parse_layer_name(name, &layer, &slot) || layer < 0 || layer >= c->n_layers) return -1;
    const int si = slot_index(slot);
    return si < 0 ? -1 : 3 + 9 * layer + si;
}

int axdec_create(const axdec_config_t* cfg, axdec_model_t** out) {
    if (!cfg || !out) return fail(AXQ8_ERR_INVALID, "axdec_create: null argument");
    const axdec_config_t cf = *cfg;
    const int tp = cf.tp_size > 1 ? cf.tp_size : 1, rank = tp > 1 ? cf.tp_rank : 0;
    if (rank < 0 || rank >= tp)
        return fail(AXQ8_ERR_INVALID, "axdec_create: tp_rank %d outside [0, %d)", cf.tp_rank, tp);
    if (cf.n_kv_heads <= 0 || cf.n_kv_heads % tp || cf.ffn % (QK * tp) || cf.vocab % tp)
        return fail(AXQ8_ERR_INVALID,
                    "axdec_create: tp_size %d must divide n_kv_heads (%d), ffn / 32 (%d) and "
                    "vocab (%d)",
                    tp, cf.n_kv_heads, cf.ffn / QK, cf.vocab);
    // this rank's dimensions
    axdec_config_t c = cf;
    c.n_heads = cf.n_heads / tp;
    c.n_kv_heads = cf.n_kv_heads / tp;
    c.ffn = cf.ffn / tp;
    c.vocab = cf.vocab / tp;
    c.tp_size = tp;
    c.tp_rank = rank;
    if (c.n_layers <= 0 || c.hidden <= 0 || c.ffn <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 ||
        c.vocab <= 0 || c.max_batch <= 0 || c.max_ctx <= 0)
        return fail(AXQ8_ERR_INVALID, "axdec_create: non-positive dimension");
    if (c.hidden % QK || c.ffn % QK || c.n_heads % c.n_kv_heads ||
        c.n_heads * c.head_dim % QK)
        return fail(AXQ8_ERR_INVALID, "axdec_create: dimensions must be multiples of 32 and "
                                      "n_heads a multiple of n_kv_heads");
    if (c.head_dim != 32 && c.head_dim != 64 && c.head_dim != 128)
        return fail(AXQ8_ERR_UNSUPPORTED, "axdec_create: head_dim %d (32, 64, 128 supported)",
                    c.head_dim);
    if (c.kv_block != 16) return fail(AXQ8_ERR_UNSUPPORTED, "axdec_create: kv_block must be 16");
    if (!rmsnorm_threads(c.hidden))
        return fail(AXQ8_ERR_UNSUPPORTED, "axdec_create: hidden %d above the norm kernel's %d",
                    c.hidden, 8 * kNormUnits * 1024);
    if (c.n_heads / c.n_kv_heads > 16)
        return fail(AXQ8_ERR_UNSUPPORTED, "axdec_create: more than 16 query heads per kv head");
    if (c.act_mode != AXQ8_ACT_Q8 && c.act_mode != AXQ8_ACT_F32)
        return fail(AXQ8_ERR_INVALID, "axdec_create: bad act_mode");
    DeviceState* ds = device_state();
    if (!ds) return AXQ8_ERR_CUDA;
    axdec_model* m = new axdec_model();
    m->c = c;
    m->cf = cf;
    m->cf.tp_size = tp;
    m->cf.tp_rank = rank;
    m->tp = tp;
    m->rank = rank;
    m->ds = ds;
    {   // AXDEC_SILU_FUSE=0: SiLU*up as a kernel of its own in wide steps (tuning, comparisons)
        const char* e = getenv("AXDEC_SILU_FUSE");
        m->silu_fused = !(e && atoi(e) == 0);
    }
    m->Nq = c.n_heads * c.head_dim;
    m->Nkv = c.n_kv_heads * c.head_dim;
    m->Nqkv = m->Nq + 2 * m->Nkv;
    m->rs_h = q8r_row_stride(c.hidden);
    m->rs_q = q8r_row_stride(m->Nq);
    m->rs_f = q8r_row_stride(c.ffn);
    m->max_blocks = (c.max_ctx + c.kv_block - 1) / c.kv_block;
    // split the context so that attention gives about four CTAs per SM at full
    // length, at most 32 splits (the merge gives one lane to each split), each
    // split at least min_pages pages: one page when the (sequence, kv head)
    // pairs are few (batch 1, 384-token context: 1 page 1,202 tokens/s, 2 pages
    // 1,166, 4 pages 998, one split 710), 32 pages from 64 pairs on, where the
    // grid is wide already and more splits only add merge work (batch 64, one
    // kv head, 2048-token context: 1 page 3.155 ms per step, 32 pages 3.081).
    // AXDEC_ATTN_MIN_PAGES overrides (tuning).
    const int pairs = c.n_kv_heads * c.max_batch;
    const int min_pages = [pairs] {
        const int dflt = pairs >= 64 ? 32 : 1;
        const char* e = getenv("AXDEC_ATTN_MIN_PAGES");
        const int v = e ? atoi(e) : dflt;
        return v >= 1 && v <= 4096 ? v : dflt;
    }();
    const int target = (4 * ds->sm_count + pairs - 1) / pairs;
    m->nsplit = std::max(1, std::min(std::min(target, (m->max_blocks + min_pages - 1) / min_pages), 32));
    m->bps = (m->max_blocks + m->nsplit - 1) / m->nsplit;
    m->nsplit = (m->max_blocks + m->bps - 1) / m->bps;
    int rc = AXQ8_OK;
    const int M = c.max_batch, H = c.hidden, F = c.ffn;
    const size_t kvsz = c.kv_fp32 ? 4 : 2;
    const int64_t pages = (int64_t)M * m->max_blocks;
    m->embd = (uint8_t*)dalloc(m, (size_t)cf.vocab * m->rs_h, &rc);   // replicated
    m->out_w = (uint8_t*)dalloc(m, (size_t)c.vocab * m->rs_h, &rc);
    m->out_norm = (float*)dalloc(m, sizeof(float) * H, &rc);
    m->L.resize(c.n_layers);
    for (int l = 0; l < c.n_layers && rc == AXQ8_OK; l++) {
        Layer& Ly = m->L[l];
        Ly.qkv = (uint8_t*)dalloc(m, (size_t)m->Nqkv * m->rs_h, &rc);
        Ly.o = (uint8_t*)dalloc(m, (size_t)H * m->rs_q, &rc);
        Ly.gu = (uint8_t*)dalloc(m, (size_t)2 * F * m->rs_h, &rc);
        Ly.down = (uint8_t*)dalloc(m, (size_t)H * m->rs_f, &rc);
        Ly.attn_norm = (float*)dalloc(m, sizeof(float) * H, &rc);
        Ly.ffn_norm = (float*)dalloc(m, sizeof(float) * H, &rc);
        Ly.kc = dalloc(m, (size_t)pages * c.n_kv_heads * c.kv_block * c.head_dim * kvsz, &rc);
        Ly.vc = dalloc(m, (size_t)pages * c.n_kv_heads * c.kv_block * c.head_dim * kvsz, &rc);
    }
    const int maxK = std::max(std::max(H, F), m->Nq);
    m->h = (float*)dalloc(m, sizeof(float) * M * H, &rc);
    m->xq = (int8_t*)dalloc(m, (size_t)M * maxK, &rc);
    // block scales: [M][K/32], or transposed [K/32][M rounded up to 4] (wide steps)
    m->dx = (float*)dalloc(m, sizeof(float) * mma_scale_pitch(M) * (maxK / QK), &rc);
    m->x32 = (float*)dalloc(m, sizeof(float) * M * maxK, &rc);
    m->qkv = (float*)dalloc(m, sizeof(float) * M * m->Nqkv, &rc);
    m->gu = (float*)dalloc(m, sizeof(float) * M * 2 * F, &rc);
    m->part = (float*)dalloc(m, sizeof(float) * (size_t)M * c.n_heads * m->nsplit * (c.head_dim + 2), &rc);
    m->logits = (float*)dalloc(m, sizeof(float) * (size_t)M * c.vocab, &rc);
    m->rope = (float2*)dalloc(m, sizeof(float2) * (size_t)c.max_ctx * (c.head_dim / 2), &rc);
    m->block_table = (int*)dalloc(m, sizeof(int) * pages, &rc);
    m->tokens = (int*)dalloc(m, sizeof(int) * M, &rc);
    m->pos = (int*)dalloc(m, sizeof(int) * M, &rc);
    m->feed = (int*)dalloc(m, sizeof(int) * (size_t)M * c.max_ctx, &rc);
    m->out_tokens = (int*)dalloc(m, sizeof(int) * (size_t)M * c.max_ctx, &rc);
    m->argmax = (int*)dalloc(m, sizeof(int) * M, &rc);
    m->ctl = (int*)dalloc(m, sizeof(int) * 4, &rc);
    m->amax_key = (unsigned long long*)dalloc(m, sizeof(unsigned long long) * M, &rc);
    m->done = (int*)dalloc(m, sizeof(int), &rc);
    m->attn_cnt = (int*)dalloc(m, sizeof(int) * M * c.n_kv_heads, &rc);
    if (tp > 1) {   // NVLink all-reduce buffers (mapped by the peers at axdec_tp_connect)
        m->ar_part = (float*)dalloc(m, sizeof(float) * M * H, &rc);
        m->ar_flags = (unsigned*)dalloc(m, sizeof(unsigned) * 2 * kArMaxRanks, &rc);
        m->ar_epoch = (unsigned*)dalloc(m, sizeof(unsigned), &rc);
        m->ar_ctas = (int*)dalloc(m, sizeof(int), &rc);
        for (void* z : {(void*)m->ar_flags, (void*)m->ar_epoch, (void*)m->ar_ctas})
            if (rc == AXQ8_OK && cudaMemset(z, 0, z == (void*)m->ar_flags ? sizeof(unsigned) * 2 * kArMaxRanks : 4) != cudaSuccess)
                rc = cuda_fail(cudaGetLastError(), "axdec: all-reduce flags");
    }
    if (rc == AXQ8_OK && c.act_mode == AXQ8_ACT_Q8 && M >= kWideMinM) {
        // split-K scratch for every width a wide step may run at
        size_t part = 0;
        int64_t cnt = 0;
        const int64_t shapes[5][2] = {{m->Nqkv, H}, {H, m->Nq}, {2 * (int64_t)F, H}, {H, F},
                                      {c.vocab, H}};
        for (int mm = kWideMinM; mm <= M; mm++)
            for (auto& sh : shapes) {
                size_t pb = 0;
                int64_t cn = 0;
                if (!use_skinny(sh[0], sh[1], mm) && mma_shape_ok(sh[0], sh[1], mm))
                    mma_split_needs(ds, sh[0], sh[1], mm, &pb, &cn);
                part = std::max(part, pb);
                cnt = std::max(cnt, cn);
            }
        if (part) {
            m->mma_sc.part = (float*)dalloc(m, part, &rc);
            m->mma_sc.part_bytes = part;
            m->mma_sc.counters = (int*)dalloc(m, sizeof(int) * cnt, &rc);
            m->mma_sc.counter_slots = cnt;
            if (rc == AXQ8_OK) {
                cudaError_t e = cudaMemset(m->mma_sc.counters, 0, sizeof(int) * cnt);
                if (e != cudaSuccess) rc = cuda_fail(e, "axdec: split counters");
            }
        }
    }
    if (rc == AXQ8_OK) {
        cudaError_t e = cudaStreamCreateWithFlags(&m->cap_stream, cudaStreamNonBlocking);
        if (e != cudaSuccess) rc = cuda_fail(e, "axdec: stream create");
    }
    if (rc == AXQ8_OK) {
        // RoPE table with the reference's expressions (mha.cpp:38-41), on the host
        const int half = c.head_dim / 2;
        std::vector<float2> tab((size_t)c.max_ctx * half);
        for (int p = 0; p < c.max_ctx; p++)
            for (int i = 0; i < half; i++) {
                const float freq = 1.0f / std::pow(c.rope_theta, (float)(2 * i) / (float)c.head_dim);
                const float angle = (float)p * freq;
                tab[(size_t)p * half + i] = make_float2(std::cos(angle), std::sin(angle));
            }
        // identity page assignment: sequence b owns pages [b*max_blocks, ...)
        std::vector<int> bt(pages);
        for (int64_t i = 0; i < pages; i++) bt[i] = (int)i;
        cudaError_t e = cudaMemcpy(m->rope, tab.data(), sizeof(float2) * tab.size(), cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(m->block_table, bt.data(), sizeof(int) * pages, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemset(m->feed, 0, sizeof(int) * (size_t)M * c.max_ctx);
        if (e == cudaSuccess) e = cudaMemset(m->tokens, 0, sizeof(int) * M);
        if (e == cudaSuccess) e = cudaMemset(m->pos, 0, sizeof(int) * M);
        if (e == cudaSuccess) e = cudaMemset(m->amax_key, 0, sizeof(unsigned long long) * M);
        if (e == cudaSuccess) e = cudaMemset(m->done, 0, sizeof(int));
        if (e == cudaSuccess) e = cudaMemset(m->attn_cnt, 0, sizeof(int) * M * c.n_kv_heads);
        // KV pages start at zero: attention multiplies the token slots past the
        // context by a zero weight, which an uninitialized NaN pattern would
        // turn into NaN
        const size_t page_bytes =
            (size_t)pages * c.n_kv_heads * c.kv_block * c.head_dim * kvsz;
        for (int l = 0; l < c.n_layers && e == cudaSuccess; l++) {
            e = cudaMemset(m->L[l].kc, 0, page_bytes);
            if (e == cudaSuccess) e = cudaMemset(m->L[l].vc, 0, page_bytes);
        }
        if (e == cudaSuccess) {
            const int ctl[4] = {1, 1, 0, 0};
            e = cudaMemcpy(m->ctl, ctl, sizeof(ctl), cudaMemcpyHostToDevice);
        }
        if (e != cudaSuccess) rc = cuda_fail(e, "axdec: init upload");
    }
    if (rc != AXQ8_OK) {
        axdec_destroy(m);
        return rc;
    }
    *out = m;
    return AXQ8_OK;
}

int axdec_destroy(axdec_model_t* m) {
    if (!m) return AXQ8_OK;
    for (auto& kv : m->graphs)
        if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    if (m->cap_stream) cudaStreamDestroy(m->cap_stream);
    for (void* p : m->ar_mapped) cudaIpcCloseMemHandle(p);
    if (m->comm) {
        const NcclApi* api = nccl_api();
        if (api) api->CommDestroy(m->comm);
    }
    for (void* p : m->allocs) cudaFree(p);
    delete m;
    return AXQ8_OK;
}

int64_t axdec_device_bytes(const axdec_model_t* m) { return m ? m->bytes : 0; }

int axdec_step_kernels(const axdec_model_t* m, int n_seq) {
    if (!m) return -1;
    auto it = m->graphs.find(n_seq);
    return it == m->graphs.end() ? -1 : it->second.kernels;
}

int64_t axdec_weight_bytes_per_step(const axdec_model_t* m) {
    if (!m) return 0;
    const axdec_config_t& c = m->c;
    const int64_t H = c.hidden, F = c.ffn;
    const int64_t per_layer = (int64_t)m->Nqkv * H + H * m->Nq + 2 * F * H + H * F;
    const int64_t params = per_layer * c.n_layers + (int64_t)c.vocab * H;   // + LM head
    return params / QK * Q8_0_BYTES;
}

int axdec_set_tensor(axdec_model_t* m, const char* name, const void* host, int ggml_type,
                     int64_t rows, int64_t cols) {
    if (!m || !name || !host) return fail(AXQ8_ERR_INVALID, "axdec_set_tensor: null argument");
    Dest d;
    int rc = resolve(m, name, &d);
    if (rc) return rc;
    if (d.f32) {
        if (ggml_type != 0 || rows * cols != d.n)
            return fail(AXQ8_ERR_INVALID, "axdec_set_tensor: '%s' must be F32 with %lld values",
                        name, (long long)d.n);
        AXQ8_CUDA_TRY(cudaMemcpy(d.f32, host, sizeof(float) * d.n, cudaMemcpyHostToDevice),
                      "axdec_set_tensor: copy");
        return AXQ8_OK;
    }
    if (ggml_type != 8 || rows != d.src_N || cols != d.src_K)
        return fail(AXQ8_ERR_INVALID,
                    "axdec_set_tensor: '%s' must be Q8_0 [%lld, %lld] (got type %d [%lld, %lld])",
                    name, (long long)d.src_N, (long long)d.src_K, ggml_type, (long long)rows,
                    (long long)cols);
    if (!strcmp(name, "output.weight")) m->out_set = true;
    // this rank's slice: rows src_row0.., whole 32-blocks from column src_col0
    std::vector<uint8_t> slice;
    if (d.N != d.src_N || d.K != d.src_K) {
        const size_t row_bytes = (size_t)(d.K / QK) * Q8_0_BYTES;
        slice.resize((size_t)d.N * row_bytes);
        const uint8_t* src = static_cast<const uint8_t*>(host);
        for (int64_t n = 0; n < d.N; n++)
            memcpy(slice.data() + (size_t)n * row_bytes,
                   src + ((size_t)(d.src_row0 + n) * (d.src_K / QK) + d.src_col0 / QK) * Q8_0_BYTES,
                   row_bytes);
        host = slice.data();
        rows = d.N;
        cols = d.K;
    }
    const size_t bytes = (size_t)rows * (cols / QK) * Q8_0_BYTES;
    void* staging = nullptr;
    void* tmp = nullptr;
    AXQ8_CUDA_TRY(cudaMalloc(&staging, bytes), "axdec_set_tensor: staging");
    cudaError_t e = cudaMalloc(&tmp, (size_t)rows * q8r_row_stride(cols));
    if (e == cudaSuccess) e = cudaMemcpy(staging, host, bytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        rc = axq8_weight_repack(staging, rows, cols, tmp, nullptr);
        if (rc == AXQ8_OK) e = cudaDeviceSynchronize();
        if (rc == AXQ8_OK && e == cudaSuccess) rc = place_rows(m, d, (const uint8_t*)tmp);
    }
    cudaFree(staging);
    if (tmp) cudaFree(tmp);
    if (e != cudaSuccess) return cuda_fail(e, "axdec_set_tensor: upload");
    if (rc) return rc;
    if (!m->out_set && !strcmp(name, "token_embd.weight")) {
        // tied LM head until output.weight arrives
        AXQ8_CUDA_TRY(cudaMemcpy(m->out_w, m->embd + (size_t)m->rank * m->c.vocab * m->rs_h,
                                 (size_t)m->c.vocab * m->rs_h,
                                 cudaMemcpyDeviceToDevice),
                      "axdec_set_tensor: tie lm head");
    }
    return AXQ8_OK;
}

int axdec_init_random(axdec_model_t* m, uint64_t seed, float stdv) {
    if (!m) return fail(AXQ8_ERR_INVALID, "axdec_init_random: null model");
    const axdec_config_t& c = m->c;
    std::vector<std::string> names = {"token_embd.weight", "output.weight", "output_norm.weight"};
    for (int l = 0; l < c.n_layers; l++)
        for (int s = 0; s < 9; s++) names.push_back("blk." + std::to_string(l) + "." + kSlots[s] + ".weight");
    for (const std::string& n : names) {
        Dest d;
        int rc = resolve(m, n.c_str(), &d);
        if (rc) return rc;
        if (d.f32) {
            fill_kernel<<<64, 256>>>(d.f32, d.n, 1.0f);
            AXQ8_CUDA_TRY(cudaGetLastError(), "axdec_init_random: fill");
            continue;
        }
        // this rank's slice of the tensor axq8_synth_q8_0(sd, src_N, src_K) generates
        const uint64_t sd = seed + (uint64_t)axdec_tensor_index(&c, n.c_str());
        if (!d.rope_perm && d.row_step == 1) {
            rc = synth_q8_0_slice(sd, d.N, d.K, d.src_row0, d.src_col0, d.src_K, 0.0f, stdv,
                                  d.rows + d.row0 * q8r_row_stride(d.K), nullptr);
            if (rc) return rc;
            continue;
        }
        void* tmp = nullptr;
        AXQ8_CUDA_TRY(cudaMalloc(&tmp, (size_t)d.N * q8r_row_stride(d.K)), "axdec_init_random: tmp");
        rc = synth_q8_0_slice(sd, d.N, d.K, d.src_row0, d.src_col0, d.src_K, 0.0f, stdv, tmp,
                              nullptr);
        if (rc == AXQ8_OK) rc = place_rows(m, d, (const uint8_t*)tmp);
        cudaFree(tmp);
        if (rc) return rc;
    }
    m->out_set = true;
    AXQ8_CUDA_TRY(cudaDeviceSynchronize(), "axdec_init_random: synchronize");
    return AXQ8_OK;
}

int axdec_generate(axdec_model_t* m, const int32_t* prompts, int32_t n_seq, int32_t n_prompt,
                   int32_t n_new, int32_t* out_tokens, float* logits_out, float* decode_ms,
                   void* stream) {
    if (!m || !prompts || !out_tokens) return fail(AXQ8_ERR_INVALID, "axdec_generate: null argument");
    if (n_seq <= 0 || n_seq > m->c.max_batch || n_prompt <= 0 || n_new <= 0)
        return fail(AXQ8_ERR_INVALID, "axdec_generate: bad sizes");
    if (n_prompt + n_new - 1 > m->c.max_ctx)
        return fail(AXQ8_ERR_INVALID, "axdec_generate: %d positions exceed max_ctx %d",
                    n_prompt + n_new - 1, m->c.max_ctx);
    if (m->tp > 1 && !m->comm)
        return fail(AXQ8_ERR_STATE, "axdec_generate: tensor-parallel model not connected");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaGraphExec_t g;
    int rc = get_graph(m, n_seq, &g);
    if (rc) return rc;
    if ((rc = reset_run(m, prompts, n_seq, n_prompt, n_prompt, n_new, s))) return rc;
    m->sess_seq = 0;
    m->sess_pos = -1;
    int r0 = 0;
    if (n_prompt >= 2 && prefill_supported(m, n_seq)) {
        // prompt positions 0 .. n_prompt - 2 in one batched pass; the last
        // prompt position goes through the step and yields the first token
        if ((rc = prefill_positions(m, n_seq, n_prompt - 1, n_prompt, s))) return rc;
        if ((rc = set_positions(m, prompts, n_seq, n_prompt, n_prompt - 1, n_prompt - 1, s))) return rc;
        r0 = n_prompt - 1;
    }
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (decode_ms) {
        AXQ8_CUDA_TRY(cudaEventCreate(&e0), "event");
        AXQ8_CUDA_TRY(cudaEventCreate(&e1), "event");
    }
    const int total = n_prompt - 1 + n_new;
    const size_t lbytes = sizeof(float) * (size_t)n_seq * m->c.vocab;
    for (int r = r0; r < total; r++) {
        if (decode_ms && r == n_prompt - 1) cudaEventRecord(e0, s);
        AXQ8_CUDA_TRY(cudaGraphLaunch(g, s), "axdec: graph launch");
        if (logits_out && r >= n_prompt - 1) {
            AXQ8_CUDA_TRY(cudaMemcpyAsync(logits_out + (size_t)(r - n_prompt + 1) * n_seq * m->c.vocab,
                                          m->logits, lbytes, cudaMemcpyDeviceToHost, s),
                          "axdec: logits copy");
        }
    }
    if (decode_ms) cudaEventRecord(e1, s);
    // generated tokens: out_tokens rows of max_out = n_new
    AXQ8_CUDA_TRY(cudaMemcpyAsync(out_tokens, m->out_tokens, sizeof(int) * (size_t)n_seq * n_new,
                                  cudaMemcpyDeviceToHost, s),
                  "axdec: tokens copy");
    AXQ8_CUDA_TRY(cudaStreamSynchronize(s), "axdec: generate");
    if (decode_ms) {
        cudaEventElapsedTime(decode_ms, e0, e1);
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
    }
    return AXQ8_OK;
}

int axdec_forced(axdec_model_t* m, const int32_t* tokens, int32_t n_seq, int32_t n_prompt,
                 int32_t n_steps, float* logits_out, void* stream) {
    if (!m || !tokens || !logits_out) return fail(AXQ8_ERR_INVALID, "axdec_forced: null argument");
    if (n_seq <= 0 || n_seq > m->c.max_batch || n_prompt <= 0 || n_steps < n_prompt ||
        n_steps > m->c.max_ctx)
        return fail(AXQ8_ERR_INVALID, "axdec_forced: bad sizes");
    if (m->tp > 1 && !m->comm)
        return fail(AXQ8_ERR_STATE, "axdec_forced: tensor-parallel model not connected");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaGraphExec_t g;
    int rc = get_graph(m, n_seq, &g);
    if (rc) return rc;
    const int n_out = n_steps - n_prompt + 1;
    if ((rc = reset_run(m, tokens, n_seq, n_steps, n_prompt, n_out, s))) return rc;
    m->sess_seq = 0;
    m->sess_pos = -1;
    const size_t lbytes = sizeof(float) * (size_t)n_seq * m->c.vocab;
    for (int r = 0; r < n_steps; r++) {
        AXQ8_CUDA_TRY(cudaGraphLaunch(g, s), "axdec: graph launch");
        if (r >= n_prompt - 1)
            AXQ8_CUDA_TRY(cudaMemcpyAsync(logits_out + (size_t)(r - n_prompt + 1) * n_seq * m->c.vocab,
                                          m->logits, lbytes, cudaMemcpyDeviceToHost, s),
                          "axdec: logits copy");
    }
    AXQ8_CUDA_TRY(cudaStreamSynchronize(s), "axdec: forced");
    return AXQ8_OK;
}

int axdec_set_prefill(axdec_model_t* m, int mode) {
    if (!m || (mode != 0 && mode != 1)) return fail(AXQ8_ERR_INVALID, "axdec_set_prefill: bad argument");
    m->prefill_mode = mode;
    return AXQ8_OK;
}

int axdec_prefill_batched(const axdec_model_t* m, int32_t n_seq) {
    return m && n_seq > 0 && n_seq <= m->c.max_batch && prefill_supported(m, n_seq) ? 1 : 0;
}

int axdec_prefill(axdec_model_t* m, const int32_t* tokens, int32_t n_seq, int32_t n_tok,
                  void* stream) {
    if (!m || (!tokens && n_tok > 0)) return fail(AXQ8_ERR_INVALID, "axdec_prefill: null argument");
    if (n_seq <= 0 || n_seq > m->c.max_batch || n_tok < 0 || n_tok >= m->c.max_ctx)
        return fail(AXQ8_ERR_INVALID, "axdec_prefill: bad sizes (n_seq %d, n_tok %d, max_ctx %d)",
                    n_seq, n_tok, m->c.max_ctx);
    if (m->tp > 1 && !m->comm)
        return fail(AXQ8_ERR_STATE, "axdec_prefill: tensor-parallel model not connected");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaGraphExec_t g;
    int rc = get_graph(m, n_seq, &g);
    if (rc) return rc;
    m->sess_seq = 0;
    m->sess_pos = -1;
    if (n_tok > 0) {
        if ((rc = reset_run(m, tokens, n_seq, n_tok, n_tok + 1, 0, s))) return rc;
        if (prefill_supported(m, n_seq)) {
            if ((rc = prefill_positions(m, n_seq, n_tok, n_tok, s))) return rc;
        } else {
            for (int r = 0; r < n_tok; r++)
                AXQ8_CUDA_TRY(cudaGraphLaunch(g, s), "axdec: graph launch");
        }
    }
    // the session continues at position n_tok with the caller's tokens: no
    // fed tokens, no recorded outputs
    std::vector<int> pos(n_seq, n_tok);
    const int ctl[3] = {0, 0, 0};
    AXQ8_CUDA_TRY(cudaMemcpyAsync(m->pos, pos.data(), sizeof(int) * n_seq, cudaMemcpyHostToDevice, s),
                  "axdec: positions upload");
    AXQ8_CUDA_TRY(cudaMemcpyAsync(m->ctl, ctl, sizeof(ctl), cudaMemcpyHostToDevice, s),
                  "axdec: ctl upload");
    AXQ8_CUDA_TRY(cudaStreamSynchronize(s), "axdec_prefill");
    m->sess_seq = n_seq;
    m->sess_pos = n_tok;
    return AXQ8_OK;
}

int axdec_decode_step(axdec_model_t* m, const int32_t* tokens, int32_t n_seq, int32_t* next_tokens,
                      float* logits_out, void* stream) {
    if (!m || !tokens || !next_tokens) return fail(AXQ8_ERR_INVALID, "axdec_decode_step: null argument");
    if (m->sess_pos < 0 || n_seq != m->sess_seq)
        return fail(AXQ8_ERR_STATE, "axdec_decode_step: no session of %d sequences (call axdec_prefill)",
                    n_seq);
    if (m->sess_pos >= m->c.max_ctx)
        return fail(AXQ8_ERR_INVALID, "axdec_decode_step: position %d reaches max_ctx %d", m->sess_pos,
                    m->c.max_ctx);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaGraphExec_t g;
    int rc = get_graph(m, n_seq, &g);
    if (rc) return rc;
    AXQ8_CUDA_TRY(cudaMemcpyAsync(m->tokens, tokens, sizeof(int) * n_seq, cudaMemcpyHostToDevice, s),
                  "axdec_decode_step: tokens upload");
    AXQ8_CUDA_TRY(cudaGraphLaunch(g, s), "axdec_decode_step: graph launch");
    AXQ8_CUDA_TRY(cudaMemcpyAsync(next_tokens, m->argmax, sizeof(int) * n_seq, cudaMemcpyDeviceToHost, s),
                  "axdec_decode_step: tokens copy");
    if (logits_out)
        AXQ8_CUDA_TRY(cudaMemcpyAsync(logits_out, m->logits, sizeof(float) * (size_t)n_seq * m->c.vocab,
                                      cudaMemcpyDeviceToHost, s),
                      "axdec_decode_step: logits copy");
    AXQ8_CUDA_TRY(cudaStreamSynchronize(s), "axdec_decode_step");
    m->sess_pos++;
    return AXQ8_OK;
}

int axdec_decode_continue(axdec_model_t* m, const int32_t* first_tokens, int32_t n_seq,
                          int32_t n_steps, int32_t* out_tokens, float* decode_ms, void* stream) {
    if (!m || !out_tokens || n_steps <= 0)
        return fail(AXQ8_ERR_INVALID, "axdec_decode_continue: bad argument");
    if (m->sess_pos < 0 || n_seq != m->sess_seq)
        return fail(AXQ8_ERR_STATE,
                    "axdec_decode_continue: no session of %d sequences (call axdec_prefill)", n_seq);
    if (m->sess_pos + n_steps > m->c.max_ctx)
        return fail(AXQ8_ERR_INVALID, "axdec_decode_continue: %d steps from position %d exceed max_ctx %d",
                    n_steps, m->sess_pos, m->c.max_ctx);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaGraphExec_t g;
    int rc = get_graph(m, n_seq, &g);
    if (rc) return rc;
    if (first_tokens)
        AXQ8_CUDA_TRY(cudaMemcpyAsync(m->tokens, first_tokens, sizeof(int) * n_seq,
                                      cudaMemcpyHostToDevice, s),
                      "axdec_decode_continue: tokens upload");
    // record the greedy tokens of positions sess_pos + 1 .. (out_tokens rows of n_steps)
    const int ctl[3] = {m->sess_pos + 1, 0, n_steps};
    AXQ8_CUDA_TRY(cudaMemcpyAsync(m->ctl, ctl, sizeof(ctl), cudaMemcpyHostToDevice, s),
                  "axdec_decode_continue: ctl upload");
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (decode_ms) {
        AXQ8_CUDA_TRY(cudaEventCreate(&e0), "event");
        AXQ8_CUDA_TRY(cudaEventCreate(&e1), "event");
        cudaEventRecord(e0, s);
    }
    for (int r = 0; r < n_steps; r++) AXQ8_CUDA_TRY(cudaGraphLaunch(g, s), "axdec: graph launch");
    if (decode_ms) cudaEventRecord(e1, s);
    AXQ8_CUDA_TRY(cudaMemcpyAsync(out_tokens, m->out_tokens, sizeof(int) * (size_t)n_seq * n_steps,
                                  cudaMemcpyDeviceToHost, s),
                  "axdec_decode_continue: tokens copy");
    const int ctl0[3] = {0, 0, 0};
    AXQ8_CUDA_TRY(cudaMemcpyAsync(m->ctl, ctl0, sizeof(ctl0), cudaMemcpyHostToDevice, s),
                  "axdec_decode_continue: ctl reset");
    AXQ8_CUDA_TRY(cudaStreamSynchronize(s), "axdec_decode_continue");
    if (decode_ms) {
        cudaEventElapsedTime(decode_ms, e0, e1);
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
    }
    m->sess_pos += n_steps;
    return AXQ8_OK;
}

int axdec_tp_unique_id(void* id_out, int64_t id_bytes) {
    if (!id_out || id_bytes < (int64_t)sizeof(ncclUniqueId))
        return fail(AXQ8_ERR_INVALID, "axdec_tp_unique_id: needs %zu bytes", sizeof(ncclUniqueId));
    const NcclApi* api = nccl_api();
    if (!api) return AXQ8_ERR_UNSUPPORTED;
    ncclUniqueId id;
    int rc = nccl_check(api->GetUniqueId(&id), "ncclGetUniqueId");
    if (rc) return rc;
    memcpy(id_out, &id, sizeof(id));
    return AXQ8_OK;
}

int axdec_tp_connect(axdec_model_t* m, const void* id) {
    if (!m || !id) return fail(AXQ8_ERR_INVALID, "axdec_tp_connect: null argument");
    if (m->tp == 1) return AXQ8_OK;
    if (m->comm) return fail(AXQ8_ERR_STATE, "axdec_tp_connect: already connected");
    const NcclApi* api = nccl_api();
    if (!api) return AXQ8_ERR_UNSUPPORTED;
    AXQ8_CUDA_TRY(cudaSetDevice(m->ds->device), "axdec_tp_connect: set device");
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    int rc = nccl_check(api->CommInitRank(&m->comm, m->tp, uid, m->rank), "ncclCommInitRank");
    if (rc) return rc;
    return setup_peer_allreduce(m);
}

int axtp_allreduce_sum(const axtp_group_t* g, int64_t n, void* stream) {
    static_assert(AXTP_MAX_RANKS == kArMaxRanks, "group size");
    if (!g || g->world < 2 || g->world > AXTP_MAX_RANKS || g->rank < 0 || g->rank >= g->world ||
        n < 0 || n % 4 || !g->epoch || !g->ctas_done)
        return fail(AXQ8_ERR_INVALID, "axtp_allreduce_sum: bad group or size");
    for (int r = 0; r < g->world; r++)
        if (!g->part[r] || !g->out[r] || !g->flags[r] ||
            (reinterpret_cast<uintptr_t>(g->part[r]) & 15) || (reinterpret_cast<uintptr_t>(g->out[r]) & 15))
            return fail(AXQ8_ERR_INVALID, "axtp_allreduce_sum: null or unaligned buffer of rank %d", r);
    if (n == 0) return AXQ8_OK;
    DeviceState* ds = device_state();
    if (!ds) return AXQ8_ERR_CUDA;
    ArPeers p{};
    for (int r = 0; r < g->world; r++) {
        p.part[r] = g->part[r];
        p.out[r] = g->out[r];
        p.flags[r] = g->flags[r];
    }
    p.epoch = g->epoch;
    p.ctas_done = g->ctas_done;
    p.status = ds->status;
    p.rank = g->rank;
    p.world = g->world;
    const int64_t per = (n / 4 + g->world - 1) / g->world;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(64, (per + kArThreads - 1) / kArThreads));
    AXQ8_CUDA_TRY(launch_k(tp_allreduce_kernel, dim3(grid), dim3(kArThreads), 0,
                           static_cast<cudaStream_t>(stream), false, p, n),
                  "axtp_allreduce_sum launch");
    return AXQ8_OK;
}

int axdec_tp_allreduce_kind(const axdec_model_t* m) {
    if (!m) return -1;
    return m->tp == 1 ? 0 : m->ar_on ? 2 : 1;
}

int axdec_tp_health(axdec_model_t* m, int* nccl_error, int* device_status) {
    if (!m) return fail(AXQ8_ERR_INVALID, "axdec_tp_health: null model");
    if (nccl_error) {
        *nccl_error = 0;
        if (m->comm) {
            const NcclApi* api = nccl_api();
            if (!api) return AXQ8_ERR_UNSUPPORTED;
            ncclResult_t r = ncclSuccess;
            int rc = nccl_check(api->CommGetAsyncError(m->comm, &r), "ncclCommGetAsyncError");
            if (rc) return rc;
            *nccl_error = (int)r;
        }
    }
    if (device_status) {
        // the status word, without synchronizing (a hung peer would block a sync)
        AXQ8_CUDA_TRY(cudaMemcpyAsync(device_status, m->ds->status, sizeof(int), cudaMemcpyDeviceToHost,
                                      m->cap_stream), "axdec_tp_health: status");
        AXQ8_CUDA_TRY(cudaStreamSynchronize(m->cap_stream), "axdec_tp_health: status");
    }
    return AXQ8_OK;
}

int axdec_tp_abort(axdec_model_t* m) {
    if (!m) return fail(AXQ8_ERR_INVALID, "axdec_tp_abort: null model");
    if (!m->comm) return AXQ8_OK;
    const NcclApi* api = nccl_api();
    if (!api) return AXQ8_ERR_UNSUPPORTED;
    int rc = nccl_check(api->CommAbort(m->comm), "ncclCommAbort");
    m->comm = nullptr;   // aborted: destroy must not touch it again
    // the step graphs hold the aborted communicator's calls: re-captured
    // after the next axdec_tp_connect
    for (auto& kv : m->graphs)
        if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    m->graphs.clear();
    for (void* p : m->ar_mapped) cudaIpcCloseMemHandle(p);
    m->ar_mapped.clear();
    m->ar_on = false;
    return rc;
}

}  // extern "C"
