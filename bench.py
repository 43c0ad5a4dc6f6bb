#!/usr/bin/env python
"""Benchmark of the B200 Q8_0 hot path; prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl axion|reference]
                    [--workload llama3|decode|gemv|prefill|skinny]

Workloads
  llama3 (default) Llama-3-8B-architecture batched decode: 32 layers, hidden
         4096, FFN 14336 SwiGLU, 32 query / 8 KV heads of 128, vocab 128256,
         RoPE theta 5e5 (Llama-3's), random-init Q8_0 weights (N(0, 0.02)
         before quantization, generated on the device), 64 sequences with
         random 2048-token prompts (batched prefill), then K (default 128)
         greedy decode steps over paged fp16 KV (block 16), tensor parallel
         over the N GPUs of the run (column-split Q/K/V/gate/up, row-split
         O/down, vocabulary-split LM head, NCCL all-reduce; strong scaling).
         One step = one decode position of all 64 sequences (64 tokens).
         Metric: decode tokens/s of the whole job, device time of K steps
         continued on the device (axdec_decode_continue).  `e2e`: the same
         steps through the public step call (axdec_decode_step) with pinned
         host token buffers, H2D of the 64 input tokens and D2H of the 64
         next tokens inside every step.  `roofline`: the step as a weight +
         KV stream per rank against the measured HBM bandwidth.
  decode TinyLlama-1.1B-architecture decode: 22 layers, hidden 2048, FFN
         5632, 32 query / 4 KV heads of 64, vocab 32000, batch 1, a random
         128-token prompt, then K (default 256) greedy steps.  Metric: decode
         tokens/s (device time of the K steps); `e2e`: the whole public
         axdec_generate call (host prompt in, host tokens out, batched prefill
         of the prompt included).
  gemv   Q8_0 GEMV, TinyLlama ffn_up shape: W [5632 x 2048] Q8_0, x [1 x 2048]
         fp32 N(0, 1) quantized on the fly, y [5632] fp32.  One step = one
         linear_from_gguf call; the weight rotates over enough copies (> 4 x
         L2) that every step streams it from HBM.  Metric: algorithmic bytes
         / s (W 34/32 B per weight + x + y = 12,285,952 B per step).
  skinny the decode-width product (q8_mmq_kernel) on the Llama-3-8B layer
         shapes [6144x4096], [4096x4096], [28672x4096], [4096x14336] at M =
         16, 32, 64 with pre-quantized activations.  One step = the 12
         products.  Metric: algorithmic bytes / s.
  prefill Q8_0 prefill GEMM sweep, Llama-2-7B linear shapes [4096x4096],
         [11008x4096], [4096x11008], [32000x4096] x M in {256, 1024, 2048,
         4096} on the tcgen05 kind::i8 path.  One step = one GEMM (cases in
         rotation; default K = 16 = the whole sweep).  Metric: int8 TOPS.

Arms
  --impl axion      the CUDA path (libaxq8.so) on N GPUs, one process per GPU
                    (torchrun for N > 1).
  --impl reference  the reference's own CPU implementation (oracle/_ref,
                    built from its unmodified sources) on the host cores, rank
                    0 only; each of the K steps is a bounded sample of the
                    workload, and the line says how its rate follows from it.
                    It loads no library of this repository.

Timing: W untimed warm-up steps, then K steps between barrier +
cudaDeviceSynchronize, CUDA events on the launching stream, max over ranks.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


# ---------------------------------------------------------------------------
# environment helpers
# ---------------------------------------------------------------------------

def measured_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except Exception:
            pass
    return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": FALLBACK_BF16_TFLOPS}, "fallback"


def ncu_traffic(workload: str):
    """DRAM bytes per launch of the dominant kernel from the committed ncu
    summary (profiles/ncu_traffic.json), or None."""
    p = ROOT / "profiles" / "ncu_traffic.json"
    try:
        return json.loads(p.read_text())[workload]["traffic_bytes"]
    except Exception:
        return None


def l3_traffic(layers: int, world: int, kv_bytes: float):
    """DRAM bytes of one Llama-3-8B decode step on one GPU: the measured
    per-layer and embedding/LM-head traffic of profiles/ncu_traffic.json
    (a 4-layer capture) scaled to `layers`, plus the K/V pages the step reads;
    None for tensor-parallel ranks (not captured: ncu runs one process)."""
    p = ROOT / "profiles" / "ncu_traffic.json"
    try:
        t = json.loads(p.read_text())["llama3_8b_arch_decode_b64_tp1"]
    except Exception:
        return None
    if world != 1:
        return None
    return int(layers * t["per_layer_bytes"] + t["embed_head_argmax_bytes"] + kv_bytes)


def use_all_host_cores() -> None:
    """The reference's OpenMP loops use every host core (torchrun sets
    OMP_NUM_THREADS=1 for its workers); called before its library loads."""
    os.environ["OMP_NUM_THREADS"] = str(host_cores())


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


class ClockSampler:
    """nvidia-smi clocks/throttle sampling while the timed region runs."""

    QUERY = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None, period_ms: int = 50):
        self.uuid = uuid
        self.period_ms = period_ms
        self.proc = None
        self.f = None

    def start(self):
        try:
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 f"-lms", str(self.period_ms)], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.flush()
        self.f.seek(0)
        rows = [r.split(", ") for r in self.f.read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        mine = [r for r in rows if len(r) >= 10 and (self.uuid is None or r[1] == self.uuid)]
        if not mine and rows:
            mine = [r for r in rows if len(r) >= 10 and r[0] == "0"]
        if not mine:
            return None
        sm = [float(r[2]) for r in mine if r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in mine if r[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in mine for n, v in zip(names, r[6:10]) if "Active" in v
                          and "Not" not in v})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(mine)}


def device_uuid(dev) -> str | None:
    import torch
    try:
        u = str(torch.cuda.get_device_properties(dev).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return None


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------

class Dist:
    def __init__(self, n_gpus: int):
        self.rank = int(os.environ.get("RANK", "0"))
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world != n_gpus:
            raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={self.world}: launch N>1 with "
                             "torch.distributed.run")
        self.pg = None

    def init(self, backend: str = "nccl"):
        import datetime
        import torch
        import torch.distributed as dist
        if backend == "nccl":
            torch.cuda.set_device(self.local)
        if self.world > 1:
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local)
                                    if backend == "nccl" else None)
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def sum(self, v: float) -> float:
        if not self.pg:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.SUM)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


# ---------------------------------------------------------------------------
# GEMV workload
# ---------------------------------------------------------------------------

GEMV_N, GEMV_K = 5632, 2048
GEMV_SEED = 0xA710


def gemv_bytes(M=1, N=GEMV_N, K=GEMV_K) -> int:
    return N * (K // 32) * 34 + M * K * 4 + M * N * 4


def run_gemv_axion(args, d: Dist) -> dict:
    import torch
    from axion_b200 import _lib, ops
    lib = _lib.load()
    dev = torch.device("cuda", d.local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(dev)
    # Every launch, graph replay, copy and event of this arm goes on `stream`
    # (CUDAGraph.replay() launches on the current stream).
    torch.cuda.set_stream(stream)
    props = torch.cuda.get_device_properties(dev)
    l2 = getattr(props, "L2_cache_size", 126 * 2**20)
    wbytes = GEMV_N * ops.row_stride(GEMV_K)
    n_copies = max(8, int(4 * l2 // wbytes) + 1)
    with torch.cuda.stream(stream):
        weights = [ops.Q8Weight.synthetic(GEMV_SEED + i, GEMV_N, GEMV_K, device=dev)
                   for i in range(n_copies)]
        g = torch.Generator(device=dev).manual_seed(1234 + d.rank)
        x = torch.randn(1, GEMV_K, generator=g, device=dev)
        y = torch.empty(1, GEMV_N, device=dev)
        xq, dx = ops.quantize_activations(x)
    s_ptr = C.c_void_p(stream.cuda_stream)
    K_steps, W_steps = args.steps, args.warmup

    def step(i):
        _lib.check(lib.axq8_linear(weights[i % n_copies].c, C.c_void_p(x.data_ptr()), 1,
                                   C.c_void_p(y.data_ptr()), _lib.AXQ8_ACT_Q8, s_ptr))

    # --- device-resident throughput: graph of one pass over the rotating copies
    torch.cuda.synchronize()
    for i in range(W_steps):
        step(i)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            for i in range(n_copies):
                step(i)
    reps = max(1, (K_steps + n_copies - 1) // n_copies)
    steps_done = reps * n_copies
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(device_uuid(dev)).start()
    time.sleep(0.15)
    d.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    d.barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    ms_max = d.max(ms)
    value = d.sum(steps_done) * gemv_bytes() / (ms_max / 1e3) / 1e9 if d.world > 1 else \
        steps_done * gemv_bytes() / (ms_max / 1e3) / 1e9

    # --- roofline: the GEMV kernel alone (pre-quantized x), back to back
    rl_graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(rl_graph, stream=stream):
            for i in range(n_copies):
                _lib.check(lib.axq8_linear_q8act(weights[i].c, C.c_void_p(xq.data_ptr()),
                                                 C.c_void_p(dx.data_ptr()), 1, None,
                                                 C.c_void_p(y.data_ptr()), s_ptr))
    rl_graph.replay()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(reps):
        rl_graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    k_ms = e0.elapsed_time(e1) / (reps * n_copies)
    peaks, peak_kind = measured_peaks()
    alg = gemv_bytes()
    achieved = alg / (k_ms / 1e3) / 1e9
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                "traffic": ncu_traffic("q8_gemv_5632x2048_m1"), "kernel": "q8_gemv_kernel<1,0,0>",
                "kernel_us": round(k_ms * 1e3, 3), "peak_source": peak_kind,
                "algorithmic_bytes": alg}

    # --- e2e through the public C-ABI call with host buffers
    xh = torch.empty(1, GEMV_K, dtype=torch.float32, pin_memory=True)
    xh.copy_(x.cpu())
    yh = torch.empty(1, GEMV_N, dtype=torch.float32, pin_memory=True)
    xd = torch.empty_like(x)
    e2e_steps = min(K_steps, 20000)

    def e2e_step(i):
        xd.copy_(xh, non_blocking=True)
        _lib.check(lib.axq8_linear(weights[i % n_copies].c, C.c_void_p(xd.data_ptr()), 1,
                                   C.c_void_p(y.data_ptr()), _lib.AXQ8_ACT_Q8, s_ptr))
        yh.copy_(y, non_blocking=True)

    with torch.cuda.stream(stream):
        for i in range(W_steps):
            e2e_step(i)
        torch.cuda.synchronize()
        d.barrier()
        e0.record(stream)
        for i in range(e2e_steps):
            e2e_step(i)
        e1.record(stream)
        torch.cuda.synchronize()
    e2e_ms = d.max(e0.elapsed_time(e1))
    e2e_val = d.sum(e2e_steps) * gemv_bytes() / (e2e_ms / 1e3) / 1e9 if d.world > 1 else \
        e2e_steps * gemv_bytes() / (e2e_ms / 1e3) / 1e9
    status = ops.status()
    return {
        "metric": "Q8_0 GEMV HBM GB/s (algorithmic bytes)", "value": round(value, 1),
        "unit": "GB/s", "n_gpus": d.world, "steps": steps_done, "warmup": W_steps,
        "ms_per_step": round(ms_max / steps_done, 6), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8 x int8 -> int32 -> fp32",
        "data": "synthetic (device-generated Q8_0 weights, N(0,0.02); x N(0,1))",
        "config": gemv_config(args, d.world),
        "l2_policy": f"rotating {n_copies} weight copies ({n_copies * wbytes / 2**20:.0f} MiB > "
                     f"4 x L2)",
        "e2e": {"value": round(e2e_val, 2), "unit": "GB/s",
                "h2d_bytes_per_step": GEMV_K * 4, "d2h_bytes_per_step": GEMV_N * 4,
                "steps": e2e_steps, "path": "axq8_linear (C ABI) + pinned H2D/D2H"},
        "roofline": roofline,
        "gpu_launches": 2 * steps_done,
        "clocks": clk,
        "device_status": status,
    }


def gemv_reference(args, steps: int) -> dict:
    """The reference's as-shipped per-token cost of this linear:
    GGUFLoader::load_tensor (read + Q8_0 dequant) + linear_from_gguf."""
    import numpy as np
    from axion_b200.gguf import Q8_0, GGUFWriter
    from oracle.oracle import Oracle, RefLib
    o, r = Oracle(), RefLib()
    tmp = Path(tempfile.mkdtemp()) / "gemv.gguf"
    gw = GGUFWriter()
    gw.add_tensor("blk.0.ffn_up.weight", o.synth_q8_0(GEMV_SEED, GEMV_N, GEMV_K),
                  (GEMV_N, GEMV_K), Q8_0)
    gw.write(tmp)
    x = np.random.default_rng(0).normal(0, 1, (1, GEMV_K)).astype(np.float32)
    r.time_linear(tmp, "blk.0.ffn_up.weight", x, GEMV_N, 2)          # warm page cache
    sec, _ = r.time_linear(tmp, "blk.0.ffn_up.weight", x, GEMV_N, steps)
    tmp.unlink()
    val = steps * gemv_bytes() / sec / 1e9
    return {"value": round(val, 4), "unit": "GB/s", "cores": host_cores(), "kind": "reference",
            "sample": f"{steps} x (GGUFLoader::load_tensor + linear_from_gguf) on "
                      f"[5632x2048] Q8_0, M=1, OpenMP threads={host_cores()}",
            "seconds": round(sec, 3)}


# ---------------------------------------------------------------------------

# ---------------------------------------------------------------------------
# TinyLlama-architecture decode workload (batch 1, 128-token prompt)
# ---------------------------------------------------------------------------

TL = dict(n_layers=22, hidden=2048, ffn=5632, n_heads=32, n_kv_heads=4, head_dim=64,
          vocab=32000, rope_theta=10000.0, rms_eps=1e-5)
TL_PROMPT, TL_NEW, TL_SEED, TL_STD = 128, 256, 0xA710, 0.02
DECODE_METRIC = "TinyLlama-arch Q8_0 decode tokens/s (batch 1, 128-token prompt, greedy)"
DECODE_CONFIG = {"workload": "tinyllama_1.1b_arch_decode_q8_0", "layers": 22, "hidden": 2048,
                 "ffn": 5632, "heads": "32q/4kv x 64", "vocab": 32000, "weights": "Q8_0",
                 "batch": 1, "prompt": TL_PROMPT, "new_tokens": TL_NEW,
                 "kv": "paged fp16, block 16",
                 "l2_policy": "weights 1.1 GB per step >> L2 (126 MB)"}


def decode_config(args, world: int) -> dict:
    return dict(DECODE_CONFIG, new_tokens=args.steps, parallelism=f"replicas x{world}")


def tl_prompt(rank: int = 0):
    import numpy as np
    return np.random.default_rng(1234 + rank).integers(0, TL["vocab"], TL_PROMPT).astype("int32")


def tl_kv_bytes(ctx: int) -> int:
    """K and V bytes one step reads at context length ctx (fp16 pages)."""
    return TL["n_layers"] * 2 * ctx * TL["n_kv_heads"] * TL["head_dim"] * 2


def run_decode_axion(args, d: Dist) -> dict:
    import torch
    from axion_b200 import ops
    from axion_b200.decoder import Decoder, DecoderConfig
    dev = torch.device("cuda", d.local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    K_new = args.steps
    cfg = DecoderConfig(**TL, max_batch=1, max_ctx=TL_PROMPT + max(K_new, args.warmup),
                        act_mode="q8")
    dec = Decoder(cfg)
    dec.init_random(TL_SEED, TL_STD)
    prompt = tl_prompt(d.rank)
    sp = stream.cuda_stream
    # warm-up: builds and instantiates the step graph, runs W decode steps
    dec.generate(prompt, args.warmup, stream=sp)
    torch.cuda.synchronize()
    clocks = ClockSampler(device_uuid(dev), period_ms=10).start()
    time.sleep(0.15)
    d.barrier()
    torch.cuda.synchronize()
    # timed: K greedy decode steps (device events inside axdec_generate)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    toks, _, decode_ms = dec.generate(prompt, K_new, stream=sp)
    e1.record(stream)
    torch.cuda.synchronize()
    d.barrier()
    clk = clocks.stop()
    call_ms = e0.elapsed_time(e1)          # the whole public call, host prompt in/tokens out
    ms_max = d.max(decode_ms)
    e2e_ms = d.max(call_ms)
    n_tok = d.sum(K_new) if d.world > 1 else K_new
    value = n_tok / (ms_max / 1e3)
    e2e_val = n_tok / (e2e_ms / 1e3)
    # roofline: the decode step is a weight stream; algorithmic bytes per step
    # = Q8_0 weights (34/32 B per weight, all linears + LM head) + KV read
    wbytes = dec.weight_bytes_per_step
    mean_kv = sum(tl_kv_bytes(TL_PROMPT + i) for i in range(K_new)) / K_new
    step_ms = ms_max / K_new
    achieved = (wbytes + mean_kv) / (step_ms / 1e3) / 1e9
    peaks, peak_kind = measured_peaks()
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                "traffic": ncu_traffic(DECODE_CONFIG["workload"]),
                "kernel": "decode step (q8_gemv_kernel dominant)", "step_us": round(step_ms * 1e3, 2),
                "algorithmic_bytes_per_step": int(wbytes + mean_kv), "peak_source": peak_kind}
    status = ops.status()
    dev_bytes = dec.device_bytes
    step_kernels = dec.step_kernels(1)
    dec.close()
    return {
        "metric": DECODE_METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": d.world,
        "steps": K_new, "warmup": args.warmup, "ms_per_step": round(step_ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 x int8 -> int32 -> fp32 (A8W8), fp16 KV",
        "data": "synthetic (device-generated Q8_0 weights N(0,0.02), norms 1.0; "
                "random prompt token ids)",
        "config": decode_config(args, d.world),
        "device_bytes": dev_bytes,
        "e2e": {"value": round(e2e_val, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": round(TL_PROMPT * 4 / K_new, 3),
                "d2h_bytes_per_step": 4,
                "path": "axdec_generate (C ABI): host prompt in, host tokens out, "
                        "batched prefill of the prompt included"},
        "roofline": roofline,
        "gpu_launches": step_kernels * K_new,
        "kernels_per_step": step_kernels,
        "clocks": clk,
        "device_status": status,
        "first_tokens": [int(t) for t in toks[0][:8]],
    }


def decode_reference(args, steps: int) -> dict:
    """ModelRunner::generate of the reference on a GGUF with the same weights
    (the oracle's generator reproduces the device weights bit for bit; the
    per-tensor seeds come from the library-free tensor_index), on the host
    cores.  Bounded sample: a 1-token prompt and `steps` new tokens, i.e.
    `steps` decode_step calls, each re-reading and dequantizing the 1.1 GB of
    Q8_0 weights as the reference does for every token (its prompt positions
    cost the same as generated ones), so the rate is tokens per second of
    decode_step."""
    import numpy as np
    from axion_b200.decoder import tensor_index
    from axion_b200.gguf import F32, Q8_0, GGUFWriter
    from oracle.oracle import Oracle, RefLib
    o, r = Oracle(), RefLib()
    H, F, V = TL["hidden"], TL["ffn"], TL["vocab"]
    hq = TL["n_heads"] * TL["head_dim"]
    hkv = TL["n_kv_heads"] * TL["head_dim"]
    g = GGUFWriter()
    g.add_string("general.architecture", "llama")
    for k, v in [("block_count", TL["n_layers"]), ("attention.head_count", TL["n_heads"]),
                 ("attention.head_count_kv", TL["n_kv_heads"]), ("embedding_length", H),
                 ("feed_forward_length", F), ("rope.dimension_count", TL["head_dim"]),
                 ("vocab_size", V)]:
        g.add_u32(f"llama.{k}", v)
    g.add_f32("llama.rope.freq_base", TL["rope_theta"])
    g.add_f32("llama.attention.layer_norm_rms_epsilon", TL["rms_eps"])

    def q8(name, N, K):
        seed = TL_SEED + tensor_index(TL["n_layers"], name)
        g.add_tensor(name, o.synth_q8_0(seed, N, K, TL_STD), (N, K), Q8_0)

    ones = np.ones(H, np.float32)
    q8("token_embd.weight", V, H)
    for i in range(TL["n_layers"]):
        p = f"blk.{i}."
        g.add_tensor(p + "attn_norm.weight", ones, (H,), F32)
        q8(p + "attn_q.weight", hq, H)
        q8(p + "attn_k.weight", hkv, H)
        q8(p + "attn_v.weight", hkv, H)
        q8(p + "attn_output.weight", H, hq)
        g.add_tensor(p + "ffn_norm.weight", ones, (H,), F32)
        q8(p + "ffn_gate.weight", F, H)
        q8(p + "ffn_up.weight", F, H)
        q8(p + "ffn_down.weight", H, F)
    g.add_tensor("output_norm.weight", ones, (H,), F32)
    q8("output.weight", V, H)
    tmp = Path(tempfile.mkdtemp()) / "tinyllama_arch_q8_0.gguf"
    g.write(tmp)
    del g
    prompt = tl_prompt(0)[:1]
    sec, toks = r.time_generate(tmp, prompt, steps)
    tmp.unlink()
    return {"value": round(steps / sec, 4), "unit": "tokens/s", "cores": host_cores(),
            "kind": "reference",
            "sample": f"ModelRunner::generate, 1-token prompt + {steps} new tokens ({steps} "
                      f"decode_step calls, each re-reading and dequantizing the 1.1 GB of Q8_0 "
                      f"weights), OpenMP threads={host_cores()}; tokens/s = {steps} / seconds",
            "seconds": round(sec, 3), "steps": steps, "step_seconds": round(sec / steps, 4)}


# ---------------------------------------------------------------------------
# Llama-3-8B-architecture batched decode (batch 64, 2048-token prompts), tensor parallel
# ---------------------------------------------------------------------------

L3 = dict(n_layers=32, hidden=4096, ffn=14336, n_heads=32, n_kv_heads=8, head_dim=128,
          vocab=128256, rope_theta=500000.0, rms_eps=1e-5)
L3_BATCH, L3_PROMPT, L3_NEW, L3_SEED = 64, 2048, 128, 0x8B
L3_METRIC = "Llama-3-8B-arch Q8_0 batched decode tokens/s (batch 64, 2048-token prompts, greedy)"
L3_CONFIG = {"workload": "llama3_8b_arch_decode_b64_tp", "layers": 32, "hidden": 4096,
             "ffn": 14336, "heads": "32q/8kv x 128", "vocab": 128256, "rope_theta": 500000.0,
             "weights": "Q8_0", "batch": L3_BATCH, "prompt": L3_PROMPT, "new_tokens": L3_NEW,
             "kv": "paged fp16, block 16",
             "l2_policy": "7.97 GB of weights + 17.7 GB of KV per step >> L2 (126 MB)"}
# Q8_0 weights one token streams: 32 layers x (Q, K, V, O, gate, up, down) + LM head
L3_LAYER_PARAMS = 4096 * 4096 * 2 + 2 * 1024 * 4096 + 3 * 14336 * 4096
L3_TOKEN_PARAMS = 32 * L3_LAYER_PARAMS + 128256 * 4096


def llama3_config(args, world: int) -> dict:
    return dict(L3_CONFIG, layers=args.layers or L3["n_layers"], prompt=args.prompt or L3_PROMPT,
                new_tokens=args.steps,
                parallelism=f"tp{world}")


def run_llama3_axion(args, d: Dist) -> dict:
    """One step = one greedy decode position of all 64 sequences; the job is
    tensor parallel over the N ranks (every rank holds 1/N of each layer's
    heads, FFN rows and LM-head vocabulary), so the whole job decodes 64
    tokens per step (strong scaling).  The 64 prompts are prefilled in one
    batched pass (timed apart, reported as `prefill`); then W warm-up and K
    timed steps through axdec_decode_step with pinned host tokens (`e2e`),
    then W + K steps continued on the device (`value`)."""
    import numpy as np
    import torch
    from axion_b200 import ops
    from axion_b200.decoder import Decoder, DecoderConfig
    dev = torch.device("cuda", d.local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    K_new, W, P = args.steps, args.warmup, args.prompt or L3_PROMPT
    arch = dict(L3, n_layers=args.layers or L3["n_layers"])
    cfg = DecoderConfig(**arch, max_batch=L3_BATCH, max_ctx=P + 2 * (W + K_new) + 1,
                        act_mode="q8", tp_size=d.world, tp_rank=d.rank)
    dec = Decoder(cfg)
    dec.init_random(L3_SEED, 0.02)
    dec.tp_connect()
    prompts = np.random.default_rng(99).integers(0, L3["vocab"], (L3_BATCH, P)).astype(np.int32)
    sp = stream.cuda_stream
    dec.generate(prompts[:, :8], W, stream=sp)      # step graph + prefill buffers + W steps
    torch.cuda.synchronize()
    d.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # batched prefill of positions 0 .. P - 2 of every prompt
    e0.record(stream)
    dec.prefill(prompts[:, :-1], stream=sp)
    e1.record(stream)
    torch.cuda.synchronize()
    prefill_ms = d.max(e0.elapsed_time(e1))
    # e2e: the public step call, host tokens in and out (pinned), every step
    tin = torch.empty(L3_BATCH, dtype=torch.int32, pin_memory=True)
    tout = torch.empty(L3_BATCH, dtype=torch.int32, pin_memory=True)
    tin.copy_(torch.from_numpy(prompts[:, -1].copy()))
    for _ in range(W):
        dec.decode_step_ptr(tin.data_ptr(), L3_BATCH, tout.data_ptr(), stream=sp)
        tin.copy_(tout)
    torch.cuda.synchronize()
    d.barrier()
    e0.record(stream)
    for _ in range(K_new):
        dec.decode_step_ptr(tin.data_ptr(), L3_BATCH, tout.data_ptr(), stream=sp)
        tin.copy_(tout)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = d.max(e0.elapsed_time(e1))
    # value: the same steps continued on the device, inputs resident
    dec.decode_continue(W, L3_BATCH, first=tin.numpy(), stream=sp)
    torch.cuda.synchronize()
    clocks = ClockSampler(device_uuid(dev), period_ms=20).start()
    time.sleep(0.15)
    d.barrier()
    torch.cuda.synchronize()
    toks, decode_ms = dec.decode_continue(K_new, L3_BATCH, stream=sp)
    torch.cuda.synchronize()
    d.barrier()
    clk = clocks.stop()
    ms_max = d.max(decode_ms)
    n_tok = L3_BATCH * K_new
    value = n_tok / (ms_max / 1e3)
    e2e_val = n_tok / (e2e_ms / 1e3)
    # roofline per rank: its weight slice + its KV heads read per step, at the
    # mean context of the timed steps
    wbytes = dec.weight_bytes_per_step
    kv_l = L3["n_kv_heads"] // d.world
    mean_ctx = P + 2 * W + K_new + (K_new - 1) / 2
    kv_bytes = arch["n_layers"] * 2 * mean_ctx * kv_l * L3["head_dim"] * 2 * L3_BATCH
    step_ms = ms_max / K_new
    achieved = (wbytes + kv_bytes) / (step_ms / 1e3) / 1e9
    peaks, peak_kind = measured_peaks()
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                "traffic": l3_traffic(arch["n_layers"], d.world, kv_bytes),
                "kernel": "decode step per rank (q8_mmq_kernel dominant)",
                "step_us": round(step_ms * 1e3, 1),
                "algorithmic_bytes_per_step_per_rank": int(wbytes + kv_bytes),
                "weight_bytes_per_step_per_rank": int(wbytes),
                "kv_bytes_per_step_per_rank": int(kv_bytes),
                "peak_source": peak_kind}
    status = ops.status()
    kernels = dec.step_kernels(L3_BATCH)
    dev_bytes = dec.device_bytes
    dec.close()
    pre_tok = L3_BATCH * (P - 1)
    return {
        "metric": L3_METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": d.world,
        "steps": K_new, "warmup": W, "ms_per_step": round(step_ms, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8 x int8 -> int32 -> fp32 (A8W8), fp16 KV",
        "data": "synthetic (device-generated Q8_0 weights N(0,0.02), norms 1.0; "
                "random prompt token ids)",
        "config": llama3_config(args, d.world),
        "tp": "column-split Q/K/V/gate/up, row-split O/down, vocabulary-split LM head; NCCL "
              "all-reduce of the hidden state after O and down, max all-reduce of the argmax keys",
        "device_bytes_per_rank": dev_bytes,
        "e2e": {"value": round(e2e_val, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": L3_BATCH * 4, "d2h_bytes_per_step": L3_BATCH * 4,
                "path": "axdec_decode_step (C ABI) per step: pinned host tokens in, H2D, step "
                        "graph, D2H of the next tokens, synchronize"},
        "prefill": {"tokens": pre_tok, "ms": round(prefill_ms, 1),
                    "tokens_per_s": round(pre_tok / (prefill_ms / 1e3), 1),
                    "path": "axdec_prefill: tcgen05 products over 4096-row chunks + causal "
                            "attention over the paged cache"},
        "roofline": roofline,
        "gpu_launches": kernels * K_new,
        "kernels_per_step": kernels,
        "clocks": clk,
        "device_status": status,
        "first_tokens": [int(t) for t in toks[0][:8]],
    }


def llama3_reference(args, steps: int) -> dict:
    """The reference decodes one sequence at a time (no batching:
    rope_apply_row_at takes one row, mha.cpp:208-211) and, per token,
    re-reads and dequantizes every weight before its M = 1 product
    (streaming_executor.cpp:299-307): its per-token cost is that of
    GGUFLoader::load_tensor + linear_from_gguf at M = 1 over all the weights.
    Each step times that on one [4096 x 4096] Q8_0 weight (host cores); the
    rate is extrapolated by weight count to a whole token (32 layers + LM
    head), attention excluded (which favours the reference)."""
    import numpy as np
    from axion_b200.gguf import Q8_0, GGUFWriter
    from oracle.oracle import Oracle, RefLib
    o, r = Oracle(), RefLib()
    tmp = Path(tempfile.mkdtemp()) / "l3.gguf"
    gw = GGUFWriter()
    gw.add_tensor("blk.0.attn_q.weight", o.synth_q8_0(L3_SEED, 4096, 4096), (4096, 4096), Q8_0)
    gw.write(tmp)
    x = np.random.default_rng(0).normal(0, 1, (1, 4096)).astype(np.float32)
    for _ in range(max(1, args.warmup)):
        r.time_linear(tmp, "blk.0.attn_q.weight", x, 4096, 1)
    secs = [r.time_linear(tmp, "blk.0.attn_q.weight", x, 4096, 1)[0] for _ in range(steps)]
    tmp.unlink()
    per_weight = statistics.mean(secs) / (4096 * 4096)
    token_s = per_weight * L3_TOKEN_PARAMS
    return {"value": round(1.0 / token_s, 5), "unit": "tokens/s", "cores": host_cores(),
            "kind": "reference", "extrapolated": True,
            "sample": f"each step: GGUFLoader::load_tensor + linear_from_gguf, [4096x4096] Q8_0, "
                      f"M=1 (OpenMP threads={host_cores()}, mean {statistics.mean(secs):.3f} s); "
                      f"tokens/s = 1 / (that time x {L3_TOKEN_PARAMS / 4096**2:.1f}, the weights "
                      f"one token streams / 4096^2), sequences one at a time",
            "seconds": round(sum(secs), 3), "steps": steps,
            "step_seconds": round(statistics.mean(secs), 4)}


# ---------------------------------------------------------------------------
# Decode-width products: the skinny Q8_0 x A8 kernel (q8_mmq_kernel) on the
# Llama-3-8B layer shapes of the batched-decode workload, M = 16 / 32 / 64
# ---------------------------------------------------------------------------

SKINNY_SHAPES = [(6144, 4096), (4096, 4096), (28672, 4096), (4096, 14336)]
SKINNY_MS = [16, 32, 64]
SKINNY_METRIC = "Q8_0 decode-width product HBM GB/s (Llama-3-8B layer shapes, M=16/32/64)"
SKINNY_CONFIG = {"workload": "q8_0_skinny_llama3_8b_layer_m16_32_64",
                 "shapes": "[6144x4096] [4096x4096] [28672x4096] [4096x14336]",
                 "M": SKINNY_MS}


def skinny_bytes(N: int, K: int, M: int) -> int:
    """Weights once (34-byte blocks), int8 activations + fp32 block scales, fp32 output."""
    return N * (K // 32) * 34 + M * K + M * (K // 32) * 4 + M * N * 4


def run_skinny_axion(args, d: Dist) -> dict:
    """One step = the 12 products (every shape at every M, M outer), each
    through axq8_linear_q8act_s (pre-quantized activations, the decode step's
    form).  Between two uses of one weight the other three stream 100-200 MB,
    more than L2, so every product reads its weight from HBM."""
    import torch
    from axion_b200 import _lib, ops
    lib = _lib.load()
    dev = torch.device("cuda", d.local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    s_ptr = C.c_void_p(stream.cuda_stream)
    g = torch.Generator(device=dev).manual_seed(77 + d.rank)
    with torch.cuda.stream(stream):
        ws = [ops.Q8Weight.synthetic(L3_SEED + i, N, K, device=dev)
              for i, (N, K) in enumerate(SKINNY_SHAPES)]
        acts = {}
        for M in SKINNY_MS:
            for K in sorted({k for _, k in SKINNY_SHAPES}):
                x = torch.randn(M, K, generator=g, device=dev)
                acts[(M, K)] = (x,) + tuple(ops.quantize_activations_t(x))
        ys = {(M, N): torch.empty(M, N, device=dev) for M in SKINNY_MS for N, _ in SKINNY_SHAPES}
    cases = [(M, i) for M in SKINNY_MS for i in range(len(SKINNY_SHAPES))]
    step_bytes = sum(skinny_bytes(*SKINNY_SHAPES[i], M) for M, i in cases)

    def product(M, i):
        N, K = SKINNY_SHAPES[i]
        _, xq, dxT = acts[(M, K)]
        _lib.check(lib.axq8_linear_q8act_s(ws[i].c, C.c_void_p(xq.data_ptr()),
                                           C.c_void_p(dxT.data_ptr()), M, None,
                                           C.c_void_p(ys[(M, N)].data_ptr()), s_ptr))

    K_steps, W_steps = args.steps, args.warmup
    for _ in range(W_steps):
        for M, i in cases:
            product(M, i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            for M, i in cases:
                product(M, i)
    graph.replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(device_uuid(dev)).start()
    time.sleep(0.15)
    d.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(K_steps):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    d.barrier()
    clk = clocks.stop()
    ms_max = d.max(e0.elapsed_time(e1))
    value = d.world * K_steps * step_bytes / (ms_max / 1e3) / 1e9

    # per-product device times (one event pair per product, same order)
    per = []
    with torch.cuda.stream(stream):
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(len(cases) + 1)]
        for rep in range(3):
            evs[0].record(stream)
            for j, (M, i) in enumerate(cases):
                product(M, i)
                evs[j + 1].record(stream)
            torch.cuda.synchronize()
            per.append([evs[j].elapsed_time(evs[j + 1]) for j in range(len(cases))])
    per_us = [min(r[j] for r in per) * 1e3 for j in range(len(cases))]
    # dominant launch: the largest weight at M = 64
    jd = cases.index((64, 2))
    alg = skinny_bytes(*SKINNY_SHAPES[2], 64)
    peaks, peak_kind = measured_peaks()
    achieved = alg / (per_us[jd] / 1e6) / 1e9
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                "traffic": ncu_traffic(SKINNY_CONFIG["workload"]),
                "kernel": "q8_mmq_kernel<8> [28672x4096] M=64", "kernel_us": round(per_us[jd], 2),
                "algorithmic_bytes": alg, "peak_source": peak_kind,
                "per_product_us": {f"M{M} [{SKINNY_SHAPES[i][0]}x{SKINNY_SHAPES[i][1]}]":
                                   round(per_us[j], 2) for j, (M, i) in enumerate(cases)}}

    # e2e: the public call (axq8_linear, fp32 activations, its own A8
    # quantization and dispatch) with pinned host input and output per product
    xh = {k: torch.empty(v[0].shape, dtype=torch.float32, pin_memory=True) for k, v in acts.items()}
    for k, v in acts.items():
        xh[k].copy_(v[0].cpu())
    yh = {k: torch.empty(v.shape, dtype=torch.float32, pin_memory=True) for k, v in ys.items()}
    xd = {k: torch.empty_like(v[0]) for k, v in acts.items()}
    h2d = sum(M * SKINNY_SHAPES[i][1] * 4 for M, i in cases)
    d2h = sum(M * SKINNY_SHAPES[i][0] * 4 for M, i in cases)

    def e2e_step():
        for M, i in cases:
            N, K = SKINNY_SHAPES[i]
            xd[(M, K)].copy_(xh[(M, K)], non_blocking=True)
            _lib.check(lib.axq8_linear(ws[i].c, C.c_void_p(xd[(M, K)].data_ptr()), M,
                                       C.c_void_p(ys[(M, N)].data_ptr()), _lib.AXQ8_ACT_Q8, s_ptr))
            yh[(M, N)].copy_(ys[(M, N)], non_blocking=True)

    with torch.cuda.stream(stream):
        for _ in range(W_steps):
            e2e_step()
        torch.cuda.synchronize()
        d.barrier()
        e0.record(stream)
        n_e2e = min(K_steps, 50)
        for _ in range(n_e2e):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
    e2e_ms = d.max(e0.elapsed_time(e1))
    e2e_val = d.world * n_e2e * step_bytes / (e2e_ms / 1e3) / 1e9
    return {
        "metric": SKINNY_METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": d.world,
        "steps": K_steps, "warmup": W_steps, "ms_per_step": round(ms_max / K_steps, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 x int8 -> int32 -> fp32 (mma.sync m16n8k32)",
        "data": "synthetic (device-generated Q8_0 weights N(0,0.02); x N(0,1))",
        "config": skinny_config(args, d.world),
        "e2e": {"value": round(e2e_val, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": n_e2e,
                "path": "axq8_linear (C ABI, A8, width dispatch) + pinned H2D/D2H per product"},
        "roofline": roofline,
        "gpu_launches": K_steps * len(cases),
        "clocks": clk,
        "device_status": ops.status(),
    }


def skinny_reference(args, rows: int) -> dict:
    """The reference's linear at a decode width: load_tensor + linear_from_gguf
    on one [4096 x 4096] Q8_0 weight at M = `rows`, host cores, as GB/s of the
    same algorithmic bytes."""
    import numpy as np
    from axion_b200.gguf import Q8_0, GGUFWriter
    from oracle.oracle import Oracle, RefLib
    o, r = Oracle(), RefLib()
    tmp = Path(tempfile.mkdtemp()) / "skinny.gguf"
    gw = GGUFWriter()
    gw.add_tensor("blk.0.attn_output.weight", o.synth_q8_0(L3_SEED + 1, 4096, 4096), (4096, 4096), Q8_0)
    gw.write(tmp)
    x = np.random.default_rng(0).normal(0, 1, (rows, 4096)).astype(np.float32)
    r.time_linear(tmp, "blk.0.attn_output.weight", x[:1], 4096, 1)
    sec, _ = r.time_linear(tmp, "blk.0.attn_output.weight", x, 4096, 1)
    tmp.unlink()
    val = skinny_bytes(4096, 4096, rows) / sec / 1e9
    return {"value": round(val, 4), "unit": "GB/s", "cores": host_cores(), "kind": "reference",
            "sample": f"GGUFLoader::load_tensor + linear_from_gguf, [4096x4096] Q8_0, M={rows}, "
                      f"OpenMP threads={host_cores()}",
            "seconds": round(sec, 3), "steps": 1}


# ---------------------------------------------------------------------------
# Prefill GEMM sweep: Llama-2-7B linear shapes on the
# tensor-core path
# ---------------------------------------------------------------------------

PREFILL_SHAPES = [(4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096)]
PREFILL_MS = [256, 1024, 2048, 4096]
PREFILL_METRIC = "Q8_0 prefill GEMM int8 TOPS (Llama-2-7B linear shapes x M sweep)"
PREFILL_CONFIG = {"workload": "q8_0_prefill_gemm_sweep_llama2_7b",
                  "shapes_NxK": [f"{n}x{k}" for n, k in PREFILL_SHAPES], "M": PREFILL_MS}


def run_prefill_axion(args, d: Dist) -> dict:
    """One step = one GEMM of the sweep (cases in rotation: 4 shapes x 4 M,
    253 MB of Q8_0 weights plus up to 180 MB of activations, so consecutive
    GEMMs never find their operands in L2).  value: sum of 2*M*N*K over the
    timed GEMMs / their summed device time through axq8_linear (activation
    quantization included).  roofline: the tcgen05 kernel alone
    (axq8_linear_q8act_t on pre-quantized activations) against the int8 dense
    peak taken as 2 x the measured bf16 GEMM peak (B200 int8:bf16 dense rate
    2:1)."""
    import torch
    from axion_b200 import _lib, ops
    lib = _lib.load()
    dev = torch.device("cuda", d.local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    s_ptr = C.c_void_p(stream.cuda_stream)
    cases = [(n, k, m) for (n, k) in PREFILL_SHAPES for m in PREFILL_MS]
    with torch.cuda.stream(stream):
        weights = {(n, k): ops.Q8Weight.synthetic(0xA710 + i, n, k, device=dev)
                   for i, (n, k) in enumerate(PREFILL_SHAPES)}
        g = torch.Generator(device=dev).manual_seed(7 + d.rank)
        xs = {k: torch.randn(max(PREFILL_MS), k, generator=g, device=dev)
              for k in {k for _, k in PREFILL_SHAPES}}
        ys = torch.empty(max(PREFILL_MS) * max(n for n, _ in PREFILL_SHAPES), device=dev)
    K_steps, W_steps = args.steps, args.warmup

    def gemm(i):
        n, k, m = cases[i % len(cases)]
        _lib.check(lib.axq8_linear(weights[(n, k)].c, C.c_void_p(xs[k].data_ptr()), m,
                                   C.c_void_p(ys.data_ptr()), _lib.AXQ8_ACT_Q8, s_ptr))
        return 2.0 * m * n * k

    # untimed set-up pass over every case: the library's workspaces reach their
    # final size here, not inside the timed region
    for i in range(len(cases)):
        gemm(i)
    for i in range(W_steps):
        gemm(i)
    torch.cuda.synchronize()
    clocks = ClockSampler(device_uuid(dev)).start()
    time.sleep(0.15)
    d.barrier()
    torch.cuda.synchronize()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(K_steps + 1)]
    ops_total = 0.0
    evs[0].record(stream)
    for i in range(K_steps):
        ops_total += gemm(W_steps + i)
        evs[i + 1].record(stream)
    torch.cuda.synchronize()
    d.barrier()
    clk = clocks.stop()
    per = [evs[i].elapsed_time(evs[i + 1]) for i in range(K_steps)]
    ms = d.max(sum(per))
    value = (d.sum(ops_total) if d.world > 1 else ops_total) / (ms / 1e3) / 1e12
    sweep = []
    for i in range(K_steps):
        n, k, m = cases[(W_steps + i) % len(cases)]
        sweep.append({"N": n, "K": k, "M": m, "us": round(per[i] * 1e3, 1),
                      "tops": round(2.0 * m * n * k / (per[i] / 1e3) / 1e12, 1)})

    # --- roofline: the tensor-core kernel alone on pre-quantized activations
    with torch.cuda.stream(stream):
        qa = {}
        for (n, k, m) in cases:
            if (k, m) not in qa:
                qa[(k, m)] = ops.quantize_activations_t(xs[k][:m])
    torch.cuda.synchronize()
    k_ops, k_ms = 0.0, 0.0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for (n, k, m) in cases:
        xq, dxT = qa[(k, m)]
        e0.record(stream)
        _lib.check(lib.axq8_linear_q8act_t(weights[(n, k)].c, C.c_void_p(xq.data_ptr()),
                                           C.c_void_p(dxT.data_ptr()), m, None,
                                           C.c_void_p(ys.data_ptr()), s_ptr))
        e1.record(stream)
        torch.cuda.synchronize()
        k_ms += e0.elapsed_time(e1)
        k_ops += 2.0 * m * n * k
    peaks, peak_kind = measured_peaks()
    int8_peak = 2.0 * peaks["bf16_tflops"]
    achieved = k_ops / (k_ms / 1e3) / 1e12
    roofline = {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(int8_peak, 1),
                "unit": "TOPS", "frac": round(achieved / int8_peak, 4),
                "traffic": ncu_traffic(PREFILL_CONFIG["workload"]),
                "kernel": "q8_mma_kernel (tcgen05.mma kind::i8)",
                "peak_source": f"2 x {peak_kind} bf16 GEMM peak (int8 dense rate = 2 x bf16)",
                "kernel_ms_sweep": round(k_ms, 3)}

    # --- e2e: the same GEMMs through axq8_linear from pinned host memory
    xh = {k: torch.empty(max(PREFILL_MS), k, pin_memory=True) for k in xs}
    for k in xs:
        xh[k].copy_(xs[k].cpu())
    yh = torch.empty(ys.numel(), pin_memory=True)
    xd = {k: torch.empty_like(xs[k]) for k in xs}
    h2d = d2h = 0
    e2e_ops = 0.0
    with torch.cuda.stream(stream):
        torch.cuda.synchronize()
        e0.record(stream)
        for i in range(K_steps):
            n, k, m = cases[(W_steps + i) % len(cases)]
            xd[k][:m].copy_(xh[k][:m], non_blocking=True)
            _lib.check(lib.axq8_linear(weights[(n, k)].c, C.c_void_p(xd[k].data_ptr()), m,
                                       C.c_void_p(ys.data_ptr()), _lib.AXQ8_ACT_Q8, s_ptr))
            yh[:m * n].copy_(ys[:m * n], non_blocking=True)
            h2d += m * k * 4
            d2h += m * n * 4
            e2e_ops += 2.0 * m * n * k
        e1.record(stream)
        torch.cuda.synchronize()
    e2e_ms = d.max(e0.elapsed_time(e1))
    e2e_val = (d.sum(e2e_ops) if d.world > 1 else e2e_ops) / (e2e_ms / 1e3) / 1e12
    return {
        "metric": PREFILL_METRIC, "value": round(value, 1), "unit": "TOPS", "n_gpus": d.world,
        "steps": K_steps, "warmup": W_steps, "ms_per_step": round(ms / K_steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 x int8 -> int32 (tcgen05 kind::i8) -> fp32 per-block rescale",
        "data": "synthetic (device-generated Q8_0 weights N(0,0.02); activations N(0,1))",
        "config": prefill_config(args, d.world),
        "e2e": {"value": round(e2e_val, 1), "unit": "TOPS", "h2d_bytes_per_step": h2d // K_steps,
                "d2h_bytes_per_step": d2h // K_steps,
                "path": "axq8_linear (C ABI), pinned H2D of x and D2H of y per GEMM"},
        "roofline": roofline,
        "gpu_launches": 2 * K_steps,
        "clocks": clk,
        "device_status": ops.status(),
        "sweep": sweep,
    }


def prefill_reference(args, steps: int) -> dict:
    """linear_from_gguf of the reference (load_tensor + fp32 GEMM) on the
    [4096 x 4096] shape with a bounded M (`steps` rows), host cores."""
    import numpy as np
    from axion_b200.gguf import Q8_0, GGUFWriter
    from oracle.oracle import Oracle, RefLib
    o, r = Oracle(), RefLib()
    tmp = Path(tempfile.mkdtemp()) / "prefill.gguf"
    gw = GGUFWriter()
    gw.add_tensor("blk.0.attn_q.weight", o.synth_q8_0(0xA710, 4096, 4096), (4096, 4096), Q8_0)
    gw.write(tmp)
    x = np.random.default_rng(0).normal(0, 1, (steps, 4096)).astype(np.float32)
    r.time_linear(tmp, "blk.0.attn_q.weight", x[:1], 4096, 1)
    sec, _ = r.time_linear(tmp, "blk.0.attn_q.weight", x, 4096, 1)
    tmp.unlink()
    ops_ = 2.0 * steps * 4096 * 4096
    return {"value": round(ops_ / sec / 1e12, 6), "unit": "TOPS", "cores": host_cores(),
            "kind": "reference",
            "sample": f"GGUFLoader::load_tensor + linear_from_gguf, [4096x4096] Q8_0, M={steps}, "
                      f"OpenMP threads={host_cores()}",
            "seconds": round(sec, 3), "steps": 1}


def gemv_config(args, world: int) -> dict:
    return {"workload": "q8_0_gemv_5632x2048_m1", "N": GEMV_N, "K": GEMV_K, "M": 1,
            "weights": "Q8_0", "parallelism": f"replicas x{world}"}


def prefill_config(args, world: int) -> dict:
    return dict(PREFILL_CONFIG, parallelism=f"replicas x{world}",
                l2_policy="cases in rotation, 253 MB of weights > L2")


def skinny_config(args, world: int) -> dict:
    return dict(SKINNY_CONFIG, parallelism=f"replicas x{world}",
                l2_policy="221 MB of weights per pass, each weight reused only after the other "
                          "three (> L2)")


WORKLOADS = {
    # name: (axion arm, reference arm, metric, config(args, n_gpus), default K,
    #        reference sample of the cpu_baseline leg, steps of the reference arm
    #        (None: K), scaling)
    "llama3": (run_llama3_axion, llama3_reference, L3_METRIC, llama3_config, L3_NEW, 8, None,
               "strong"),
    "decode": (run_decode_axion, decode_reference, DECODE_METRIC, decode_config, TL_NEW, 3, 24,
               "weak"),
    "gemv": (run_gemv_axion, gemv_reference, "Q8_0 GEMV HBM GB/s (algorithmic bytes)",
             gemv_config, 200000, 300, 300, "weak"),
    "prefill": (run_prefill_axion, prefill_reference, PREFILL_METRIC, prefill_config, 16, 64, 64,
                "weak"),
    "skinny": (run_skinny_axion, skinny_reference, SKINNY_METRIC, skinny_config, 20, 16, 16,
               "weak"),
}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["axion", "reference"], default="axion")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="llama3")
    ap.add_argument("--layers", type=int, default=None,
                    help="llama3 workload: decoder layers (default 32; fewer only for small "
                         "profiler captures, and the config says so)")
    ap.add_argument("--prompt", type=int, default=None,
                    help="llama3 workload: prompt length (default 2048)")
    ap.add_argument("--cpu-sample", type=int, default=None,
                    help="size of the reference sample timed for cpu_baseline")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    (run_axion, run_ref, metric, config_fn, k_default, sample_default, ref_steps,
     scaling) = WORKLOADS[args.workload]
    if args.steps is None:
        args.steps = k_default
    d = Dist(args.gpus)

    if args.impl == "reference":
        # rank 0 alone, on the host cores; loads no library of this repository
        if d.rank != 0:
            return 0
        use_all_host_cores()
        sample = args.cpu_sample or (ref_steps if ref_steps is not None else args.steps)
        cb = run_ref(args, sample)
        steps = cb.get("steps", sample)
        step_s = cb.get("step_seconds", cb["seconds"] / steps)
        out = {"impl": "reference", "metric": metric, "value": cb["value"], "unit": cb["unit"],
               "n_gpus": args.gpus, "steps": steps, "warmup": args.warmup,
               "ms_per_step": round(step_s * 1e3, 3),
               "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
               "dtype": "fp32 (the reference dequantizes Q8_0 to fp32)",
               "data": "synthetic (host-generated Q8_0 GGUF, same weights as the axion arm)",
               "config": config_fn(args, args.gpus),
               "reference_run": f"host OpenMP x{cb['cores']}, rank 0 only: {cb['sample']}",
               "extrapolated": bool(cb.get("extrapolated", False)),
               "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
               "e2e": {"value": cb["value"], "unit": cb["unit"], "h2d_bytes_per_step": 0,
                       "d2h_bytes_per_step": 0}}
        print(json.dumps(out))
        return 0

    d.init("nccl")
    res = run_axion(args, d)
    if d.rank == 0:
        try:
            use_all_host_cores()
            cb = run_ref(args, args.cpu_sample or sample_default)
            res["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
        except Exception as e:  # the reference library did not travel / build
            res["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
        print(json.dumps(res))
    d.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
