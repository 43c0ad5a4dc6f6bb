#!/usr/bin/env python
"""Benchmark of the B200 Q8_0 hot path; prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl axion|reference]
                    [--workload gemv]

Workloads
  gemv   Q8_0 GEMV, TinyLlama ffn_up shape: W [5632 x 2048] Q8_0 (random init,
         N(0, 0.02) before quantization), x [1 x 2048] fp32 N(0, 1) quantized on
         the fly, y [5632] fp32.  One step = one linear_from_gguf call.  The
         weight rotates over enough copies (> 4 x L2) that every step streams
         its weight from HBM.  Metric: algorithmic bytes / s (W 34/32 B per
         weight + x + y = 12,285,952 B per step).

Arms
  --impl axion      the CUDA path (libaxq8.so) on N GPUs, one process per GPU
                    (torchrun for N > 1; each rank runs its own replica: the
                    GEMV does not shard, scaling "weak").
  --impl reference  the reference's own CPU implementation (oracle/_ref,
                    built from its sources) on the host cores, rank 0 only.

Timing: W untimed warm-up steps, then K steps between barrier +
cudaDeviceSynchronize, CUDA events on the launching stream, max over ranks.
`e2e` is the same metric through the public C-ABI entry point with host
(pinned) buffers, H2D of x and D2H of y inside the timed region.
`roofline` is the GEMV kernel alone (pre-quantized activation, CUDA events
over back-to-back launches) against the measured HBM copy bandwidth.
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
        "config": {"workload": "q8_0_gemv_5632x2048_m1", "N": GEMV_N, "K": GEMV_K, "M": 1,
                   "act": "q8", "l2_policy": f"rotating {n_copies} weight copies "
                   f"({n_copies * wbytes / 2**20:.0f} MiB > 4 x L2)",
                   "parallelism": f"replicas x{d.world}"},
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

WORKLOADS = {"gemv": (run_gemv_axion, gemv_reference)}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["axion", "reference"], default="axion")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="gemv")
    ap.add_argument("--cpu-sample", type=int, default=None,
                    help="reference calls timed for cpu_baseline")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    run_axion, run_ref = WORKLOADS[args.workload]
    d = Dist(args.gpus)

    if args.impl == "reference":
        if d.rank != 0:
            return 0
        steps = args.steps or 30
        cb = run_ref(args, steps)
        out = {"impl": "reference", "metric": "Q8_0 GEMV HBM GB/s (algorithmic bytes)",
               "value": cb["value"], "unit": cb["unit"], "n_gpus": args.gpus, "steps": steps,
               "warmup": args.warmup, "ms_per_step": round(cb["seconds"] * 1e3 / steps, 3),
               "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
               "dtype": "fp32 (reference dequantizes Q8_0 to fp32)",
               "data": "synthetic (host-generated Q8_0 GGUF, same recipe)",
               "config": {"workload": "q8_0_gemv_5632x2048_m1", "N": GEMV_N, "K": GEMV_K,
                          "M": 1, "parallelism": "host OpenMP"},
               "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
               "e2e": {"value": cb["value"], "unit": cb["unit"], "h2d_bytes_per_step": 0,
                       "d2h_bytes_per_step": 0}}
        print(json.dumps(out))
        return 0

    if args.steps is None:
        args.steps = 200000
    d.init("nccl")
    res = run_axion(args, d)
    if d.rank == 0:
        sample = args.cpu_sample or 300
        try:
            res["cpu_baseline"] = {k: v for k, v in run_ref(args, sample).items()
                                   if k != "seconds"}
        except Exception as e:  # the reference library did not travel / build
            res["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
        print(json.dumps(res))
    d.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
