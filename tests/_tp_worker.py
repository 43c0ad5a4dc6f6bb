"""Child-process bodies of the tensor-parallel tests (one process per rank).

Each worker joins a torch.distributed group (gloo on 127.0.0.1, used only to
pass the NCCL id), builds its rank's slice of the model, connects the
decoder's own NCCL communicator and writes its results to `out_dir`.
"""
from __future__ import annotations

import os
from pathlib import Path

import numpy as np


def _init(rank: int, world: int, port: int, use_cuda: bool):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    if use_cuda:
        torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    return dist


def id_exchange(rank: int, world: int, port: int, out_dir: str) -> None:
    """CPU only: rank 0's id reaches every rank unchanged."""
    dist = _init(rank, world, port, use_cuda=False)
    from axion_b200.decoder import share_tp_id
    uid = share_tp_id(rank, lambda: bytes(range(128)), None)
    Path(out_dir, f"id{rank}.bin").write_bytes(uid)
    dist.destroy_process_group()


def _allreduce(ar: str) -> None:
    """Which hidden-state all-reduce the decoder connects with (nvlink | nccl)."""
    os.environ["AXDEC_TP_AR"] = ar


def tiny_gguf(rank: int, world: int, port: int, out_dir: str, gguf: str, act: str, kv32: bool,
              prompt: list, n_new: int, ar: str = "nvlink") -> None:
    dist = _init(rank, world, port, use_cuda=True)
    from axion_b200.decoder import Decoder
    _allreduce(ar)
    d = Decoder.from_gguf(gguf, act_mode=act, kv_fp32=kv32, max_ctx=32, tp_size=world,
                          tp_rank=rank)
    d.tp_connect()
    Path(out_dir, f"ar{rank}.txt").write_text(d.tp_allreduce)
    toks, lg, _ = d.generate(prompt, n_new, logits=True)
    np.save(Path(out_dir, f"tok{rank}.npy"), toks)
    np.save(Path(out_dir, f"lg{rank}.npy"), lg)
    d.close()
    dist.barrier()
    dist.destroy_process_group()


def synthetic(rank: int, world: int, port: int, out_dir: str, cfg_kw: dict, seed: int,
              prompts, n_new: int, ar: str = "nvlink") -> None:
    dist = _init(rank, world, port, use_cuda=True)
    from axion_b200.decoder import Decoder, DecoderConfig
    _allreduce(ar)
    d = Decoder(DecoderConfig(tp_size=world, tp_rank=rank, **cfg_kw))
    d.init_random(seed, std=0.02)
    d.tp_connect()
    Path(out_dir, f"ar{rank}.txt").write_text(d.tp_allreduce)
    toks, lg, _ = d.generate(np.asarray(prompts, np.int32), n_new, logits=True)
    np.save(Path(out_dir, f"tok{rank}.npy"), toks)
    np.save(Path(out_dir, f"lg{rank}.npy"), lg)
    d.close()
    dist.barrier()
    dist.destroy_process_group()


class _FakeDecoder:
    """Stands in for Decoder in the host-only failure test: records aborts."""

    def __init__(self):
        self.aborted = False

    def tp_abort(self):
        self.aborted = True

    def tp_health(self):
        return 0, 0


def heartbeat_failure(rank: int, world: int, port: int, out_dir: str, steps_before_exit: int,
                      timeout: float) -> None:
    """CPU only (gloo): rank 1 leaves after a few steps without a word; rank 0
    must notice through the stale heartbeat before its next step and abort."""
    import time
    dist = _init(rank, world, port, use_cuda=False)
    from axion_b200.tp_watchdog import Heartbeat, PeerFailure, guarded_step
    store = dist.distributed_c10d._get_default_store()
    hb = Heartbeat(store, rank, world, timeout=timeout)
    dec = _FakeDecoder()
    for _ in range(steps_before_exit):
        guarded_step(dec, hb, lambda: None)
        time.sleep(0.05)
    dist.barrier()          # both ranks finished the healthy steps
    if rank == 1:
        Path(out_dir, "left1.txt").write_text("left")
        return              # leaves between steps, no collective in flight
    t0 = time.time()
    outcome = "no failure seen"
    while time.time() - t0 < 10 * timeout:
        try:
            guarded_step(dec, hb, lambda: None)
        except PeerFailure as e:
            outcome = f"peer failure {e.ranks} after {time.time() - t0:.2f} s, aborted {dec.aborted}"
            break
        time.sleep(0.05)
    Path(out_dir, "outcome0.txt").write_text(outcome)
