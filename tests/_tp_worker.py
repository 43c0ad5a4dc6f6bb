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


def tiny_gguf(rank: int, world: int, port: int, out_dir: str, gguf: str, act: str, kv32: bool,
              prompt: list, n_new: int) -> None:
    dist = _init(rank, world, port, use_cuda=True)
    from axion_b200.decoder import Decoder
    d = Decoder.from_gguf(gguf, act_mode=act, kv_fp32=kv32, max_ctx=32, tp_size=world,
                          tp_rank=rank)
    d.tp_connect()
    toks, lg, _ = d.generate(prompt, n_new, logits=True)
    np.save(Path(out_dir, f"tok{rank}.npy"), toks)
    np.save(Path(out_dir, f"lg{rank}.npy"), lg)
    d.close()
    dist.barrier()
    dist.destroy_process_group()


def synthetic(rank: int, world: int, port: int, out_dir: str, cfg_kw: dict, seed: int,
              prompts, n_new: int) -> None:
    dist = _init(rank, world, port, use_cuda=True)
    from axion_b200.decoder import Decoder, DecoderConfig
    d = Decoder(DecoderConfig(tp_size=world, tp_rank=rank, **cfg_kw))
    d.init_random(seed, std=0.02)
    d.tp_connect()
    toks, lg, _ = d.generate(np.asarray(prompts, np.int32), n_new, logits=True)
    np.save(Path(out_dir, f"tok{rank}.npy"), toks)
    np.save(Path(out_dir, f"lg{rank}.npy"), lg)
    d.close()
    dist.barrier()
    dist.destroy_process_group()
