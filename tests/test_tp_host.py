"""Host-side logic of tensor-parallel decoding, without a GPU: configuration
validation (before any device work) and the communicator-id exchange over
two gloo ranks on 127.0.0.1."""
from __future__ import annotations

import ctypes
import socket

import pytest


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_create_rejects_bad_tp_configs():
    from axion_b200 import _lib
    from axion_b200.decoder import DecoderConfig
    lib = _lib.load()
    base = dict(n_layers=1, hidden=128, ffn=256, n_heads=4, n_kv_heads=2, head_dim=32, vocab=96)
    h = ctypes.c_void_p()
    for kw, what in [(dict(tp_size=2, tp_rank=2), b"tp_rank"),
                     (dict(tp_size=4, tp_rank=0), b"tp_size"),       # n_kv_heads 2
                     (dict(tp_size=2, tp_rank=0, vocab=97), b"tp_size"),
                     (dict(tp_size=3, tp_rank=0, n_kv_heads=3, n_heads=3, head_dim=32), b"tp_size")]:
        cfg = DecoderConfig(**{**base, **kw}).c()
        rc = lib.axdec_create(ctypes.byref(cfg), ctypes.byref(h))
        assert rc == _lib.AXQ8_ERR_INVALID, kw
        assert what in lib.axq8_last_error(), (kw, lib.axq8_last_error())


def test_connect_and_id_need_valid_arguments():
    from axion_b200 import _lib
    lib = _lib.load()
    assert lib.axdec_tp_connect(None, None) == _lib.AXQ8_ERR_INVALID
    buf = (ctypes.c_ubyte * 16)()
    assert lib.axdec_tp_unique_id(ctypes.cast(buf, ctypes.c_void_p), 16) == _lib.AXQ8_ERR_INVALID


def test_id_exchange_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp
    import _tp_worker
    mp.spawn(_tp_worker.id_exchange, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    ids = [(tmp_path / f"id{r}.bin").read_bytes() for r in range(2)]
    assert ids[0] == ids[1] == bytes(range(128))


def test_peer_that_leaves_is_detected_before_the_next_step(tmp_path):
    """Two gloo ranks exchange heartbeats between steps; rank 1 leaves
    without a word, rank 0 sees its heartbeat go stale before its next step,
    aborts the (fake) communicator and stops."""
    import torch.multiprocessing as mp
    import _tp_worker
    mp.spawn(_tp_worker.heartbeat_failure, args=(2, _port(), str(tmp_path), 5, 0.5), nprocs=2,
             join=True)
    outcome = (tmp_path / "outcome0.txt").read_text()
    assert outcome.startswith("peer failure [1]") and outcome.endswith("aborted True"), outcome
    assert (tmp_path / "left1.txt").exists()


def test_heartbeat_marks_a_silent_peer():
    from axion_b200.tp_watchdog import Heartbeat
    import time
    import torch.distributed as dist
    store = dist.HashStore()
    a = Heartbeat(store, 0, 2, timeout=0.2)
    b = Heartbeat(store, 1, 2, timeout=0.2)
    a.beat()
    b.beat()
    assert a.dead_peers() == [] and b.dead_peers() == []
    time.sleep(0.3)
    a.beat()
    assert a.dead_peers() == [1]        # rank 1 stopped beating
    assert b.dead_peers() == []         # rank 0 is fresh
