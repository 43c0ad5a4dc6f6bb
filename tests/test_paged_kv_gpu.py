"""Paged KV entry points (include/axkv.h) against the oracle.

PagedKVCache.append over caller-owned pages (ragged appends across page
boundaries, several sequences) must store every row (fp16-rounded on fp16
pages, exact on fp32 pages), and the decode attention over the pages must
equal the oracle's mha_attention_incremental restatement (pinned to the
reference by tests/test_oracle.py) on the same cached values.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3


@pytest.mark.parametrize("n_seq", [1, 3])       # 1: the scalar kernel, 3: the tensor-core one
# groups of 8 and 4 query heads take the transposed tensor-core kernel, 16 the
# one with a head per MMA row
@pytest.mark.parametrize("hd,n_heads,n_kv,fp32", [(64, 32, 4, False), (128, 32, 8, False),
                                                 (128, 16, 2, False), (128, 32, 2, False),
                                                 (128, 8, 2, True), (32, 4, 2, False)])
def test_append_and_decode_attention_vs_oracle(cuda, oracle, hd, n_heads, n_kv, fp32, n_seq):
    from axion_b200 import ops
    from axion_b200.paged_kv import PagedKVCache
    rng = np.random.default_rng(hd + n_heads)
    lens = [150, 17, 1][:n_seq]
    kv = PagedKVCache(n_kv, hd, max_seqs=n_seq, max_tokens=160, kv_fp32=fp32)
    kv.initialize(n_kv * hd, 16)
    ks, vs = [], []
    for s, n in enumerate(lens):
        k = rng.normal(0, 1, (n, n_kv * hd)).astype(np.float32)
        v = rng.normal(0, 1, (n, n_kv * hd)).astype(np.float32)
        ks.append(k)
        vs.append(v)
        cut = [0, n // 3, n // 3 + 1, n]          # ragged appends
        for a, b in zip(cut[:-1], cut[1:]):
            if b > a:
                kv.append(torch.from_numpy(k[a:b]).cuda(), torch.from_numpy(v[a:b]).cuda(), seq=s)
    q = rng.normal(0, 1, (n_seq, n_heads * hd)).astype(np.float32)
    out = kv.attention(torch.from_numpy(q).cuda(), n_heads).cpu().numpy()
    for s in range(n_seq):
        kr = ks[s] if fp32 else ks[s].astype(np.float16).astype(np.float32)
        vr = vs[s] if fp32 else vs[s].astype(np.float16).astype(np.float32)
        assert np.array_equal(kv.materialize_keys(s).cpu().numpy(), kr)
        assert np.array_equal(kv.materialize_values(s).cpu().numpy(), vr)
        ref = oracle.attention(q[s], kr, vr, n_heads, n_kv, hd)
        err = np.max(np.abs(out[s] - ref)) / np.max(np.abs(ref))
        print(f"hd {hd} G {n_heads // n_kv} n_seq {n_seq} seq {s} ({lens[s]} tokens): rel err {err:.2e}")
        assert err <= REL_TOL
    assert ops.status() == 0
    # a second call reuses the workspace (its counters were left at zero)
    out2 = kv.attention(torch.from_numpy(q).cuda(), n_heads).cpu().numpy()
    assert np.array_equal(out, out2)


def test_append_outside_the_table_is_reported(cuda):
    from axion_b200 import _lib, ops
    from axion_b200.paged_kv import PagedKVCache
    import ctypes as C
    kv = PagedKVCache(2, 64, max_seqs=1, max_tokens=32)
    lib = _lib.load()
    k = torch.zeros(1, 128, device="cuda")
    seq = torch.zeros(1, dtype=torch.int32, device="cuda")
    pos = torch.full((1,), 40, dtype=torch.int32, device="cuda")     # past max_blocks * 16
    ops.status_clear()
    _lib.check(lib.axkv_paged_append(C.byref(kv.c), C.c_void_p(k.data_ptr()),
                                     C.c_void_p(k.data_ptr()), 1, C.c_void_p(seq.data_ptr()),
                                     C.c_void_p(pos.data_ptr()), None))
    assert ops.status() == _lib.AXQ8_ERR_INVALID
    ops.status_clear()


@pytest.mark.parametrize("hd,n_heads,n_kv", [(64, 32, 4), (128, 32, 8), (128, 16, 2),
                                             (128, 8, 4), (64, 16, 16), (128, 16, 1)])
@pytest.mark.parametrize("T,p0", [(40, 0), (23, 23), (16, 70), (70, 20)])
def test_prefill_attention_vs_oracle(cuda, oracle, hd, n_heads, n_kv, T, p0):
    """Causal attention of a prompt chunk (axkv_paged_prefill_attn, the
    batched prefill's kernel with fp32 output): every position of the chunk
    against the oracle's attention over keys 0 .. position."""
    from axion_b200 import ops
    from axion_b200.paged_kv import PagedKVCache
    rng = np.random.default_rng(hd + n_heads + T + p0)
    n_seq, n = 2, p0 + T
    kv = PagedKVCache(n_kv, hd, max_seqs=n_seq, max_tokens=n + 16)
    ks = [rng.normal(0, 1, (n, n_kv * hd)).astype(np.float32) for _ in range(n_seq)]
    vs = [rng.normal(0, 1, (n, n_kv * hd)).astype(np.float32) for _ in range(n_seq)]
    for s in range(n_seq):
        kv.append(torch.from_numpy(ks[s]).cuda(), torch.from_numpy(vs[s]).cuda(), seq=s)
    q = rng.normal(0, 1, (n_seq * T, n_heads * hd)).astype(np.float32)
    out = kv.prefill_attention(torch.from_numpy(q).cuda(), n_heads, T, p0).cpu().numpy()
    worst = 0.0
    for s in range(n_seq):
        kr = ks[s].astype(np.float16).astype(np.float32)
        vr = vs[s].astype(np.float16).astype(np.float32)
        for t in range(T):
            p = p0 + t
            ref = oracle.attention(q[s * T + t], kr[:p + 1], vr[:p + 1], n_heads, n_kv, hd)
            worst = max(worst, float(np.max(np.abs(out[s * T + t] - ref)) / np.max(np.abs(ref))))
    print(f"prefill attention hd {hd} G {n_heads // n_kv} T {T} p0 {p0}: rel err {worst:.2e}")
    assert worst <= REL_TOL
    # the fused A8 output (the O projection's input) is the A8 quantization of
    # those same fp32 rows, bit for bit
    xq, dxT = kv.prefill_attention(torch.from_numpy(q).cuda(), n_heads, T, p0, quantize=True)
    oq, od = oracle.quantize_act(out)
    assert np.array_equal(xq.cpu().numpy(), oq)
    assert np.array_equal(dxT.cpu().numpy()[:, :n_seq * T], od.T)
    assert ops.status() == 0
