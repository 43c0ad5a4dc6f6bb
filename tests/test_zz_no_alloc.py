"""axq8_linear_noalloc, the A8 linear for callers that cannot allocate.

Callers that run under a fixed device-memory budget (an allocator owning all
of HBM) or that must not trigger the device synchronization a cudaMalloc can
cause use this entry point: its scratch is a fixed static device array, so it
allocates nothing.  This test calls it through the C ABI and checks it
against axq8_linear (A8 mode) and against the oracle's A8 linear on two calls
in a row — the second call reuses the array the first call left behind — at
widths that run the GEMV and the skinny product, plus the size limit.

Kept in a file of its own, named to be collected last; it must pass run alone
in a fresh process as well as after the other tests.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3          # the linear-path tolerance of tests/test_linear_gpu.py
MAX_MK = 1 << 20        # activation elements the fixed scratch holds


def _call_noalloc(lib, w, x: torch.Tensor, y: torch.Tensor) -> int:
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    return lib.axq8_linear_noalloc(w.c, C.c_void_p(x.data_ptr()), x.shape[0],
                                   C.c_void_p(y.data_ptr()), s)


@pytest.mark.parametrize("N,K,Ms", [
    (1500, 2048, (3, 1)),       # the GEMV, one and several 4-row passes
    (1500, 4096, (16, 64)),     # the skinny product (axq8_linear's kernel at these widths)
    (640, 4096, (80, 96)),      # above 64 rows: the GEMV here, tcgen05 in axq8_linear
])
def test_noalloc_matches_linear_two_calls(cuda, oracle, N, K, Ms):
    from axion_b200 import _lib, ops
    lib = _lib.load()
    rng = np.random.default_rng(21 + K + N)
    blocks = oracle.quantize_weight_blocks(rng.normal(0, 0.02, (N, K)).astype(np.float32))
    w = ops.Q8Weight.from_blocks(blocks, N, K)
    wd = w.dequantize().cpu().numpy().astype(np.float64)
    # two different inputs in a row: the second call must not see the first's data
    for call, M in enumerate(Ms):
        x = torch.from_numpy(rng.normal(0, 1, (M, K)).astype(np.float32)).cuda()
        y = torch.full((M, N), float("nan"), device="cuda")
        _lib.check(_call_noalloc(lib, w, x, y))
        got = y.cpu().numpy()
        xn = x.cpu().numpy()
        scale = np.abs(xn.astype(np.float64)) @ np.abs(wd).T
        # against the existing entry point (axq8_linear, A8) ...
        ref = ops.linear_from_gguf(x, w, act_mode="q8").cpu().numpy().astype(np.float64)
        assert rel_err(got, ref, scale) <= REL_TOL, (call, M)
        # ... and against the oracle's A8 linear on the same quantized input
        xq, dx = oracle.quantize_act(xn)
        want = oracle.linear_a8(blocks, N, K, xq, dx).astype(np.float64)
        assert rel_err(got, want, scale) <= REL_TOL, (call, M)
    assert ops.status() == 0


def test_noalloc_rejects_oversize(cuda, oracle):
    from axion_b200 import _lib, ops
    lib = _lib.load()
    K = 4096
    blocks = oracle.quantize_weight_blocks(np.zeros((2, K), np.float32))
    w = ops.Q8Weight.from_blocks(blocks, 2, K)
    M = MAX_MK // K + 1
    x = torch.zeros(M, K, device="cuda")
    y = torch.zeros(M, 2, device="cuda")
    rc = _call_noalloc(lib, w, x, y)
    assert rc == _lib.AXQ8_ERR_INVALID
    assert b"exceeds" in lib.axq8_last_error()
    # the largest accepted size still runs
    M = MAX_MK // K
    x = torch.zeros(M, K, device="cuda")
    y = torch.ones(M, 2, device="cuda")
    _lib.check(_call_noalloc(lib, w, x, y))
    torch.cuda.synchronize()
    assert torch.count_nonzero(y).item() == 0
