"""axq8_linear_noalloc, the A8 linear for callers that cannot allocate.

Callers that run under a fixed device-memory budget (an allocator owning all
of HBM) or that must not trigger the device synchronization a cudaMalloc can
cause use this entry point: its scratch is a fixed static device array, so it
allocates nothing.  This test calls it through the C ABI and checks it
against axq8_linear (A8 mode) on two calls in a row — the second call reuses
the array the first call left behind — plus the size limit.

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


def test_noalloc_matches_linear_two_calls(cuda, oracle):
    from axion_b200 import _lib, ops
    lib = _lib.load()
    N, K = 1500, 2048
    rng = np.random.default_rng(21)
    blocks = oracle.quantize_weight_blocks(rng.normal(0, 0.02, (N, K)).astype(np.float32))
    w = ops.Q8Weight.from_blocks(blocks, N, K)
    wd = w.dequantize().cpu().numpy().astype(np.float64)
    # two different inputs in a row: the second call must not see the first's data
    for call, M in enumerate((3, 1)):
        x = torch.from_numpy(rng.normal(0, 1, (M, K)).astype(np.float32)).cuda()
        y = torch.full((M, N), float("nan"), device="cuda")
        _lib.check(_call_noalloc(lib, w, x, y))
        ref = ops.linear_from_gguf(x, w, act_mode="q8")
        xn = x.cpu().numpy()
        scale = np.abs(xn.astype(np.float64)) @ np.abs(wd).T
        assert rel_err(y.cpu().numpy(), ref.cpu().numpy().astype(np.float64), scale) <= REL_TOL, call
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
