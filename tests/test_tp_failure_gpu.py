"""Bounded waits of the NVLink all-reduce (include/axtp.h), on one GPU.

A group of two ranks whose second rank never runs: this rank's kernel
announces its partial and waits for the other rank's announcement, which
nothing writes.  The wait gives up after its bound (about two seconds), the
device status word reads AXQ8_ERR_WAIT_TIMEOUT and the device stays usable.
No GPU fault, trap or hang is involved: the missing peer is a flag that
nothing sets.
"""
from __future__ import annotations

import ctypes as C
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_missing_peer_times_out_with_status(cuda):
    from axion_b200 import _lib, ops
    lib = _lib.load()
    n = 4096
    part = [torch.randn(n, device="cuda"), torch.zeros(n, device="cuda")]
    out = [torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")]
    flags = [torch.zeros(16, dtype=torch.int32, device="cuda") for _ in range(2)]
    epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
    ctas = torch.zeros(1, dtype=torch.int32, device="cuda")
    # axtp_group_t: part[8], out[8], flags[8], epoch, ctas_done, rank, world
    buf = C.create_string_buffer(8 * 26 + 8)
    ptrs = [t.data_ptr() for t in part] + [0] * 6 + [t.data_ptr() for t in out] + [0] * 6 + \
        [t.data_ptr() for t in flags] + [0] * 6 + [epoch.data_ptr(), ctas.data_ptr()]
    C.memmove(buf, (C.c_uint64 * len(ptrs))(*ptrs), 8 * len(ptrs))
    C.memmove(C.addressof(buf) + 8 * len(ptrs), (C.c_int32 * 2)(0, 2), 8)
    ops.status_clear()
    torch.cuda.synchronize()
    t0 = time.time()
    _lib.check(lib.axtp_allreduce_sum(C.cast(buf, C.c_void_p), n, None))
    torch.cuda.synchronize()
    dt = time.time() - t0
    print(f"missing peer: kernel returned after {dt:.2f} s")
    assert ops.status() == _lib.AXQ8_ERR_WAIT_TIMEOUT
    assert dt < 30
    ops.status_clear()
    # the device still works
    assert int((torch.ones(n, device="cuda") * 3).sum().item()) == 3 * n
    # bad groups are refused on the host
    C.memmove(C.addressof(buf) + 8 * len(ptrs), (C.c_int32 * 2)(2, 2), 8)
    assert lib.axtp_allreduce_sum(C.cast(buf, C.c_void_p), n, None) == _lib.AXQ8_ERR_INVALID
