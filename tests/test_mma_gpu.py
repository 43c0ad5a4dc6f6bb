"""Parity of the tensor-core Q8_0 x A8 product (tcgen05 kind::i8, the
prefill / batched-decode path of axq8_linear) with the oracle.

* Activation quantization with transposed scales: bit-exact with the oracle.
* int32 block dots read back from TMEM: bit-exact with the oracle's
  sum_i qw*qx per (m, n, block) (the reference's Q8_0 bytes, gguf.cpp:870-882).
* fp32 outputs: against the oracle's A8 linear (same block dots, fp32
  combination in another order), error normalised by sum_k |x'_k w_k|
  <= 1e-5; against linear_from_gguf's arithmetic (linear.cpp:27-71) on the
  dequantized activation x' <= 1e-3 (REL_TOL).
* Shapes cover ragged M and N tiles, every BN (32/64/128), split-K, and
  deterministic results across calls.
* The skinny decode-width product (mma.sync, M <= 64) to the same bar.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3
A8_COMBINE_TOL = 1e-5

# (N, K, M): BN 32 / 64 / 128, ragged tiles, split-K (few tiles, long K)
SHAPES = [
    (128, 128, 32),
    (200, 1024, 100),
    (256, 512, 64),
    (384, 2048, 129),
    (1024, 4096, 33),
    (4096, 4096, 64),
    (512, 1024, 1000),
]


def _ops():
    from axion_b200 import ops
    return ops


def _case(oracle, N, K, M, seed):
    rng = np.random.default_rng(seed)
    blocks = oracle.quantize_weight_blocks(rng.normal(0, 0.02, (N, K)).astype(np.float32))
    x = rng.normal(0, 1, (M, K)).astype(np.float32)
    w = _ops().Q8Weight.from_blocks(blocks, N, K)
    return blocks, x, w


def _xdeq(xq: np.ndarray, dx: np.ndarray) -> np.ndarray:
    M, K = xq.shape
    return (xq.reshape(M, K // 32, 32).astype(np.float32) * dx[:, :, None]).reshape(M, K)


def test_quantize_act_t_bit_exact(cuda, oracle):
    ops = _ops()
    rng = np.random.default_rng(1)
    for M, K in [(33, 256), (64, 2048), (130, 4096)]:
        x = rng.normal(0, 1, (M, K)).astype(np.float32)
        x[0, :32] = 0.0
        xq, dxT = ops.quantize_activations_t(torch.from_numpy(x).cuda())
        oq, od = oracle.quantize_act(x)
        assert dxT.shape == (K // 32, ops.scale_pitch(M))
        assert np.array_equal(xq.cpu().numpy(), oq)
        assert np.array_equal(dxT.cpu().numpy()[:, :M].view(np.uint32), od.T.view(np.uint32))


@pytest.mark.parametrize("N,K,M", [(128, 128, 32), (200, 1024, 100), (384, 512, 129), (256, 256, 520)])
def test_tensor_core_block_dots_bit_exact(cuda, oracle, N, K, M):
    ops = _ops()
    blocks, x, w = _case(oracle, N, K, M, seed=N + M)
    xq, dxT = ops.quantize_activations_t(torch.from_numpy(x).cuda())
    dots, y = ops.block_dots_tc(w, xq, dxT)
    ref = oracle.block_dots(blocks, N, K, xq.cpu().numpy())
    assert np.array_equal(dots.cpu().numpy(), ref)
    assert ops.status() == 0


@pytest.mark.parametrize("N,K,M", SHAPES)
def test_tensor_core_linear_vs_oracle(cuda, oracle, N, K, M):
    ops = _ops()
    blocks, x, w = _case(oracle, N, K, M, seed=7 * N + M)
    xt = torch.from_numpy(x).cuda()
    assert ops.linear_path(w, M) == ("skinny" if M <= 64 else "tensor_core")
    xq, dxT = ops.quantize_activations_t(xt)
    y = ops.linear_q8act_t(w, xq, dxT).cpu().numpy()      # the tcgen05 product at every M
    oq, od = oracle.quantize_act(x)
    ref = oracle.linear_a8(blocks, N, K, oq, od)
    xd = _xdeq(oq, od)
    wdeq = oracle.dequant(blocks, N * K).reshape(N, K)
    scale = np.abs(xd.astype(np.float64)) @ np.abs(wdeq.astype(np.float64)).T
    err = rel_err(y, ref.astype(np.float64), scale)
    print(f"[{N}x{K}] M={M}: A8 combine err vs oracle {err:.2e}")
    assert err <= A8_COMBINE_TOL
    # the reference's fp32 arithmetic on the same (dequantized) activation
    ref32 = oracle.linear_f32(xd, wdeq)
    assert rel_err(y, ref32.astype(np.float64), scale) <= REL_TOL
    assert ops.status() == 0


@pytest.mark.parametrize("M", [65, 300])
def test_tensor_core_entry_points_agree(cuda, oracle, M):
    """axq8_linear (A8, M > 64) == axq8_linear_q8act_t bit for bit; the
    residual is one fp32 add; repeated calls (split-K) are deterministic."""
    ops = _ops()
    N, K = 1024, 4096
    blocks, x, w = _case(oracle, N, K, M, seed=3)
    xt = torch.from_numpy(x).cuda()
    y1 = ops.linear_from_gguf(xt, w)
    xq, dxT = ops.quantize_activations_t(xt)
    y2 = ops.linear_q8act_t(w, xq, dxT)
    y3 = ops.linear_q8act_t(w, xq, dxT)
    assert torch.equal(y1, y2) and torch.equal(y2, y3)
    res = torch.randn(M, N, device="cuda")
    y4 = ops.linear_q8act_t(w, xq, dxT, residual=res)
    assert torch.equal(y4, res + y2)
    assert ops.status() == 0


# (N, K, M): one 8-row tile to all eight, ragged 16-row tiles, split-K over
# CTAs (few tiles, long K) and over the warps only
SKINNY = [(200, 1024, 1), (257, 512, 5), (1000, 4096, 9), (768, 4096, 16), (4096, 512, 31),
          (2048, 5632, 33), (128, 14336, 64), (6144, 4096, 64)]


@pytest.mark.parametrize("N,K,M", SKINNY)
def test_skinny_product_vs_oracle(cuda, oracle, N, K, M):
    """The decode-width product (mma.sync m16n8k32, register accumulators):
    against the oracle's A8 linear within the combination tolerance, equal to
    axq8_linear for 8 < M <= 64, deterministic, residual = one fp32 add."""
    ops = _ops()
    blocks, x, w = _case(oracle, N, K, M, seed=11 * N + M)
    xt = torch.from_numpy(x).cuda()
    xq, dxT = ops.quantize_activations_t(xt)
    y = ops.linear_q8act_s(w, xq, dxT)
    assert torch.equal(y, ops.linear_q8act_s(w, xq, dxT))
    oq, od = oracle.quantize_act(x)
    ref = oracle.linear_a8(blocks, N, K, oq, od)
    xd = _xdeq(oq, od)
    wdeq = oracle.dequant(blocks, N * K).reshape(N, K)
    scale = np.abs(xd.astype(np.float64)) @ np.abs(wdeq.astype(np.float64)).T
    err = rel_err(y.cpu().numpy(), ref.astype(np.float64), scale)
    print(f"skinny [{N}x{K}] M={M}: err vs oracle {err:.2e}")
    assert err <= A8_COMBINE_TOL
    if ops.linear_path(w, M) == "skinny":
        assert torch.equal(ops.linear_from_gguf(xt, w), y)
    res = torch.randn(M, N, device="cuda")
    assert torch.equal(ops.linear_q8act_s(w, xq, dxT, residual=res), res + y)
    assert ops.status() == 0


def test_dispatch_by_width(cuda, oracle):
    ops = _ops()
    _, _, w = _case(oracle, 256, 256, 1, seed=0)
    assert ops.linear_path(w, 1) == "gemv"
    assert ops.linear_path(w, 8) == "gemv"
    assert ops.linear_path(w, 9) == "skinny"
    assert ops.linear_path(w, 32) == "skinny"
    assert ops.linear_path(w, 64) == "skinny"
    assert ops.linear_path(w, 65) == "tensor_core"
    assert ops.linear_path(w, 64, "f32") == "gemv"
    _, _, w2 = _case(oracle, 64, 256, 1, seed=0)
    assert ops.linear_path(w2, 256) == "gemv"        # N < 128
    assert ops.linear_path(w2, 40) == "skinny"       # any N


# The prefill sweep's Llama-2-7B linear shapes at M = 256 and 2048: the
# product through axq8_linear (A8, tcgen05 at these widths) on sampled output
# rows against the oracle's A8 linear and the reference's fp32 arithmetic.
SWEEP = [(4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096)]


@pytest.mark.parametrize("M", [256, 2048])
@pytest.mark.parametrize("N,K", SWEEP)
def test_prefill_sweep_shapes_vs_oracle(cuda, oracle, N, K, M):
    ops = _ops()
    blocks = oracle.synth_q8_0(0xA710 + N + K, N, K, 0.02)
    w = ops.Q8Weight.from_blocks(blocks, N, K)
    rng = np.random.default_rng(N + M)
    x = rng.normal(0, 1, (M, K)).astype(np.float32)
    assert ops.linear_path(w, M) == "tensor_core"
    y = ops.linear_from_gguf(torch.from_numpy(x).cuda(), w).cpu().numpy()
    rows = np.sort(rng.choice(M, 6, replace=False))
    rows[0], rows[-1] = 0, M - 1             # first and last tile rows always
    oq, od = oracle.quantize_act(x[rows])
    ref = oracle.linear_a8(blocks, N, K, oq, od)
    xd = _xdeq(oq, od)
    wdeq = oracle.dequant(blocks, N * K).reshape(N, K)
    scale = np.abs(xd.astype(np.float64)) @ np.abs(wdeq.astype(np.float64)).T
    err = rel_err(y[rows], ref.astype(np.float64), scale)
    print(f"sweep [{N}x{K}] M={M}: rows {rows.tolist()} err vs oracle {err:.2e}")
    assert err <= A8_COMBINE_TOL
    assert rel_err(y[rows], oracle.linear_f32(xd, wdeq).astype(np.float64), scale) <= REL_TOL
    assert np.isfinite(y).all()
    assert ops.status() == 0
