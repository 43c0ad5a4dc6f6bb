"""Parity of the CUDA Q8_0 linear path with the oracle and the reference's
golden outputs (all calls go through the C ABI of libaxq8.so).

Tolerances: integer/byte results (repack, dequantized values, activation
quantization, int32 block dots, synthetic weights, per-tensor quantized
matmul) are bit-exact.  fp32 linear outputs differ from the reference only by
summation order; the contract is a relative error <= 1e-3 normalised by
sum_k |x_k * w_k| (REL_TOL), and the measured error is ~1e-6.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden, rel_err

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _ops():
    from axion_b200 import ops
    return ops


def _scale(x: np.ndarray, wdeq: np.ndarray) -> np.ndarray:
    return np.abs(x.astype(np.float64)) @ np.abs(wdeq.astype(np.float64)).T


def _weight(oracle, N, K, seed=0, std=0.02):
    rng = np.random.default_rng(seed)
    blocks = oracle.quantize_weight_blocks(rng.normal(0, std, (N, K)).astype(np.float32))
    return blocks, _ops().Q8Weight.from_blocks(blocks, N, K)


def test_repack_round_trip(cuda, oracle):
    for (N, K) in [(1, 32), (7, 96), (33, 2048), (5, 5632)]:
        blocks, w = _weight(oracle, N, K, seed=N)
        torch.cuda.synchronize()
        assert np.array_equal(w.blocks_host(), blocks)


def test_dequantize_matches_reference(cuda):
    g = golden("linear_cases.npz")
    ops = _ops()
    for i in range(int(g["n"])):
        if f"c{i}_wdeq" not in g:
            continue
        M, N, K = (int(v) for v in g[f"c{i}_shape"])
        w = ops.Q8Weight.from_blocks(g[f"c{i}_blocks"], N, K)
        assert np.array_equal(bits(w.dequantize().cpu().numpy()), bits(g[f"c{i}_wdeq"])), i


def test_known_answer_block(cuda):
    ka = golden("q8_known_answer.npz")
    w = _ops().Q8Weight.from_blocks(ka["block"], 1, 32)
    vals = w.dequantize().cpu().numpy().reshape(-1)
    assert np.array_equal(bits(vals), bits(ka["values"]))


def test_quantize_act_bit_exact(cuda, oracle):
    rng = np.random.default_rng(5)
    x = rng.normal(0, 1, (5, 2048)).astype(np.float32)
    x[0, :32] = 0.0
    x[1, 64:96] = 1e-30
    x[2, 128:160] *= 1e6
    x[3, 0:32] = np.linspace(-1, 1, 32)         # exact halves after scaling
    xq, dx = _ops().quantize_activations(torch.from_numpy(x).cuda())
    oq, od = oracle.quantize_act(x)
    assert np.array_equal(xq.cpu().numpy(), oq)
    assert np.array_equal(bits(dx.cpu().numpy()), bits(od))


def test_block_dots_bit_exact(cuda, oracle):
    for (M, N, K) in [(1, 3, 32), (2, 17, 256), (3, 64, 2048)]:
        blocks, w = _weight(oracle, N, K, seed=K)
        x = np.random.default_rng(M).normal(0, 1, (M, K)).astype(np.float32)
        oq, _ = oracle.quantize_act(x)
        d = _ops().block_dots(w, torch.from_numpy(oq).cuda()).cpu().numpy()
        assert np.array_equal(d, oracle.block_dots(blocks, N, K, oq)), (M, N, K)


def test_linear_f32_matches_reference_golden(cuda):
    """A32 mode against the reference's linear_from_gguf outputs."""
    g = golden("linear_cases.npz")
    ops = _ops()
    for i in range(int(g["n"])):
        M, N, K = (int(v) for v in g[f"c{i}_shape"])
        w = ops.Q8Weight.from_blocks(g[f"c{i}_blocks"], N, K)
        x = g[f"c{i}_x"]
        y = ops.linear_from_gguf(torch.from_numpy(x).cuda(), w, act_mode="f32").cpu().numpy()
        wd = w.dequantize().cpu().numpy()
        assert rel_err(y, g[f"c{i}_y"], _scale(x, wd)) <= REL_TOL, (i, M, N, K)


def test_linear_q8_matches_reference_on_quantized_input(cuda, oracle, ):
    """A8 mode equals the reference's linear_from_gguf applied to the
    dequantized Q8 activation x' = q_x * d_x (only summation order differs)."""
    g = golden("linear_cases.npz")
    ops = _ops()
    for i in range(int(g["n"])):
        M, N, K = (int(v) for v in g[f"c{i}_shape"])
        w = ops.Q8Weight.from_blocks(g[f"c{i}_blocks"], N, K)
        x = g[f"c{i}_x"]
        y = ops.linear_from_gguf(torch.from_numpy(x).cuda(), w, act_mode="q8").cpu().numpy()
        oq, od = oracle.quantize_act(x)
        xd = (oq.reshape(M, K // 32, 32) * od[:, :, None]).reshape(M, K).astype(np.float32)
        wd = w.dequantize().cpu().numpy()
        ref = oracle.linear_f32(xd, wd)         # == reference linear_from_gguf bit for bit
        assert rel_err(y, ref, _scale(xd, wd)) <= REL_TOL, (i, M, N, K)
        a8 = oracle.linear_a8(g[f"c{i}_blocks"], N, K, oq, od)
        assert rel_err(y, a8, _scale(xd, wd)) <= REL_TOL


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8, 9, 16, 33, 64])
def test_linear_batch_sizes(cuda, oracle, M):
    N, K = 257, 1024
    blocks, w = _weight(oracle, N, K, seed=M)
    x = np.random.default_rng(100 + M).normal(0, 1, (M, K)).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    wd = w.dequantize().cpu().numpy()
    for mode in ("q8", "f32"):
        y = _ops().linear_from_gguf(xt, w, act_mode=mode).cpu().numpy()
        if mode == "q8":
            oq, od = oracle.quantize_act(x)
            ref = oracle.linear_a8(blocks, N, K, oq, od)
        else:
            ref = oracle.linear_a32(x, blocks, N)
        assert rel_err(y, ref, _scale(x, wd)) <= REL_TOL, mode


@pytest.mark.parametrize("N,K", [(1, 32), (2, 28672), (3, 14336), (1000, 64), (5632, 2048)])
def test_linear_edge_shapes(cuda, oracle, N, K):
    blocks, w = _weight(oracle, N, K, seed=N + K)
    x = np.random.default_rng(7).normal(0, 1, (1, K)).astype(np.float32)
    y = _ops().linear_from_gguf(torch.from_numpy(x).cuda(), w).cpu().numpy()
    oq, od = oracle.quantize_act(x)
    ref = oracle.linear_a8(blocks, N, K, oq, od)
    wd = oracle.dequant(blocks, N * K).reshape(N, K)
    assert rel_err(y, ref, _scale(x, wd)) <= REL_TOL


def test_q8act_with_residual(cuda, oracle):
    N, K, M = 300, 512, 2
    blocks, w = _weight(oracle, N, K)
    x = np.random.default_rng(1).normal(0, 1, (M, K)).astype(np.float32)
    r = np.random.default_rng(2).normal(0, 1, (M, N)).astype(np.float32)
    oq, od = oracle.quantize_act(x)
    y = _ops().linear_q8act(w, torch.from_numpy(oq).cuda(), torch.from_numpy(od).cuda(),
                            residual=torch.from_numpy(r).cuda()).cpu().numpy()
    ref = oracle.linear_a8(blocks, N, K, oq, od) + r
    assert np.allclose(y, ref, rtol=1e-5, atol=1e-5)


def test_full_size_gemv_and_linearity(cuda, oracle):
    """TinyLlama ffn_up shape [5632 x 2048] with device-generated weights:
    oracle agreement plus exact homogeneity y(2x) == 2 y(x) (A8 scales by
    powers of two exactly)."""
    ops = _ops()
    N, K = 5632, 2048
    w = ops.Q8Weight.synthetic(0xA710, N, K)
    x = torch.randn(1, K, generator=torch.Generator().manual_seed(0)).cuda()
    y1 = ops.linear_from_gguf(x, w)
    y2 = ops.linear_from_gguf(2 * x, w)
    assert torch.equal(y2, 2 * y1)
    blocks = w.blocks_host()
    xn = x.cpu().numpy()
    oq, od = oracle.quantize_act(xn)
    ref = oracle.linear_a8(blocks, N, K, oq, od)
    wd = oracle.dequant(blocks, N * K).reshape(N, K)
    assert rel_err(y1.cpu().numpy(), ref, _scale(xn, wd)) <= REL_TOL


def test_synth_weights_bit_exact(cuda, oracle):
    ops = _ops()
    for (N, K, seed) in [(3, 64, 1), (40, 2048, 0xA710)]:
        dev = ops.synth_q8_0_blocks(seed, N, K).cpu().numpy()
        host = oracle.synth_q8_0(seed, N, K)
        assert np.array_equal(dev, host)
        w = ops.Q8Weight.synthetic(seed, N, K)
        assert np.array_equal(w.blocks_host(), host)


def test_quantized_matmul_matches_reference(cuda):
    g = golden("quantized_matmul.npz")
    ops = _ops()
    for i in range(int(g["n"])):
        W = ops.quantize_weight(torch.from_numpy(g[f"c{i}_w"]).cuda(), ops.QuantType.Q8_0)
        assert np.array_equal(W.q8.cpu().numpy(), g[f"c{i}_q"])
        assert np.float32(W.scale) == g[f"c{i}_scale"]
        y = ops.quantized_matmul(torch.from_numpy(g[f"c{i}_x"]).cuda(), W).cpu().numpy()
        assert np.array_equal(bits(y), bits(g[f"c{i}_y"])), i
        # runtime_validation.cpp:527-528: the Q8 payload is 4x smaller than FP32
        assert W.payload_bytes() * 4 == g[f"c{i}_w"].size * 4


def test_error_behaviour(cuda, oracle):
    ops = _ops()
    _, w = _weight(oracle, 8, 64)
    with pytest.raises(RuntimeError, match="dimension mismatch"):
        ops.linear_from_gguf(torch.zeros(1, 32, device="cuda"), w)
    with pytest.raises(RuntimeError, match="expects 2D"):
        ops.linear_from_gguf(torch.zeros(64, device="cuda"), w)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        ops.linear_from_gguf(torch.zeros(1, 64), w)
    with pytest.raises(RuntimeError):
        ops.Q8Weight.from_blocks(np.zeros(33, np.uint8), 1, 32)
    y = ops.linear_from_gguf(torch.zeros(0, 64, device="cuda"), w)
    assert y.shape == (0, 8)


def test_no_wait_timeouts_recorded(cuda):
    torch.cuda.synchronize()
    assert _ops().status() == 0
