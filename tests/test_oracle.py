"""Pin the C restatement (oracle/q8_oracle.c) to the reference.

Against the committed golden vectors (made by running the reference itself,
tests/golden/make_golden.py) everywhere, and against the reference library
directly when it is built in this checkout.  The fp32 functions must agree
bit for bit: same operations, same order, same rounding.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import golden


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_fp16_table_matches_reference(oracle):
    table = golden("fp16_table.npy")
    mine = np.array([oracle.fp16_to_fp32(h) for h in range(65536)], np.float32)
    assert np.array_equal(bits(mine), table)


def test_known_answer_block(oracle):
    ka = golden("q8_known_answer.npz")
    vals = oracle.dequant(ka["block"], 32)
    assert np.array_equal(bits(vals), bits(ka["values"]))
    # runtime_validation.cpp:848-852 expectation: (i-16)*0.5
    assert np.allclose(vals, (np.arange(32) - 16) * 0.5, atol=1e-3)


def test_q8_0_byte_size(oracle):
    assert oracle.q8_0_byte_size(32) == 34
    assert oracle.q8_0_byte_size(5632 * 2048) == 12_255_232


def test_linear_cases_bit_exact(oracle):
    g = golden("linear_cases.npz")
    for i in range(int(g["n"])):
        M, N, K = (int(v) for v in g[f"c{i}_shape"])
        blocks, x = g[f"c{i}_blocks"], g[f"c{i}_x"]
        if f"c{i}_wdeq" in g:
            assert np.array_equal(bits(oracle.dequant(blocks, N * K)),
                                  bits(g[f"c{i}_wdeq"].reshape(-1))), i
        y = oracle.linear_a32(x, blocks, N)
        assert np.array_equal(bits(y), bits(g[f"c{i}_y"])), (i, M, N, K)


def test_ops_bit_exact(oracle):
    g = golden("ops_cases.npz")
    assert np.array_equal(bits(oracle.rmsnorm(g["rms_x"], g["rms_w"], 1e-5)), bits(g["rms_y"]))
    assert np.array_equal(bits(oracle.rope_row(g["rope_x"], 8, 64, 10000.0, 77)),
                          bits(g["rope_y"]))
    att = oracle.attention(g["att_q"], g["att_k"], g["att_v"], 8, 2, 64)
    assert np.array_equal(bits(att), bits(g["att_y"]))
    assert np.array_equal(bits(oracle.silu_mul(g["silu_g"], g["silu_u"])), bits(g["silu_y"]))


def test_tiny_llama_decode_bit_exact(oracle):
    """The oracle's full incremental decode reproduces the reference's logits
    and greedy tokens bit for bit (fp32 contiguous KV, A32 arithmetic)."""
    from oracle.model import OracleLlama
    ref = golden("tiny_llama_ref.npz")
    m = OracleLlama.from_gguf(golden("tiny_llama.gguf"), oracle)
    prompt = ref["prompt"].tolist()
    n_new = len(ref["tokens"]) - len(prompt)
    logits, toks = m.decode(prompt, n_new, act="f32", kv="f32")
    assert toks == ref["tokens"][len(prompt):].tolist()
    assert np.array_equal(bits(logits), bits(ref["logits"]))


def test_quantize_act_convention(oracle):
    rng = np.random.default_rng(3)
    x = rng.normal(0, 1, (3, 128)).astype(np.float32)
    x[1, 32:64] = 0.0                       # an all-zero block: d = 0, q = 0
    x[2, 0] = 2.5 * (x[2, :32].max() or 1)  # a block dominated by one value
    q, d = oracle.quantize_act(x)
    assert q.dtype == np.int8 and d.shape == (3, 4)
    assert np.all(q[1, 32:64] == 0) and d[1, 1] == 0.0
    assert np.abs(q).max() <= 127
    # reconstruction error bounded by half a quantization step
    xr = q.reshape(3, 4, 32) * d[:, :, None]
    assert np.all(np.abs(xr - x.reshape(3, 4, 32)) <= d[:, :, None] * 0.5 + 1e-7)


def test_block_dots_and_a8_consistency(oracle):
    rng = np.random.default_rng(4)
    N, K, M = 9, 96, 2
    blocks = oracle.quantize_weight_blocks(rng.normal(0, 0.02, (N, K)).astype(np.float32))
    xq, dx = oracle.quantize_act(rng.normal(0, 1, (M, K)).astype(np.float32))
    dots = oracle.block_dots(blocks, N, K, xq)
    qw = blocks.reshape(N, K // 32, 34)[:, :, 2:].view(np.int8).astype(np.int64)
    ref_dots = np.einsum("nbi,mbi->mnb", qw, xq.reshape(M, K // 32, 32).astype(np.int64))
    assert np.array_equal(dots, ref_dots)
    y = oracle.linear_a8(blocks, N, K, xq, dx)
    dw = blocks.reshape(N, K // 32, 34)[:, :, :2].copy().view(np.float16)[:, :, 0].astype(np.float64)
    y64 = np.einsum("nb,mb,mnb->mn", dw, dx.astype(np.float64), dots.astype(np.float64))
    assert np.allclose(y, y64, rtol=1e-5, atol=1e-6)


def test_synth_generator_statistics(oracle):
    v = oracle.gen_normal(0xA710, 1 << 20, std=0.02)
    assert abs(v.mean()) < 1e-4 and abs(v.std() - 0.02) < 2e-4
    assert np.abs(v).max() <= 6 * 0.02 + 1e-6      # Irwin-Hall(12) support


def test_oracle_vs_reference_live(oracle, reflib):
    """Direct comparison with the reference library on fresh random inputs."""
    rng = np.random.default_rng(11)
    for (M, N, K) in [(1, 17, 64), (3, 40, 320), (2, 5, 32)]:
        w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
        blocks = oracle.quantize_weight_blocks(w)
        wd = oracle.dequant(blocks, N * K).reshape(N, K)
        x = rng.normal(0, 1, (M, K)).astype(np.float32)
        assert np.array_equal(bits(reflib.linear_from_gguf(x, wd)),
                              bits(oracle.linear_a32(x, blocks, N)))


def test_reference_runtime_validation_passes():
    """The reference's own known-answer harness, built from its sources."""
    import subprocess
    from oracle.oracle import REF_VALIDATION
    if not REF_VALIDATION.exists():
        pytest.skip("reference harness not built here")
    r = subprocess.run([str(REF_VALIDATION)], capture_output=True, text=True,
                       cwd=str(REF_VALIDATION.parent))
    assert r.returncode == 0, r.stdout[-2000:]
    assert "AXION RUNTIME VALIDATION PASSED (0 failures)" in r.stdout
