"""Batched prefill (axdec_prefill / axdec_generate) and step-wise decoding.

The prompt runs as wide products over chunks of (sequence, position) rows and
a causal GQA attention kernel over the paged fp16 cache, in place of the
reference's one-position-at-a-time prompt loop (ModelRunner::generate,
inference/cpp/runtime/model_runner.cpp:291-295; the whole-sequence form is
StreamingExecutor::execute_layer + mha_attention, streaming_executor.cpp:110-238,
mha.cpp:167-198).  Checked against:

* the same model with the prompt fed through the decode step (set_prefill(False));
* the oracle's sequential A8 decode with fp16 KV (oracle/model.py), which
  regenerates the device weights bit for bit;
* generate() versus prefill() + decode_step() (the step-wise public API).

Head dims 64 (TinyLlama shape, 8 query heads per kv head) and 128 (Llama-3
shape, 4 per kv head), several sequences, prompts spanning several chunks.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3
A8_TOL = 5e-2       # A8 decode tolerance of tests/test_decode_gpu.py (quantization flips)


def _rel(a, b) -> float:
    a = a.reshape(a.shape[0], -1).astype(np.float64)
    b = b.reshape(b.shape[0], -1).astype(np.float64)
    return float(np.max(np.max(np.abs(a - b), axis=1) / np.max(np.abs(b), axis=1)))


def _top1_consistent(lg, ref, tol) -> bool:
    for a, r in zip(lg.reshape(lg.shape[0], -1), ref.reshape(ref.shape[0], -1)):
        ia, ir = int(np.argmax(a)), int(np.argmax(r))
        if ia != ir and abs(r[ia] - r[ir]) > tol * np.max(np.abs(r)):
            return False
    return True


ARCH = {
    # name: (hidden, ffn, n_heads, n_kv, head_dim, vocab)
    "hd64": (2048, 5632, 32, 4, 64, 32000),      # TinyLlama widths
    "hd128": (1024, 2048, 8, 2, 128, 4096),      # Llama-3 head shape (GQA 4)
}
SEED = 0x5EED


def _decoder(arch, n_layers=2, **kw):
    from axion_b200.decoder import Decoder, DecoderConfig
    H, F, nh, nkv, hd, V = ARCH[arch]
    cfg = DecoderConfig(n_layers=n_layers, hidden=H, ffn=F, n_heads=nh, n_kv_heads=nkv,
                        head_dim=hd, vocab=V, rope_theta=10000.0, rms_eps=1e-5, **kw)
    d = Decoder(cfg)
    d.init_random(SEED, std=0.02)
    return d


def _oracle_model(d, oracle):
    from oracle.model import LlamaConfig, OracleLlama
    c = d.cfg
    H, F, nq, nkv = c.hidden, c.ffn, c.n_heads * c.head_dim, c.n_kv_heads * c.head_dim
    shapes = {"attn_q": (nq, H), "attn_k": (nkv, H), "attn_v": (nkv, H), "attn_output": (H, nq),
              "ffn_gate": (F, H), "ffn_up": (F, H), "ffn_down": (H, F)}
    t = {}
    for n in ["token_embd.weight", "output.weight"]:
        t[n] = ("q8", oracle.synth_q8_0(SEED + d.tensor_index(n), c.vocab, H, 0.02), c.vocab, H)
    for i in range(c.n_layers):
        for k, (N, K) in shapes.items():
            n = f"blk.{i}.{k}.weight"
            t[n] = ("q8", oracle.synth_q8_0(SEED + d.tensor_index(n), N, K, 0.02), N, K)
        t[f"blk.{i}.attn_norm.weight"] = ("f32", np.ones(H, np.float32))
        t[f"blk.{i}.ffn_norm.weight"] = ("f32", np.ones(H, np.float32))
    t["output_norm.weight"] = ("f32", np.ones(H, np.float32))
    return OracleLlama(LlamaConfig(c.n_layers, H, c.n_heads, c.n_kv_heads, c.head_dim, F, c.vocab,
                                   c.rope_theta, c.rms_eps), t, oracle)


@pytest.mark.parametrize("arch,n_seq,n_prompt", [("hd64", 2, 40), ("hd128", 3, 37)])
def test_prefill_matches_stepwise_and_oracle(cuda, oracle, arch, n_seq, n_prompt):
    from axion_b200 import ops
    d = _decoder(arch, max_batch=n_seq, max_ctx=64)
    assert d.prefill_batched(n_seq)
    prompts = np.random.default_rng(4).integers(0, d.cfg.vocab, (n_seq, n_prompt)).astype(np.int32)
    toks, lg, _ = d.generate(prompts, 4, logits=True)
    d.set_prefill(False)
    assert not d.prefill_batched(n_seq)
    toks_s, lg_s, _ = d.generate(prompts, 4, logits=True)
    assert ops.status() == 0
    for b in range(n_seq):
        # the first generated step's logits come straight from the prefilled cache
        assert _rel(lg[:1, b, :], lg_s[:1, b, :]) <= A8_TOL
        assert _top1_consistent(lg[:, b, :], lg_s[:, b, :], A8_TOL)
    # the oracle, teacher-forced with the device's tokens (one prompt each)
    om = _oracle_model(d, oracle)
    for b in range(n_seq):
        o_lg, _ = om.decode(prompts[b].tolist(), 4, act="q8", kv="f16",
                            forced=toks[b][:-1].tolist())
        err = _rel(lg[:, b, :], o_lg)
        print(f"{arch} seq {b}: prefill+decode vs oracle rel err {err:.2e}")
        assert err <= A8_TOL
        assert _top1_consistent(lg[:, b, :], o_lg, A8_TOL)
    d.close()


def test_prefill_chunks_match_single_chunk(cuda, monkeypatch):
    """Prompt split over many chunks (chunk boundaries inside pages and
    across them) equals one chunk: K/V of earlier chunks are read back from
    the pages by the causal attention."""
    from axion_b200 import ops
    prompts = np.random.default_rng(6).integers(0, 4096, (2, 90)).astype(np.int32)
    d = _decoder("hd128", max_batch=2, max_ctx=128)
    one, lg1, _ = d.generate(prompts, 3, logits=True)
    monkeypatch.setenv("AXDEC_PREFILL_ROWS", "46")      # 23 positions per chunk
    many, lgm, _ = d.generate(prompts, 3, logits=True)
    monkeypatch.setenv("AXDEC_PREFILL_ROWS", "14")      # 7 positions: the skinny product
    few, lgf, _ = d.generate(prompts, 3, logits=True)
    assert ops.status() == 0
    for b in range(2):
        assert _rel(lgm[:, b, :], lg1[:, b, :]) <= A8_TOL
        assert _rel(lgf[:, b, :], lg1[:, b, :]) <= A8_TOL
        assert _top1_consistent(lgm[:, b, :], lg1[:, b, :], A8_TOL)
    d.close()


def test_prefill_then_decode_steps_equal_generate(cuda):
    """prefill(prompt[:, :-1]) then decode_step from the last prompt token
    reproduces generate() token for token and logit for logit."""
    d = _decoder("hd64", max_batch=4, max_ctx=64)
    prompts = np.random.default_rng(5).integers(0, 32000, (4, 21)).astype(np.int32)
    toks, lg, _ = d.generate(prompts, 5, logits=True)
    d.prefill(prompts[:, :-1])
    cur = prompts[:, -1].copy()
    for i in range(5):
        cur, l = d.decode_step(cur, logits=True)
        assert cur.tolist() == toks[:, i].tolist()
        assert np.array_equal(l, lg[i])
    # the device-side continuation: first 2 steps from the host, 3 fed back
    d.prefill(prompts[:, :-1])
    first = d.decode_step(prompts[:, -1])
    cont, ms = d.decode_continue(4, 4, first=first)
    assert np.array_equal(cont, toks[:, 1:5]) and ms > 0
    d.close()


def test_decode_step_needs_a_session(cuda):
    from axion_b200._lib import AxionCudaError
    d = _decoder("hd64", max_batch=2, max_ctx=32)
    with pytest.raises(AxionCudaError):
        d.decode_step(np.array([1, 2], np.int32))
    d.prefill(np.array([[1, 2, 3], [4, 5, 6]], np.int32))
    with pytest.raises(AxionCudaError):
        d.decode_step(np.array([1], np.int32))          # the session has 2 sequences
    d.decode_step(np.array([7, 8], np.int32))
    d.generate(np.array([[1, 2, 3]], np.int32), 1)       # ends the session
    with pytest.raises(AxionCudaError):
        d.decode_step(np.array([1, 2], np.int32))
    d.close()
