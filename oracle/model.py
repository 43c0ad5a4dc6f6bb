"""Oracle of the whole incremental decode (test infrastructure only).

Composes the C restatement's operators in the order of the reference's
decode path, so that with fp32 activations and an fp32 contiguous KV cache
it reproduces the reference's logits bit for bit:

* ModelRunner::generate            inference/cpp/runtime/model_runner.cpp:245-317
* StreamingExecutor::decode_step   inference/cpp/runtime/streaming_executor.cpp:403-420
* StreamingExecutor::decode_layer  inference/cpp/runtime/streaming_executor.cpp:268-401
* logits_from_hidden_row           inference/cpp/runtime/model_runner.cpp:237-243
* compute_logits / argmax          inference/cpp/runtime/logits.cpp:11-79

Two switches select the device path's numerics instead:
``act="q8"`` quantizes every linear's input to Q8 blocks (the A8 convention of
q8_oracle.h), ``kv="f16"`` stores K/V rounded to fp16 (the paged cache).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .oracle import Q8_0_BYTES, QK, Oracle


@dataclass
class LlamaConfig:
    n_layers: int
    hidden: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    rope_theta: float = 10000.0
    rms_eps: float = 1e-5


class OracleLlama:
    def __init__(self, cfg: LlamaConfig, tensors: dict, o: Oracle):
        self.cfg = cfg
        self.t = tensors          # name -> ("q8", blocks, N, K) | ("f32", array)
        self.o = o

    @classmethod
    def from_gguf(cls, path, o: Oracle | None = None) -> "OracleLlama":
        from axion_b200.gguf import F32, Q8_0, GGUFLoader
        o = o or Oracle()
        g = GGUFLoader()
        g.load_file(path)
        a = g.architecture() or "llama"
        n_heads = g.get_u32(f"{a}.attention.head_count", 1)
        hidden = g.get_u32(f"{a}.embedding_length", 0)
        hd = g.get_u32(f"{a}.rope.dimension_count", 0) or hidden // n_heads
        vocab = g.get_u32(f"{a}.vocab_size", 0) or g.tensor_shape("token_embd.weight")[0]
        cfg = LlamaConfig(
            n_layers=g.get_u32(f"{a}.block_count", 0), hidden=hidden, n_heads=n_heads,
            n_kv_heads=g.get_u32(f"{a}.attention.head_count_kv", n_heads), head_dim=hd,
            ffn=g.tensor_shape("blk.0.ffn_up.weight")[0], vocab=vocab,
            rope_theta=g.get_f32(f"{a}.rope.freq_base", 10000.0),
            rms_eps=g.get_f32(f"{a}.attention.layer_norm_rms_epsilon", 1e-6))
        t = {}
        for name in g.tensor_names():
            info = g.tensor_info(name)
            raw = np.array(g.load_tensor_raw(name))
            if info.type == Q8_0:
                N, K = info.shape
                t[name] = ("q8", raw, N, K)
            elif info.type == F32:
                t[name] = ("f32", g.load_tensor_f32(name))
            else:
                raise RuntimeError(f"oracle model: unsupported tensor type {info.type}")
        if "output.weight" not in t:
            t["output.weight"] = t["token_embd.weight"]
        return cls(cfg, t, o)

    # ------------------------------------------------------------------
    def _linear(self, x: np.ndarray, name: str, act: str) -> np.ndarray:
        kind, blocks, N, K = self.t[name]
        x2 = x.reshape(1, -1).astype(np.float32)
        if act == "q8":
            xq, dx = self.o.quantize_act(x2)
            return self.o.linear_a8(blocks, N, K, xq, dx)[0]
        return self.o.linear_a32(x2, blocks, N)[0]

    def embed(self, tok: int) -> np.ndarray:
        _, blocks, V, H = self.t["token_embd.weight"]
        if not 0 <= tok < V:
            raise RuntimeError("Invalid token id")
        row = blocks[tok * (H // QK) * Q8_0_BYTES:(tok + 1) * (H // QK) * Q8_0_BYTES]
        return self.o.dequant(row, H)

    def decode(self, prompt, n_new: int, act: str = "f32", kv: str = "f32", forced=None):
        """Greedy incremental decode; returns (logits [n_new, vocab], new tokens).
        With `forced` (n_new - 1 tokens) step s + 1 is fed forced[s] instead of
        the argmax of step s (teacher forcing); the argmaxes are still returned."""
        c = self.cfg
        o = self.o
        kc = [np.zeros((0, c.n_kv_heads * c.head_dim), np.float32) for _ in range(c.n_layers)]
        vc = [np.zeros((0, c.n_kv_heads * c.head_dim), np.float32) for _ in range(c.n_layers)]
        pos = 0

        def step(h):
            nonlocal pos
            for li in range(c.n_layers):
                p = f"blk.{li}."
                x = o.rmsnorm(h.reshape(1, -1), self.t[p + "attn_norm.weight"][1], c.rms_eps)[0]
                q = self._linear(x, p + "attn_q.weight", act)
                k = self._linear(x, p + "attn_k.weight", act)
                v = self._linear(x, p + "attn_v.weight", act)
                q = o.rope_row(q, c.n_heads, c.head_dim, c.rope_theta, pos)
                k = o.rope_row(k, c.n_kv_heads, c.head_dim, c.rope_theta, pos)
                if kv == "f16":
                    k = k.astype(np.float16).astype(np.float32)
                    v = v.astype(np.float16).astype(np.float32)
                kc[li] = np.vstack([kc[li], k[None]])
                vc[li] = np.vstack([vc[li], v[None]])
                ctx = o.attention(q, kc[li], vc[li], c.n_heads, c.n_kv_heads, c.head_dim)
                after = h + self._linear(ctx, p + "attn_output.weight", act)
                f = o.rmsnorm(after.reshape(1, -1), self.t[p + "ffn_norm.weight"][1],
                              c.rms_eps)[0]
                g = self._linear(f, p + "ffn_gate.weight", act)
                u = self._linear(f, p + "ffn_up.weight", act)
                a = o.silu_mul(g, u)
                h = after + self._linear(a, p + "ffn_down.weight", act)
            pos += 1
            return h

        last = None
        for tok in prompt:
            last = step(self.embed(int(tok)))
        logits = np.zeros((n_new, c.vocab), np.float32)
        toks = []
        for s in range(n_new):
            normed = o.rmsnorm(last.reshape(1, -1), self.t["output_norm.weight"][1], c.rms_eps)[0]
            lg = self._linear(normed, "output.weight", act)
            logits[s] = lg
            nxt = o.argmax(lg)
            toks.append(nxt)
            if s + 1 < n_new:
                last = step(self.embed(int(forced[s]) if forced is not None else nxt))
        return logits, toks
