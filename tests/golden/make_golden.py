"""Generate the golden fixtures in tests/golden/ by running the reference itself.

Run in a container where the reference sources are present (they are not on
the GPU machines, which only read the committed fixtures):

    make -C oracle ref && python tests/golden/make_golden.py

Every output value below comes from the reference's own C++ code path
(oracle/_ref/libaxion_ref.so, built from its unmodified sources by
oracle/Makefile) called through oracle/ref_shim.cpp:

* fp16_table.npy            fp16_to_fp32 over all 65536 bit patterns
                            (inference/cpp/core/fp16.cpp:5-66)
* q8_known_answer.npz       the known-answer Q8_0 block of the reference's own
                            harness (inference/cpp/tests/runtime_validation.cpp
                            :768-852: d = 0.5, q[i] = i - 16) read back through
                            GGUFLoader::load_tensor
* linear_cases.npz          GGUFLoader::load_tensor + linear_from_gguf on
                            seeded Q8_0 weights, several shapes incl. edge
                            cases (K = 32, N = 1, M = 1..5, ragged N)
* quantized_matmul.npz      quantize_weight(Q8_0) + quantized_matmul
                            (inference/cpp/runtime/quantized_matmul.cpp)
* ops_cases.npz             rmsnorm, NEOX RoPE, mha_attention_incremental,
                            silu*up on seeded inputs
* tiny_llama.gguf           a 2-layer Llama-architecture model with Q8_0
                            linears (written by axion_b200.gguf.GGUFWriter)
* tiny_llama_ref.npz        ModelRunner::generate greedy tokens and the
                            per-step logits of the same incremental decode
* tinyllama_width_256.npz   256 greedy steps of ModelRunner::generate (and the
                            per-step logits) on a 2-layer model of TinyLlama's
                            layer widths (hidden 2048, FFN 5632, 32/4 heads of
                            64) with a 2048-token vocabulary, whose Q8_0
                            weights are the device generator's
                            (axq8_synth_q8_0 seed + tensor index, std 0.02;
                            norms 1.0), so the GPU test rebuilds the same model
                            with axdec_init_random instead of reading a file.
                            `python tests/golden/make_golden.py --long` writes
                            it alone (about two minutes of host time).
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from axion_b200.gguf import F32, Q8_0, GGUFWriter  # noqa: E402
from oracle.oracle import Oracle, RefLib  # noqa: E402

SEED = 0xA710

# tiny Llama-architecture model (shapes chosen so every linear is Q8_0-legal)
TINY = dict(n_layers=2, hidden=128, n_heads=4, n_kv_heads=2, head_dim=32, ffn=256, vocab=96,
            rope_theta=10000.0, rms_eps=1e-5)
TINY_PROMPT = [5, 17, 3, 88, 42, 9]
TINY_NEW = 12

LINEAR_SHAPES = [  # (M, N, K)
    (1, 1, 32), (1, 5, 32), (2, 7, 64), (3, 33, 96), (1, 64, 512), (4, 129, 256),
    (5, 48, 1024), (1, 300, 2048),
]


def write_tiny_llama(o: Oracle, path: Path, seed: int = SEED) -> dict:
    """Seeded random-init tiny model in GGUF; returns the fp32 norm weights."""
    c = TINY
    H, F, V = c["hidden"], c["ffn"], c["vocab"]
    hq = c["n_heads"] * c["head_dim"]
    hkv = c["n_kv_heads"] * c["head_dim"]
    g = GGUFWriter()
    g.add_string("general.architecture", "llama")
    g.add_u32("llama.block_count", c["n_layers"])
    g.add_u32("llama.attention.head_count", c["n_heads"])
    g.add_u32("llama.attention.head_count_kv", c["n_kv_heads"])
    g.add_u32("llama.embedding_length", H)
    g.add_u32("llama.feed_forward_length", F)
    g.add_u32("llama.rope.dimension_count", c["head_dim"])
    g.add_u32("llama.vocab_size", V)
    g.add_f32("llama.rope.freq_base", c["rope_theta"])
    g.add_f32("llama.attention.layer_norm_rms_epsilon", c["rms_eps"])
    rng = np.random.default_rng(seed)

    def q8(name, rows, cols, std=0.02):
        w = rng.normal(0.0, std, (rows, cols)).astype(np.float32)
        g.add_tensor(name, o.quantize_weight_blocks(w), (rows, cols), Q8_0)

    def norm(name):
        w = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
        g.add_tensor(name, w, (H,), F32)

    # larger embedding / head scale so the logits have clear top-1 margins
    q8("token_embd.weight", V, H, std=0.5)
    for i in range(c["n_layers"]):
        p = f"blk.{i}."
        norm(p + "attn_norm.weight")
        q8(p + "attn_q.weight", hq, H, std=0.2)
        q8(p + "attn_k.weight", hkv, H, std=0.2)
        q8(p + "attn_v.weight", hkv, H, std=0.2)
        q8(p + "attn_output.weight", H, hq, std=0.2)
        norm(p + "ffn_norm.weight")
        q8(p + "ffn_gate.weight", F, H, std=0.2)
        q8(p + "ffn_up.weight", F, H, std=0.2)
        q8(p + "ffn_down.weight", H, F, std=0.2)
    norm("output_norm.weight")
    q8("output.weight", V, H, std=0.2)
    g.write(path)
    return c


# 256-step greedy fixture: TinyLlama layer widths, 2 layers, small vocabulary
LONG = dict(n_layers=2, hidden=2048, n_heads=32, n_kv_heads=4, head_dim=64, ffn=5632, vocab=2048,
            rope_theta=10000.0, rms_eps=1e-5)
LONG_SEED = 0x256
LONG_PROMPT_LEN = 16
LONG_NEW = 256


def long_index(name: str) -> int:
    from axion_b200.decoder import tensor_index
    return tensor_index(LONG["n_layers"], name)


def write_long_model(o: Oracle, path: Path) -> None:
    c = LONG
    H, F, V = c["hidden"], c["ffn"], c["vocab"]
    hq, hkv = c["n_heads"] * c["head_dim"], c["n_kv_heads"] * c["head_dim"]
    g = GGUFWriter()
    g.add_string("general.architecture", "llama")
    for k, v in [("block_count", c["n_layers"]), ("attention.head_count", c["n_heads"]),
                 ("attention.head_count_kv", c["n_kv_heads"]), ("embedding_length", H),
                 ("feed_forward_length", F), ("rope.dimension_count", c["head_dim"]),
                 ("vocab_size", V)]:
        g.add_u32(f"llama.{k}", v)
    g.add_f32("llama.rope.freq_base", c["rope_theta"])
    g.add_f32("llama.attention.layer_norm_rms_epsilon", c["rms_eps"])

    def q8(name, N, K):
        g.add_tensor(name, o.synth_q8_0(LONG_SEED + long_index(name), N, K, 0.02), (N, K), Q8_0)

    ones = np.ones(H, np.float32)
    q8("token_embd.weight", V, H)
    for i in range(c["n_layers"]):
        p = f"blk.{i}."
        g.add_tensor(p + "attn_norm.weight", ones, (H,), F32)
        q8(p + "attn_q.weight", hq, H)
        q8(p + "attn_k.weight", hkv, H)
        q8(p + "attn_v.weight", hkv, H)
        q8(p + "attn_output.weight", H, hq)
        g.add_tensor(p + "ffn_norm.weight", ones, (H,), F32)
        q8(p + "ffn_gate.weight", F, H)
        q8(p + "ffn_up.weight", F, H)
        q8(p + "ffn_down.weight", H, F)
    g.add_tensor("output_norm.weight", ones, (H,), F32)
    q8("output.weight", V, H)
    g.write(path)


def make_long(o: Oracle, r: RefLib) -> None:
    path = HERE / "_long.gguf"
    write_long_model(o, path)
    prompt = np.random.default_rng(LONG_SEED).integers(0, LONG["vocab"], LONG_PROMPT_LEN)
    prompt = prompt.astype(np.int32)
    toks = r.generate(path, prompt, LONG_NEW)
    logits, am = r.decode_logits(path, prompt, LONG_NEW, LONG["vocab"])
    path.unlink()
    assert toks[LONG_PROMPT_LEN:] == am.tolist(), "generate and the per-step decode disagree"
    srt = np.sort(logits, axis=1)
    margin = (srt[:, -1] - srt[:, -2]) / np.max(np.abs(logits), axis=1)
    np.savez_compressed(HERE / "tinyllama_width_256.npz", prompt=prompt,
                        tokens=np.array(toks[LONG_PROMPT_LEN:], np.int32), logits=logits,
                        seed=np.int64(LONG_SEED), min_margin=np.float32(margin.min()),
                        config=np.array([LONG[k] for k in ("n_layers", "hidden", "n_heads",
                                                           "n_kv_heads", "head_dim", "ffn",
                                                           "vocab")], np.int64))
    print("long run: smallest top-2 margin (relative)", float(margin.min()))


def main() -> None:
    o = Oracle()
    r = RefLib()
    rng = np.random.default_rng(SEED)

    # 1. fp16 table
    table = np.array([r.fp16_to_fp32(h) for h in range(65536)], dtype=np.float32)
    np.save(HERE / "fp16_table.npy", table.view(np.uint32))

    # 2. known-answer block through the reference loader
    tmp = HERE / "_ka.gguf"
    blk = np.zeros(34, np.uint8)
    blk[0:2] = np.frombuffer(np.float16(0.5).tobytes(), np.uint8)
    blk[2:] = (np.arange(32) - 16).astype(np.int8).view(np.uint8)
    g = GGUFWriter()
    g.add_tensor("q8_0", blk, (32,), Q8_0)
    g.write(tmp)
    ka = r.load_tensor(tmp, "q8_0")
    tmp.unlink()
    np.savez(HERE / "q8_known_answer.npz", block=blk, values=ka)

    # 3. linear cases
    cases = {}
    tmp = HERE / "_lin.gguf"
    for i, (M, N, K) in enumerate(LINEAR_SHAPES):
        w = rng.normal(0.0, 0.02, (N, K)).astype(np.float32)
        x = rng.normal(0.0, 1.0, (M, K)).astype(np.float32)
        blocks = o.quantize_weight_blocks(w)
        g = GGUFWriter()
        g.add_tensor("w", blocks, (N, K), Q8_0)
        g.write(tmp)
        wd = r.load_tensor(tmp, "w")
        y = r.linear_from_gguf(x, wd)
        cases[f"c{i}_blocks"] = blocks
        cases[f"c{i}_x"] = x
        if N * K <= 65536:   # keep the fixture small: dequant values of the small cases
            cases[f"c{i}_wdeq"] = wd
        cases[f"c{i}_y"] = y
        cases[f"c{i}_shape"] = np.array([M, N, K], np.int64)
    tmp.unlink()
    np.savez_compressed(HERE / "linear_cases.npz", n=len(LINEAR_SHAPES), **cases)

    # 4. quantize_weight / quantized_matmul (per-tensor Q8_0, W is [K, N])
    qm = {}
    for i, (M, K, N) in enumerate([(2, 4, 3), (3, 64, 17), (1, 256, 40)]):
        x = rng.normal(0.0, 1.0, (M, K)).astype(np.float32)
        w = rng.normal(0.0, 0.05, (K, N)).astype(np.float32)
        y, q, s = r.quantized_matmul_q8(x, w)
        qm.update({f"c{i}_x": x, f"c{i}_w": w, f"c{i}_y": y, f"c{i}_q": q,
                   f"c{i}_scale": np.float32(s)})
    np.savez(HERE / "quantized_matmul.npz", n=3, **qm)

    # 5. decode-layer operators
    ops = {}
    x = rng.normal(0.0, 1.0, (2, 256)).astype(np.float32)
    wn = (1.0 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    ops["rms_x"], ops["rms_w"], ops["rms_y"] = x, wn, r.rmsnorm(x, wn, 1e-5)
    q = rng.normal(0.0, 1.0, 8 * 64).astype(np.float32)
    ops["rope_x"], ops["rope_y"] = q, r.rope_row(q, 8, 64, 10000.0, 77)
    kc = rng.normal(0.0, 1.0, (40, 2 * 64)).astype(np.float32)
    vc = rng.normal(0.0, 1.0, (40, 2 * 64)).astype(np.float32)
    ops["att_q"], ops["att_k"], ops["att_v"] = q, kc, vc
    ops["att_y"] = r.attention(q, kc, vc, 8, 2, 64)
    gg = rng.normal(0.0, 2.0, 1000).astype(np.float32)
    uu = rng.normal(0.0, 1.0, 1000).astype(np.float32)
    ops["silu_g"], ops["silu_u"], ops["silu_y"] = gg, uu, r.silu_mul(gg, uu)
    np.savez(HERE / "ops_cases.npz", **ops)

    # 6. tiny llama end to end
    path = HERE / "tiny_llama.gguf"
    write_tiny_llama(o, path)
    toks = r.generate(path, TINY_PROMPT, TINY_NEW)
    logits, am = r.decode_logits(path, TINY_PROMPT, TINY_NEW, TINY["vocab"])
    np.savez(HERE / "tiny_llama_ref.npz", prompt=np.array(TINY_PROMPT, np.int32),
             tokens=np.array(toks, np.int32), logits=logits, argmax=am)
    print("generated", toks)
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    if "--long" in sys.argv:
        make_long(Oracle(), RefLib())
    else:
        main()
        make_long(Oracle(), RefLib())
