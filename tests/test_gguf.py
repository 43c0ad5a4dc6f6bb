"""GGUF reader/writer: round trips, the reference loader's rules, malformed files."""
from __future__ import annotations

import numpy as np
import pytest

from axion_b200 import gguf
from conftest import golden


def test_byte_sizes_match_reference_table():
    # runtime_validation.cpp:271-291 and :662-669
    assert gguf.tensor_byte_size(gguf.F16, 32) == 64
    assert gguf.tensor_byte_size(gguf.Q4_0, 32) == 18
    assert gguf.tensor_byte_size(gguf.Q8_0, 32) == 34
    assert gguf.tensor_byte_size(gguf.Q8_1, 32) == 36
    assert gguf.tensor_byte_size(gguf.Q2_K, 256) == 84
    assert gguf.tensor_byte_size(gguf.Q4_K, 256) == 144
    assert gguf.tensor_byte_size(gguf.Q6_K, 256) == 210
    assert gguf.tensor_byte_size(gguf.Q8_K, 256) == 292
    assert gguf.tensor_byte_size(gguf.Q4_1, 32) == 20
    assert gguf.tensor_byte_size(gguf.Q5_0, 32) == 22
    assert gguf.tensor_byte_size(gguf.Q5_1, 32) == 24
    assert gguf.tensor_byte_size(gguf.Q3_K, 256) == 110
    assert gguf.tensor_byte_size(gguf.Q5_K, 256) == 176
    with pytest.raises(RuntimeError):
        gguf.tensor_byte_size(99, 32)


def test_round_trip(tmp_path, oracle):
    rng = np.random.default_rng(1)
    w = rng.normal(0, 0.02, (7, 64)).astype(np.float32)
    blocks = oracle.quantize_weight_blocks(w)
    g = gguf.GGUFWriter()
    g.add_string("general.architecture", "llama")
    g.add_u32("llama.block_count", 3)
    g.add_f32("llama.rope.freq_base", 500000.0)
    g.add_str_array("tokenizer.ggml.tokens", ["a", "b", "c"])
    g.add_tensor("w", blocks, (7, 64), gguf.Q8_0)
    g.add_tensor("n", np.arange(64, dtype=np.float32), (64,), gguf.F32)
    p = tmp_path / "t.gguf"
    g.write(p)
    r = gguf.GGUFLoader()
    assert r.load_file(p)
    assert r.architecture() == "llama"
    assert r.get_u32("llama.block_count") == 3
    assert r.get_f32("llama.rope.freq_base") == 500000.0
    assert r.get_arr_len("tokenizer.ggml.tokens") == 3
    assert r.tensor_shape("w") == [7, 64]
    assert r.tensor_shape("missing") == []
    assert bytes(r.load_tensor_raw("w")) == blocks.tobytes()
    assert np.array_equal(r.load_tensor_f32("n"), np.arange(64, dtype=np.float32))
    assert r.tensor_data_offset % 32 == 0
    with pytest.raises(RuntimeError, match="Tensor not found"):
        r.load_tensor_raw("missing")


def test_reads_golden_model_like_reference(reflib, oracle):
    """Our loader and the reference loader agree on shapes and dequantized values."""
    p = golden("tiny_llama.gguf")
    r = gguf.GGUFLoader()
    r.load_file(p)
    for name in ["token_embd.weight", "blk.0.attn_q.weight", "blk.1.ffn_down.weight",
                 "output.weight"]:
        info = r.tensor_info(name)
        ref = reflib.load_tensor(p, name)
        assert list(ref.shape) == list(info.shape)
        mine = oracle.dequant(np.array(r.load_tensor_raw(name)), info.element_count)
        assert np.array_equal(mine.view(np.uint32), ref.reshape(-1).view(np.uint32))


def test_malformed_files(tmp_path):
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUX" + b"\0" * 32)
    with pytest.raises(RuntimeError, match="Invalid GGUF"):
        gguf.GGUFLoader().load_file(bad)
    with pytest.raises(RuntimeError, match="Failed to open"):
        gguf.GGUFLoader().load_file(tmp_path / "nope.gguf")
    # truncated: header claims a tensor whose data is missing
    g = gguf.GGUFWriter()
    g.add_tensor("w", np.zeros(34 * 4, np.uint8), (4, 32), gguf.Q8_0)
    p = tmp_path / "trunc.gguf"
    g.write(p)
    data = p.read_bytes()
    p.write_bytes(data[:-40])
    with pytest.raises(RuntimeError):
        gguf.GGUFLoader().load_file(p)
    p.write_bytes(data[:20])
    with pytest.raises(RuntimeError, match="Truncated"):
        gguf.GGUFLoader().load_file(p)


def test_writer_rejects_wrong_size():
    g = gguf.GGUFWriter()
    with pytest.raises(ValueError):
        g.add_tensor("w", np.zeros(33, np.uint8), (32,), gguf.Q8_0)
