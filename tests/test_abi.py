"""The C-ABI library loads and exports every function its headers declare.

No compute call is made here (no GPU needed).
"""
from __future__ import annotations

import ctypes
import re
import subprocess

from conftest import ROOT

HEADERS = sorted((ROOT / "include").glob("*.h"))
DECL = re.compile(r"^[A-Za-z_][\w \t\*]*?\b(ax[a-z0-9]*_\w+)\s*\(", re.M)


def declared_functions() -> set[str]:
    names = set()
    for h in HEADERS:
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names.update(DECL.findall(text))
    return names


def test_headers_declare_functions():
    names = declared_functions()
    assert "axq8_linear" in names and "axq8_weight_upload" in names
    assert len(names) >= 15


def test_library_exports_every_declared_symbol():
    from axion_b200 import _lib
    lib = _lib.load()
    missing = [n for n in sorted(declared_functions()) if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_bindings_cover_declarations():
    from axion_b200 import _lib
    missing = sorted(declared_functions() - set(_lib.SIGNATURES))
    assert not missing, f"no ctypes signature for: {missing}"


def test_library_is_sm100a_only():
    """The fatbin carries sm_100a code only (no PTX, no other SM)."""
    so = ROOT / "axion_b200" / "libaxq8.so"
    r = subprocess.run(["cuobjdump", "--list-elf", str(so)], capture_output=True, text=True)
    if r.returncode != 0:
        import pytest
        pytest.skip("cuobjdump unavailable")
    arches = set(re.findall(r"sm_(\d+a?)", r.stdout))
    assert arches == {"100a"}, arches


def test_pure_host_entry_points():
    """Size helpers need no device."""
    from axion_b200 import _lib
    lib = _lib.load()
    assert lib.axq8_q8_0_byte_size(32) == 34
    assert lib.axq8_q8_0_byte_size(5632 * 2048) == 12_255_232
    assert lib.axq8_row_stride(2048) == 2048 + 128
    assert lib.axq8_row_stride(32) == 32 + 16
    assert lib.axq8_row_stride(5632) % 16 == 0
    assert b"sm_100a" in lib.axq8_version()


def test_invalid_arguments_fail_cleanly():
    """Argument validation runs before any device work and reports a message."""
    from axion_b200 import _lib
    lib = _lib.load()
    w = _lib.axq8_weight_t()
    rc = lib.axq8_weight_wrap(None, 4, 33, ctypes.byref(w))
    assert rc == _lib.AXQ8_ERR_INVALID
    assert b"K" in lib.axq8_last_error() or b"null" in lib.axq8_last_error()
    rc = lib.axq8_linear(None, None, 1, None, 0, None)
    assert rc == _lib.AXQ8_ERR_INVALID


def test_tensor_core_entry_points_validate_shapes():
    """The tensor-core product refuses shapes it does not tile (M < 32,
    N < 128, K % 128 != 0) before touching the device; axq8_linear_path is
    pure host logic."""
    from axion_b200 import _lib
    lib = _lib.load()
    w = _lib.axq8_weight_t()
    w.rows = 4096                      # never dereferenced on these paths
    w.N, w.K, w.row_stride = 256, 256, lib.axq8_row_stride(256)
    w.owns, w.device = 0, 0
    rc = lib.axq8_linear_q8act_t(ctypes.byref(w), 4096, 4096, 16, None, 4096, None)
    assert rc == _lib.AXQ8_ERR_UNSUPPORTED and b"M >= 32" in lib.axq8_last_error()
    w.N = 64
    rc = lib.axq8_linear_q8act_t(ctypes.byref(w), 4096, 4096, 64, None, 4096, None)
    assert rc == _lib.AXQ8_ERR_UNSUPPORTED
    w.N, w.K, w.row_stride = 256, 96, lib.axq8_row_stride(96)
    rc = lib.axq8_block_dots_tc(ctypes.byref(w), 4096, 4096, 64, 4096, 4096, None)
    assert rc == _lib.AXQ8_ERR_UNSUPPORTED
    w.K, w.row_stride = 256, lib.axq8_row_stride(256)
    assert lib.axq8_linear_path(ctypes.byref(w), 1, _lib.AXQ8_ACT_Q8) == _lib.AXQ8_PATH_GEMV
    assert lib.axq8_linear_path(ctypes.byref(w), 32, _lib.AXQ8_ACT_Q8) == _lib.AXQ8_PATH_SKINNY
    # up to 64 rows the skinny product for every shape, the tcgen05 product beyond
    assert lib.axq8_linear_path(ctypes.byref(w), 64, _lib.AXQ8_ACT_Q8) == _lib.AXQ8_PATH_SKINNY
    assert lib.axq8_linear_path(ctypes.byref(w), 65, _lib.AXQ8_ACT_Q8) == _lib.AXQ8_PATH_TENSOR_CORE
    w.N = 131072
    assert lib.axq8_linear_path(ctypes.byref(w), 64, _lib.AXQ8_ACT_Q8) == _lib.AXQ8_PATH_SKINNY
    assert lib.axq8_linear_path(ctypes.byref(w), 65, _lib.AXQ8_ACT_Q8) == _lib.AXQ8_PATH_TENSOR_CORE
    w.N = 256
    rc = lib.axq8_linear_q8act_s(ctypes.byref(w), 4096, 4096, 65, None, 4096, None)
    assert rc == _lib.AXQ8_ERR_UNSUPPORTED and b"M <= 64" in lib.axq8_last_error()
    assert lib.axq8_linear_path(ctypes.byref(w), 64, _lib.AXQ8_ACT_F32) == _lib.AXQ8_PATH_GEMV
    assert lib.axq8_quantize_act_t(None, 4, 33, None, None, None) == _lib.AXQ8_ERR_INVALID


def test_tensor_index_matches_library():
    """The library-free axdec_tensor_index twin (used by the reference arm of
    the benchmark, which must not load libaxq8.so) agrees on every name."""
    import ctypes as C
    from axion_b200 import _lib
    from axion_b200.decoder import DecoderConfig, tensor_index
    lib = _lib.load()
    cc = DecoderConfig(n_layers=5, hidden=64, ffn=64, n_heads=2, n_kv_heads=1, head_dim=32,
                       vocab=64).c()
    names = ["token_embd.weight", "output.weight", "output_norm.weight", "blk.5.attn_q.weight",
             "blk.0.bogus.weight", "blk.x.attn_q.weight", "nothing"]
    names += [f"blk.{i}.{s}.weight" for i in range(5) for s in
              ("attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "ffn_norm", "ffn_gate",
               "ffn_up", "ffn_down")]
    for n in names:
        assert tensor_index(5, n) == lib.axdec_tensor_index(C.byref(cc), n.encode()), n
