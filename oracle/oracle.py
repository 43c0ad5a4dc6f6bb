"""numpy-level wrappers of the two CPU checkers (test infrastructure only).

``Oracle``  — liboracle.so, the C restatement in q8_oracle.c.
``RefLib``  — _ref/libaxion_ref.so, the reference's own C++ path.

Each wrapper function names the reference file:line it follows in its C
implementation (see q8_oracle.h / ref_shim.cpp).
"""
from __future__ import annotations

import ctypes as C
import os
import re
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libaxion_ref.so"
REF_VALIDATION = HERE / "_ref" / "axion_runtime_validation"


def _ref_src() -> Path:
    """The reference's inference/cpp source tree: $AXION_REF_SRC, else the
    `REF ?=` default of the Makefile that builds the reference library (one
    place names the location; `make REF=...` and this variable override it)."""
    env = os.environ.get("AXION_REF_SRC")
    if env:
        return Path(env)
    try:
        m = re.search(r"^REF\s*\?=\s*(\S+)", (HERE / "Makefile").read_text(), re.M)
        if m:
            return Path(m.group(1))
    except OSError:
        pass
    return HERE / "_ref" / "src-not-configured"


REF_SRC = _ref_src()

QK = 32
Q8_0_BYTES = 34

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_I64 = C.c_int64


def build(ref: bool | None = None) -> None:
    """Build liboracle.so (always) and the reference library (when its sources exist)."""
    targets = ["oracle"]
    if ref is None:
        ref = REF_SRC.exists()
    if ref:
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", str(HERE), f"REF={REF_SRC}", *targets], check=True)


class Oracle:
    def __init__(self) -> None:
        if not ORACLE_SO.exists():
            build(ref=False)
        L = C.CDLL(str(ORACLE_SO))
        sig = {
            "axo_fp16_to_fp32": (C.c_float, [C.c_uint16]),
            "axo_fp32_to_fp16": (C.c_uint16, [C.c_float]),
            "axo_q8_0_byte_size": (C.c_uint64, [C.c_uint64]),
            "axo_q8_0_dequant": (None, [_u8p, C.c_uint64, _f32p]),
            "axo_q8_0_quantize": (None, [_f32p, _I64, _I64, _u8p]),
            "axo_quantize_act": (None, [_f32p, _I64, _I64, _i8p, _f32p]),
            "axo_block_dots": (None, [_u8p, _I64, _I64, _i8p, _I64, _i32p]),
            "axo_linear_a8": (None, [_u8p, _I64, _I64, _i8p, _f32p, _I64, _f32p]),
            "axo_linear_a32": (None, [_f32p, _I64, _I64, _u8p, _I64, _f32p]),
            "axo_linear_f32": (None, [_f32p, _I64, _I64, _f32p, _I64, _f32p]),
            "axo_rmsnorm": (None, [_f32p, _I64, _I64, _f32p, C.c_float, _f32p]),
            "axo_rope_neox_row": (None, [_f32p, C.c_int, C.c_int, C.c_float, C.c_int]),
            "axo_attention_decode": (None, [_f32p, _f32p, _f32p, _I64, C.c_int, C.c_int,
                                            C.c_int, _f32p]),
            "axo_silu_mul": (None, [_f32p, _f32p, _I64, _f32p]),
            "axo_residual_add": (None, [_f32p, _f32p, _I64, _f32p]),
            "axo_argmax": (_I64, [_f32p, _I64]),
            "axo_gen_normal": (None, [C.c_uint64, C.c_uint64, _I64, C.c_float, C.c_float, _f32p]),
        }
        for n, (r, a) in sig.items():
            f = getattr(L, n)
            f.restype = r
            f.argtypes = a
        self.L = L

    # --- format ---
    def fp16_to_fp32(self, h: int) -> float:
        return self.L.axo_fp16_to_fp32(h)

    def q8_0_byte_size(self, n: int) -> int:
        return self.L.axo_q8_0_byte_size(n)

    def dequant(self, blocks: np.ndarray, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        self.L.axo_q8_0_dequant(np.ascontiguousarray(blocks, np.uint8), n, out)
        return out

    def quantize_weight_blocks(self, w: np.ndarray) -> np.ndarray:
        w = np.ascontiguousarray(w, np.float32)
        rows, K = w.shape
        out = np.empty(rows * (K // QK) * Q8_0_BYTES, np.uint8)
        self.L.axo_q8_0_quantize(w, rows, K, out)
        return out

    def gen_normal(self, seed: int, n: int, std: float = 0.02, mean: float = 0.0,
                   start: int = 0) -> np.ndarray:
        out = np.empty(n, np.float32)
        self.L.axo_gen_normal(seed, start, n, mean, std, out)
        return out

    def synth_q8_0(self, seed: int, N: int, K: int, std: float = 0.02) -> np.ndarray:
        """Host twin of axq8_synth_q8_0 (GGUF block layout)."""
        return self.quantize_weight_blocks(self.gen_normal(seed, N * K, std).reshape(N, K))

    # --- linear ---
    def quantize_act(self, x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
        x = np.ascontiguousarray(x, np.float32)
        M, K = x.shape
        q = np.empty((M, K), np.int8)
        d = np.empty((M, K // QK), np.float32)
        self.L.axo_quantize_act(x, M, K, q, d)
        return q, d

    def block_dots(self, blocks: np.ndarray, N: int, K: int, xq: np.ndarray) -> np.ndarray:
        M = xq.shape[0]
        out = np.empty((M, N, K // QK), np.int32)
        self.L.axo_block_dots(np.ascontiguousarray(blocks, np.uint8), N, K,
                              np.ascontiguousarray(xq, np.int8), M, out)
        return out

    def linear_a8(self, blocks: np.ndarray, N: int, K: int, xq: np.ndarray,
                  dx: np.ndarray) -> np.ndarray:
        M = xq.shape[0]
        y = np.empty((M, N), np.float32)
        self.L.axo_linear_a8(np.ascontiguousarray(blocks, np.uint8), N, K,
                             np.ascontiguousarray(xq, np.int8),
                             np.ascontiguousarray(dx, np.float32), M, y)
        return y

    def linear_a32(self, x: np.ndarray, blocks: np.ndarray, N: int) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        M, K = x.shape
        y = np.empty((M, N), np.float32)
        self.L.axo_linear_a32(x, M, K, np.ascontiguousarray(blocks, np.uint8), N, y)
        return y

    def linear_f32(self, x: np.ndarray, w: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        M, K = x.shape
        N = w.shape[0]
        y = np.empty((M, N), np.float32)
        self.L.axo_linear_f32(x, M, K, w, N, y)
        return y

    # --- decode-layer ops ---
    def rmsnorm(self, x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        self.L.axo_rmsnorm(x, x.shape[0], x.shape[1], np.ascontiguousarray(w, np.float32),
                           eps, out)
        return out

    def rope_row(self, x: np.ndarray, n_heads: int, hd: int, theta: float, pos: int) -> np.ndarray:
        y = np.ascontiguousarray(x, np.float32).copy()
        self.L.axo_rope_neox_row(y, n_heads, hd, theta, pos)
        return y

    def attention(self, q: np.ndarray, k: np.ndarray, v: np.ndarray, n_head: int, n_kv: int,
                  hd: int) -> np.ndarray:
        out = np.empty(n_head * hd, np.float32)
        self.L.axo_attention_decode(np.ascontiguousarray(q, np.float32),
                                    np.ascontiguousarray(k, np.float32),
                                    np.ascontiguousarray(v, np.float32), k.shape[0],
                                    n_head, n_kv, hd, out)
        return out

    def silu_mul(self, g: np.ndarray, u: np.ndarray) -> np.ndarray:
        g = np.ascontiguousarray(g, np.float32)
        out = np.empty_like(g)
        self.L.axo_silu_mul(g, np.ascontiguousarray(u, np.float32), g.size, out)
        return out

    def argmax(self, x: np.ndarray) -> int:
        x = np.ascontiguousarray(x, np.float32)
        return int(self.L.axo_argmax(x, x.size))


class RefLib:
    """The reference's own C++ implementation (built by oracle/Makefile)."""

    def __init__(self) -> None:
        if not REF_SO.exists():
            if not REF_SRC.exists():
                raise FileNotFoundError("reference library not built and sources absent")
            build(ref=True)
        L = C.CDLL(str(REF_SO))
        sig = {
            "axref_last_error": (C.c_char_p, []),
            "axref_fp16_to_fp32": (C.c_float, [C.c_uint16]),
            "axref_q8_0_byte_size": (C.c_uint64, [C.c_uint64]),
            "axref_gguf_open": (C.c_void_p, [C.c_char_p]),
            "axref_gguf_close": (None, [C.c_void_p]),
            "axref_gguf_shape": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_int64)]),
            "axref_gguf_load_tensor": (C.c_int, [C.c_void_p, C.c_char_p, _f32p, _I64]),
            "axref_linear_from_gguf": (C.c_int, [_f32p, _I64, _I64, _f32p, _I64, _I64, _f32p]),
            "axref_quantized_matmul_q8": (C.c_int, [_f32p, _I64, _I64, _f32p, _I64, _f32p, _i8p,
                                                    C.POINTER(C.c_float)]),
            "axref_rmsnorm": (C.c_int, [_f32p, _I64, _I64, _f32p, C.c_float, _f32p]),
            "axref_silu_mul": (C.c_int, [_f32p, _f32p, _I64, _f32p]),
            "axref_rope_row_at": (C.c_int, [_f32p, C.c_int, C.c_int, C.c_float, C.c_int]),
            "axref_mha_incremental": (C.c_int, [_f32p, _f32p, _f32p, _I64, C.c_int, C.c_int,
                                                C.c_int, _f32p]),
            "axref_generate": (C.c_int, [C.c_char_p, _i32p, C.c_int, C.c_int, _i32p,
                                         C.POINTER(C.c_int)]),
            "axref_decode_logits": (C.c_int, [C.c_char_p, _i32p, C.c_int, C.c_int, C.c_void_p,
                                              _f32p, _i32p]),
            "axref_time_linear": (C.c_int, [C.c_char_p, C.c_char_p, _f32p, _I64, C.c_int,
                                            C.c_int, _f32p, C.POINTER(C.c_double)]),
            "axref_time_generate": (C.c_int, [C.c_char_p, _i32p, C.c_int, C.c_int, _i32p,
                                              C.POINTER(C.c_int), C.POINTER(C.c_double)]),
        }
        for n, (r, a) in sig.items():
            f = getattr(L, n)
            f.restype = r
            f.argtypes = a
        self.L = L

    def _check(self, rc: int) -> None:
        if rc != 0:
            raise RuntimeError(self.L.axref_last_error().decode())

    def fp16_to_fp32(self, h: int) -> float:
        return self.L.axref_fp16_to_fp32(h)

    def load_tensor(self, path: str, name: str) -> np.ndarray:
        h = self.L.axref_gguf_open(str(path).encode())
        if not h:
            raise RuntimeError(self.L.axref_last_error().decode())
        try:
            shp = (C.c_int64 * 4)()
            nd = self.L.axref_gguf_shape(h, name.encode(), shp)
            if nd < 0:
                raise RuntimeError("Tensor not found")
            shape = tuple(shp[i] for i in range(nd))
            out = np.empty(int(np.prod(shape)), np.float32)
            self._check(self.L.axref_gguf_load_tensor(h, name.encode(), out, out.size))
            return out.reshape(shape)
        finally:
            self.L.axref_gguf_close(h)

    def linear_from_gguf(self, x: np.ndarray, w: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        M, K = x.shape
        N, Kw = w.shape
        y = np.empty((M, N), np.float32)
        self._check(self.L.axref_linear_from_gguf(x, M, K, w, N, Kw, y))
        return y

    def quantized_matmul_q8(self, x: np.ndarray, w_kn: np.ndarray):
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w_kn, np.float32)
        M, K = x.shape
        N = w.shape[1]
        y = np.empty((M, N), np.float32)
        q = np.empty(K * N, np.int8)
        s = C.c_float(0)
        self._check(self.L.axref_quantized_matmul_q8(x, M, K, w, N, y, q, C.byref(s)))
        return y, q.reshape(K, N), s.value

    def rmsnorm(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        self._check(self.L.axref_rmsnorm(x, x.shape[0], x.shape[1],
                                         np.ascontiguousarray(w, np.float32), eps, out))
        return out

    def silu_mul(self, g, u):
        g = np.ascontiguousarray(g, np.float32)
        out = np.empty_like(g)
        self._check(self.L.axref_silu_mul(g, np.ascontiguousarray(u, np.float32), g.size, out))
        return out

    def rope_row(self, x, n_heads, hd, theta, pos):
        y = np.ascontiguousarray(x, np.float32).copy()
        self._check(self.L.axref_rope_row_at(y, n_heads, hd, theta, pos))
        return y

    def attention(self, q, k, v, n_head, n_kv, hd):
        out = np.empty(n_head * hd, np.float32)
        self._check(self.L.axref_mha_incremental(
            np.ascontiguousarray(q, np.float32), np.ascontiguousarray(k, np.float32),
            np.ascontiguousarray(v, np.float32), k.shape[0], n_head, n_kv, hd, out))
        return out

    def generate(self, path: str, prompt, max_new: int) -> list[int]:
        pr = np.ascontiguousarray(prompt, np.int32)
        out = np.empty(len(pr) + max_new, np.int32)
        n = C.c_int(0)
        self._check(self.L.axref_generate(str(path).encode(), pr, len(pr), max_new, out,
                                          C.byref(n)))
        return out[:n.value].tolist()

    def decode_logits(self, path: str, prompt, n_steps: int, vocab: int, forced=None):
        pr = np.ascontiguousarray(prompt, np.int32)
        logits = np.empty((n_steps, vocab), np.float32)
        am = np.empty(n_steps, np.int32)
        fp = None
        if forced is not None:
            forced = np.ascontiguousarray(forced, np.int32)
            fp = forced.ctypes.data_as(C.c_void_p)
        self._check(self.L.axref_decode_logits(str(path).encode(), pr, len(pr), n_steps, fp,
                                               logits, am))
        return logits, am

    def time_linear(self, path: str, name: str, x: np.ndarray, N: int, iters: int,
                    with_load: bool = True):
        """Seconds for `iters` x [load_tensor +] linear_from_gguf, and the last output."""
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty((x.shape[0], N), np.float32)
        sec = C.c_double(0)
        self._check(self.L.axref_time_linear(str(path).encode(), name.encode(), x, x.shape[0],
                                             iters, int(with_load), y, C.byref(sec)))
        return sec.value, y

    def time_generate(self, path: str, prompt, max_new: int):
        """Seconds of one ModelRunner::generate call, and the tokens it returned."""
        pr = np.ascontiguousarray(prompt, np.int32)
        out = np.empty(len(pr) + max_new, np.int32)
        n = C.c_int(0)
        sec = C.c_double(0)
        self._check(self.L.axref_time_generate(str(path).encode(), pr, len(pr), max_new, out,
                                               C.byref(n), C.byref(sec)))
        return sec.value, out[:n.value].tolist()
