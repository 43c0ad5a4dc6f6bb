"""ctypes binding of libaxq8.so, the C ABI declared in include/axq8.h, axdec.h and axkv.h.

Loading fails loudly: there is no CPU fallback for any entry point.  If the
shared library is missing, build it with ``python -m axion_b200.build``.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "libaxq8.so"

AXQ8_OK = 0
AXQ8_ERR_INVALID = -1
AXQ8_ERR_CUDA = -2
AXQ8_ERR_ALLOC = -3
AXQ8_ERR_WAIT_TIMEOUT = -4
AXQ8_ERR_UNSUPPORTED = -5
AXQ8_ERR_STATE = -6

AXQ8_ACT_Q8 = 0
AXQ8_ACT_F32 = 1

AXQ8_PATH_GEMV = 0
AXQ8_PATH_TENSOR_CORE = 1
AXQ8_PATH_SKINNY = 2


class axq8_weight_t(C.Structure):
    _fields_ = [
        ("rows", C.c_void_p),
        ("N", C.c_int64),
        ("K", C.c_int64),
        ("row_stride", C.c_int64),
        ("owns", C.c_int32),
        ("device", C.c_int32),
    ]


class axkv_cache_t(C.Structure):
    _fields_ = [
        ("k_pages", C.c_void_p), ("v_pages", C.c_void_p), ("block_table", C.c_void_p),
        ("n_pages", C.c_int32), ("max_blocks", C.c_int32), ("n_kv_heads", C.c_int32),
        ("head_dim", C.c_int32), ("page_tokens", C.c_int32), ("kv_fp32", C.c_int32),
    ]


class axdec_config_t(C.Structure):
    _fields_ = [
        ("n_layers", C.c_int32), ("hidden", C.c_int32), ("ffn", C.c_int32),
        ("n_heads", C.c_int32), ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32),
        ("vocab", C.c_int32), ("rope_theta", C.c_float), ("rms_eps", C.c_float),
        ("max_batch", C.c_int32), ("max_ctx", C.c_int32), ("kv_block", C.c_int32),
        ("act_mode", C.c_int32), ("kv_fp32", C.c_int32),
        ("tp_size", C.c_int32), ("tp_rank", C.c_int32),
    ]


_P = C.c_void_p
_I64 = C.c_int64
_I32 = C.c_int
_W = C.POINTER(axq8_weight_t)

# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple] = {
    "axq8_q8_0_byte_size": (C.c_uint64, [C.c_uint64]),
    "axq8_row_stride": (_I64, [_I64]),
    "axq8_weight_upload": (_I32, [_P, _I64, _I64, _P, _W]),
    "axq8_weight_repack": (_I32, [_P, _I64, _I64, _P, _P]),
    "axq8_weight_wrap": (_I32, [_P, _I64, _I64, _W]),
    "axq8_weight_free": (_I32, [_W]),
    "axq8_dequantize": (_I32, [_W, _P, _P]),
    "axq8_quantize_act": (_I32, [_P, _I64, _I64, _P, _P, _P]),
    "axq8_linear": (_I32, [_W, _P, _I64, _P, _I32, _P]),
    "axq8_linear_q8act": (_I32, [_W, _P, _P, _I64, _P, _P, _P]),
    "axq8_linear_noalloc": (_I32, [_W, _P, _I64, _P, _P]),
    "axq8_block_dots": (_I32, [_W, _P, _I64, _P, _P]),
    "axq8_block_dots_tc": (_I32, [_W, _P, _P, _I64, _P, _P, _P]),
    "axq8_linear_path": (_I32, [_W, _I64, _I32]),
    "axq8_quantize_act_t": (_I32, [_P, _I64, _I64, _P, _P, _P]),
    "axq8_linear_q8act_t": (_I32, [_W, _P, _P, _I64, _P, _P, _P]),
    "axq8_linear_q8act_s": (_I32, [_W, _P, _P, _I64, _P, _P, _P]),
    "axq8_quantize_weight_tensor": (_I32, [_P, _I64, _I64, _P, _P, _P]),
    "axq8_quantized_matmul": (_I32, [_P, _I64, _I64, _P, _P, _I64, _P, _P]),
    "axq8_synth_q8_0": (_I32, [C.c_uint64, _I64, _I64, C.c_float, C.c_float, _I32, _P, _P]),
    "axdec_create": (_I32, [C.POINTER(axdec_config_t), C.POINTER(C.c_void_p)]),
    "axdec_destroy": (_I32, [_P]),
    "axdec_set_tensor": (_I32, [_P, C.c_char_p, _P, _I32, _I64, _I64]),
    "axdec_init_random": (_I32, [_P, C.c_uint64, C.c_float]),
    "axdec_tensor_index": (_I32, [C.POINTER(axdec_config_t), C.c_char_p]),
    "axdec_generate": (_I32, [_P, _P, _I32, _I32, _I32, _P, _P, C.POINTER(C.c_float), _P]),
    "axdec_forced": (_I32, [_P, _P, _I32, _I32, _I32, _P, _P]),
    "axdec_device_bytes": (_I64, [_P]),
    "axdec_weight_bytes_per_step": (_I64, [_P]),
    "axdec_step_kernels": (_I32, [_P, _I32]),
    "axdec_tp_unique_id": (_I32, [_P, _I64]),
    "axdec_tp_connect": (_I32, [_P, _P]),
    "axkv_pages_bytes": (_I64, [C.POINTER(axkv_cache_t)]),
    "axkv_paged_append": (_I32, [C.POINTER(axkv_cache_t), _P, _P, _I32, _P, _P, _P]),
    "axkv_decode_attn_workspace": (_I64, [C.POINTER(axkv_cache_t), _I32, _I32]),
    "axkv_paged_decode_attn": (_I32, [C.POINTER(axkv_cache_t), _P, _I32, _I32, _P, _P, _P, _I64,
                                      _P]),
    "axkv_paged_prefill_attn": (_I32, [C.POINTER(axkv_cache_t), _P, _I64, _I32, _I32, _I32, _I32,
                                       _P, _P, _P, _P]),
    "axtp_allreduce_sum": (_I32, [_P, _I64, _P]),
    "axdec_tp_allreduce_kind": (_I32, [_P]),
    "axdec_tp_health": (_I32, [_P, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "axdec_tp_abort": (_I32, [_P]),
    "axdec_set_prefill": (_I32, [_P, _I32]),
    "axdec_prefill_batched": (_I32, [_P, _I32]),
    "axdec_prefill": (_I32, [_P, _P, _I32, _I32, _P]),
    "axdec_decode_step": (_I32, [_P, _P, _I32, _P, _P, _P]),
    "axdec_decode_continue": (_I32, [_P, _P, _I32, _I32, _P, C.POINTER(C.c_float), _P]),
    "axq8_status_read": (_I32, [C.POINTER(C.c_int)]),
    "axq8_status_clear": (_I32, []),
    "axq8_last_error": (C.c_char_p, []),
    "axq8_version": (C.c_char_p, []),
}

_lib: C.CDLL | None = None


def lib_path() -> Path:
    return _LIB_PATH


def load() -> C.CDLL:
    """Load libaxq8.so and declare every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    if not _LIB_PATH.exists():
        raise RuntimeError(
            f"axion_b200: CUDA library {_LIB_PATH} is missing; "
            "build it with `python -m axion_b200.build` (no CPU fallback exists)")
    lib = C.CDLL(str(_LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class AxionCudaError(RuntimeError):
    """A C-ABI call returned a negative status."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


def check(rc: int) -> None:
    if rc != AXQ8_OK:
        msg = load().axq8_last_error().decode(errors="replace")
        raise AxionCudaError(rc, msg or f"axion_b200 error {rc}")
