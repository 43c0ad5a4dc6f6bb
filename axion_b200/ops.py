"""Reference-named operator API over the C ABI (torch tensors for device memory).

Mirrors the names, argument meaning and error behaviour of the reference's
operator API for the Q8_0 linear path:

* ``linear_from_gguf(input[M,K], weight[N,K]) -> [M,N]``
  (inference/cpp/runtime/linear.hpp:22-25; errors linear.cpp:31-44);
* ``QuantType`` / ``QuantizedWeight`` / ``quantize_weight`` / ``quantized_matmul``
  (inference/cpp/runtime/quantized_matmul.hpp:14-48), Q8_0 per-tensor format;
* ``gguf_tensor_byte_size`` (inference/cpp/gguf/gguf.hpp:34-37).

The weight of ``linear_from_gguf`` is a :class:`Q8Weight`: the GGUF Q8_0
blocks kept resident on the device in the repacked row layout, instead of the
fp32 tensor the reference's loader produces by dequantizing on every call.
Every operator runs a CUDA kernel of libaxq8.so on the current torch stream;
inputs must already be CUDA tensors.  There is no CPU path.
"""
from __future__ import annotations

import ctypes as C
import enum
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import check

QK = 32
Q8_0_BYTES = 34


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _require_cuda(t: torch.Tensor, what: str) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise RuntimeError(f"{what} must be a CUDA tensor (axion_b200 has no CPU path)")


def gguf_tensor_byte_size_q8_0(n: int) -> int:
    """gguf_tensor_byte_size(GGUFType::Q8_0, n) (gguf.cpp:51)."""
    return int(_lib.load().axq8_q8_0_byte_size(n))


def row_stride(K: int) -> int:
    return int(_lib.load().axq8_row_stride(K))


class Q8Weight:
    """A GGUF Q8_0 weight [N, K] resident on the device (repacked rows)."""

    def __init__(self, rows: torch.Tensor, N: int, K: int):
        if K % QK:
            raise RuntimeError(f"Q8_0 weight K={K} is not a multiple of 32")
        _require_cuda(rows, "Q8Weight rows")
        if rows.dtype != torch.uint8 or rows.numel() != N * row_stride(K):
            raise RuntimeError("Q8Weight rows: wrong dtype or size")
        self.rows = rows
        self.N = int(N)
        self.K = int(K)
        self._c = _lib.axq8_weight_t()
        check(_lib.load().axq8_weight_wrap(C.c_void_p(rows.data_ptr()), self.N, self.K,
                                           C.byref(self._c)))

    @property
    def shape(self) -> tuple[int, int]:
        return (self.N, self.K)

    @property
    def c(self) -> C.POINTER(_lib.axq8_weight_t):
        return C.byref(self._c)

    @classmethod
    def empty(cls, N: int, K: int, device=None) -> "Q8Weight":
        dev = torch.device(device) if device is not None else torch.device("cuda")
        rows = torch.empty(N * row_stride(K), dtype=torch.uint8, device=dev)
        return cls(rows, N, K)

    @classmethod
    def from_blocks(cls, blocks, N: int, K: int, device=None) -> "Q8Weight":
        """Upload GGUF Q8_0 blocks (host bytes / ndarray, or a CUDA uint8 tensor)."""
        nbytes = N * (K // QK) * Q8_0_BYTES
        if isinstance(blocks, torch.Tensor) and blocks.is_cuda:
            src = blocks.reshape(-1)
            device = src.device
        else:
            arr = np.frombuffer(blocks, dtype=np.uint8) if not isinstance(blocks, np.ndarray) \
                else blocks.reshape(-1).view(np.uint8)
            if arr.size != nbytes:
                raise RuntimeError(f"Q8_0 blocks: {arr.size} bytes, expected {nbytes}")
            dev = torch.device(device) if device is not None else torch.device("cuda")
            src = torch.from_numpy(np.ascontiguousarray(arr)).to(dev, non_blocking=False)
            device = dev
        if src.numel() != nbytes:
            raise RuntimeError(f"Q8_0 blocks: {src.numel()} bytes, expected {nbytes}")
        w = cls.empty(N, K, device)
        with torch.cuda.device(w.rows.device):
            check(_lib.load().axq8_weight_repack(C.c_void_p(src.data_ptr()), N, K,
                                                 C.c_void_p(w.rows.data_ptr()),
                                                 C.c_void_p(_stream())))
        w._src_keepalive = src   # the repack is asynchronous on the stream
        return w

    @classmethod
    def synthetic(cls, seed: int, N: int, K: int, std: float = 0.02, mean: float = 0.0,
                  device=None) -> "Q8Weight":
        """Random-init Q8_0 weight generated on the device (axq8_synth_q8_0)."""
        w = cls.empty(N, K, device)
        with torch.cuda.device(w.rows.device):
            check(_lib.load().axq8_synth_q8_0(seed, N, K, mean, std, 1,
                                              C.c_void_p(w.rows.data_ptr()),
                                              C.c_void_p(_stream())))
        return w

    def dequantize(self) -> torch.Tensor:
        """fp32 [N, K]: the values GGUFLoader::load_tensor gives for this tensor."""
        out = torch.empty(self.N, self.K, dtype=torch.float32, device=self.rows.device)
        with torch.cuda.device(self.rows.device):
            check(_lib.load().axq8_dequantize(self.c, C.c_void_p(out.data_ptr()),
                                              C.c_void_p(_stream())))
        return out

    def blocks_host(self) -> np.ndarray:
        """The weight back in GGUF block order (host bytes), for round-trip checks."""
        rs = row_stride(self.K)
        nb = self.K // QK
        rows = self.rows.view(self.N, rs).cpu().numpy()
        out = np.empty((self.N, nb, Q8_0_BYTES), dtype=np.uint8)
        out[:, :, 2:] = rows[:, :self.K].reshape(self.N, nb, QK)
        out[:, :, :2] = rows[:, self.K:self.K + 2 * nb].reshape(self.N, nb, 2)
        return out.reshape(-1)


def synth_q8_0_blocks(seed: int, N: int, K: int, std: float = 0.02, mean: float = 0.0,
                      device=None) -> torch.Tensor:
    """Device-generated random-init weight in GGUF block layout (uint8 CUDA)."""
    dev = torch.device(device) if device is not None else torch.device("cuda")
    out = torch.empty(N * (K // QK) * Q8_0_BYTES, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        check(_lib.load().axq8_synth_q8_0(seed, N, K, mean, std, 0, C.c_void_p(out.data_ptr()),
                                          C.c_void_p(_stream())))
    return out


def _check_linear_shapes(input: torch.Tensor, N: int, K: int) -> None:
    if input.dim() != 2:
        raise RuntimeError("linear_from_gguf expects 2D input [M,K] and weight [N,K]")
    if input.shape[1] != K:
        raise RuntimeError("linear_from_gguf dimension mismatch: input K != weight K")


ACT_MODES = {"q8": _lib.AXQ8_ACT_Q8, "f32": _lib.AXQ8_ACT_F32}


def linear_from_gguf(input: torch.Tensor, weight: Q8Weight, act_mode: str = "q8") -> torch.Tensor:
    """out[M, N] = input[M, K] . weight[N, K]^T with the weight kept in Q8_0.

    act_mode "q8": activations quantized to Q8 blocks, exact int32 block dots
    (the decode default); "f32": fp32 activations against the dequantized
    weight, the reference's own arithmetic.
    """
    if not isinstance(weight, Q8Weight):
        raise RuntimeError("linear_from_gguf expects 2D input [M,K] and weight [N,K]")
    _require_cuda(input, "linear_from_gguf input")
    _check_linear_shapes(input, weight.N, weight.K)
    if input.dtype != torch.float32:
        raise RuntimeError("linear_from_gguf: input must be float32")
    x = input.contiguous()
    M = x.shape[0]
    out = torch.empty(M, weight.N, dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        check(_lib.load().axq8_linear(weight.c, C.c_void_p(x.data_ptr()), M,
                                      C.c_void_p(out.data_ptr()), ACT_MODES[act_mode],
                                      C.c_void_p(_stream())))
    return out


def quantize_activations(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """A8 quantization: (xq int8 [M,K], dx fp32 [M,K/32])."""
    _require_cuda(x, "quantize_activations input")
    if x.dim() != 2 or x.shape[1] % QK or x.dtype != torch.float32:
        raise RuntimeError("quantize_activations expects float32 [M, K] with K % 32 == 0")
    x = x.contiguous()
    M, K = x.shape
    xq = torch.empty(M, K, dtype=torch.int8, device=x.device)
    dx = torch.empty(M, K // QK, dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        check(_lib.load().axq8_quantize_act(C.c_void_p(x.data_ptr()), M, K,
                                            C.c_void_p(xq.data_ptr()), C.c_void_p(dx.data_ptr()),
                                            C.c_void_p(_stream())))
    return xq, dx


def linear_q8act(weight: Q8Weight, xq: torch.Tensor, dx: torch.Tensor,
                 residual: torch.Tensor | None = None) -> torch.Tensor:
    """y = residual + dequant(xq, dx) . W^T with exact int32 block dots."""
    _require_cuda(xq, "xq")
    M = xq.shape[0]
    if xq.shape[1] != weight.K:
        raise RuntimeError("linear_from_gguf dimension mismatch: input K != weight K")
    out = torch.empty(M, weight.N, dtype=torch.float32, device=xq.device)
    res = residual.contiguous() if residual is not None else None
    with torch.cuda.device(xq.device):
        check(_lib.load().axq8_linear_q8act(weight.c, C.c_void_p(xq.data_ptr()),
                                            C.c_void_p(dx.data_ptr()), M,
                                            C.c_void_p(_ptr(res)) if res is not None else None,
                                            C.c_void_p(out.data_ptr()), C.c_void_p(_stream())))
    return out


def block_dots(weight: Q8Weight, xq: torch.Tensor) -> torch.Tensor:
    """Exact int32 block dot products [M, N, K/32]."""
    _require_cuda(xq, "xq")
    M = xq.shape[0]
    out = torch.empty(M, weight.N, weight.K // QK, dtype=torch.int32, device=xq.device)
    with torch.cuda.device(xq.device):
        check(_lib.load().axq8_block_dots(weight.c, C.c_void_p(xq.contiguous().data_ptr()), M,
                                          C.c_void_p(out.data_ptr()), C.c_void_p(_stream())))
    return out


PATHS = {_lib.AXQ8_PATH_GEMV: "gemv", _lib.AXQ8_PATH_TENSOR_CORE: "tensor_core",
         _lib.AXQ8_PATH_SKINNY: "skinny"}


def linear_path(weight: Q8Weight, M: int, act_mode: str = "q8") -> str:
    """Which kernel linear_from_gguf runs at M rows: "gemv", "skinny" (decode
    widths) or "tensor_core" (tcgen05)."""
    rc = _lib.load().axq8_linear_path(weight.c, M, ACT_MODES[act_mode])
    if rc < 0:
        check(rc)
    return PATHS[rc]


def scale_pitch(M: int) -> int:
    """Row pitch of the transposed activation scales (M rounded up to 4)."""
    return (M + 3) // 4 * 4


def quantize_activations_t(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """A8 quantization for the tensor-core product: (xq int8 [M,K],
    dxT fp32 [K/32, Mp]) with the scales transposed."""
    _require_cuda(x, "quantize_activations_t input")
    if x.dim() != 2 or x.shape[1] % QK or x.dtype != torch.float32:
        raise RuntimeError("quantize_activations_t expects float32 [M, K] with K % 32 == 0")
    x = x.contiguous()
    M, K = x.shape
    xq = torch.empty(M, K, dtype=torch.int8, device=x.device)
    dxT = torch.empty(K // QK, scale_pitch(M), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        check(_lib.load().axq8_quantize_act_t(C.c_void_p(x.data_ptr()), M, K,
                                              C.c_void_p(xq.data_ptr()),
                                              C.c_void_p(dxT.data_ptr()), C.c_void_p(_stream())))
    return xq, dxT


def linear_q8act_t(weight: Q8Weight, xq: torch.Tensor, dxT: torch.Tensor,
                   residual: torch.Tensor | None = None) -> torch.Tensor:
    """Tensor-core product y = residual + dequant(xq, dxT) . W^T (M >= 32)."""
    _require_cuda(xq, "xq")
    M = xq.shape[0]
    if xq.shape[1] != weight.K:
        raise RuntimeError("linear_from_gguf dimension mismatch: input K != weight K")
    out = torch.empty(M, weight.N, dtype=torch.float32, device=xq.device)
    res = residual.contiguous() if residual is not None else None
    with torch.cuda.device(xq.device):
        check(_lib.load().axq8_linear_q8act_t(weight.c, C.c_void_p(xq.data_ptr()),
                                              C.c_void_p(dxT.data_ptr()), M,
                                              C.c_void_p(_ptr(res)) if res is not None else None,
                                              C.c_void_p(out.data_ptr()), C.c_void_p(_stream())))
    return out


def linear_q8act_s(weight: Q8Weight, xq: torch.Tensor, dxT: torch.Tensor,
                   residual: torch.Tensor | None = None) -> torch.Tensor:
    """Skinny tensor-core product (1 <= M <= 64), same inputs as linear_q8act_t."""
    _require_cuda(xq, "xq")
    M = xq.shape[0]
    if xq.shape[1] != weight.K:
        raise RuntimeError("linear_from_gguf dimension mismatch: input K != weight K")
    out = torch.empty(M, weight.N, dtype=torch.float32, device=xq.device)
    res = residual.contiguous() if residual is not None else None
    with torch.cuda.device(xq.device):
        check(_lib.load().axq8_linear_q8act_s(weight.c, C.c_void_p(xq.data_ptr()),
                                              C.c_void_p(dxT.data_ptr()), M,
                                              C.c_void_p(_ptr(res)) if res is not None else None,
                                              C.c_void_p(out.data_ptr()), C.c_void_p(_stream())))
    return out


def block_dots_tc(weight: Q8Weight, xq: torch.Tensor,
                  dxT: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Block dots read back from the tensor cores: (dots int32 [M, N, K/32], y)."""
    _require_cuda(xq, "xq")
    M = xq.shape[0]
    dots = torch.empty(M, weight.N, weight.K // QK, dtype=torch.int32, device=xq.device)
    y = torch.empty(M, weight.N, dtype=torch.float32, device=xq.device)
    with torch.cuda.device(xq.device):
        check(_lib.load().axq8_block_dots_tc(weight.c, C.c_void_p(xq.contiguous().data_ptr()),
                                             C.c_void_p(dxT.data_ptr()), M,
                                             C.c_void_p(dots.data_ptr()), C.c_void_p(y.data_ptr()),
                                             C.c_void_p(_stream())))
    return dots, y


class QuantType(enum.Enum):
    """Runtime per-tensor formats (quantized_matmul.hpp:14-19); Q8_0 runs on device."""
    FP32 = 0
    Q4_0 = 1
    Q8_0 = 2
    Q8_1 = 3


@dataclass
class QuantizedWeight:
    """A weight [K, N] in a per-tensor runtime format (quantized_matmul.hpp:22-34)."""
    type: QuantType
    K: int
    N: int
    q8: torch.Tensor          # int8 [K, N] on the device
    scale_dev: torch.Tensor   # fp32 [1] on the device

    @property
    def scale(self) -> float:
        return float(self.scale_dev.item())

    def payload_bytes(self) -> int:
        return self.q8.numel()


def quantize_weight(weight: torch.Tensor, type: QuantType = QuantType.Q8_0) -> QuantizedWeight:
    """quantize_weight (quantized_matmul.cpp:35-108) for QuantType.Q8_0."""
    if weight.dim() != 2:
        raise RuntimeError("quantize_weight expects a 2D [K, N] weight")
    if type != QuantType.Q8_0:
        raise RuntimeError(f"quantize_weight: {type.name} is not implemented on the device")
    _require_cuda(weight, "quantize_weight weight")
    w = weight.contiguous().float()
    K, N = w.shape
    q = torch.empty(K, N, dtype=torch.int8, device=w.device)
    s = torch.empty(1, dtype=torch.float32, device=w.device)
    with torch.cuda.device(w.device):
        check(_lib.load().axq8_quantize_weight_tensor(C.c_void_p(w.data_ptr()), K, N,
                                                      C.c_void_p(q.data_ptr()),
                                                      C.c_void_p(s.data_ptr()),
                                                      C.c_void_p(_stream())))
    return QuantizedWeight(QuantType.Q8_0, K, N, q, s)


def quantized_matmul(input: torch.Tensor, W: QuantizedWeight) -> torch.Tensor:
    """quantized_matmul (quantized_matmul.cpp:110-204), Q8_0: out = (x . q) * scale."""
    if input.dim() != 2:
        raise RuntimeError("quantized_matmul expects a 2D [M, K] input")
    if input.shape[1] != W.K:
        raise RuntimeError("quantized_matmul dimension mismatch (K)")
    _require_cuda(input, "quantized_matmul input")
    x = input.contiguous().float()
    M = x.shape[0]
    out = torch.empty(M, W.N, dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        check(_lib.load().axq8_quantized_matmul(C.c_void_p(x.data_ptr()), M, W.K,
                                                C.c_void_p(W.q8.data_ptr()),
                                                C.c_void_p(W.scale_dev.data_ptr()), W.N,
                                                C.c_void_p(out.data_ptr()), C.c_void_p(_stream())))
    return out


def status() -> int:
    """Device status word (0, or the code of a bounded wait that gave up)."""
    code = C.c_int(0)
    check(_lib.load().axq8_status_read(C.byref(code)))
    return code.value


def status_clear() -> None:
    check(_lib.load().axq8_status_clear())
