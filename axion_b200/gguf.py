"""GGUF v3 reader and writer (host side of the Q8_0 weight boundary).

``GGUFLoader`` mirrors the reference loader's interface
(inference/cpp/gguf/gguf.hpp:87-210: load_file, tensor_names, tensor_shape,
get_u32/get_f32/get_str/get_arr_len, architecture) and the same on-disk rules
(gguf.cpp:643-758): dims are stored GGML-order (inner first) and reversed to
row-major ``[outer, ..., inner]``; the tensor data section starts at the next
32-byte boundary after the directory; Q8_0 tensors occupy (n/32)*34 bytes.
Unlike the reference, ``load_tensor_raw`` returns the undecoded blocks (a
read-only memory map), so Q8_0 weights can be uploaded once and kept in
their quantized form on the device instead of being re-read and dequantized
per token (gguf.cpp:784-882).

``GGUFWriter`` writes the files the tests and benchmarks feed to both the
reference loader and this one.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

GGUF_MAGIC = b"GGUF"
GGUF_VERSION = 3
ALIGNMENT = 32

# GGUFType (inference/cpp/gguf/gguf.hpp:13-28)
F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q8_1 = 0, 1, 2, 3, 6, 7, 8, 9
Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, Q8_K = 10, 11, 12, 13, 14, 15

# (elements per block, bytes per block): gguf.cpp:36-67
_BLOCK = {
    F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q4_1: (32, 20), Q5_0: (32, 22),
    Q5_1: (32, 24), Q8_0: (32, 34), Q8_1: (32, 36), Q2_K: (256, 84),
    Q3_K: (256, 110), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210),
    Q8_K: (256, 292),
}

# metadata value types
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)
_SCALAR = {_U8: "<B", _I8: "<b", _U16: "<H", _I16: "<h", _U32: "<I", _I32: "<i",
           _F32: "<f", _BOOL: "<?", _U64: "<Q", _I64: "<q", _F64: "<d"}


def tensor_byte_size(ggml_type: int, n: int) -> int:
    """gguf_tensor_byte_size (gguf.cpp:36-67)."""
    if ggml_type not in _BLOCK:
        raise RuntimeError("Unsupported GGUF tensor type")
    per, nbytes = _BLOCK[ggml_type]
    return (n // per) * nbytes


@dataclass
class TensorInfo:
    name: str
    type: int
    shape: tuple[int, ...]      # row-major [outer, ..., inner]
    offset: int                 # relative to the data section
    element_count: int
    byte_size: int


class GGUFLoader:
    """Parses a GGUF v3 file; tensor data is memory-mapped, never copied."""

    def __init__(self) -> None:
        self.path: Path | None = None
        self.version = 0
        self.metadata: dict[str, object] = {}
        self.tensors: dict[str, TensorInfo] = {}
        self.tensor_data_offset = 0
        self._map: np.memmap | None = None

    # -- parsing -------------------------------------------------------------
    def load_file(self, path: str | Path) -> bool:
        self.path = Path(path)
        if not self.path.is_file():
            raise RuntimeError("Failed to open GGUF")
        with open(self.path, "rb") as f:
            if f.read(4) != GGUF_MAGIC:
                raise RuntimeError("Invalid GGUF file")
            (self.version,) = struct.unpack("<I", _read(f, 4))
            n_tensors, n_kv = struct.unpack("<QQ", _read(f, 16))
            for _ in range(n_kv):
                key = _read_str(f)
                (vt,) = struct.unpack("<I", _read(f, 4))
                self.metadata[key] = _read_value(f, vt)
            for _ in range(n_tensors):
                name = _read_str(f)
                (nd,) = struct.unpack("<I", _read(f, 4))
                dims = struct.unpack(f"<{nd}Q", _read(f, 8 * nd)) if nd else ()
                ttype, off = struct.unpack("<IQ", _read(f, 12))
                n = 1
                for d in dims:
                    n *= d
                shape = tuple(int(d) for d in reversed(dims))
                self.tensors[name] = TensorInfo(name, ttype, shape, off, n,
                                                tensor_byte_size(ttype, n))
            pos = f.tell()
        self.tensor_data_offset = (pos + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT
        size = self.path.stat().st_size
        for t in self.tensors.values():
            if self.tensor_data_offset + t.offset + t.byte_size > size:
                raise RuntimeError(f"GGUF tensor {t.name} extends past end of file")
        self._map = np.memmap(self.path, dtype=np.uint8, mode="r")
        return True

    # -- accessors (gguf.hpp:96-206) -----------------------------------------
    def tensor_names(self) -> list[str]:
        return list(self.tensors)

    def tensor_shape(self, name: str) -> list[int]:
        t = self.tensors.get(name)
        return list(t.shape) if t else []

    def has_metadata(self, key: str) -> bool:
        return key in self.metadata

    def get_u32(self, key: str, fallback: int = 0) -> int:
        v = self.metadata.get(key)
        return int(v) if isinstance(v, (int, float, bool)) else fallback

    get_i32 = get_u32
    get_u64 = get_u32

    def get_f32(self, key: str, fallback: float = 0.0) -> float:
        v = self.metadata.get(key)
        return float(v) if isinstance(v, (int, float, bool)) else fallback

    def get_str(self, key: str, fallback: str = "") -> str:
        v = self.metadata.get(key)
        return v if isinstance(v, str) else fallback

    def get_arr_len(self, key: str, fallback: int = 0) -> int:
        v = self.metadata.get(key)
        return len(v) if isinstance(v, list) else fallback

    def architecture(self) -> str:
        return self.get_str("general.architecture", "")

    # -- tensor data ----------------------------------------------------------
    def load_tensor_raw(self, name: str) -> np.ndarray:
        """Undecoded bytes of `name` (read-only uint8 view of the file)."""
        t = self.tensors.get(name)
        if t is None:
            raise RuntimeError("Tensor not found")
        start = self.tensor_data_offset + t.offset
        return self._map[start:start + t.byte_size]

    def tensor_info(self, name: str) -> TensorInfo:
        t = self.tensors.get(name)
        if t is None:
            raise RuntimeError("Tensor not found")
        return t

    def load_tensor_f32(self, name: str) -> np.ndarray:
        """F32 / F16 tensors decoded on the host (norm weights)."""
        t = self.tensor_info(name)
        raw = self.load_tensor_raw(name)
        if t.type == F32:
            return np.frombuffer(raw, dtype="<f4").reshape(t.shape).copy()
        if t.type == F16:
            return np.frombuffer(raw, dtype="<f2").astype(np.float32).reshape(t.shape)
        raise RuntimeError(f"load_tensor_f32: {name} has quantized type {t.type}")


def _read(f, n: int) -> bytes:
    b = f.read(n)
    if len(b) != n:
        raise RuntimeError("Truncated GGUF file")
    return b


def _read_str(f) -> str:
    (n,) = struct.unpack("<Q", _read(f, 8))
    if n > (1 << 30):
        raise RuntimeError("Corrupt GGUF string length")
    return _read(f, n).decode("utf-8", errors="replace")


def _read_value(f, vt: int):
    if vt in _SCALAR:
        fmt = _SCALAR[vt]
        (v,) = struct.unpack(fmt, _read(f, struct.calcsize(fmt)))
        return v
    if vt == _STR:
        return _read_str(f)
    if vt == _ARR:
        et, n = struct.unpack("<IQ", _read(f, 12))
        if n > (1 << 31):
            raise RuntimeError("Corrupt GGUF array length")
        return [_read_value(f, et) for _ in range(n)]
    raise RuntimeError(f"Unknown GGUF metadata type {vt}")


class GGUFWriter:
    """Minimal GGUF v3 writer: scalar/string/array metadata and tensors."""

    def __init__(self) -> None:
        self._kv: list[tuple[str, int, object]] = []
        self._tensors: list[tuple[str, int, tuple[int, ...], bytes]] = []

    def add_u32(self, key: str, v: int) -> None:
        self._kv.append((key, _U32, int(v)))

    def add_f32(self, key: str, v: float) -> None:
        self._kv.append((key, _F32, float(v)))

    def add_string(self, key: str, v: str) -> None:
        self._kv.append((key, _STR, v))

    def add_str_array(self, key: str, v: list[str]) -> None:
        self._kv.append((key, _ARR, (_STR, list(v))))

    def add_tensor(self, name: str, data: bytes | np.ndarray, shape: tuple[int, ...],
                   ggml_type: int) -> None:
        """`shape` is row-major [outer, ..., inner]; stored reversed (GGML order)."""
        raw = data.tobytes() if isinstance(data, np.ndarray) else bytes(data)
        n = 1
        for d in shape:
            n *= int(d)
        if len(raw) != tensor_byte_size(ggml_type, n):
            raise ValueError(f"{name}: {len(raw)} bytes, expected "
                             f"{tensor_byte_size(ggml_type, n)}")
        self._tensors.append((name, ggml_type, tuple(int(d) for d in shape), raw))

    def write(self, path: str | Path) -> None:
        out = bytearray()
        out += GGUF_MAGIC + struct.pack("<IQQ", GGUF_VERSION, len(self._tensors), len(self._kv))
        for key, vt, v in self._kv:
            out += _pack_str(key) + struct.pack("<I", vt) + _pack_value(vt, v)
        offsets, off = [], 0
        for _, _, _, raw in self._tensors:
            offsets.append(off)
            off += (len(raw) + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT
        for (name, tt, shape, _), o in zip(self._tensors, offsets):
            dims = tuple(reversed(shape))
            out += _pack_str(name) + struct.pack(f"<I{len(dims)}Q", len(dims), *dims)
            out += struct.pack("<IQ", tt, o)
        out += b"\0" * ((-len(out)) % ALIGNMENT)
        with open(path, "wb") as f:
            f.write(out)
            for (_, _, _, raw), o in zip(self._tensors, offsets):
                f.write(raw)
                f.write(b"\0" * ((-len(raw)) % ALIGNMENT))


def _pack_str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _pack_value(vt: int, v) -> bytes:
    if vt in _SCALAR:
        return struct.pack(_SCALAR[vt], v)
    if vt == _STR:
        return _pack_str(v)
    if vt == _ARR:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(_pack_value(et, x) for x in items)
    raise ValueError(vt)
