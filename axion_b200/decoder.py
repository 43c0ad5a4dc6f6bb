"""Llama-architecture greedy decoder over the C ABI of include/axdec.h.

Mirrors the reference's ``ModelRunner`` (inference/cpp/runtime/model_runner.hpp:39-106):
configuration resolved from GGUF metadata the same way (``resolve_config``,
model_runner.cpp:22-97), ``generate`` with greedy sampling, plus a
teacher-forced logits mode for parity tests.  Weights are uploaded once and
stay on the device.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import check
from .gguf import F32, Q8_0, GGUFLoader


@dataclass
class DecoderConfig:
    n_layers: int
    hidden: int
    ffn: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    vocab: int
    rope_theta: float = 10000.0
    rms_eps: float = 1e-5
    max_batch: int = 1
    max_ctx: int = 512
    kv_block: int = 16
    act_mode: str = "q8"         # "q8" (A8, decode default) or "f32" (reference arithmetic)
    kv_fp32: bool = False        # fp16 KV pages by default
    tp_size: int = 1             # tensor-parallel ranks (one process per GPU)
    tp_rank: int = 0

    def c(self) -> _lib.axdec_config_t:
        return _lib.axdec_config_t(
            self.n_layers, self.hidden, self.ffn, self.n_heads, self.n_kv_heads, self.head_dim,
            self.vocab, self.rope_theta, self.rms_eps, self.max_batch, self.max_ctx,
            self.kv_block, _lib.AXQ8_ACT_Q8 if self.act_mode == "q8" else _lib.AXQ8_ACT_F32,
            1 if self.kv_fp32 else 0, self.tp_size, self.tp_rank)

    @property
    def vocab_local(self) -> int:
        """Vocabulary rows of this rank's LM-head slice (logits width)."""
        return self.vocab // max(1, self.tp_size)


def config_from_gguf(g: GGUFLoader, **kw) -> DecoderConfig:
    """resolve_config (model_runner.cpp:22-97) on our loader."""
    a = g.architecture() or "llama"
    n_heads = g.get_u32(f"{a}.attention.head_count", 1) or 1
    hidden = g.get_u32(f"{a}.embedding_length", 0)
    hd = g.get_u32(f"{a}.rope.dimension_count", 0) or (hidden // n_heads if hidden else 0)
    vocab = g.get_u32(f"{a}.vocab_size", 0) or g.get_arr_len("tokenizer.ggml.tokens", 0) \
        or g.tensor_shape("token_embd.weight")[0]
    ffn = g.get_u32(f"{a}.feed_forward_length", 0) or g.tensor_shape("blk.0.ffn_up.weight")[0]
    return DecoderConfig(
        n_layers=g.get_u32(f"{a}.block_count", 0), hidden=hidden, ffn=ffn, n_heads=n_heads,
        n_kv_heads=g.get_u32(f"{a}.attention.head_count_kv", n_heads), head_dim=hd, vocab=vocab,
        rope_theta=g.get_f32(f"{a}.rope.freq_base", 10000.0),
        rms_eps=g.get_f32(f"{a}.attention.layer_norm_rms_epsilon", 1e-6), **kw)


class Decoder:
    def __init__(self, cfg: DecoderConfig):
        import torch  # noqa: F401  (initialises the CUDA context torch also uses)
        self.cfg = cfg
        self.lib = _lib.load()
        self._cc = cfg.c()
        h = C.c_void_p()
        check(self.lib.axdec_create(C.byref(self._cc), C.byref(h)))
        self.h = h

    def close(self) -> None:
        if self.h:
            self.lib.axdec_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- weights ---------------------------------------------------------------
    @classmethod
    def from_gguf(cls, path, **kw) -> "Decoder":
        g = GGUFLoader()
        g.load_file(path)
        d = cls(config_from_gguf(g, **kw))
        for name in g.tensor_names():
            info = g.tensor_info(name)
            if info.type not in (Q8_0, F32):
                raise RuntimeError(f"{name}: GGUF type {info.type} not supported (Q8_0/F32)")
            raw = np.ascontiguousarray(g.load_tensor_raw(name))
            rows, cols = (info.shape if len(info.shape) == 2 else (1, info.shape[0]))
            check(d.lib.axdec_set_tensor(d.h, name.encode(), raw.ctypes.data_as(C.c_void_p),
                                         info.type, rows, cols))
        return d

    def init_random(self, seed: int, std: float = 0.02) -> None:
        check(self.lib.axdec_init_random(self.h, seed, std))

    def tensor_index(self, name: str) -> int:
        return self.lib.axdec_tensor_index(C.byref(self._cc), name.encode())

    @property
    def device_bytes(self) -> int:
        return self.lib.axdec_device_bytes(self.h)

    @property
    def weight_bytes_per_step(self) -> int:
        return self.lib.axdec_weight_bytes_per_step(self.h)

    # -- tensor parallelism ---------------------------------------------------------
    def tp_connect(self, group=None) -> None:
        """Join the tensor-parallel communicator: rank 0 draws the NCCL id,
        every rank of `group` (torch.distributed, any backend) receives it and
        connects.  Collective over the tp_size ranks."""
        if self.cfg.tp_size <= 1:
            return
        uid = share_tp_id(self.cfg.tp_rank, self._new_id, group)
        buf = (C.c_ubyte * len(uid)).from_buffer_copy(uid)
        check(self.lib.axdec_tp_connect(self.h, C.cast(buf, C.c_void_p)))

    @property
    def tp_allreduce(self) -> str:
        """Hidden-state all-reduce in use: "none", "nccl" or "nvlink"."""
        return ("none", "nccl", "nvlink")[self.lib.axdec_tp_allreduce_kind(self.h)]

    def tp_health(self) -> tuple[int, int]:
        """(NCCL asynchronous error, device status word), without a device sync."""
        e, st = C.c_int(0), C.c_int(0)
        check(self.lib.axdec_tp_health(self.h, C.byref(e), C.byref(st)))
        return e.value, st.value

    def tp_abort(self) -> None:
        """Abort the communicator (a peer failed); tp_connect again before stepping."""
        check(self.lib.axdec_tp_abort(self.h))

    def _new_id(self) -> bytes:
        buf = (C.c_ubyte * 128)()
        check(self.lib.axdec_tp_unique_id(C.cast(buf, C.c_void_p), 128))
        return bytes(buf)

    def step_kernels(self, n_seq: int = 1) -> int:
        """Kernels one decode step of n_seq sequences launches (-1 before the
        first generate/forced call with that n_seq)."""
        return self.lib.axdec_step_kernels(self.h, n_seq)

    # -- decoding --------------------------------------------------------------
    def generate(self, prompts, n_new: int, logits: bool = False, stream=None):
        """Greedy continuation of prompts [n_seq, n_prompt] (or one prompt).
        Returns (tokens [n_seq, n_new], logits [n_new, n_seq, vocab] | None,
        decode_ms of the n_new generation steps)."""
        p = np.ascontiguousarray(np.atleast_2d(np.asarray(prompts, np.int32)))
        n_seq, n_prompt = p.shape
        out = np.empty((n_seq, n_new), np.int32)
        lg = np.empty((n_new, n_seq, self.cfg.vocab_local), np.float32) if logits else None
        ms = C.c_float(0)
        check(self.lib.axdec_generate(
            self.h, p.ctypes.data_as(C.c_void_p), n_seq, n_prompt, n_new,
            out.ctypes.data_as(C.c_void_p),
            lg.ctypes.data_as(C.c_void_p) if lg is not None else None, C.byref(ms),
            C.c_void_p(stream) if stream else None))
        return out, lg, ms.value

    def set_prefill(self, batched: bool) -> None:
        """Batched prefill of prompts (default, where supported) or one
        position at a time through the decode step."""
        check(self.lib.axdec_set_prefill(self.h, 1 if batched else 0))

    def prefill_batched(self, n_seq: int) -> bool:
        return bool(self.lib.axdec_prefill_batched(self.h, n_seq))

    def prefill(self, tokens, stream=None) -> None:
        """Start a step-wise session: tokens [n_seq, n_tok] fill the KV cache
        at positions 0 .. n_tok - 1 (StreamingExecutor::begin_decode plus the
        prompt); decode_step continues at position n_tok."""
        t = np.ascontiguousarray(np.atleast_2d(np.asarray(tokens, np.int32)))
        n_seq, n_tok = t.shape
        check(self.lib.axdec_prefill(self.h, t.ctypes.data_as(C.c_void_p), n_seq, n_tok,
                                     C.c_void_p(stream) if stream else None))

    def decode_step(self, tokens, logits: bool = False, stream=None):
        """One decode position for every sequence of the session
        (StreamingExecutor::decode_step): input token per sequence in, greedy
        next token per sequence out (and the step's logits [n_seq, vocab])."""
        t = np.ascontiguousarray(np.asarray(tokens, np.int32).reshape(-1))
        nxt = np.empty_like(t)
        lg = np.empty((t.size, self.cfg.vocab_local), np.float32) if logits else None
        check(self.lib.axdec_decode_step(self.h, t.ctypes.data_as(C.c_void_p), t.size,
                                         nxt.ctypes.data_as(C.c_void_p),
                                         lg.ctypes.data_as(C.c_void_p) if lg is not None else None,
                                         C.c_void_p(stream) if stream else None))
        return (nxt, lg) if logits else nxt

    def decode_step_ptr(self, tokens_ptr: int, n_seq: int, next_ptr: int, stream=None) -> None:
        """decode_step on caller-owned host buffers (e.g. pinned memory)."""
        check(self.lib.axdec_decode_step(self.h, C.c_void_p(tokens_ptr), n_seq,
                                         C.c_void_p(next_ptr), None,
                                         C.c_void_p(stream) if stream else None))

    def decode_continue(self, n_steps: int, n_seq: int, first=None, stream=None):
        """n_steps greedy steps of the session on the device, tokens fed back
        on the device; returns (tokens [n_seq, n_steps], device ms)."""
        out = np.empty((n_seq, n_steps), np.int32)
        f = None
        if first is not None:
            f = np.ascontiguousarray(np.asarray(first, np.int32).reshape(-1))
            assert f.size == n_seq
        ms = C.c_float(0)
        check(self.lib.axdec_decode_continue(self.h, f.ctypes.data_as(C.c_void_p) if f is not None
                                             else None, n_seq, n_steps,
                                             out.ctypes.data_as(C.c_void_p), C.byref(ms),
                                             C.c_void_p(stream) if stream else None))
        return out, ms.value

    def forced(self, tokens, n_prompt: int, stream=None) -> np.ndarray:
        """Teacher-forced logits [n_steps - n_prompt + 1, n_seq, vocab] (this
        rank's vocabulary slice under tensor parallelism)."""
        t = np.ascontiguousarray(np.atleast_2d(np.asarray(tokens, np.int32)))
        n_seq, n_steps = t.shape
        lg = np.empty((n_steps - n_prompt + 1, n_seq, self.cfg.vocab_local), np.float32)
        check(self.lib.axdec_forced(self.h, t.ctypes.data_as(C.c_void_p), n_seq, n_prompt,
                                    n_steps, lg.ctypes.data_as(C.c_void_p),
                                    C.c_void_p(stream) if stream else None))
        return lg


_SLOTS = ("attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "ffn_norm", "ffn_gate",
          "ffn_up", "ffn_down")


def tensor_index(n_layers: int, name: str) -> int:
    """axdec_tensor_index without the library: token_embd 0, output 1,
    output_norm 2, then 3 + 9 * layer + slot (the per-tensor seed offset of
    axdec_init_random), -1 for an unknown name."""
    fixed = {"token_embd.weight": 0, "output.weight": 1, "output_norm.weight": 2}
    if name in fixed:
        return fixed[name]
    parts = name.split(".")
    if len(parts) != 4 or parts[0] != "blk" or parts[3] != "weight" or not parts[1].isdigit():
        return -1
    layer = int(parts[1])
    if layer >= n_layers or parts[2] not in _SLOTS:
        return -1
    return 3 + 9 * layer + _SLOTS.index(parts[2])


def share_tp_id(rank: int, make_id, group=None) -> bytes:
    """The communicator id of rank 0, on every rank of `group`: rank 0 calls
    make_id(), the bytes travel by a torch.distributed object broadcast."""
    import torch.distributed as dist
    obj = [make_id() if rank == 0 else None]
    src = 0 if group is None else dist.get_global_rank(group, 0)
    dist.broadcast_object_list(obj, src=src, group=group)
    uid = obj[0]
    if not isinstance(uid, (bytes, bytearray)) or len(uid) != 128:
        raise RuntimeError("tensor-parallel id exchange failed")
    return bytes(uid)
