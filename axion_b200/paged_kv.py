"""Paged KV cache over the C ABI of include/axkv.h, under the reference's names.

Mirrors PagedKVCache (inference/cpp/runtime/paged_kv.hpp:18-41, paged_kv.cpp):
``initialize(hidden, page)``, ``append(K, V)``, ``materialize_keys()``,
``materialize_values()``, for several sequences at once, plus the decode
attention over the cache (mha_attention_incremental, mha.cpp:227-285).  Pages
are fp16 (or fp32) per KV head, 16 tokens each, in device memory owned here;
sequence s owns pages s * max_blocks onwards (identity block table).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._lib import check


class PagedKVCache:
    page_size = 16

    def __init__(self, n_kv_heads: int, head_dim: int, max_seqs: int = 1, max_tokens: int = 4096,
                 kv_fp32: bool = False, device=None):
        self.n_kv_heads, self.head_dim = n_kv_heads, head_dim
        self.hidden_size = n_kv_heads * head_dim
        self.max_seqs = max_seqs
        self.max_blocks = (max_tokens + self.page_size - 1) // self.page_size
        dev = torch.device(device) if device is not None else torch.device("cuda")
        dt = torch.float32 if kv_fp32 else torch.float16
        n_pages = max_seqs * self.max_blocks
        shape = (n_pages, n_kv_heads, self.page_size, head_dim)
        self.k = torch.zeros(shape, dtype=dt, device=dev)
        self.v = torch.zeros(shape, dtype=dt, device=dev)
        self.block_table = torch.arange(n_pages, dtype=torch.int32, device=dev)
        self.used = [0] * max_seqs
        self.c = _lib.axkv_cache_t(self.k.data_ptr(), self.v.data_ptr(),
                                   self.block_table.data_ptr(), n_pages, self.max_blocks,
                                   n_kv_heads, head_dim, self.page_size, 1 if kv_fp32 else 0)
        self._ws = None
        self._lib = _lib.load()

    def initialize(self, hidden: int, page: int = 16) -> None:
        """PagedKVCache::initialize: empties the cache; hidden must be
        n_kv_heads * head_dim and page 16 (the device page)."""
        if hidden != self.hidden_size or page != self.page_size:
            raise RuntimeError(f"PagedKVCache: hidden {hidden} / page {page} do not match "
                               f"{self.hidden_size} / {self.page_size}")
        self.used = [0] * self.max_seqs

    def _stream(self) -> C.c_void_p:
        return C.c_void_p(torch.cuda.current_stream(self.k.device).cuda_stream)

    def append(self, K: torch.Tensor, V: torch.Tensor, seq: int = 0) -> None:
        """Append rows K, V [rows, hidden] (fp32, device) to sequence `seq`."""
        if K.shape != V.shape or K.dim() != 2 or K.shape[1] != self.hidden_size:
            raise RuntimeError("PagedKVCache::append: K and V must be [rows, hidden]")
        n = K.shape[0]
        if self.used[seq] + n > self.max_blocks * self.page_size:
            raise RuntimeError("PagedKVCache::append: sequence full")
        pos = torch.arange(self.used[seq], self.used[seq] + n, dtype=torch.int32,
                           device=self.k.device)
        sq = torch.full((n,), seq, dtype=torch.int32, device=self.k.device)
        Kc, Vc = K.float().contiguous(), V.float().contiguous()
        check(self._lib.axkv_paged_append(C.byref(self.c), C.c_void_p(Kc.data_ptr()),
                                          C.c_void_p(Vc.data_ptr()), n, C.c_void_p(sq.data_ptr()),
                                          C.c_void_p(pos.data_ptr()), self._stream()))
        self.used[seq] += n

    def _gather(self, pages: torch.Tensor, seq: int) -> torch.Tensor:
        n = self.used[seq]
        nb = (n + self.page_size - 1) // self.page_size
        p = pages[seq * self.max_blocks: seq * self.max_blocks + nb]      # [nb, kv, 16, hd]
        return p.permute(0, 2, 1, 3).reshape(nb * self.page_size, self.hidden_size)[:n].float()

    def materialize_keys(self, seq: int = 0) -> torch.Tensor:
        return self._gather(self.k, seq)

    def materialize_values(self, seq: int = 0) -> torch.Tensor:
        return self._gather(self.v, seq)

    def attention(self, q: torch.Tensor, n_heads: int) -> torch.Tensor:
        """Decode attention of one query row per sequence ([n_seq, n_heads *
        head_dim], fp32, device) over all its cached tokens."""
        n_seq = q.shape[0]
        qpos = torch.tensor([self.used[s] - 1 for s in range(n_seq)], dtype=torch.int32,
                            device=self.k.device)
        if min(self.used[:n_seq]) <= 0:
            raise RuntimeError("PagedKVCache: attention over an empty sequence")
        need = self._lib.axkv_decode_attn_workspace(C.byref(self.c), n_seq, n_heads)
        if need < 0:
            raise RuntimeError("PagedKVCache: unsupported attention shape")
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.zeros(need, dtype=torch.uint8, device=self.k.device)
        qc = q.float().contiguous()
        out = torch.empty_like(qc)
        check(self._lib.axkv_paged_decode_attn(C.byref(self.c), C.c_void_p(qc.data_ptr()), n_seq,
                                               n_heads, C.c_void_p(qpos.data_ptr()),
                                               C.c_void_p(out.data_ptr()),
                                               C.c_void_p(self._ws.data_ptr()), self._ws.numel(),
                                               self._stream()))
        return out

    def prefill_attention(self, q: torch.Tensor, n_heads: int, T: int, p0: int,
                          quantize: bool = False):
        """Causal attention (mha_attention, mha.cpp:126-198) of positions p0 ..
        p0 + T - 1 of every sequence: q rows [n_seq * T, n_heads * head_dim]
        (row s * T + t = sequence s, position p0 + t), their K/V already
        appended.  quantize: (xq int8 rows, dxT transposed block scales) for
        the next Q8_0 product instead of fp32 rows."""
        n_seq = q.shape[0] // T
        if n_seq * T != q.shape[0] or any(self.used[s] < p0 + T for s in range(n_seq)):
            raise RuntimeError("PagedKVCache: prefill rows must be appended first")
        qc = q.float().contiguous()
        dev = self.k.device
        if quantize:
            rows, width = qc.shape[0], n_heads * self.head_dim
            xq = torch.empty(rows, width, dtype=torch.int8, device=dev)
            dxT = torch.empty(width // 32, (rows + 3) // 4 * 4, dtype=torch.float32, device=dev)
            check(self._lib.axkv_paged_prefill_attn(
                C.byref(self.c), C.c_void_p(qc.data_ptr()), qc.shape[1], n_seq, T, p0, n_heads,
                None, C.c_void_p(xq.data_ptr()), C.c_void_p(dxT.data_ptr()), self._stream()))
            return xq, dxT
        out = torch.empty_like(qc)
        check(self._lib.axkv_paged_prefill_attn(C.byref(self.c), C.c_void_p(qc.data_ptr()),
                                                qc.shape[1], n_seq, T, p0, n_heads,
                                                C.c_void_p(out.data_ptr()), None, None,
                                                self._stream()))
        return out
