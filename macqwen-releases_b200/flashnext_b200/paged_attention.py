"""Paged-KV decode attention on sm_100a.

Replaces the decode branch (L == 1) of ``paged_attention(queries, cache,
scale, mask)`` (``models/qwen27b/paged_kv.py:417-495``): per-page partial
softmax statistics in float32 merged online, output ``o / l`` in the query
dtype.  Here the cache is HBM-resident pages addressed through a block table
(bfloat16 K/V pages of ``page_size`` tokens, ``[pages, page_size, kv_heads,
head_dim]``), and the merge is a split-K flash decode: one CTA streams the
K/V rows of ``split_tokens`` contiguous tokens of one (sequence, kv head)
through a TMA ring into tensor-core MMAs, a second kernel merges the splits
of a sequence.
"""
from __future__ import annotations

import ctypes

from . import _lib
from .cuda_runtime import _bf16, _dev, _stream, _Workspace

_ws = _Workspace()


def _torch():
    import torch

    return torch


def auto_split(batch: int, kv_heads: int, capacity_tokens: int, sms: int = 148) -> int:
    """Tokens per split-K chunk: the longest power of two in [64, 2048]
    whose (sequence, kv head, split) work items -- counted at full capacity
    -- still give every SM three CTAs (1.5 waves of the two resident per
    SM).  Longer splits mean fewer CTA start-ups and partials to merge;
    enough items keep every SM streaming."""
    split = 2048
    while split > 64 and batch * kv_heads * -(-capacity_tokens // split) < 3 * sms:
        split //= 2
    return split


def paged_decode(q, k_cache, v_cache, block_table, context_lens, scale: float,
                 split_tokens: int | None = None, out=None, workspace=None):
    """q [B, Hq, D] bf16 -> out [B, Hq, D] bf16 (one query token per sequence).

    ``split_tokens`` defaults to :func:`auto_split` of the batch, kv heads
    and block-table capacity."""
    torch = _torch()
    lib = _lib.ensure_device()
    qt = _bf16(q, "q")
    kt = _bf16(k_cache, "k_cache")
    vt = _bf16(v_cache, "v_cache")
    bt = _dev(block_table, torch.int32)
    cl = _dev(context_lens, torch.int32)
    if qt.dim() != 3 or kt.dim() != 4 or kt.shape != vt.shape:
        raise ValueError("q must be [B, Hq, D] and caches [pages, page_size, Hkv, D]")
    batch, q_heads, head_dim = (int(v) for v in qt.shape)
    num_pages, page_size, kv_heads, kd = (int(v) for v in kt.shape)
    if kd != head_dim:
        raise ValueError("cache head_dim differs from q")
    if bt.dim() != 2 or bt.shape[0] != batch or cl.shape != (batch,):
        raise ValueError("block_table must be [B, max_pages] and context_lens [B]")
    a = _lib.FnPagedArgs()
    a.abi_version = _lib.ABI_VERSION
    a.batch, a.q_heads, a.kv_heads, a.head_dim = batch, q_heads, kv_heads, head_dim
    a.page_size, a.max_pages, a.num_pages = page_size, int(bt.shape[1]), num_pages
    a.scale = float(scale)
    if split_tokens is None:
        split_tokens = auto_split(batch, kv_heads, int(bt.shape[1]) * page_size,
                                  torch.cuda.get_device_properties(qt.device).multi_processor_count)
    a.split_tokens = int(split_tokens)
    a.q, a.k_cache, a.v_cache = qt.data_ptr(), kt.data_ptr(), vt.data_ptr()
    a.block_table, a.context_lens = bt.data_ptr(), cl.data_ptr()
    if out is None:
        out = torch.empty_like(qt)
    a.out = out.data_ptr()
    need = ctypes.c_uint64(0)
    _lib.check(lib.fnmoe_paged_decode_workspace_size(ctypes.byref(a), ctypes.byref(need)), "paged workspace")
    ws = workspace if workspace is not None else _ws.get(need.value)
    a.workspace = ws.data_ptr()
    a.workspace_bytes = ws.numel()
    _lib.check(lib.fnmoe_paged_decode(ctypes.byref(a), _stream()), "paged_decode")
    return out


class PagedKVCache:
    """HBM page pool + per-sequence block tables (decode-side of ``PagedKVCache``,
    ``models/qwen27b/paged_kv.py:54-400``, without SSD spill or page selection)."""

    def __init__(self, num_pages: int, page_size: int, kv_heads: int, head_dim: int,
                 max_pages_per_seq: int, batch: int, device="cuda"):
        torch = _torch()
        self.page_size = page_size
        self.k = torch.zeros((num_pages, page_size, kv_heads, head_dim), dtype=torch.bfloat16, device=device)
        self.v = torch.zeros_like(self.k)
        self.block_table = torch.full((batch, max_pages_per_seq), -1, dtype=torch.int32, device=device)
        self.context_lens = torch.zeros((batch,), dtype=torch.int32, device=device)
        self._free = list(range(num_pages - 1, -1, -1))
        self._host_lens = [0] * batch

    def append(self, seq: int, k, v) -> None:
        """Append K/V rows [n, kv_heads, head_dim] to sequence ``seq``."""
        n = int(k.shape[0])
        pos = self._host_lens[seq]
        done = 0
        while done < n:
            page_idx, slot = divmod(pos + done, self.page_size)
            if slot == 0:
                if not self._free:
                    raise RuntimeError("page pool exhausted")
                self.block_table[seq, page_idx] = self._free.pop()
            page = int(self.block_table[seq, page_idx])
            take = min(self.page_size - slot, n - done)
            self.k[page, slot:slot + take] = k[done:done + take]
            self.v[page, slot:slot + take] = v[done:done + take]
            done += take
        self._host_lens[seq] = pos + n
        self.context_lens[seq] = pos + n


def paged_attention(queries, cache: PagedKVCache, scale: float, mask=None):
    """Decode form of the reference ``paged_attention`` (paged_kv.py:417).

    ``queries`` [B, Hq, 1, D]; returns [B, Hq, 1, D].  Only the decode case
    (one query token, no mask) runs here; prefill uses a fused SDPA kernel in
    the reference and is outside this path.
    """
    if mask is not None or queries.shape[2] != 1:
        raise ValueError("paged decode attention takes one query token and no mask")
    q = queries[:, :, 0, :]
    out = paged_decode(q, cache.k, cache.v, cache.block_table, cache.context_lens, scale)
    return out.unsqueeze(2)
