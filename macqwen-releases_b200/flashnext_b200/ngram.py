"""Quantized embedding and n-gram rows gathered from HBM-resident tables.

Replaces ``models/flashnext/ngram.py``: ``StreamingQuantizedEmbedding``
(ngram.py:28-69, also the streamed input embedding of loader.py:266-283) and
``StreamingShardedEmbedding`` (ngram.py:82-188).  The reference keeps these
tables on disk and, per lookup, reads the requested packed rows and runs
``mx.dequantize`` on them.  Here each table is loaded into HBM once -- the
shards of a sharded table concatenated in shard order -- and a lookup is one
``fnmoe_rows_dequantize`` launch: a warp per row gathers the packed row, its
scales and biases, and writes ``bf16(s*q + b)``.  Indices stay on the device.

Index semantics follow the sharded lookup (ngram.py:106-119): an index in
``[0, rows)`` reads that row; any other index reads shard 0's row
``clamp(index, 0, shard0_rows - 1)``.  (The single-table reference class would
fail or wrap on such an index; here it is clamped the same way.)
"""
from __future__ import annotations

import ctypes

from . import _lib
from .cuda_runtime import _stream


def _torch():
    import torch

    return torch


def infer_quantization(store, prefix: str, dims: int) -> tuple[int, int]:
    """(group_size, bits) from the packed and scale widths (ngram.py:19-25)."""
    packed = store.shape(f"{prefix}.weight")[-1]
    groups = store.shape(f"{prefix}.scales")[-1]
    return dims // groups, packed * 32 // dims


def rows_dequantize(weight, scales, biases, indices, dims: int, bits: int, group_size: int, *,
                    first_shard_rows: int | None = None, out=None):
    """Gather and dequantise rows of a device table.

    ``weight`` [rows, dims * bits / 32] int32/uint32, ``scales``/``biases``
    [rows, dims / group_size] bf16, ``indices`` any integer shape (device or
    host) -> ``[*indices.shape, dims]`` bf16 on the table's device."""
    torch = _torch()
    lib = _lib.ensure_device()
    dev = weight.device
    if weight.dtype not in (torch.int32, torch.uint32) or scales.dtype != torch.bfloat16 or \
            biases.dtype != torch.bfloat16:
        raise TypeError("weight must be int32/uint32 and scales/biases bfloat16")
    rows = int(weight.shape[0])
    if weight.dim() != 2 or int(weight.shape[1]) * 32 != dims * bits:
        raise ValueError("weight must be [rows, dims * bits / 32]")
    if tuple(scales.shape) != (rows, dims // group_size) or scales.shape != biases.shape:
        raise ValueError("scales and biases must be [rows, dims / group_size]")
    idx = torch.as_tensor(indices, device=dev).to(torch.int64).contiguous()
    shape = tuple(idx.shape)
    flat = idx.reshape(-1)
    if out is None:
        out = torch.empty((*shape, dims), dtype=torch.bfloat16, device=dev)
    if flat.numel() == 0:
        return out
    a = _lib.FnRowsArgs()
    a.abi_version = _lib.ABI_VERSION
    a.dims, a.bits, a.group_size = int(dims), int(bits), int(group_size)
    a.table_rows = rows
    a.first_shard_rows = rows if first_shard_rows is None else int(first_shard_rows)
    a.count = int(flat.numel())
    w, s, b = weight.contiguous(), scales.contiguous(), biases.contiguous()
    a.weight, a.scales, a.biases = w.data_ptr(), s.data_ptr(), b.data_ptr()
    a.indices, a.out = flat.data_ptr(), out.data_ptr()
    _lib.check(lib.fnmoe_rows_dequantize(ctypes.byref(a), _stream()), "rows_dequantize")
    return out


class StreamingQuantizedEmbedding:
    """A quantized embedding table resident in HBM (ngram.py:28-69).

    ``StreamingQuantizedEmbedding(store, prefix, dims, mode="affine")`` loads
    ``{prefix}.weight/.scales/.biases`` from a :class:`~.store.SafeTensorStore`
    (or any object with ``shape`` and ``to_device``); ``from_arrays`` takes
    device tensors directly.  Calling it with indices returns
    ``[*indices.shape, dims]`` bfloat16 rows."""

    def __init__(self, store, prefix: str, dims: int, mode: str = "affine", *, device="cuda"):
        if mode != "affine":
            raise ValueError("only the affine quantization mode is supported")
        self.prefix = prefix
        self.dims = int(dims)
        self.mode = mode
        self.group_size, self.bits = infer_quantization(store, prefix, self.dims)
        self.weight = store.to_device(f"{prefix}.weight", device)
        self.scales = store.to_device(f"{prefix}.scales", device)
        self.biases = store.to_device(f"{prefix}.biases", device)
        self.first_shard_rows = int(self.weight.shape[0])

    @classmethod
    def from_arrays(cls, weight, scales, biases, dims: int, mode: str = "affine"):
        self = cls.__new__(cls)
        if mode != "affine":
            raise ValueError("only the affine quantization mode is supported")
        self.prefix = None
        self.dims = int(dims)
        self.mode = mode
        self.bits = int(weight.shape[-1]) * 32 // self.dims
        self.group_size = self.dims // int(scales.shape[-1])
        self.weight, self.scales, self.biases = weight, scales, biases
        self.first_shard_rows = int(weight.shape[0])
        return self

    @property
    def rows(self) -> int:
        return int(self.weight.shape[0])

    def __call__(self, indices, out=None):
        return rows_dequantize(self.weight, self.scales, self.biases, indices, self.dims, self.bits,
                               self.group_size, first_shard_rows=self.first_shard_rows, out=out)


class StreamingShardedEmbedding:
    """Hashed n-gram rows spread over shards (ngram.py:82-188), held as one
    HBM table: the shards' rows concatenated in shard order, so global row
    ``offsets[k] + l`` is shard ``k``'s row ``l``.  ``shards`` are
    :class:`StreamingQuantizedEmbedding` tables of one quantization."""

    def __init__(self, shards, shard_sizes, dims: int):
        torch = _torch()
        self.shard_sizes = tuple(int(size) for size in shard_sizes)
        if len(self.shard_sizes) != len(shards) or not shards:
            raise ValueError("one size per shard is required")
        offsets = [0]
        for size in self.shard_sizes:
            offsets.append(offsets[-1] + size)
        self.shard_offsets = tuple(offsets)
        self.dims = int(dims)
        first = shards[0]
        self.bits, self.group_size = first.bits, first.group_size
        for shard, size in zip(shards, self.shard_sizes):
            if (shard.bits, shard.group_size, shard.dims) != (self.bits, self.group_size, self.dims):
                raise ValueError("every shard must share bits, group size and dims")
            if shard.rows != size:
                raise ValueError("shard_sizes disagree with the shards' row counts")
        self.weight = torch.cat([s.weight for s in shards])
        self.scales = torch.cat([s.scales for s in shards])
        self.biases = torch.cat([s.biases for s in shards])

    def __call__(self, indices, out=None):
        return rows_dequantize(self.weight, self.scales, self.biases, indices, self.dims, self.bits,
                               self.group_size, first_shard_rows=self.shard_sizes[0], out=out)
