"""Read-only view over a safetensors checkpoint, for filling HBM tables.

Mirrors the reading side of ``SafeTensorStore`` (``models/flashnext/
store.py:100-118,127-200,297-313,531-565,604``): the same constructor (a model
directory holding ``model.safetensors.index.json`` or one
``model.safetensors``), ``refs`` of ``TensorRef(shard, dtype, shape, start)``,
``shape(name)``, ``rows_np(name, rows)``, ``whole_np(name)``,
``empty_rows`` and ``expert_record_view``.  The reference streams expert rows
from this store on every decode step; on a B200 every table is loaded into HBM
once (``to_device``), so only positioned reads and the host -> device copy
remain.  No MLX: bfloat16 tensors come back as ``uint16`` arrays (the
reference's NumPy view of them too) and as ``torch.bfloat16`` on the device.
"""
from __future__ import annotations

import json
import mmap
import os
import struct
from typing import Sequence

import numpy as np

# safetensors dtype -> NumPy dtype of the raw bytes (store.py:28-41)
DTYPES = {
    "F32": np.dtype("<f4"), "F16": np.dtype("<f2"), "BF16": np.dtype("<u2"), "U32": np.dtype("<u4"),
    "I32": np.dtype("<i4"), "I64": np.dtype("<i8"), "U64": np.dtype("<u8"), "F64": np.dtype("<f8"),
    "BOOL": np.dtype("?"), "U16": np.dtype("<u2"), "U8": np.dtype("u1"), "I8": np.dtype("i1"),
}


class TensorRef:
    """Where one tensor lives: shard file, dtype, shape, absolute byte offset."""

    __slots__ = ("shard", "dtype", "shape", "start", "row_bytes")

    def __init__(self, shard: str, dtype: str, shape: Sequence[int], start: int):
        self.shard = shard
        self.dtype = dtype
        self.shape = tuple(int(v) for v in shape)
        self.start = int(start)
        trailing = int(np.prod(self.shape[1:])) if len(self.shape) > 1 else 1
        self.row_bytes = trailing * DTYPES[dtype].itemsize


def read_header(path: str) -> tuple[dict, int]:
    """(header dict, byte offset of the data section) of one safetensors file."""
    with open(path, "rb") as f:
        head = f.read(8)
        if len(head) != 8:
            raise ValueError(f"{path}: not a safetensors file")
        (n,) = struct.unpack("<Q", head)
        meta = json.loads(f.read(n))
    return meta, 8 + n


class SafeTensorStore:
    """Memory-mapped view over every shard of a safetensors checkpoint."""

    def __init__(self, model_dir: str):
        self.dir = os.path.expanduser(model_dir)
        self.refs: dict[str, TensorRef] = {}
        self._maps: dict[str, mmap.mmap] = {}
        index_path = os.path.join(self.dir, "model.safetensors.index.json")
        if os.path.exists(index_path):
            with open(index_path) as handle:
                shards = sorted(set(json.load(handle)["weight_map"].values()))
        elif os.path.exists(os.path.join(self.dir, "model.safetensors")):
            shards = ["model.safetensors"]
        else:
            raise FileNotFoundError(f"{self.dir}: no model.safetensors.index.json or model.safetensors")
        for shard in shards:
            self.add_shard(shard)

    def add_shard(self, shard: str) -> None:
        meta, data_start = read_header(os.path.join(self.dir, shard))
        for name, info in meta.items():
            if name == "__metadata__":
                continue
            if info["dtype"] not in DTYPES:
                raise ValueError(f"{name}: unsupported dtype {info['dtype']}")
            begin, end = (int(v) for v in info["data_offsets"])
            ref = TensorRef(shard, info["dtype"], info["shape"], data_start + begin)
            if end - begin != int(np.prod(ref.shape)) * DTYPES[ref.dtype].itemsize:
                raise ValueError(f"{name}: data_offsets disagree with shape and dtype")
            self.refs[name] = ref

    def _map(self, shard: str) -> mmap.mmap:
        m = self._maps.get(shard)
        if m is None:
            with open(os.path.join(self.dir, shard), "rb") as f:
                m = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
            self._maps[shard] = m
        return m

    def _view(self, name: str) -> np.ndarray:
        ref = self.refs[name]
        count = int(np.prod(ref.shape))
        return np.frombuffer(self._map(ref.shard), dtype=DTYPES[ref.dtype], count=count,
                             offset=ref.start).reshape(ref.shape)

    def shape(self, name: str) -> tuple[int, ...]:
        return self.refs[name].shape

    def rows_np(self, name: str, indices: Sequence[int]) -> np.ndarray:
        """The requested rows of ``name`` stacked along axis 0 (a copy)."""
        return np.ascontiguousarray(self._view(name)[list(indices)])

    def whole_np(self, name: str) -> np.ndarray:
        """The whole tensor as a read-only NumPy view of the mapped file."""
        return self._view(name)

    def empty_rows(self, name: str, count: int) -> np.ndarray:
        ref = self.refs[name]
        return np.empty((count, *ref.shape[1:]), dtype=DTYPES[ref.dtype])

    def expert_record_view(self, name: str, buffer: np.ndarray, count: int, offset: int,
                           record_stride: int) -> np.ndarray:
        """View one tensor row inside each expert-major record of ``buffer``
        (store.py:537-564)."""
        ref = self.refs[name]
        dtype = DTYPES[ref.dtype]
        if buffer.dtype != np.uint8 or not buffer.flags.c_contiguous:
            raise ValueError("expert record buffer must be contiguous uint8")
        if offset < 0 or record_stride < ref.row_bytes:
            raise ValueError("expert record layout cannot contain the tensor row")
        tail = []
        stride = dtype.itemsize
        for dim in reversed(ref.shape[1:]):
            tail.append(stride)
            stride *= dim
        tail.reverse()
        return np.ndarray(shape=(count, *ref.shape[1:]), dtype=dtype, buffer=buffer, offset=offset,
                          strides=(record_stride, *tail))

    def to_device(self, name: str, device="cuda", rows: Sequence[int] | None = None):
        """The tensor (or the given rows) as a torch tensor on ``device``:
        ``bfloat16`` for BF16, ``int32`` for U32 packed words (same bits), the
        matching dtype otherwise."""
        import torch

        ref = self.refs[name]
        host = self.whole_np(name) if rows is None else self.rows_np(name, rows)
        if ref.dtype == "U32":
            host = host.view(np.int32)
        elif ref.dtype in ("U16", "BF16"):
            host = host.view(np.int16)
        if not host.flags.writeable:  # a view of the read-only mapping
            host = np.array(host)
        t = torch.from_numpy(np.ascontiguousarray(host))
        if ref.dtype == "BF16":
            t = t.view(torch.bfloat16)
        return t.to(device)

    def close(self) -> None:
        for m in self._maps.values():
            m.close()
        self._maps.clear()
