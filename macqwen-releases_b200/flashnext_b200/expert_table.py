"""HBM-resident expert tables: the reference's slab-pack record layout on the GPU.

The reference streams experts from SSD into a slab pack / expert pool laid out
as a 4 KiB header followed by fixed-stride records of nine tensors
(``models/flashnext/slab_pack.py:1-25,96-153``; ``expert_pool.py:57-110``).
Kernels address a record in place when a route has bit 31 set
(``SLOT_BIT``, ``expert_pool.py:38``; pointer math ``metal_runtime.py:198-228``).

On a B200 the whole expert bank fits in HBM (48 layers x 512 experts at
3072/640 is 90.6 GB of 180 GB), so the table is simply filled once.  The
record layout generalises the reference's (which hard-codes hidden 2560 /
intermediate 640) to any shape; at 2560/640 the offsets and the 3,072,000 B
stride are identical to ``slab_pack.get_slab_layout``.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass

import numpy as np

HEADER_SIZE = 4096
SLOT_BIT = 0x80000000
HEADER_MAGIC = 0x4D4F4553  # "MOES" (slab_pack.py:50)
PARTS = (
    ("gate_proj", "weight"), ("gate_proj", "scales"), ("gate_proj", "biases"),
    ("up_proj", "weight"), ("up_proj", "scales"), ("up_proj", "biases"),
    ("down_proj", "weight"), ("down_proj", "scales"), ("down_proj", "biases"),
)


@dataclass(frozen=True)
class RecordLayout:
    """Byte layout of one expert record."""

    hidden_size: int
    inter_size: int
    group_size: int
    offsets: tuple[int, ...]   # nine part offsets, PARTS order
    sizes: tuple[int, ...]
    record_stride: int

    def offset(self, projection: str, part: str) -> int:
        return self.offsets[PARTS.index((projection, part))]

    def shape(self, projection: str, part: str) -> tuple[int, int]:
        rows, cols = self._rows_cols(projection)
        if part == "weight":
            return rows, cols // 8
        return rows, cols // self.group_size

    def _rows_cols(self, projection: str) -> tuple[int, int]:
        if projection == "down_proj":
            return self.hidden_size, self.inter_size
        return self.inter_size, self.hidden_size


def record_layout(hidden_size: int, inter_size: int, group_size: int = 32,
                  page: int = 4096) -> RecordLayout:
    """Record layout for the given shape (slab_pack.py:96-153, generalised).

    Parts follow gate/up/down x weight/scales/biases order, each at a 16-byte
    aligned offset; the stride is rounded up to ``page``.
    """
    if hidden_size % group_size or inter_size % group_size:
        raise ValueError("hidden and intermediate sizes must be group aligned")
    sizes = []
    for projection in ("gate_proj", "up_proj", "down_proj"):
        rows, cols = (hidden_size, inter_size) if projection == "down_proj" else (inter_size, hidden_size)
        sizes.extend([rows * cols // 2, rows * (cols // group_size) * 2, rows * (cols // group_size) * 2])
    offsets = []
    off = 0
    for size in sizes:
        off = (off + 15) & ~15
        offsets.append(off)
        off += size
    stride = -(-off // page) * page
    return RecordLayout(hidden_size, inter_size, group_size, tuple(offsets), tuple(sizes), stride)


def _as_u8(t):
    import torch

    return t.contiguous().view(torch.uint8).reshape(-1)


class ExpertTable:
    """A device buffer of ``records`` expert records plus a 4 KiB header.

    ``buffer`` is a ``torch.uint8`` CUDA tensor.  Rows are written with
    :meth:`write` (device-to-device copies); :meth:`routes` encodes record
    slots with bit 31 for the executor.
    """

    def __init__(self, records: int, hidden_size: int, inter_size: int,
                 group_size: int = 32, *, device=None, header_size: int = HEADER_SIZE):
        import torch

        if records <= 0:
            raise ValueError("records must be positive")
        self.layout = record_layout(hidden_size, inter_size, group_size)
        self.records = int(records)
        self.header_size = int(header_size)
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        total = self.header_size + self.records * self.layout.record_stride
        self.buffer = torch.zeros(total, dtype=torch.uint8, device=self.device)
        header = struct.pack("<IIIII", HEADER_MAGIC, 1 if group_size == 32 else 2, self.records,
                             self.layout.record_stride, self.header_size)
        self.buffer[: len(header)] = torch.frombuffer(bytearray(header), dtype=torch.uint8).to(self.device)

    @property
    def nbytes(self) -> int:
        return int(self.buffer.numel())

    def record_view(self, slot: int):
        base = self.header_size + slot * self.layout.record_stride
        return self.buffer[base: base + self.layout.record_stride]

    def write(self, slot: int, gate, up, down) -> None:
        """Copy one expert's (weight, scales, biases) triples into record ``slot``."""
        if not 0 <= slot < self.records:
            raise ValueError("slot outside the table")
        rec = self.record_view(slot)
        for i, t in enumerate((*gate, *up, *down)):
            data = _as_u8(t)
            if data.numel() != self.layout.sizes[i]:
                raise ValueError(f"part {PARTS[i]} has {data.numel()} bytes, layout wants {self.layout.sizes[i]}")
            off = self.layout.offsets[i]
            rec[off: off + data.numel()].copy_(data)

    def write_bank(self, gate, up, down, experts=None, slots=None) -> None:
        """Write experts of (E, rows, cols) projection arrays into the table."""
        n = int(gate[0].shape[0])
        experts = list(range(n)) if experts is None else list(experts)
        slots = list(range(len(experts))) if slots is None else list(slots)
        for e, s in zip(experts, slots):
            self.write(s, tuple(t[e] for t in gate), tuple(t[e] for t in up), tuple(t[e] for t in down))

    @classmethod
    def from_projections(cls, gate, up, down, group_size: int = 32, *, header_size: int = HEADER_SIZE):
        n, inter, hcols = (int(v) for v in gate[0].shape)
        table = cls(n, hcols * 8, inter, group_size, device=gate[0].device, header_size=header_size)
        table.write_bank(gate, up, down)
        return table

    def routes(self, slots) -> "object":
        """uint32 routes addressing ``slots`` in this table (bit 31 set)."""
        import torch

        s = torch.as_tensor(slots, dtype=torch.int64, device=self.device)
        if bool(((s < 0) | (s >= self.records)).any()):
            raise ValueError("slot outside the table")
        # int32 tensor carrying the uint32 bit pattern (bit 31 set).
        return ((s | SLOT_BIT) - (1 << 32)).to(torch.int32)

    def abi(self, lib_struct, *, header: bool = True):
        """Fill an FnExpertTable ctypes struct describing this table."""
        t = lib_struct()
        t.base = self.buffer.data_ptr()
        t.header_bytes = self.header_size if header else 0
        t.record_stride = self.layout.record_stride
        for i, off in enumerate(self.layout.offsets):
            t.part_offset[i] = off
        t.records = self.records
        return t


def reference_layout_matches(layout: RecordLayout, offsets, stride) -> bool:
    """True when ``layout`` equals a reference slab layout (offsets, stride)."""
    return tuple(int(o) for o in offsets) == layout.offsets and int(stride) == layout.record_stride


def host_records(gate, up, down, layout: RecordLayout) -> np.ndarray:
    """Pack NumPy projection arrays into expert-major records (no header)."""
    n = gate[0].shape[0]
    out = np.zeros(n * layout.record_stride, dtype=np.uint8)
    for e in range(n):
        for i, arr in enumerate((*gate, *up, *down)):
            payload = np.ascontiguousarray(arr[e]).view(np.uint8).reshape(-1)
            start = e * layout.record_stride + layout.offsets[i]
            out[start: start + payload.size] = payload
    return out
