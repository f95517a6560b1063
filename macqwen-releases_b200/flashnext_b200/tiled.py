"""HBM-resident tile-major expert tables for the decode kernels.

The reference keeps hot experts in packed records so a layer reads each
expert's projections with few large transfers (``models/flashnext/
slab_pack.py:96-153``, ``expert_pool.py:57-162``).  The B200 analogue repacks
a layer's experts once (``fnmoe_tile_experts``) into one 2560-byte chunk per
(row group, 128-byte block) in MMA fragment order -- 8 gate + 8 up rows for
gate/up, 16 rows for down, scales and biases included -- so that a warp moves
each block of its rows with a single bulk copy.  Records hold the routed
experts in order, then (optionally) the shared expert.
"""
from __future__ import annotations

import ctypes
from typing import Mapping

from . import _lib
from .cuda_runtime import _bf16, _dev, _stream


def _torch():
    import torch

    return torch


def _triple(p):
    if isinstance(p, Mapping):
        return p["weight"], p["scales"], p["biases"]
    return tuple(p)


def record_bytes(hidden: int, inter: int, group: int = 32):
    """(gate_up, down) bytes per tiled record."""
    lib = _lib.load()
    gu, dn = ctypes.c_uint64(0), ctypes.c_uint64(0)
    _lib.check(lib.fnmoe_tiled_record_bytes(hidden, inter, group, ctypes.byref(gu), ctypes.byref(dn)),
               "tiled_record_bytes")
    return int(gu.value), int(dn.value)


class TiledExperts:
    """Tiled copy of routed experts ``{gate_proj, up_proj, down_proj}`` (expert-major
    arrays) and, optionally, a shared expert (same mapping without the expert axis)."""

    def __init__(self, experts: Mapping, shared: Mapping | None = None, *, group_size: int = 32):
        torch = _torch()
        lib = _lib.ensure_device()
        parts = {}
        for name in ("gate_proj", "up_proj", "down_proj"):
            w, s, b = _triple(experts[name])
            parts[name] = (_dev(w), _bf16(s, f"{name} scales"), _bf16(b, f"{name} biases"))
        E, inter, hw = (int(v) for v in parts["gate_proj"][0].shape)
        self.hidden_size = hw * 8
        self.inter_size = inter
        self.group_size = int(group_size)
        self.expert_count = E
        self.has_shared = shared is not None
        self.records = E + (1 if self.has_shared else 0)
        self.gate_up_record_bytes, self.down_record_bytes = record_bytes(self.hidden_size, inter, self.group_size)
        self.gate_up = torch.empty(self.records * self.gate_up_record_bytes, dtype=torch.uint8, device="cuda")
        self.down = torch.empty(self.records * self.down_record_bytes, dtype=torch.uint8, device="cuda")
        self._tile(lib, parts, 0)
        if self.has_shared:
            sp = {}
            for name in ("gate_proj", "up_proj", "down_proj"):
                w, s, b = _triple(shared[name])
                sp[name] = (_dev(w).unsqueeze(0), _bf16(s, f"shared {name} scales").unsqueeze(0),
                            _bf16(b, f"shared {name} biases").unsqueeze(0))
            if int(sp["gate_proj"][0].shape[1]) != inter:
                raise ValueError("shared expert intermediate must equal the routed intermediate")
            self._tile(lib, sp, E)
        torch.cuda.current_stream().synchronize()

    def abi(self):
        t = _lib.FnTiledExperts()
        t.gate_up = self.gate_up.data_ptr()
        t.down = self.down.data_ptr()
        t.gate_up_record_bytes = self.gate_up_record_bytes
        t.down_record_bytes = self.down_record_bytes
        t.records = self.records
        t.has_shared = 1 if self.has_shared else 0
        return t

    def _tile(self, lib, parts, first):
        a = _lib.FnTileArgs()
        a.abi_version = _lib.ABI_VERSION
        a.experts = int(parts["gate_proj"][0].shape[0])
        a.hidden_size = self.hidden_size
        a.inter_size = self.inter_size
        a.group_size = self.group_size
        a.first_record = first
        for name, key in (("gate_proj", "gate"), ("up_proj", "up"), ("down_proj", "down")):
            w, s, b = (t.contiguous() for t in parts[name])
            setattr(a, f"{key}_weight", w.data_ptr())
            setattr(a, f"{key}_scales", s.data_ptr())
            setattr(a, f"{key}_biases", b.data_ptr())
        a.tiled = self.abi()
        _lib.check(lib.fnmoe_tile_experts(ctypes.byref(a), _stream()), "tile_experts")
