"""The patched sparse-MoE block as one C-ABI call per layer.

Replaces ``Qwen3_5MoeSparseMoeBlock.__call__ = _moe_call``
(``models/flashnext/adaptive_topk.py:53-292``) together with the expert block
it dispatches to (``StreamingSwitchGLU``, ``models/flashnext/expert_cache.py:
1584-1810``) at routing threshold 1.0:

    logits = bf16(x @ W_router^T)          (adaptive_topk.py:59,61)
    softmax -> top-k -> renorm             (adaptive_topk.py:61-64,256-261)
    shared = SwiGLU-MLP(x); g = sigmoid(x . w_g)   (adaptive_topk.py:263-264)
    out = combine(experts) + bf16(g * shared)       (adaptive_topk.py:288-289)

All tokens of the batch go through the same grouped kernels, whatever the
batch size (the reference switches to ``gather_qmm`` above 8 tokens), so a
token's output does not depend on the rest of the batch.
"""
from __future__ import annotations

import ctypes
from typing import Any, Mapping

from . import _lib
from .cuda_runtime import _bf16, _dev, _stream, _Workspace
from .expert_table import ExpertTable
from .tiled import TiledExperts


def _torch():
    import torch

    return torch


def _triple(p):
    if isinstance(p, Mapping):
        return p["weight"], p["scales"], p["biases"]
    return tuple(p)


class SparseMoEBlock:
    """Router + routed Q4 experts + sigmoid-gated shared expert on sm_100a.

    ``experts`` is a mapping ``{"gate_proj", "up_proj", "down_proj"}`` of
    (weight [E,O,K/8] int32/uint32, scales bf16, biases bf16) triples, or an
    :class:`ExpertTable` whose record ``e`` holds expert ``e`` (or
    ``route_map[e]`` when given).  ``shared`` is the same mapping for the
    shared expert ([O,K/8] etc. without the expert axis) or None.

    With ``tiled`` (the default for array experts whose sizes allow it) the
    experts are repacked once into :class:`TiledExperts` and the layer reads
    only those; ``tiled=False`` keeps reading the reference-layout arrays.
    ``path`` selects the expert kernels: "auto" (tcgen05 GEMMs on dequantised
    bf16 weights for prefill-sized batches, the exact decode kernels
    otherwise), "prefill" or "decode".  ``keep_threshold`` < 1 turns on the
    adaptive keep of ``adaptive_topk.py:43-50,75-261`` (``_THRESHOLD`` /
    ``_MIN_KEEP``): each token keeps the fewest top-k slots whose share of the
    top-k mass reaches the threshold (at least ``min_keep``), computed on the
    GPU without a host sync; dropped slots report slot 0's expert with score 0.
    """

    def __init__(self, router_weight, experts: Any, *, top_k: int = 10, shared: Mapping | None = None,
                 shared_expert_gate=None, group_size: int = 32, renorm_blend: float = 1.0,
                 route_map=None, tiled: bool = True, path: str = "auto", keep_threshold: float = 1.0,
                 min_keep: int = 1):
        torch = _torch()
        self.router_weight = _bf16(router_weight, "router_weight")
        self.expert_count, self.hidden_size = (int(v) for v in self.router_weight.shape)
        self.top_k = int(top_k)
        self.group_size = int(group_size)
        self.renorm_blend = float(renorm_blend)
        self.keep_threshold = float(keep_threshold)
        self.min_keep = int(min_keep)
        if path not in ("auto", "prefill", "decode"):
            raise ValueError("path must be 'auto', 'prefill' or 'decode'")
        self.path = path
        self.table = experts if isinstance(experts, ExpertTable) else None
        self.route_map = None if route_map is None else _dev(route_map, torch.int32)
        if self.table is not None:
            self.inter_size = self.table.layout.inter_size
            self.experts = None
        else:
            self.experts = {}
            for name in ("gate_proj", "up_proj", "down_proj"):
                w, s, b = _triple(experts[name])
                self.experts[name] = (_dev(w), _bf16(s, f"{name} scales"), _bf16(b, f"{name} biases"))
            self.inter_size = int(self.experts["gate_proj"][0].shape[1])
        self.shared = None
        if shared is not None:
            self.shared = {}
            for name in ("gate_proj", "up_proj", "down_proj"):
                w, s, b = _triple(shared[name])
                self.shared[name] = (_dev(w), _bf16(s, f"shared {name} scales"), _bf16(b, f"shared {name} biases"))
            if shared_expert_gate is None:
                raise ValueError("shared expert needs its sigmoid gate weight")
            self.shared_expert_gate = _bf16(shared_expert_gate, "shared_expert_gate").reshape(-1)
        self.tiled = None
        if (tiled and self.experts is not None and self.inter_size % 8 == 0 and self.hidden_size % 16 == 0):
            self.tiled = TiledExperts(self.experts, self.shared, group_size=self.group_size)
            self.experts = None
        self._ws = _Workspace()
        self.last_inds = None
        self.last_scores = None
        self.last_logits = None

    def _args(self, x, out, inds, scores, logits):
        a = _lib.FnMoELayerArgs()
        a.abi_version = _lib.ABI_VERSION
        a.top_k = self.top_k
        a.x = x.data_ptr()
        a.router_weight = self.router_weight.data_ptr()
        a.renorm_blend = self.renorm_blend
        a.tokens = x.shape[0]
        a.hidden_size = self.hidden_size
        a.inter_size = self.inter_size
        a.expert_count = self.expert_count
        a.group_size = self.group_size
        if self.tiled is not None:
            a.tiled = self.tiled.abi()
        elif self.experts is not None:
            for name, key in (("gate_proj", "gate"), ("up_proj", "up"), ("down_proj", "down")):
                w, s, b = self.experts[name]
                setattr(a, f"{key}_weight", w.data_ptr())
                setattr(a, f"{key}_scales", s.data_ptr())
                setattr(a, f"{key}_biases", b.data_ptr())
        else:
            a.table = self.table.abi(_lib.FnExpertTable)
            if self.route_map is not None:
                a.table_routes_of_expert = self.route_map.data_ptr()
        if self.shared is not None:
            a.shared_inter_size = int(self.shared["gate_proj"][0].shape[0])
            for name, key in (("gate_proj", "gate"), ("up_proj", "up"), ("down_proj", "down")):
                if self.tiled is not None:
                    break
                w, s, b = self.shared[name]
                setattr(a, f"shared_{key}_weight", w.data_ptr())
                setattr(a, f"shared_{key}_scales", s.data_ptr())
                setattr(a, f"shared_{key}_biases", b.data_ptr())
            a.shared_expert_gate = self.shared_expert_gate.data_ptr()
        a.flags = {"auto": 0, "prefill": _lib.LAYER_FORCE_PREFILL, "decode": _lib.LAYER_FORCE_DECODE}[self.path]
        a.keep_threshold = self.keep_threshold if 0.0 < self.keep_threshold < 1.0 else 0.0
        a.min_keep = max(0, self.min_keep)
        a.output = out.data_ptr()
        a.logits_out = logits.data_ptr()
        a.inds_out = inds.data_ptr()
        a.scores_out = scores.data_ptr()
        return a

    def workspace_bytes(self, tokens: int) -> int:
        torch = _torch()
        dummy = torch.empty(1, dtype=torch.bfloat16, device="cuda")
        a = self._args(dummy, dummy, dummy, dummy, dummy)
        a.tokens = tokens
        need = ctypes.c_uint64(0)
        lib = _lib.ensure_device()
        _lib.check(lib.fnmoe_moe_layer_workspace_size(ctypes.byref(a), ctypes.byref(need)), "layer workspace")
        return int(need.value)

    def __call__(self, x, out=None):
        torch = _torch()
        lib = _lib.ensure_device()
        xt = _bf16(x, "x")
        lead = xt.shape[:-1]
        xt = xt.reshape(-1, self.hidden_size)
        tokens = xt.shape[0]
        if out is None:
            out = torch.empty((tokens, self.hidden_size), dtype=torch.bfloat16, device="cuda")
        inds = torch.empty((tokens, self.top_k), dtype=torch.int32, device="cuda")
        scores = torch.empty((tokens, self.top_k), dtype=torch.bfloat16, device="cuda")
        logits = torch.empty((tokens, self.expert_count), dtype=torch.bfloat16, device="cuda")
        a = self._args(xt, out, inds, scores, logits)
        need = ctypes.c_uint64(0)
        _lib.check(lib.fnmoe_moe_layer_workspace_size(ctypes.byref(a), ctypes.byref(need)), "layer workspace")
        ws = self._ws.get(need.value)
        a.workspace = ws.data_ptr()
        a.workspace_bytes = ws.numel()
        _lib.check(lib.fnmoe_moe_layer(ctypes.byref(a), _stream()), "moe_layer")
        self.last_inds, self.last_scores, self.last_logits = inds, scores, logits
        return out.reshape(*lead, self.hidden_size)
