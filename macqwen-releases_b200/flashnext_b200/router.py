"""Router chain on the GPU: BF16 router linear, precise softmax, top-k, renorm.

Mirrors ``models/flashnext/compiled.py:61-112`` (``router(logits, k)``,
``renorm(scores, topk_mass, blend)``) and the router part of
``adaptive_topk._moe_call`` (``models/flashnext/adaptive_topk.py:53-64,256-261``).
MLX's ``argpartition`` leaves the slot order and tie-break unspecified; here
slots come out by decreasing probability, ties to the lower expert index.
"""
from __future__ import annotations

from . import _lib
from .cuda_runtime import _bf16, _stream


def _torch():
    import torch

    return torch


def router(logits, k: int):
    """``compiled.router``: (inds uint32-as-int32 [T,k], scores bf16 [T,k], topk_mass bf16 [T,1])."""
    torch = _torch()
    lib = _lib.ensure_device()
    lt = _bf16(logits, "logits")
    shape = lt.shape
    lt = lt.reshape(-1, shape[-1])
    tokens, experts = lt.shape
    inds = torch.empty((tokens, k), dtype=torch.int32, device="cuda")
    raw = torch.empty((tokens, k), dtype=torch.bfloat16, device="cuda")
    mass = torch.empty((tokens,), dtype=torch.bfloat16, device="cuda")
    _lib.check(lib.fnmoe_softmax_topk(lt.data_ptr(), tokens, experts, k, 1.0, inds.data_ptr(),
                                      raw.data_ptr(), None, mass.data_ptr(), _stream()), "softmax_topk")
    lead = tuple(shape[:-1])
    return inds.reshape(*lead, k), raw.reshape(*lead, k), mass.reshape(*lead, 1)


def renorm(scores, topk_mass, blend: float = 1.0):
    """``compiled.renorm``: bfloat16 elementwise, one rounding per operation.

    The ops are a handful of bfloat16 elements per token, so they run as
    torch CUDA bfloat16 arithmetic (float32 compute, bfloat16 result per op),
    the same rounding the fused router kernel applies.
    """
    torch = _torch()
    sc = _bf16(scores, "scores")
    mass = _bf16(topk_mass, "topk_mass")
    selected = sc.float().sum(dim=-1, keepdim=True).to(torch.bfloat16)
    b = torch.tensor(blend, dtype=torch.bfloat16, device=sc.device)
    normalizer = mass + b * (selected - mass)
    return sc / normalizer, normalizer


def router_topk(x, router_weight, k: int, blend: float = 1.0):
    """Fused router: logits = bf16(x W^T) -> softmax -> top-k -> renorm.

    Returns (inds int32 [T,k], renormalised scores bf16 [T,k], topk_mass bf16
    [T], logits bf16 [T,E]).
    """
    torch = _torch()
    lib = _lib.ensure_device()
    xt = _bf16(x, "x")
    wt = _bf16(router_weight, "router_weight")
    tokens, hidden = xt.shape
    experts = wt.shape[0]
    if wt.shape[1] != hidden:
        raise ValueError("router_weight must have shape (experts, hidden)")
    inds = torch.empty((tokens, k), dtype=torch.int32, device="cuda")
    scores = torch.empty((tokens, k), dtype=torch.bfloat16, device="cuda")
    mass = torch.empty((tokens,), dtype=torch.bfloat16, device="cuda")
    logits = torch.empty((tokens, experts), dtype=torch.bfloat16, device="cuda")
    _lib.check(lib.fnmoe_router_topk(xt.data_ptr(), wt.data_ptr(), tokens, hidden, experts, k, float(blend),
                                     inds.data_ptr(), scores.data_ptr(), mass.data_ptr(), logits.data_ptr(),
                                     _stream()), "router_topk")
    return inds, scores, mass, logits


def group_tokens(routes, array_experts: int, table_records: int = 0):
    """GPU grouping of (token, slot) pairs by expert (``_gather_sort`` analogue).

    Returns (counts [keys], offsets [keys+1], order [T*S]) int32 tensors;
    ``order`` lists flattened pair indices sorted by expert, ties by index.
    """
    torch = _torch()
    lib = _lib.ensure_device()
    rt = routes if routes.dtype == torch.int32 else routes.to(torch.int32)
    rt = rt.contiguous().reshape(-1)
    pairs = rt.numel()
    keys = array_experts + table_records
    counts = torch.empty(keys, dtype=torch.int32, device="cuda")
    offsets = torch.empty(keys + 1, dtype=torch.int32, device="cuda")
    order = torch.empty(pairs, dtype=torch.int32, device="cuda")
    ws = torch.empty((2 * pairs + 4 * keys + 64) * 16 + 4096, dtype=torch.uint8, device="cuda")
    _lib.check(lib.fnmoe_group_tokens(rt.data_ptr(), pairs, array_experts, table_records, counts.data_ptr(),
                                      offsets.data_ptr(), order.data_ptr(), ws.data_ptr(), ws.numel(),
                                      _stream()), "group_tokens")
    return counts, offsets, order
