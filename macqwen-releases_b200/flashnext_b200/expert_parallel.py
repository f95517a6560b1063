"""Expert-parallel sparse-MoE layer over torch.distributed (one process per GPU).

Rank r of W owns routed experts [r*E/W, (r+1)*E/W) (tiled tables on the GPU);
the router and the shared expert are replicated, and each rank routes its own
tokens (data parallel over tokens).  One layer step:

1. route locally: logits -> softmax -> top-k -> renorm, plus the shared
   expert's sigmoid gate (``fnmoe_router_topk_shared``; the reference computes
   the same on one device, ``models/flashnext/adaptive_topk.py:53-64,263-264``);
2. dispatch: the (token, slot) pairs are ordered by owner rank (stable in pair
   order) and written into a fixed-capacity send buffer, ``capacity * top_k``
   slots per peer (enough when every pair goes to one owner; the capacity is
   the largest per-rank token count, given at construction or agreed per call
   by an all-reduce); a slot carries the input row and the owner-local expert
   id, or ``ROUTE_NONE`` when unused.  One ``all_to_all_single`` with equal
   splits moves it; with a given capacity nothing is read back to the host
   and the step can be captured in a CUDA graph;
3. the owner runs its experts on the received rows, one slot per row (empty
   slots are skipped by the grouping), together with the shared expert on its
   own tokens (the shared expert is one more record of its tiled table;
   ``fnmoe_moe_execute`` with per-slot outputs);
4. the bfloat16 outputs come back along the reverse all-to-all and land in
   their (token, slot) places;
5. the token's rank combines in slot order and adds the gated shared expert
   (``fnmoe_combine``, ``metal_runtime.py:301-333``).

Every kernel gives a row's result independently of the rest of its batch, so
the output is bit-identical to the single-device layer (``fnmoe_moe_layer``).
Rows travel as int32 words (pairs of bfloat16), which every backend carries.

The compute steps go through a backend object: ``CudaBackend`` (the product)
or, for multi-process tests of the dispatch/combine logic on CPU ranks, any
object with the same three methods (route, experts, combine).
"""
from __future__ import annotations

import ctypes
from typing import Mapping

from . import _lib
from .cuda_runtime import _bf16, _dev, _stream, _Workspace
from .tiled import TiledExperts


def _torch():
    import torch

    return torch


def _triple(p):
    if isinstance(p, Mapping):
        return p["weight"], p["scales"], p["biases"]
    return tuple(p)


class CudaBackend:
    """The sm_100a kernels behind the four compute steps."""

    def __init__(self, router_weight, local_experts: Mapping, shared: Mapping, shared_expert_gate,
                 *, top_k: int, group_size: int = 32, renorm_blend: float = 1.0):
        self.router_weight = _bf16(router_weight, "router_weight")
        self.expert_count, self.hidden_size = (int(v) for v in self.router_weight.shape)
        self.top_k = int(top_k)
        self.group_size = int(group_size)
        self.renorm_blend = float(renorm_blend)
        # Local records: this rank's routed experts, then the shared expert as
        # one more record (an ordinary expert to the executor), so received
        # pairs and this rank's shared-expert rows go through one call.
        torch = _torch()
        merged = {}
        for name in ("gate_proj", "up_proj", "down_proj"):
            lw, ls, lb = (t for t in _triple(local_experts[name]))
            sw, ss, sb = _triple(shared[name])
            merged[name] = (torch.cat([_dev(lw), _dev(sw).unsqueeze(0)]),
                            torch.cat([_bf16(ls, "scales"), _bf16(ss, "shared scales").unsqueeze(0)]),
                            torch.cat([_bf16(lb, "biases"), _bf16(sb, "shared biases").unsqueeze(0)]))
        self.local = TiledExperts(merged, None, group_size=group_size)
        self.local_count = self.local.expert_count - 1  # routed experts; the shared one is record local_count
        self.inter_size = self.local.inter_size
        self.shared_gate_weight = _bf16(shared_expert_gate, "shared_expert_gate").reshape(-1)
        self._ws = _Workspace()

    def route(self, x):
        torch = _torch()
        lib = _lib.ensure_device()
        T = x.shape[0]
        inds = torch.empty((T, self.top_k), dtype=torch.int32, device="cuda")
        scores = torch.empty((T, self.top_k), dtype=torch.bfloat16, device="cuda")
        mass = torch.empty((T,), dtype=torch.bfloat16, device="cuda")
        logits = torch.empty((T, self.expert_count), dtype=torch.bfloat16, device="cuda")
        sl = torch.empty((T,), dtype=torch.bfloat16, device="cuda")
        sg = torch.empty((T,), dtype=torch.bfloat16, device="cuda")
        _lib.check(lib.fnmoe_router_topk_shared(
            x.data_ptr(), self.router_weight.data_ptr(), self.shared_gate_weight.data_ptr(), T, self.hidden_size,
            self.expert_count, self.top_k, self.renorm_blend, inds.data_ptr(), scores.data_ptr(), mass.data_ptr(),
            logits.data_ptr(), sl.data_ptr(), sg.data_ptr(), _stream()), "router_topk_shared")
        return inds, scores, sg

    def _execute(self, x, routes, tiled, weights, expert_count, ws):
        """Per-slot outputs [rows, H] of routes [rows, 1] (one slot per row)."""
        torch = _torch()
        lib = _lib.ensure_device()
        rows = x.shape[0]
        out = torch.empty((rows, self.hidden_size), dtype=torch.bfloat16, device="cuda")
        if rows == 0:
            return out
        a = _lib.FnMoEArgs()
        a.abi_version = _lib.ABI_VERSION
        a.flags = _lib.FLAG_NO_COMBINE
        a.x = x.data_ptr()
        if tiled is not None:
            a.tiled = tiled.abi()
        else:
            for name, key in (("gate_proj", "gate"), ("up_proj", "up"), ("down_proj", "down")):
                w, s, b = weights[name]
                setattr(a, f"{key}_weight", w.data_ptr())
                setattr(a, f"{key}_scales", s.data_ptr())
                setattr(a, f"{key}_biases", b.data_ptr())
        a.routes = routes.data_ptr()
        a.tokens, a.slots = rows, 1
        a.hidden_size, a.inter_size, a.expert_count = self.hidden_size, self.inter_size, expert_count
        a.group_size = self.group_size
        a.x_dtype = _lib.DTYPE_BF16
        a.down_out = out.data_ptr()
        need = ctypes.c_uint64(0)
        _lib.check(lib.fnmoe_moe_workspace_size(ctypes.byref(a), ctypes.byref(need)), "workspace_size")
        w = ws.get(need.value)
        a.workspace, a.workspace_bytes = w.data_ptr(), w.numel()
        _lib.check(lib.fnmoe_moe_execute(ctypes.byref(a), _stream()), "moe_execute")
        return out

    def experts(self, rows, local_ids, x):
        """Per-pair outputs of the received rows, and the shared expert on x."""
        torch = _torch()
        n = rows.shape[0]
        all_rows = torch.cat([rows, x]).contiguous()
        routes = torch.cat([local_ids.to(torch.int32),
                            torch.full((x.shape[0],), self.local_count, dtype=torch.int32, device=x.device)])
        out = self._execute(all_rows, routes.reshape(-1, 1).contiguous(), self.local, None, self.local_count + 1,
                            self._ws)
        return out[:n], out[n:]

    def combine(self, d, inds, scores, shared, shared_gate):
        torch = _torch()
        lib = _lib.ensure_device()
        T, S, H = d.shape
        out = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")
        _lib.check(lib.fnmoe_combine(d.data_ptr(), inds.data_ptr(), scores.data_ptr(), _lib.DTYPE_BF16, T, S, H,
                                     self.expert_count, None, shared.data_ptr(), shared_gate.data_ptr(),
                                     out.data_ptr(), _stream()), "combine")
        return out


class ExpertParallelMoE:
    """One sparse-MoE layer with experts sharded over the ranks of `group`."""

    def __init__(self, backend, *, expert_count: int, hidden_size: int, top_k: int, group=None,
                 capacity_tokens: int | None = None):
        import torch.distributed as dist

        self.backend = backend
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if expert_count % self.world:
            raise ValueError("expert_count must be divisible by the number of ranks")
        self.expert_count = expert_count
        self.per_rank = expert_count // self.world
        self.hidden_size = hidden_size
        self.top_k = top_k
        # tokens per rank and call that every rank's send buffer can hold; None:
        # agreed per call with an all-reduce of the ranks' token counts
        self.capacity_tokens = capacity_tokens

    def _capacity(self, T, device):
        torch = _torch()
        import torch.distributed as dist

        if self.capacity_tokens is not None:
            if T > self.capacity_tokens:
                raise ValueError(f"{T} tokens exceed capacity_tokens={self.capacity_tokens}")
            return self.capacity_tokens
        t = torch.tensor([T], dtype=torch.int64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return int(t.item())

    def _a2a(self, out, inp, out_splits, in_splits):
        import torch.distributed as dist

        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)
        return out

    def __call__(self, x):
        torch = _torch()
        T, H = x.shape
        k = self.top_k
        W = self.world
        dev = x.device
        inds, scores, sg = self.backend.route(x)
        flat = inds.reshape(-1).to(torch.int64)
        owner = torch.div(flat, self.per_rank, rounding_mode="floor")
        order = torch.sort(owner, stable=True).indices  # pairs grouped by owner, pair order kept
        so = owner[order]
        # pairs per owner (scatter_add into a fixed-size tensor: bincount would read its size back to the host)
        counts = torch.zeros(W, dtype=torch.int64, device=dev).scatter_add_(0, owner, torch.ones_like(owner))
        starts = torch.cumsum(counts, 0) - counts
        pos = torch.arange(T * k, device=dev) - starts[so]  # slot inside the owner's segment
        cap = self._capacity(T, dev) * k
        w = H // 2
        # one payload row per slot: the input row as H/2 int32 words, then the
        # owner-local expert id (ROUTE_NONE when the slot is empty) and 3 pad words
        send = torch.zeros((W, cap, w + 4), dtype=torch.int32, device=dev)
        send[:, :, w] = -1  # ROUTE_NONE as int32
        send[so, pos, :w] = x.view(torch.int32)[torch.div(order, k, rounding_mode="floor")]
        send[so, pos, w] = (flat[order] - so * self.per_rank).to(torch.int32)
        recv = torch.empty_like(send)
        self._a2a(recv.view(W * cap, w + 4), send.view(W * cap, w + 4), None, None)
        recv_rows = recv[:, :, :w].reshape(W * cap, w).view(x.dtype)
        d_recv, shared = self.backend.experts(recv_rows, recv[:, :, w].reshape(-1).contiguous(), x)
        back = torch.empty((W, cap, H), dtype=d_recv.dtype, device=dev)
        self._a2a(back.view(W * cap, H).view(torch.int32), d_recv.reshape(W * cap, H).contiguous().view(torch.int32),
                  None, None)
        d = torch.empty((T * k, H), dtype=back.dtype, device=dev)
        d[order] = back[so, pos]
        return self.backend.combine(d.view(T, k, H), inds, scores, shared, sg)
