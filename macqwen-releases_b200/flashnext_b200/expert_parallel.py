"""Expert-parallel sparse-MoE layer over torch.distributed (one process per GPU).

Rank r of W owns routed experts [r*E/W, (r+1)*E/W) (tiled tables on the GPU);
the router and the shared expert are replicated, and each rank routes its own
tokens (data parallel over tokens).  The reference runs the layer on one
device (``models/flashnext/adaptive_topk.py:53-292``); this file distributes
it without changing a bit of its result.  One layer step:

1. route locally: logits -> softmax -> top-k -> renorm, plus the shared
   expert's sigmoid gate (``fnmoe_router_topk_shared``; the reference
   computes the same on one device, ``adaptive_topk.py:53-64,263-264``);
2. dispatch: for every (token t, destination rank d) one row -- t's input
   row and the k + 1 owner-local expert ids of t's slots on d
   (``ROUTE_NONE`` elsewhere); slot k is the shared expert, which the
   token's own rank runs (the shared expert is the last record of every
   rank's tiled table).  A token's row crosses to a rank once, however many
   of its slots that rank owns;
3. every rank runs its experts on the rows it received, one executor call
   with k + 1 slots per row (empty slots are skipped);
4. return: each live routed (row, slot) output goes back to the token's
   rank, into place [t][slot];
5. the token's rank combines in slot order and adds the gated shared expert
   (``metal_runtime.py:301-333``).

Every kernel gives a row's result independently of the rest of its batch, so
the output is bit-identical to the single-device layer (``fnmoe_moe_layer``).

Two transports carry steps 2 and 4:

* ``PeerExchange`` (CUDA, the product): each rank's exchange window is
  mapped into its peers through CUDA IPC; dispatch and return are kernels
  that store straight into the peers' windows over NVLink, exactly the rows
  that must move, with epoch flags and bounded waits (``fnmoe_ep_*``).  No
  host synchronisation, so a step can be captured in a CUDA graph.
* the collective path (``ExpertParallelMoE._collective``): the same protocol
  over ``all_to_all_single`` with fixed-size buffers (any backend, e.g. gloo
  ranks on CPU in the tests).

The compute steps go through a backend object: ``CudaBackend`` (the product)
or, for multi-process tests on CPU ranks, any object with the same methods.
"""
from __future__ import annotations

import ctypes
from typing import Mapping

from . import _lib
from .cuda_runtime import _bf16, _dev, _stream, _Workspace
from .tiled import TiledExperts

ROUTE_NONE_I32 = -1  # FNMOE_ROUTE_NONE as int32


def _torch():
    import torch

    return torch


def _triple(p):
    if isinstance(p, Mapping):
        return p["weight"], p["scales"], p["biases"]
    return tuple(p)


def _capturing() -> bool:
    torch = _torch()
    return torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()


class CudaBackend:
    """The sm_100a kernels behind the compute steps."""

    def __init__(self, router_weight, local_experts: Mapping, shared: Mapping, shared_expert_gate,
                 *, top_k: int, group_size: int = 32, renorm_blend: float = 1.0):
        self.router_weight = _bf16(router_weight, "router_weight")
        self.expert_count, self.hidden_size = (int(v) for v in self.router_weight.shape)
        self.top_k = int(top_k)
        self.group_size = int(group_size)
        self.renorm_blend = float(renorm_blend)
        # Local records: this rank's routed experts, then the shared expert as
        # one more record (an ordinary expert to the executor), so received
        # rows and this rank's shared-expert slots go through one call.
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
        self._rws = _Workspace()  # the router's: byte planes of the fixed points from 64 tokens

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
        if T:
            need = ctypes.c_uint64(0)
            _lib.check(lib.fnmoe_router_workspace_size(T, self.hidden_size, self.expert_count, 1, ctypes.byref(need)),
                       "router_workspace_size")
            w = self._rws.get(need.value) if need.value else None
            _lib.check(lib.fnmoe_router_topk_shared_ws(
                x.data_ptr(), self.router_weight.data_ptr(), self.shared_gate_weight.data_ptr(), T,
                self.hidden_size, self.expert_count, self.top_k, self.renorm_blend, inds.data_ptr(),
                scores.data_ptr(), mass.data_ptr(), logits.data_ptr(), sl.data_ptr(), sg.data_ptr(),
                w.data_ptr() if w is not None else None, w.numel() if w is not None else 0, _stream()),
                "router_topk_shared_ws")
        return inds, scores, sg

    def run_experts(self, x_ptr: int, ids_ptr: int, rows: int, slots: int, out_ptr: int) -> None:
        """Per-slot outputs [rows, slots, H] of rows [rows, H] with local ids [rows, slots]."""
        lib = _lib.ensure_device()
        a = _lib.FnMoEArgs()
        a.abi_version = _lib.ABI_VERSION
        a.flags = _lib.FLAG_NO_COMBINE
        a.x = x_ptr
        a.tiled = self.local.abi()
        a.routes = ids_ptr
        a.tokens, a.slots = rows, slots
        a.hidden_size, a.inter_size, a.expert_count = self.hidden_size, self.inter_size, self.local_count + 1
        a.group_size = self.group_size
        a.x_dtype = _lib.DTYPE_BF16
        a.down_out = out_ptr
        need = ctypes.c_uint64(0)
        _lib.check(lib.fnmoe_moe_workspace_size(ctypes.byref(a), ctypes.byref(need)), "workspace_size")
        w = self._ws.get(need.value)
        a.workspace, a.workspace_bytes = w.data_ptr(), w.numel()
        _lib.check(lib.fnmoe_moe_execute(ctypes.byref(a), _stream()), "moe_execute")

    def experts(self, rows, ids):
        """Per-slot outputs [R, S, H] of the received rows [R, H] (ids [R, S], -1 = empty)."""
        torch = _torch()
        R, S = ids.shape
        out = torch.empty((R, S, self.hidden_size), dtype=torch.bfloat16, device="cuda")
        if R:
            self.run_experts(rows.data_ptr(), ids.contiguous().data_ptr(), R, S, out.data_ptr())
        return out

    def combine(self, d, inds, scores, shared, shared_gate):
        torch = _torch()
        lib = _lib.ensure_device()
        T, S, H = d.shape
        out = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")
        if T:
            _lib.check(lib.fnmoe_combine(d.data_ptr(), inds.data_ptr(), scores.data_ptr(), _lib.DTYPE_BF16, T, S, H,
                                         self.expert_count, None, shared.data_ptr(), shared_gate.data_ptr(),
                                         out.data_ptr(), _stream()), "combine")
        return out


class PeerExchange:
    """Dispatch and return over NVLink peer memory (``fnmoe_ep_*``).

    Creating it is collective (every rank of ``group``): each rank allocates
    its window, the IPC handles go round with ``all_gather_object``, and
    every rank maps its peers' windows.  ``close()`` is collective too."""

    def __init__(self, group, *, capacity_tokens: int, hidden_size: int, top_k: int, experts_per_rank: int):
        import torch.distributed as dist

        lib = _lib.ensure_device()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        cfg = _lib.FnEpConfig()
        cfg.abi_version = _lib.ABI_VERSION
        cfg.world, cfg.rank = self.world, self.rank
        cfg.capacity_tokens, cfg.hidden_size, cfg.top_k = capacity_tokens, hidden_size, top_k
        cfg.experts_per_rank = experts_per_rank
        handle = ctypes.c_void_p()
        _lib.check(lib.fnmoe_ep_create(ctypes.byref(cfg), ctypes.byref(handle)), "ep_create")
        self.handle = handle
        ipc = (ctypes.c_char * _lib.EP_IPC_BYTES)()
        _lib.check(lib.fnmoe_ep_ipc_handle(handle, ipc), "ep_ipc_handle")
        gathered = [None] * self.world
        dist.all_gather_object(gathered, bytes(ipc), group=group)
        blob = b"".join(gathered)
        _lib.check(lib.fnmoe_ep_open_peers(handle, blob), "ep_open_peers")
        dist.barrier(group=group)
        self.window = _lib.FnEpWindow()
        _lib.check(lib.fnmoe_ep_window(handle, ctypes.byref(self.window)), "ep_window")
        self.capacity_tokens = capacity_tokens
        self.top_k = top_k
        self.hidden_size = hidden_size

    def dispatch(self, x, inds) -> None:
        lib = _lib.ensure_device()
        _lib.check(lib.fnmoe_ep_dispatch(self.handle, x.data_ptr(), inds.data_ptr(), x.shape[0], _stream()),
                   "ep_dispatch")

    def return_combine(self, scores, shared_gate, out) -> None:
        lib = _lib.ensure_device()
        _lib.check(lib.fnmoe_ep_return_combine(self.handle, scores.data_ptr(), shared_gate.data_ptr(), out.shape[0],
                                               out.data_ptr(), _stream()), "ep_return_combine")

    def close(self) -> None:
        import torch.distributed as dist

        if self.handle is None:
            return
        dist.barrier(group=self.group)  # no peer writes into this window any more
        _lib.check(_lib.ensure_device().fnmoe_ep_destroy(self.handle), "ep_destroy")
        self.handle = None


class ExpertParallelMoE:
    """One sparse-MoE layer with experts sharded over the ranks of `group`.

    ``capacity_tokens`` bounds the tokens a rank routes per call.  With it
    given, a CUDA backend exchanges over NVLink peer memory (``PeerExchange``,
    graph-capturable); otherwise, or with ``peer=False``, the protocol runs
    over ``all_to_all_single`` with the capacity agreed per call.  Outside
    graph capture the ranks first agree on the largest token count, so a call
    that exceeds the capacity raises ``ValueError`` on every rank (instead of
    one rank raising while the others wait in a collective)."""

    def __init__(self, backend, *, expert_count: int, hidden_size: int, top_k: int, group=None,
                 capacity_tokens: int | None = None, peer: bool | None = None):
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
        self.capacity_tokens = capacity_tokens
        use_peer = peer if peer is not None else (isinstance(backend, CudaBackend) and capacity_tokens is not None)
        if use_peer and capacity_tokens is None:
            raise ValueError("the peer-memory exchange needs capacity_tokens")
        self.exchange = (PeerExchange(group, capacity_tokens=capacity_tokens, hidden_size=hidden_size, top_k=top_k,
                                      experts_per_rank=self.per_rank) if use_peer else None)

    def close(self) -> None:
        if self.exchange is not None:
            self.exchange.close()
            self.exchange = None

    def _agree(self, T, device):
        """Largest token count over the ranks (one all-reduce); raises on every
        rank when it exceeds the fixed capacity."""
        torch = _torch()
        import torch.distributed as dist

        t = torch.tensor([T], dtype=torch.int64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        most = int(t.item())
        if self.capacity_tokens is not None and most > self.capacity_tokens:
            raise ValueError(f"{most} tokens on some rank exceed capacity_tokens={self.capacity_tokens}")
        return most

    def __call__(self, x):
        torch = _torch()
        T = x.shape[0]
        if self.capacity_tokens is None or not _capturing():
            cap = self._agree(T, x.device)
        else:
            cap = self.capacity_tokens
        inds, scores, sg = self.backend.route(x)
        if self.exchange is not None:
            ex = self.exchange
            ex.dispatch(x, inds)
            w = ex.window
            self.backend.run_experts(w.rows, w.ids, w.row_count, w.slots, w.slot_outputs)
            out = torch.empty((T, self.hidden_size), dtype=torch.bfloat16, device=x.device)
            ex.return_combine(scores, sg, out)
            return out
        return self._collective(x, inds, scores, sg, self.capacity_tokens or cap)

    # -- the same protocol over all_to_all_single (fixed-size buffers) --------

    def _a2a(self, out, inp):
        import torch.distributed as dist

        dist.all_to_all_single(out, inp, None, None, group=self.group)
        return out

    def _collective(self, x, inds, scores, sg, cap):
        torch = _torch()
        T, H = x.shape
        k, W, dev = self.top_k, self.world, x.device
        cap = max(int(cap), 1)
        flat = inds.to(torch.int64)
        owner = torch.div(flat, self.per_rank, rounding_mode="floor")       # [T, k]
        ranks = torch.arange(W, device=dev)
        # ids[d, t, s]: owner-local expert id of slot s on rank d, or none; slot k: shared expert on the own rank
        ids = torch.full((W, cap, k + 1), ROUTE_NONE_I32, dtype=torch.int32, device=dev)
        local = (flat - owner * self.per_rank).to(torch.int32)
        mine = owner[None, :, :] == ranks[:, None, None]                      # [W, T, k]
        ids[:, :T, :k] = torch.where(mine, local[None].expand(W, T, k), torch.full_like(local[None].expand(W, T, k),
                                                                                       ROUTE_NONE_I32))
        ids[self.rank, :T, k] = self.per_rank
        rows = torch.zeros((W, cap, H), dtype=x.dtype, device=dev)
        rows[:, :T] = x[None]
        # rows travel as int32 words (pairs of bfloat16), which every backend carries
        r_rows = self._a2a(torch.empty((W * cap, H // 2), dtype=torch.int32, device=dev),
                           rows.view(W * cap, H).view(torch.int32)).view(x.dtype)
        r_ids = self._a2a(torch.empty_like(ids).view(W * cap, k + 1), ids.view(W * cap, k + 1))
        d = self.backend.experts(r_rows, r_ids)                               # [W*cap, k+1, H]
        d = d.view(W, cap, k + 1, H)
        back = self._a2a(torch.empty((W * cap * k, H // 2), dtype=torch.int32, device=dev),
                         d[:, :, :k].contiguous().view(W * cap * k, H).view(torch.int32)).view(d.dtype)
        back = back.view(W, cap, k, H)                                        # [owner, t, slot, H]
        tok = torch.arange(T, device=dev)[:, None].expand(T, k)
        slot = torch.arange(k, device=dev)[None, :].expand(T, k)
        d_slots = back[owner, tok, slot]                                      # [T, k, H]
        shared = d[self.rank, :T, k]                                          # [T, H]
        return self.backend.combine(d_slots.contiguous(), inds, scores, shared.contiguous(), sg)
