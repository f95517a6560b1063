"""B200 executor with the op-level API of ``models/flashnext/metal_runtime.py``.

``MoEExecutor`` (alias ``MetalMoEExecutor``) keeps the reference's
constructor arguments, ``execute`` keywords, attributes (``available``,
``last_path``, ``fallback_reason``, ``capabilities``), bounds and error
types (metal_runtime.py:425-932), so ``StreamingSwitchGLU`` style callers
(``models/flashnext/expert_cache.py:1543-1554,1679,1728,1776``) can swap it
in.  Differences, all deliberate:

* there is no reference/NumPy fallback path: when the CUDA library or an
  sm_100 device is missing, ``execute`` raises ``RuntimeError``;
* ``slab_pack``/``stream_pack`` are device expert tables
  (:class:`~flashnext_b200.expert_table.ExpertTable`, or raw uint8 CUDA
  buffers in the same record layout) and are not limited to 2560/640;
* Q4/G64 uses the same fused down+combine as G32.

Arrays are torch CUDA tensors (bfloat16 activations and metadata, uint32
packed weights stored as int32/uint32 tensors).  NumPy inputs are accepted
for convenience: they are copied to the device, run through the same
kernels, and the result is copied back.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import Any, Mapping, Sequence

import numpy as np

from . import _lib
from .expert_table import ExpertTable, record_layout

MAX_TOKENS = 8
MAX_EXPERTS = 512
MAX_TOP_K = 10
MAX_WIDTH = 16_384
GROUP_SIZE = 32
SUPPORTED_GROUP_SIZES = (32, 64)
BITS = 4


@dataclass(frozen=True)
class Q4G32Projection:
    """Packed expert rows consumed by one gate, up, or down projection."""

    weight: Any
    scales: Any
    biases: Any


@dataclass(frozen=True)
class CudaCapabilities:
    """Backend probe result exposed as attributes and mapping-like keys."""

    available: bool
    supports_custom_moe: bool
    backend: str
    reason: str

    @property
    def custom_cuda(self) -> bool:
        return self.supports_custom_moe

    custom_metal = custom_cuda  # attribute name used by the reference callers

    def __getitem__(self, key: str) -> Any:
        return getattr(self, key)


def probe_capabilities(backend: Any = None) -> CudaCapabilities:
    """Capability flags without compiling or allocating (metal_runtime.py:65-96)."""
    if backend == "reference":
        return CudaCapabilities(False, False, "reference", "reference backend requested")
    if backend is not None and hasattr(backend, "available"):
        available = bool(getattr(backend, "available"))
        supports = bool(getattr(backend, "supports_custom_moe", False))
        reason = "injected backend capability"
        if not available:
            reason = "injected backend is unavailable"
        elif not supports:
            reason = "backend does not provide custom MoE"
        return CudaCapabilities(available and supports, supports, "injected", reason)
    if backend not in (None, "cuda"):
        return CudaCapabilities(False, False, str(backend), "unknown backend")
    try:
        import torch

        if not torch.cuda.is_available():
            return CudaCapabilities(False, False, "cuda", "no CUDA device")
        lib = _lib.load()
        if lib.fnmoe_available() != 1:
            return CudaCapabilities(False, False, "cuda", _lib.last_error(lib))
        return CudaCapabilities(True, True, "cuda", "sm_100 device detected")
    except Exception as exc:  # library missing or unloadable
        return CudaCapabilities(False, False, "cuda", f"CUDA library unavailable: {exc}")


def _as_projection(value: Any) -> Q4G32Projection:
    if isinstance(value, Q4G32Projection):
        return value
    if isinstance(value, Mapping):
        return Q4G32Projection(value["weight"], value["scales"], value["biases"])
    if isinstance(value, Sequence) and len(value) == 3:
        return Q4G32Projection(value[0], value[1], value[2])
    raise TypeError("projection must be (weight, scales, biases)")


def _shape(value: Any) -> tuple[int, ...]:
    return tuple(int(item) for item in value.shape)


def _validate_projection(projection, expert_count, input_width, output_width, group_size=GROUP_SIZE):
    """Shape/dtype checks of metal_runtime.py:119-142."""
    weight_shape = _shape(projection.weight)
    count = weight_shape[0] if expert_count is None else expert_count
    expected_weight = (count, output_width, input_width // 8)
    expected_meta = (count, output_width, input_width // group_size)
    if weight_shape != expected_weight:
        raise ValueError(f"weight shape {weight_shape} != {expected_weight}")
    if _shape(projection.scales) != expected_meta or _shape(projection.biases) != expected_meta:
        raise ValueError(f"Q4/G{group_size} scales and biases have an invalid shape")
    dt = str(getattr(projection.weight, "dtype", ""))
    if dt not in ("torch.int32", "torch.uint32", "uint32", "int32"):
        raise TypeError("Q4 weights must use uint32 packed values")


# -- tensor plumbing ----------------------------------------------------------


def _torch():
    import torch

    return torch


def _dev(a, dtype=None):
    """Return a contiguous CUDA tensor view of ``a`` (NumPy inputs are copied)."""
    torch = _torch()
    if isinstance(a, np.ndarray):
        if a.dtype == np.uint32:
            t = torch.from_numpy(a.view(np.int32).copy())
        else:
            t = torch.from_numpy(np.ascontiguousarray(a))
        t = t.cuda()
    else:
        t = a if a.is_cuda else a.cuda()
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    return t.contiguous()


def _bf16(a, what):
    """bfloat16 CUDA tensor; float32 values must already be bfloat16-exact."""
    torch = _torch()
    t = _dev(a)
    if t.dtype == torch.bfloat16:
        return t
    if t.dtype == torch.float32:
        b = t.to(torch.bfloat16)
        if not torch.equal(b.float(), t):
            raise ValueError(f"{what} must be bfloat16 (float32 activations are not supported)")
        return b
    raise TypeError(f"{what} must be a bfloat16 tensor")


def _u32(a, what):
    torch = _torch()
    t = _dev(a)
    if t.dtype in (torch.int32, getattr(torch, "uint32", torch.int32)):
        return t
    if t.dtype == torch.int64:
        if bool(((t < 0) | (t > 0xFFFFFFFF)).any()):
            raise ValueError(f"{what} outside uint32")
        return torch.where(t >= 2 ** 31, t - 2 ** 32, t).to(torch.int32)
    raise TypeError(f"{what} must be an integer tensor")


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return _torch().cuda.current_stream().cuda_stream


class _Workspace:
    """Grow-only device scratch buffer owned by one executor/op."""

    def __init__(self):
        self.buf = None

    def get(self, nbytes: int):
        torch = _torch()
        if self.buf is None or self.buf.numel() < nbytes or self.buf.device != torch.device("cuda", torch.cuda.current_device()):
            self.buf = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device="cuda")
        return self.buf


def _table_struct(table, layout_shape, group_size, *, header: bool):
    """FnExpertTable for an ExpertTable or a raw uint8 record buffer."""
    if table is None:
        return _lib.FnExpertTable()
    if isinstance(table, ExpertTable):
        return table.abi(_lib.FnExpertTable, header=header)
    torch = _torch()
    buf = _dev(table)
    if buf.dtype != torch.uint8:
        buf = buf.view(torch.uint8)
    hidden, inter = layout_shape
    lay = record_layout(hidden, inter, group_size)
    hdr = 4096 if header else 0
    t = _lib.FnExpertTable()
    t.base = buf.data_ptr()
    t.header_bytes = hdr
    t.record_stride = lay.record_stride
    for i, off in enumerate(lay.offsets):
        t.part_offset[i] = off
    t.records = max(0, (buf.numel() - hdr) // lay.record_stride)
    return t


def weighted_combine(expert_outputs: Any, routes: Any, scores: Any) -> Any:
    """Combine routed expert outputs using the router scores (metal_runtime.py:145-191).

    ``expert_outputs`` is ``[..., slots, hidden]`` or ``[..., experts, hidden]``
    (``routes`` then selects the slots).  Computed in float32 on the GPU.
    """
    torch = _torch()
    host = isinstance(expert_outputs, np.ndarray)
    output_shape = _shape(expert_outputs)
    route_shape = _shape(routes)
    score_shape = _shape(scores)
    if len(output_shape) < 2 or len(route_shape) == 0:
        raise ValueError("expert_outputs and routes need at least one dimension")
    if score_shape != route_shape:
        raise ValueError("routes and scores must have identical shapes")
    slots = route_shape[-1]
    if output_shape[:-1] == route_shape:
        experts = 0
    elif len(output_shape) == len(route_shape) + 1 and output_shape[-2] >= slots:
        experts = output_shape[-2]
        r = np.asarray(routes) if isinstance(routes, np.ndarray) else None
        if r is not None and r.size and (r.min() < 0 or r.max() >= experts):
            raise ValueError("routes contain an expert outside expert_outputs")
    else:
        raise ValueError(f"expert_outputs shape {output_shape} does not match routes {route_shape}")
    lib = _lib.ensure_device()
    hidden = output_shape[-1]
    tokens = int(np.prod(route_shape[:-1])) if len(route_shape) > 1 else 1
    out_t = _dev(expert_outputs, torch.float32)
    sc_t = _dev(scores, torch.float32)
    rt = _dev(routes, torch.int32) if experts else None
    if rt is not None and not host:
        if bool(((rt < 0) | (rt >= experts)).any()):
            raise ValueError("routes contain an expert outside expert_outputs")
    res = torch.empty((tokens, hidden), dtype=torch.float32, device="cuda")
    _lib.check(lib.fnmoe_weighted_combine(out_t.data_ptr(), _ptr(rt), sc_t.data_ptr(), res.data_ptr(),
                                          tokens, slots, experts, hidden, _stream()), "weighted_combine")
    res = res.reshape(*route_shape[:-1], hidden)
    return res.cpu().numpy() if host else res


class MoEExecutor:
    """Bounded three-projection executor on sm_100a (metal_runtime.py:422-932)."""

    def __init__(
        self,
        expert_count: int,
        hidden_size: int,
        top_k: int,
        backend: Any = None,
        *,
        max_tokens: int = MAX_TOKENS,
        max_width: int = MAX_WIDTH,
        profile_boundaries: bool | None = None,
        profile_boundary: str | None = None,
        fused_up_swiglu: bool | None = None,
        group_size: int = GROUP_SIZE,
        header_size: int = 4096,
    ) -> None:
        if not 1 <= expert_count <= MAX_EXPERTS:
            raise ValueError(f"expert_count must be in 1..{MAX_EXPERTS}")
        if hidden_size <= 0:
            raise ValueError("hidden_size must be positive")
        if not 1 <= top_k <= MAX_TOP_K:
            raise ValueError(f"top_k must be in 1..{MAX_TOP_K}")
        if top_k > expert_count:
            raise ValueError("top_k cannot exceed expert_count")
        if not 1 <= max_tokens <= MAX_TOKENS:
            raise ValueError(f"max_tokens must be in 1..{MAX_TOKENS}")
        if not 1 <= max_width <= MAX_WIDTH:
            raise ValueError(f"max_width must be in 1..{MAX_WIDTH}")
        if group_size not in SUPPORTED_GROUP_SIZES:
            raise ValueError(f"group_size must be one of {SUPPORTED_GROUP_SIZES}")
        self.expert_count = int(expert_count)
        self.hidden_size = int(hidden_size)
        self.top_k = int(top_k)
        self.max_tokens = int(max_tokens)
        self.max_width = int(max_width)
        self.group_size = int(group_size)
        self.header_size = int(header_size)
        self.backend = backend
        self.capabilities = probe_capabilities(backend)
        self.last_path = "cuda"
        self.fallback_reason = self.capabilities["reason"]
        if fused_up_swiglu is None:
            fused_up_swiglu = os.environ.get("FLASHNEXT_FUSED_UP_SWIGLU") == "1"
        # gate/up/SwiGLU always run as one kernel here; the flag is kept so
        # callers that set it keep working.
        self.fused_up_swiglu = bool(fused_up_swiglu)
        self._ws = _Workspace()
        self._profile = bool(profile_boundaries)
        self._events: list[tuple[Any, Any]] = []

    @property
    def available(self) -> bool:
        return bool(self.capabilities["available"])

    @property
    def boundary_profile(self) -> dict[str, Any]:
        """Device milliseconds of the latest profiled ``execute`` calls."""
        events = []
        for start, end in self._events:
            end.synchronize()
            events.append({"label": "execute", "device_ms": start.elapsed_time(end)})
        return {"events": events, "total_ms": sum(e["device_ms"] for e in events)}

    def reset_boundary_profile(self) -> None:
        self._events.clear()

    def execute(
        self,
        x: Any,
        routes: Any,
        projections: Mapping[str, Any] | Sequence[Any] | Any = None,
        *,
        return_all: bool = False,
        scores: Any = None,
        slab_pack: Any = None,
        stream_pack: Any = None,
        shared_y: Any = None,
        shared: Any = None,
        shared_gate: Any = None,
    ) -> Any:
        """Run gate, up, SwiGLU and down for bounded flattened inputs.

        ``x`` [tokens, hidden_size]; ``routes`` [tokens, top_k] expert indices
        (bit 31 = record of ``slab_pack``).  Returns the combined [tokens,
        hidden] output when ``scores`` is given, the per-slot down outputs
        [tokens, top_k, hidden] otherwise, or ``(gate, up, down)`` with
        ``return_all``.
        """
        # Combine-only probes (metal_runtime.py:784-798).
        if projections is not None and not isinstance(projections, (Mapping, list, tuple)):
            if not self.capabilities.supports_custom_moe:
                raise RuntimeError("custom MoE is unavailable on this backend")
            self.last_path = "cuda"
            self.fallback_reason = None
            return weighted_combine(x, routes, projections)
        if projections is None and scores is not None:
            if not self.capabilities.supports_custom_moe:
                raise RuntimeError("custom MoE is unavailable on this backend")
            self.last_path = "cuda"
            self.fallback_reason = None
            return weighted_combine(x, routes, scores)
        if projections is None:
            raise TypeError("packed execution needs gate, up, and down projections")
        x_shape = _shape(x)
        route_shape = _shape(routes)
        if len(x_shape) != 2 or x_shape[1] != self.hidden_size:
            raise ValueError("x must have shape (tokens, hidden_size)")
        if len(route_shape) != 2 or route_shape[1] != self.top_k:
            raise ValueError("routes must have shape (tokens, top_k)")
        if scores is not None and _shape(scores) != route_shape:
            raise ValueError("scores must have the same shape as routes")
        if (shared is None) != (shared_gate is None):
            raise ValueError("shared and shared_gate must be provided together")
        if shared_y is not None and shared is not None:
            raise ValueError("provide shared_y or shared parts, not both")
        if stream_pack is not None and slab_pack is None:
            raise ValueError("stream pack requires a resident slab pack")
        tokens = x_shape[0]
        if route_shape[0] != tokens:
            raise ValueError("x and routes must have the same token count")
        if not 1 <= tokens <= self.max_tokens:
            raise ValueError(f"tokens must be in 1..{self.max_tokens}")
        if isinstance(routes, np.ndarray) and np.any(routes.astype(np.int64) < 0):
            raise ValueError("routes contain an expert outside the configured bank")
        if isinstance(projections, Mapping):
            gate = _as_projection(projections["gate_proj"])
            up = _as_projection(projections["up_proj"])
            down = _as_projection(projections["down_proj"])
        else:
            if len(projections) != 3:
                raise ValueError("projections must contain gate, up, and down")
            gate, up, down = (_as_projection(item) for item in projections)
        gate_width = _shape(gate.weight)[1]
        inter_width = _shape(up.weight)[1]
        if gate_width != inter_width or gate_width > self.max_width:
            raise ValueError("gate and up projection widths must match the bound")
        _validate_projection(gate, None, self.hidden_size, gate_width, self.group_size)
        _validate_projection(up, None, self.hidden_size, inter_width, self.group_size)
        if self.hidden_size % self.group_size or inter_width % self.group_size:
            raise ValueError(f"Q4/G{self.group_size} projection inputs must be group aligned")
        _validate_projection(down, None, inter_width, self.hidden_size, self.group_size)
        if not self.available:
            raise RuntimeError(f"CUDA MoE executor unavailable: {self.fallback_reason}")
        return self._run(x, routes, gate, up, down, inter_width, return_all, scores,
                         slab_pack, stream_pack, shared_y, shared, shared_gate)

    def _run(self, x, routes, gate, up, down, inter, return_all, scores, slab_pack,
             stream_pack, shared_y, shared, shared_gate):
        torch = _torch()
        lib = _lib.ensure_device()
        host = isinstance(x, np.ndarray)
        # float32 activations keep float32 arithmetic end to end (the
        # reference's kernels with T = float, metal_runtime.py:371-373);
        # bfloat16 activations the bfloat16 sequence
        f32 = (x.dtype == np.float32) if host else (x.dtype == torch.float32)
        act = torch.float32 if f32 else torch.bfloat16
        xt = _dev(x, torch.float32) if f32 else _bf16(x, "x")
        rt = _u32(routes, "routes")
        tokens, slots = _shape(rt)
        H = self.hidden_size
        keep = [xt, rt]
        a = _lib.FnMoEArgs()
        a.abi_version = _lib.ABI_VERSION
        a.x = xt.data_ptr()
        for name, proj in (("gate", gate), ("up", up), ("down", down)):
            w = _dev(proj.weight)
            if w.dtype not in (torch.int32, getattr(torch, "uint32", torch.int32)):
                raise TypeError("Q4 weights must use uint32 packed values")
            s = _bf16(proj.scales, f"{name} scales")
            b = _bf16(proj.biases, f"{name} biases")
            keep += [w, s, b]
            setattr(a, f"{name}_weight", w.data_ptr())
            setattr(a, f"{name}_scales", s.data_ptr())
            setattr(a, f"{name}_biases", b.data_ptr())
        a.routes = rt.data_ptr()
        a.tokens = tokens
        a.slots = slots
        a.hidden_size = H
        a.inter_size = inter
        a.expert_count = _shape(gate.weight)[0]
        a.group_size = self.group_size
        a.x_dtype = _lib.DTYPE_F32 if f32 else _lib.DTYPE_BF16
        if scores is not None:
            st = _dev(scores)
            if st.dtype not in (torch.float32, torch.bfloat16):
                st = st.to(torch.float32)
            keep.append(st)
            a.scores = st.data_ptr()
            a.scores_dtype = _lib.DTYPE_F32 if st.dtype == torch.float32 else _lib.DTYPE_BF16
        as_act = (lambda v, what: _dev(v, torch.float32)) if f32 else _bf16
        if shared_y is not None:
            sy = as_act(shared_y, "shared_y").reshape(tokens, H)
            keep.append(sy)
            a.shared_y = sy.data_ptr()
        if shared is not None:
            sh = as_act(shared, "shared").reshape(tokens, H)
            sg = as_act(shared_gate, "shared_gate").reshape(tokens)
            keep += [sh, sg]
            a.shared = sh.data_ptr()
            a.shared_gate = sg.data_ptr()
        if slab_pack is not None:
            a.table = _table_struct(slab_pack, (H, inter), self.group_size, header=True)
            keep.append(slab_pack)
        if stream_pack is not None:
            a.stream_table = _table_struct(stream_pack, (H, inter), self.group_size, header=False)
            keep.append(stream_pack)
        out = None
        g_out = u_out = d_out = None
        if return_all:
            a.flags |= _lib.FLAG_RETURN_ALL
            g_out = torch.empty((tokens, slots, inter), dtype=act, device="cuda")
            u_out = torch.empty_like(g_out)
            d_out = torch.empty((tokens, slots, H), dtype=act, device="cuda")
            a.gate_out, a.up_out, a.down_out = g_out.data_ptr(), u_out.data_ptr(), d_out.data_ptr()
        elif scores is None:
            a.flags |= _lib.FLAG_NO_COMBINE
            d_out = torch.empty((tokens, slots, H), dtype=act, device="cuda")
            a.down_out = d_out.data_ptr()
        else:
            out = torch.empty((tokens, H), dtype=act, device="cuda")
            a.output = out.data_ptr()
        need = ctypes.c_uint64(0)
        _lib.check(lib.fnmoe_moe_workspace_size(ctypes.byref(a), ctypes.byref(need)), "workspace_size")
        ws = self._ws.get(need.value)
        a.workspace = ws.data_ptr()
        a.workspace_bytes = ws.numel()
        if self._profile:
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
        _lib.check(lib.fnmoe_moe_execute(ctypes.byref(a), _stream()), "moe_execute")
        if self._profile:
            end.record()
            self._events.append((start, end))
        self.last_path = "cuda"
        self.fallback_reason = None
        if return_all:
            res = (g_out, u_out, d_out)
            return tuple(r.float().cpu().numpy() for r in res) if host else res
        res = d_out if out is None else out
        return res.float().cpu().numpy() if host else res


MetalMoEExecutor = MoEExecutor

__all__ = [
    "BITS", "GROUP_SIZE", "MAX_EXPERTS", "MAX_TOKENS", "MAX_TOP_K", "MAX_WIDTH",
    "CudaCapabilities", "MetalMoEExecutor", "MoEExecutor", "Q4G32Projection",
    "SUPPORTED_GROUP_SIZES", "probe_capabilities", "weighted_combine",
]
