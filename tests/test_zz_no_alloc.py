"""fnmoe_moe_execute_static: the executor path on library-owned static scratch.

Collected last (file name) so that it also runs after every other GPU test
has used the device; it passes alone in a fresh process as well.
"""
from __future__ import annotations

import ctypes

import pytest

pytestmark = pytest.mark.gpu


def _args(lib_mod, x, routes, scores, bank, out, tokens, slots, hidden, inter, experts):
    a = lib_mod.FnMoEArgs()
    a.abi_version = lib_mod.ABI_VERSION
    a.x = x.data_ptr()
    for name, key in (("gate_proj", "gate"), ("up_proj", "up"), ("down_proj", "down")):
        w, s, b = bank[name]
        setattr(a, f"{key}_weight", w.data_ptr())
        setattr(a, f"{key}_scales", s.data_ptr())
        setattr(a, f"{key}_biases", b.data_ptr())
    a.routes = routes.data_ptr()
    a.scores = scores.data_ptr()
    a.scores_dtype = lib_mod.DTYPE_F32
    a.output = out.data_ptr()
    a.tokens, a.slots = tokens, slots
    a.hidden_size, a.inter_size, a.expert_count = hidden, inter, experts
    a.group_size = 32
    a.x_dtype = lib_mod.DTYPE_BF16
    return a


def test_static_scratch_matches_workspace_path(cuda_lib):
    """Same inputs through fnmoe_moe_execute (caller workspace) and, twice in
    a row, fnmoe_moe_execute_static: the outputs agree bit for bit (tolerance:
    zero bf16 ulps -- both run the same kernels in the same order)."""
    import torch

    from flashnext_b200 import _lib, synthetic

    lib = cuda_lib
    tokens, slots, hidden, inter, experts = 6, 10, 2048, 512, 64
    bank = synthetic.expert_bank(experts, hidden, inter, 32, seed=23)
    x = synthetic.bf16_normal((tokens, hidden), seed=24)
    g = torch.Generator(device="cuda")
    g.manual_seed(25)
    routes = torch.stack([torch.randperm(experts, generator=g, device="cuda")[:slots] for _ in range(tokens)])
    routes = routes.to(torch.int32).contiguous()
    scores = torch.rand((tokens, slots), generator=g, device="cuda").contiguous()
    stream = torch.cuda.current_stream().cuda_stream

    ref = torch.empty((tokens, hidden), dtype=torch.bfloat16, device="cuda")
    a = _args(_lib, x, routes, scores, bank, ref, tokens, slots, hidden, inter, experts)
    need = ctypes.c_uint64(0)
    _lib.check(lib.fnmoe_moe_workspace_size(ctypes.byref(a), ctypes.byref(need)), "workspace_size")
    assert need.value <= _lib.STATIC_SCRATCH_BYTES
    ws = torch.empty(need.value, dtype=torch.uint8, device="cuda")
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.check(lib.fnmoe_moe_execute(ctypes.byref(a), stream), "moe_execute")

    outs = []
    for _ in range(2):
        o = torch.full((tokens, hidden), float("nan"), dtype=torch.bfloat16, device="cuda")
        b = _args(_lib, x, routes, scores, bank, o, tokens, slots, hidden, inter, experts)
        _lib.check(lib.fnmoe_moe_execute_static(ctypes.byref(b), stream), "moe_execute_static")
        outs.append(o)
    torch.cuda.synchronize()
    assert torch.isfinite(ref.float()).all()
    for o in outs:
        assert torch.equal(o.view(torch.int16), ref.view(torch.int16))


def test_static_scratch_rejects_oversize_calls(cuda_lib):
    """A call whose scratch need exceeds the static array fails with
    FNMOE_ERR_WORKSPACE and says so; nothing is launched."""
    import torch

    from flashnext_b200 import _lib, synthetic

    lib = cuda_lib
    tokens, slots, hidden, inter, experts = 1024, 10, 2048, 512, 4
    bank = synthetic.expert_bank(experts, hidden, inter, 32, seed=31)
    x = torch.zeros((tokens, hidden), dtype=torch.bfloat16, device="cuda")
    routes = torch.zeros((tokens, slots), dtype=torch.int32, device="cuda")
    scores = torch.zeros((tokens, slots), dtype=torch.float32, device="cuda")
    out = torch.empty((tokens, hidden), dtype=torch.bfloat16, device="cuda")
    a = _args(_lib, x, routes, scores, bank, out, tokens, slots, hidden, inter, experts)
    need = ctypes.c_uint64(0)
    _lib.check(lib.fnmoe_moe_workspace_size(ctypes.byref(a), ctypes.byref(need)), "workspace_size")
    assert need.value > _lib.STATIC_SCRATCH_BYTES
    rc = lib.fnmoe_moe_execute_static(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.ERR_WORKSPACE
    assert "static scratch" in _lib.last_error(lib)
