"""CUDA path vs the CPU oracle, through the C ABI (B200 only).

Integer/index results must be bit-exact; the projections, SwiGLU, router
and combine follow the oracle's canonical arithmetic and must be bit-exact
too.  Every floating-point comparison also states the north-star tolerance
(max-abs 2e-2 relative to the output scale, mean-rel 5e-3) it implies.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import bf16, moe

pytestmark = pytest.mark.gpu

TOL_MAX_ABS = 2e-2
TOL_MEAN_REL = 5e-3


def _np(t):
    import torch

    if t.dtype == torch.bfloat16:
        return t.float().cpu().numpy()
    if t.dtype == torch.int32:
        return t.cpu().numpy().view(np.uint32)
    return t.cpu().numpy()


def _bits(a):
    return bf16.f32_to_bits(np.asarray(a, np.float32))


def assert_bf16_equal(got, want, what=""):
    g, w = _bits(got), _bits(want)
    bad = np.count_nonzero(g != w)
    if bad:
        gi = np.asarray(got, np.float64)
        wi = np.asarray(want, np.float64)
        raise AssertionError(f"{what}: {bad}/{g.size} bf16 mismatches, max abs {np.abs(gi - wi).max():.3g}")


def assert_north_star(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    err = np.abs(got - want)
    assert err.max() <= TOL_MAX_ABS * max(1.0, np.abs(want).max())
    assert err.mean() <= TOL_MEAN_REL * max(np.abs(want).mean(), 1e-30)


def _bank_np(bank):
    """torch expert bank -> oracle triples (uint32 words, f32 scales, f32 biases)."""
    out = {}
    for k, (w, s, b) in bank.items():
        out[k] = (_np(w), _np(s), _np(b))
    return out


# --------------------------------------------------------------------------
# elementwise / small kernels
# --------------------------------------------------------------------------


def test_dequantize_bit_exact(cuda_lib):
    import torch

    from flashnext_b200 import _lib, synthetic
    w, s, b = synthetic.q4_projection(3, 64, 256, 32, seed=11)
    out = torch.empty((3, 64, 256), dtype=torch.bfloat16, device="cuda")
    _lib.check(cuda_lib.fnmoe_dequantize(w.data_ptr(), s.data_ptr(), b.data_ptr(), out.data_ptr(), 3 * 64, 256, 32,
                                         torch.cuda.current_stream().cuda_stream), "dequantize")
    want = bf16.bits_to_f32(moe.dequantize(_np(w), _np(s), _np(b), 32))
    assert_bf16_equal(_np(out), want, "dequantize")


@pytest.mark.parametrize("up_bits", [0x3F80, 0x3F9E, 0xC0A0])
def test_swiglu_exhaustive_bit_exact(cuda_lib, up_bits):
    """All 65,536 gate encodings (tests/unit/test_swiglu_contract.py:63-83 contract)."""
    import torch

    from flashnext_b200 import _lib
    gates = torch.arange(65536, dtype=torch.int32, device="cuda").to(torch.int16).view(torch.bfloat16)
    up = torch.full((65536,), 0, dtype=torch.int16, device="cuda")
    up.fill_(up_bits - 65536 if up_bits >= 32768 else up_bits)
    up = up.view(torch.bfloat16)
    out = torch.empty_like(gates)
    _lib.check(cuda_lib.fnmoe_swiglu(gates.data_ptr(), up.data_ptr(), out.data_ptr(), 65536,
                                     torch.cuda.current_stream().cuda_stream), "swiglu")
    want = moe.swiglu_bf16(_np(gates), _np(up))
    got = _np(out)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert_bf16_equal(got[~nan], want[~nan], "swiglu")


def test_weighted_combine_known_answer_on_gpu(golden):
    import torch

    from flashnext_b200 import weighted_combine
    out = weighted_combine(torch.tensor(golden["combine_outputs"]).cuda(), torch.tensor(golden["combine_routes"]).cuda(),
                           torch.tensor(golden["combine_scores"]).cuda())
    np.testing.assert_array_equal(out.cpu().numpy(), golden["combine_result"])
    host = weighted_combine(golden["combine_outputs"], golden["combine_routes"], golden["combine_scores"])
    np.testing.assert_array_equal(host, golden["combine_result"])


# --------------------------------------------------------------------------
# router
# --------------------------------------------------------------------------


@pytest.mark.parametrize("tokens,hidden,experts,zipf", [(1, 2048, 512, None), (64, 2048, 512, 1.1),
                                                        (5, 3072, 512, None), (3, 256, 40, None),
                                                        (100, 2176, 40, None), (70, 3072, 512, None)])
def test_router_topk_bit_exact(cuda_lib, tokens, hidden, experts, zipf):
    from flashnext_b200 import router, synthetic
    if zipf:
        x, w = synthetic.zipf_router(tokens, hidden, experts, zipf, seed=3)
    else:
        x = synthetic.bf16_normal((tokens, hidden), seed=4)
        w = synthetic.bf16_normal((experts, hidden), 0.02, seed=5)
    k = min(10, experts)
    inds, scores, mass, logits = router.router_topk(x, w, k)
    o_inds, o_scores, o_mass, o_logits = moe.router(_np(x), _np(w), k)
    assert_bf16_equal(_np(logits), o_logits, "logits")
    np.testing.assert_array_equal(_np(inds), o_inds)
    assert_bf16_equal(_np(scores), o_scores, "renormalised scores")
    assert_bf16_equal(_np(mass), o_mass[:, 0], "topk mass")


@pytest.mark.parametrize("tokens,hidden", [(64, 2048), (200, 1024), (5, 2048), (70, 2056)])
def test_router_topk_shared_workspace_bit_exact(cuda_lib, tokens, hidden):
    """fnmoe_router_topk_shared_ws (the expert-parallel layer's router): the
    tensor-core path from 64 tokens, the GEMV below or off the 128-byte grid;
    logits, shared logit, top-k and shared gate bit for bit against the
    oracle; a workspace one byte short is refused."""
    import ctypes

    import torch

    from flashnext_b200 import _lib, synthetic
    lib = _lib.ensure_device()
    E, k = 512, 10
    x = synthetic.bf16_normal((tokens, hidden), seed=61)
    w = synthetic.bf16_normal((E, hidden), 0.02, seed=62)
    wg = synthetic.bf16_normal((hidden,), 0.02, seed=63)
    need = ctypes.c_uint64(0)
    assert lib.fnmoe_router_workspace_size(tokens, hidden, E, 1, ctypes.byref(need)) == _lib.OK
    assert (need.value > 0) == (tokens >= 64 and hidden % 128 == 0)
    ws = torch.empty(max(need.value, 1), dtype=torch.uint8, device="cuda")
    inds = torch.empty((tokens, k), dtype=torch.int32, device="cuda")
    scores = torch.empty((tokens, k), dtype=torch.bfloat16, device="cuda")
    mass = torch.empty((tokens,), dtype=torch.bfloat16, device="cuda")
    logits = torch.empty((tokens, E), dtype=torch.bfloat16, device="cuda")
    sl = torch.empty((tokens,), dtype=torch.bfloat16, device="cuda")
    sg = torch.empty((tokens,), dtype=torch.bfloat16, device="cuda")

    def call(nbytes):
        return lib.fnmoe_router_topk_shared_ws(x.data_ptr(), w.data_ptr(), wg.data_ptr(), tokens, hidden, E, k, 1.0,
                                               inds.data_ptr(), scores.data_ptr(), mass.data_ptr(), logits.data_ptr(),
                                               sl.data_ptr(), sg.data_ptr(), ws.data_ptr(), nbytes, None)

    if need.value:
        assert call(need.value - 1) == _lib.ERR_WORKSPACE
    for _ in range(2):  # twice: the split-K partial sums must start from zero again
        assert call(need.value) == _lib.OK
        torch.cuda.synchronize()
        o_inds, o_scores, _, o_logits = moe.router(_np(x), _np(w), k)
        assert_bf16_equal(_np(logits), o_logits, "logits")
        np.testing.assert_array_equal(_np(inds), o_inds)
        assert_bf16_equal(_np(scores), o_scores, "renormalised scores")
        o_sl = moe.router_logits(_np(x), _np(wg).reshape(1, -1))[:, 0]
        assert_bf16_equal(_np(sl), o_sl, "shared logit")


@pytest.mark.parametrize("tokens", [3, 20])
def test_router_topk_limits_bit_exact(cuda_lib, tokens):
    """The interface limits: 1,024 experts (32 logits per lane) and top-k 16,
    through the one-CTA (<= 8 tokens) and the warp-per-token top-k."""
    from flashnext_b200 import router, synthetic
    x = synthetic.bf16_normal((tokens, 1024), seed=41)
    w = synthetic.bf16_normal((1024, 1024), 0.02, seed=42)
    inds, scores, mass, logits = router.router_topk(x, w, 16)
    o_inds, o_scores, o_mass, o_logits = moe.router(_np(x), _np(w), 16)
    assert_bf16_equal(_np(logits), o_logits, "logits")
    np.testing.assert_array_equal(_np(inds), o_inds)
    assert_bf16_equal(_np(scores), o_scores, "renormalised scores")


@pytest.mark.parametrize("tokens", [2, 24])
def test_moe_layer_limits_bit_exact(cuda_lib, tokens):
    """A layer with 1,024 experts and top-k 16 (grouping over 1,025 bins)."""
    from flashnext_b200 import synthetic
    from flashnext_b200.moe_block import SparseMoEBlock
    L = synthetic.moe_layer(tokens, 512, 256, 1024, 16, 32, seed=tokens + 90)
    block = SparseMoEBlock(L.router_weight, L.experts, top_k=16, shared=L.shared,
                           shared_expert_gate=L.shared_expert_gate)
    out = block(L.x)
    nb = _bank_np(L.experts)
    sh = {k: (_np(w), _np(s), _np(b)) for k, (w, s, b) in L.shared.items()}
    ref = moe.moe_block(_np(L.x), _np(L.router_weight), 16, nb["gate_proj"], nb["up_proj"], nb["down_proj"],
                        (sh["gate_proj"], sh["up_proj"], sh["down_proj"]), _np(L.shared_expert_gate))
    np.testing.assert_array_equal(_np(block.last_inds), ref["inds"])
    assert_bf16_equal(_np(out), ref["out"], "layer output")


def test_router_ties_resolve_to_lower_expert(cuda_lib):
    import torch

    from flashnext_b200 import router
    logits = torch.zeros((2, 64), dtype=torch.bfloat16, device="cuda")
    logits[0, [5, 9, 17, 33]] = 3.0
    logits[1, 60] = 1.0
    inds, raw, mass = router.router(logits, 6)
    o_inds, o_raw, o_mass = moe.topk(moe.softmax_bf16(_np(logits)), 6)
    np.testing.assert_array_equal(_np(inds), o_inds)
    assert _np(inds)[0].tolist()[:4] == [5, 9, 17, 33]
    assert_bf16_equal(_np(raw), o_raw)


def test_group_tokens_exact(cuda_lib):
    import torch

    from flashnext_b200 import router
    rng = np.random.default_rng(9)
    routes = rng.integers(0, 37, (50, 10)).astype(np.int32)
    counts, offsets, order = router.group_tokens(torch.tensor(routes).cuda(), 37)
    o_counts, o_offsets, o_order = moe.group_tokens(routes, 37)
    np.testing.assert_array_equal(counts.cpu().numpy(), o_counts)
    np.testing.assert_array_equal(offsets.cpu().numpy(), o_offsets)
    np.testing.assert_array_equal(order.cpu().numpy(), o_order)


# --------------------------------------------------------------------------
# executor (metal_runtime.execute contract)
# --------------------------------------------------------------------------


def _executor_case(tokens, slots, hidden, inter, experts, group, seed):
    from flashnext_b200 import synthetic
    bank = synthetic.expert_bank(experts, hidden, inter, group, seed=seed)
    x = synthetic.bf16_normal((tokens, hidden), seed=seed + 50)
    rng = np.random.default_rng(seed)
    routes = np.stack([rng.permutation(experts)[:slots] for _ in range(tokens)]).astype(np.int32)
    scores = rng.dirichlet(np.ones(slots), size=tokens).astype(np.float32)
    return bank, x, routes, scores


@pytest.mark.parametrize("tokens,slots,hidden,inter,experts,group", [
    (1, 10, 2048, 512, 64, 32),
    (3, 2, 64, 32, 4, 32),
    (8, 10, 256, 128, 16, 32),
    (2, 7, 2560, 640, 8, 32),
    (4, 3, 256, 128, 6, 64),
    (1, 1, 32, 32, 1, 32),
])
def test_executor_bit_exact(cuda_lib, tokens, slots, hidden, inter, experts, group):
    import torch

    from flashnext_b200 import MoEExecutor
    bank, x, routes, scores = _executor_case(tokens, slots, hidden, inter, experts, group, seed=tokens * 7 + slots)
    ex = MoEExecutor(experts, hidden, slots, group_size=group)
    out = ex.execute(x, torch.tensor(routes).cuda(), bank, scores=torch.tensor(scores).cuda())
    assert ex.last_path == "cuda"
    nb = _bank_np(bank)
    want = moe.executor(_np(x), routes, nb["gate_proj"], nb["up_proj"], nb["down_proj"], scores=scores,
                        group_size=group)
    assert_bf16_equal(_np(out), want, "combined output")
    assert_north_star(_np(out), want)
    g, u, d = ex.execute(x, torch.tensor(routes).cuda(), bank, return_all=True)
    og, ou, od = moe.executor(_np(x), routes, nb["gate_proj"], nb["up_proj"], nb["down_proj"], group_size=group,
                              return_all=True)
    assert_bf16_equal(_np(g), og, "gate")
    assert_bf16_equal(_np(u), ou, "up")
    assert_bf16_equal(_np(d), od, "down")
    per_slot = ex.execute(x, torch.tensor(routes).cuda(), bank)
    assert_bf16_equal(_np(per_slot), od, "per-slot down")


@pytest.mark.parametrize("offset", [8, 100, 255])
def test_executor_misaligned_workspace(cuda_lib, offset):
    """A workspace pointer on any byte boundary works: the library rounds its
    start up to 256 bytes within the reported size (which includes that
    slack); the result equals the oracle's."""
    import torch

    from flashnext_b200 import _lib
    bank, x, routes, scores = _executor_case(3, 4, 256, 128, 6, 32, seed=61)
    r = torch.tensor(routes).cuda()
    sc = torch.tensor(scores).cuda()
    out = torch.empty((3, 256), dtype=torch.bfloat16, device="cuda")
    a = _lib.FnMoEArgs()
    a.abi_version = _lib.ABI_VERSION
    a.x = x.data_ptr()
    for name, key in (("gate_proj", "gate"), ("up_proj", "up"), ("down_proj", "down")):
        w, s, b = bank[name]
        setattr(a, f"{key}_weight", w.data_ptr())
        setattr(a, f"{key}_scales", s.data_ptr())
        setattr(a, f"{key}_biases", b.data_ptr())
    a.routes, a.scores, a.scores_dtype, a.output = r.data_ptr(), sc.data_ptr(), _lib.DTYPE_F32, out.data_ptr()
    a.tokens, a.slots, a.hidden_size, a.inter_size, a.expert_count, a.group_size = 3, 4, 256, 128, 6, 32
    need = ctypes.c_uint64(0)
    _lib.check(cuda_lib.fnmoe_moe_workspace_size(ctypes.byref(a), ctypes.byref(need)), "workspace_size")
    ws = torch.empty(need.value + offset, dtype=torch.uint8, device="cuda")
    a.workspace, a.workspace_bytes = ws.data_ptr() + offset, need.value
    _lib.check(cuda_lib.fnmoe_moe_execute(ctypes.byref(a), torch.cuda.current_stream().cuda_stream), "execute")
    a.workspace_bytes = need.value - 256 - 1  # below the aligned carves themselves: rejected, nothing runs
    assert cuda_lib.fnmoe_moe_execute(ctypes.byref(a), torch.cuda.current_stream().cuda_stream) == _lib.ERR_WORKSPACE
    nb = _bank_np(bank)
    want = moe.executor(_np(x), routes, nb["gate_proj"], nb["up_proj"], nb["down_proj"], scores=scores)
    assert_bf16_equal(_np(out), want, "combined output")


def test_executor_shared_epilogues_bit_exact(cuda_lib):
    import torch

    from flashnext_b200 import MoEExecutor, synthetic
    bank, x, routes, scores = _executor_case(2, 4, 256, 128, 8, 32, seed=21)
    sy = synthetic.bf16_normal((2, 256), 0.5, seed=22)
    sh = synthetic.bf16_normal((2, 256), 0.5, seed=23)
    sg = torch.tensor([[0.333984375], [0.75]], dtype=torch.bfloat16, device="cuda")
    ex = MoEExecutor(8, 256, 4)
    nb = _bank_np(bank)
    r = torch.tensor(routes).cuda()
    sc_bf = torch.tensor(scores).cuda().to(torch.bfloat16)
    for kw, okw in (({"shared_y": sy}, {"shared_y": _np(sy)}),
                    ({"shared": sh, "shared_gate": sg}, {"shared": _np(sh), "shared_gate": _np(sg)})):
        out = ex.execute(x, r, bank, scores=sc_bf, **kw)
        want = moe.executor(_np(x), routes, nb["gate_proj"], nb["up_proj"], nb["down_proj"], scores=_np(sc_bf), **okw)
        assert_bf16_equal(_np(out), want, str(list(kw)))
        # fused epilogue == unfused + add, bit for bit (test_metal_runtime.py:641-662)
        unfused = ex.execute(x, r, bank, scores=sc_bf)
        if "shared_y" in kw:
            ref = (unfused.float() + sy.float()).to(torch.bfloat16)
        else:
            ref = (unfused.float() + (sh.float() * sg.float()).to(torch.bfloat16).float()).to(torch.bfloat16)
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


def test_table_routes_match_projection_buffers(cuda_lib):
    """Bit-31 table records and stream records give the array result
    (test_metal_runtime.py:664-827)."""
    import torch

    from flashnext_b200 import ExpertTable, MoEExecutor
    bank, x, routes, scores = _executor_case(3, 4, 256, 128, 6, 32, seed=31)
    ex = MoEExecutor(6, 256, 4)
    r = torch.tensor(routes).cuda()
    sc = torch.tensor(scores).cuda()
    base = ex.execute(x, r, bank, scores=sc)
    table = ExpertTable.from_projections(bank["gate_proj"], bank["up_proj"], bank["down_proj"], 32)
    slot_routes = table.routes(routes.astype(np.int64))
    via_table = ex.execute(x, slot_routes, bank, scores=sc, slab_pack=table)
    assert torch.equal(base.view(torch.int16), via_table.view(torch.int16))
    # stream records: routes without bit 31 address a header-less record buffer
    stream = table.buffer[table.header_size:]
    mixed = slot_routes.clone()
    mixed[:, ::2] = r[:, ::2]
    via_stream = ex.execute(x, mixed, bank, scores=sc, slab_pack=table, stream_pack=stream)
    assert torch.equal(base.view(torch.int16), via_stream.view(torch.int16))


def test_out_of_range_routes_are_flagged_not_read(cuda_lib):
    import torch

    from flashnext_b200 import MoEExecutor, _lib
    bank, x, routes, scores = _executor_case(2, 3, 64, 32, 4, 32, seed=41)
    routes[1, 2] = 9  # outside the 4-expert bank
    _lib.read_device_errors(clear=True)
    ex = MoEExecutor(4, 64, 3)
    out = ex.execute(x, torch.tensor(routes).cuda(), bank, scores=torch.tensor(scores).cuda())
    flags = _lib.read_device_errors(clear=True)
    assert flags & _lib.ERR_BAD_ROUTE
    nb = _bank_np(bank)
    # token 0 is untouched; token 1 combines only its valid slots
    want0 = moe.executor(_np(x)[:1], routes[:1], nb["gate_proj"], nb["up_proj"], nb["down_proj"], scores=scores[:1])
    assert_bf16_equal(_np(out)[:1], want0, "valid token")


# --------------------------------------------------------------------------
# full layer (router + experts + shared)
# --------------------------------------------------------------------------


def _layer_inputs(tokens, hidden=2048, inter=512, experts=512, zipf=None, seed=0):
    from flashnext_b200 import synthetic
    return synthetic.moe_layer(tokens, hidden, inter, experts, 10, 32, zipf=zipf, seed=seed)


def _oracle_layer(L):
    nb = _bank_np(L.experts)
    sh = {k: (_np(w), _np(s), _np(b)) for k, (w, s, b) in L.shared.items()}
    return moe.moe_block(_np(L.x), _np(L.router_weight), L.top_k, nb["gate_proj"], nb["up_proj"], nb["down_proj"],
                         (sh["gate_proj"], sh["up_proj"], sh["down_proj"]), _np(L.shared_expert_gate))


@pytest.mark.parametrize("tokens,zipf", [(1, None), (64, 1.1), (9, None)])
def test_moe_layer_bit_exact(cuda_lib, tokens, zipf):
    from flashnext_b200.moe_block import SparseMoEBlock
    L = _layer_inputs(tokens, zipf=zipf, seed=tokens)
    block = SparseMoEBlock(L.router_weight, L.experts, top_k=10, shared=L.shared,
                           shared_expert_gate=L.shared_expert_gate)
    out = block(L.x)
    ref = _oracle_layer(L)
    np.testing.assert_array_equal(_np(block.last_inds), ref["inds"])
    assert_bf16_equal(_np(block.last_logits), ref["logits"], "logits")
    assert_bf16_equal(_np(block.last_scores), ref["scores"], "scores")
    assert_bf16_equal(_np(out), ref["out"], "layer output")
    assert_north_star(_np(out), ref["out"])


@pytest.mark.parametrize("tokens,zipf,threshold,min_keep", [(1, None, 0.5, 1), (5, None, 0.85, 2),
                                                              (64, 1.1, 0.5, 1), (64, 1.1, 0.9, 3)])
def test_moe_layer_adaptive_keep_bit_exact(cuda_lib, tokens, zipf, threshold, min_keep):
    """Adaptive keep (adaptive_topk.py:43-50,75-261) on the GPU: kept slot
    counts, indices (dropped -> slot 0's expert), renormalised scores and the
    layer output against the oracle, bit for bit."""
    from flashnext_b200 import _lib
    from flashnext_b200.moe_block import SparseMoEBlock
    _lib.read_device_errors()  # start from a clear error word
    L = _layer_inputs(tokens, zipf=zipf, seed=tokens + 31)
    block = SparseMoEBlock(L.router_weight, L.experts, top_k=10, shared=L.shared,
                           shared_expert_gate=L.shared_expert_gate, keep_threshold=threshold, min_keep=min_keep)
    out = block(L.x)
    nb = _bank_np(L.experts)
    sh = {k: (_np(w), _np(s), _np(b)) for k, (w, s, b) in L.shared.items()}
    ref = moe.moe_block(_np(L.x), _np(L.router_weight), 10, nb["gate_proj"], nb["up_proj"], nb["down_proj"],
                        (sh["gate_proj"], sh["up_proj"], sh["down_proj"]), _np(L.shared_expert_gate),
                        threshold=threshold, min_keep=min_keep)
    # some tokens really drop slots at these thresholds
    assert (ref["scores"] == 0).any()
    np.testing.assert_array_equal(_np(block.last_inds), ref["inds"])
    assert_bf16_equal(_np(block.last_scores), ref["scores"], "scores")
    assert_bf16_equal(_np(out), ref["out"], "layer output")
    assert _lib.read_device_errors() == 0


def test_moe_layer_adaptive_keep_prefill_within_tolerance(cuda_lib):
    from flashnext_b200 import _lib
    from flashnext_b200.moe_block import SparseMoEBlock
    _lib.read_device_errors()
    L = _layer_inputs(64, zipf=None, seed=77)
    kw = dict(top_k=10, shared=L.shared, shared_expert_gate=L.shared_expert_gate, keep_threshold=0.6)
    pre = SparseMoEBlock(L.router_weight, L.experts, path="prefill", **kw)
    dec = SparseMoEBlock(L.router_weight, L.experts, path="decode", **kw)
    out_p, out_d = _np(pre(L.x)), _np(dec(L.x))
    np.testing.assert_array_equal(_np(pre.last_inds), _np(dec.last_inds))
    assert_north_star(out_p, out_d)
    assert _lib.read_device_errors() == 0


def test_moe_layer_is_batch_invariant(cuda_lib):
    import torch

    from flashnext_b200.moe_block import SparseMoEBlock
    L = _layer_inputs(12, hidden=512, inter=256, experts=64, seed=5)
    block = SparseMoEBlock(L.router_weight, L.experts, top_k=10, shared=L.shared,
                           shared_expert_gate=L.shared_expert_gate)
    full = block(L.x).clone()
    for t in (0, 5, 11):
        one = block(L.x[t:t + 1])
        assert torch.equal(one.view(torch.int16), full[t:t + 1].view(torch.int16))


def test_moe_layer_with_expert_table(cuda_lib):
    import torch

    from flashnext_b200 import ExpertTable
    from flashnext_b200.moe_block import SparseMoEBlock
    L = _layer_inputs(4, hidden=512, inter=256, experts=32, seed=8)
    arrays = SparseMoEBlock(L.router_weight, L.experts, top_k=10, shared=L.shared,
                            shared_expert_gate=L.shared_expert_gate)(L.x).clone()
    # records in a shuffled order; the route map sends expert e to its record
    perm = np.random.default_rng(0).permutation(32)
    table = ExpertTable(32, 512, 256, 32)
    table.write_bank(L.experts["gate_proj"], L.experts["up_proj"], L.experts["down_proj"],
                     experts=range(32), slots=perm.tolist())
    route_map = torch.tensor(((perm.astype(np.int64) | 0x80000000) - (1 << 32)), dtype=torch.int32).cuda()
    via = SparseMoEBlock(L.router_weight, table, top_k=10, shared=L.shared,
                         shared_expert_gate=L.shared_expert_gate, route_map=route_map)(L.x)
    assert torch.equal(arrays.view(torch.int16), via.view(torch.int16))


@pytest.mark.parametrize("tokens,hidden,inter,experts,group", [
    (64, 2048, 512, 512, 32),   # headline layer, Zipf routing
    (5, 2560, 640, 24, 32),     # down rows (320 bytes) end in a partial block; Gc = 20
    (7, 1024, 256, 16, 64),     # group size 64
    (2, 1024, 256, 16, 64),     # group size 64, small-batch K-split path
    (3, 3072, 640, 12, 32),     # qwen4 full-depth layer shape
])
def test_tiled_layer_matches_arrays_and_oracle(cuda_lib, tokens, hidden, inter, experts, group):
    """The tiled tables (one bulk-copied chunk per row group and block) give
    the same bits as the reference-layout arrays, and both match the oracle."""
    import torch

    from flashnext_b200 import synthetic
    from flashnext_b200.moe_block import SparseMoEBlock
    k = min(10, experts)
    L = synthetic.moe_layer(tokens, hidden, inter, experts, k, group, zipf=1.1 if tokens >= 64 else None,
                            seed=tokens + hidden)
    kw = dict(top_k=k, shared=L.shared, shared_expert_gate=L.shared_expert_gate, group_size=group)
    tiled = SparseMoEBlock(L.router_weight, L.experts, **kw)
    assert tiled.tiled is not None
    arrays = SparseMoEBlock(L.router_weight, L.experts, tiled=False, **kw)
    assert arrays.tiled is None
    a = arrays(L.x).clone()
    t = tiled(L.x)
    assert torch.equal(a.view(torch.int16), t.view(torch.int16))
    if tokens <= 7:
        nb = _bank_np(L.experts)
        sh = {n: (_np(w), _np(s), _np(b)) for n, (w, s, b) in L.shared.items()}
        ref = moe.moe_block(_np(L.x), _np(L.router_weight), k, nb["gate_proj"], nb["up_proj"], nb["down_proj"],
                            (sh["gate_proj"], sh["up_proj"], sh["down_proj"]), _np(L.shared_expert_gate),
                            group_size=group)
        assert_bf16_equal(_np(t), ref["out"], "tiled layer output")


@pytest.mark.parametrize("tokens,experts,zipf", [(64, 64, None), (200, 32, 1.1), (13, 16, None)])
def test_prefill_gemm_layer_within_tolerance(cuda_lib, tokens, experts, zipf):
    """tcgen05 prefill path (dequantised bf16 weights, float32 tensor-core
    accumulation) against the exact oracle layer and the exact decode path:
    the north-star tolerance (max-abs 2e-2, mean-rel 5e-3), same routing."""
    import torch

    from flashnext_b200 import synthetic
    from flashnext_b200.moe_block import SparseMoEBlock
    L = synthetic.moe_layer(tokens, 2048, 512, experts, 10, 32, zipf=zipf, seed=tokens + 5)
    kw = dict(top_k=10, shared=L.shared, shared_expert_gate=L.shared_expert_gate)
    pre = SparseMoEBlock(L.router_weight, L.experts, path="prefill", **kw)
    dec = SparseMoEBlock(L.router_weight, L.experts, path="decode", **kw)
    out_p = pre(L.x).clone()
    out_d = dec(L.x).clone()
    assert torch.equal(pre.last_inds, dec.last_inds)
    assert torch.isfinite(out_p.float()).all()
    ref = _oracle_layer(L)
    np.testing.assert_array_equal(_np(pre.last_inds), ref["inds"])
    assert_north_star(_np(out_p), ref["out"])
    assert_north_star(_np(out_p), _np(out_d))


# --------------------------------------------------------------------------
# paged attention
# --------------------------------------------------------------------------


@pytest.mark.parametrize("batch,hq,hkv,d,page,ctx", [
    (2, 16, 2, 256, 64, (1000, 1000)),
    (3, 24, 4, 256, 64, (256, 300)),
    (4, 8, 8, 128, 16, (1, 40)),
    (2, 16, 2, 64, 64, (5000, 7000)),
])
def test_paged_decode_matches_oracle_and_truth(cuda_lib, batch, hq, hkv, d, page, ctx):
    from flashnext_b200 import synthetic
    from flashnext_b200.paged_attention import paged_decode
    from oracle import attention as attn
    P = synthetic.paged_decode_inputs(batch, hq, hkv, d, page, ctx, seed=batch * 13 + d)
    out = paged_decode(P.q, P.k_cache, P.v_cache, P.block_table, P.context_lens, P.scale)
    got = _np(out)
    want = attn.paged_decode_oracle(_np(P.q), _np(P.k_cache), _np(P.v_cache), P.block_table.cpu().numpy(),
                                    P.context_lens.cpu().numpy(), P.scale)
    assert_north_star(got, want)
    table = P.block_table.cpu().numpy()
    kc, vc = _np(P.k_cache), _np(P.v_cache)
    for b in range(batch):
        n = int(P.context_lens[b])
        pages = table[b, : -(-n // page)]
        k = kc[pages].reshape(-1, hkv, d)[:n]
        v = vc[pages].reshape(-1, hkv, d)[:n]
        truth = attn.dense_truth(_np(P.q)[b], k, v, P.scale)
        assert np.abs(got[b] - truth).max() / np.abs(truth).max() < 1.5e-2


def test_executor_tiny_and_subnormal_activations_bit_exact(cuda_lib):
    """Groups whose largest activation is below 2^-104 take the two-step
    power-of-two scaling; bfloat16 subnormals enter the fixed point exactly."""
    import torch

    from flashnext_b200 import MoEExecutor
    bank, x, routes, scores = _executor_case(3, 4, 256, 128, 6, 32, seed=51)
    x = x.clone()
    x[0] = (x[0].float() * 2.0 ** -110).to(torch.bfloat16)      # tiny but normal
    x[1, :64] = (x[1, :64].float() * 2.0 ** -128).to(torch.bfloat16)  # partly subnormal
    x[2, 32:64] = 0                                              # an all-zero group
    ex = MoEExecutor(6, 256, 4)
    nb = _bank_np(bank)
    g, u, d = ex.execute(x, torch.tensor(routes).cuda(), bank, return_all=True)
    og, ou, od = moe.executor(_np(x), routes, nb["gate_proj"], nb["up_proj"], nb["down_proj"], return_all=True)
    assert_bf16_equal(_np(g), og, "gate")
    assert_bf16_equal(_np(u), ou, "up")
    assert_bf16_equal(_np(d), od, "down")


# --------------------------------------------------------------------------
# float32 activations (metal_runtime.py:371-373; test_metal_runtime.py:516-557)
# --------------------------------------------------------------------------


@pytest.mark.parametrize("tokens,slots,hidden,inter,experts,group", [
    (1, 10, 2048, 512, 64, 32),   # batch 1 (4-warp row kernel on the reference-layout arrays)
    (8, 10, 512, 256, 16, 32),    # 16-warp grouped row kernel (>= 64 pairs)
    (3, 3, 256, 128, 6, 64),      # group size 64
])
def test_executor_float32_activations_bit_exact(cuda_lib, tokens, slots, hidden, inter, experts, group):
    """float32 x: the executor keeps float32 arithmetic (every intermediate
    rounded to float32, the float32 SwiGLU sequence) and returns float32,
    bit for bit equal to the oracle's float32 executor -- combined, per-slot,
    return_all and both shared epilogues."""
    import torch

    from flashnext_b200 import MoEExecutor, synthetic
    bank = synthetic.expert_bank(experts, hidden, inter, group, seed=tokens + 400)
    g = torch.Generator(device="cuda")
    g.manual_seed(tokens + 401)
    x = torch.randn((tokens, hidden), generator=g, device="cuda")  # full float32 mantissas
    rng = np.random.default_rng(tokens)
    routes = np.stack([rng.permutation(experts)[:slots] for _ in range(tokens)]).astype(np.int32)
    scores = rng.dirichlet(np.ones(slots), size=tokens).astype(np.float32)
    sy = rng.normal(0, 0.5, (tokens, hidden)).astype(np.float32)
    sh = rng.normal(0, 0.5, (tokens, hidden)).astype(np.float32)
    sgate = rng.uniform(0, 1, (tokens, 1)).astype(np.float32)
    ex = MoEExecutor(experts, hidden, slots, group_size=group)
    nb = _bank_np(bank)
    r = torch.tensor(routes).cuda()
    xn = x.cpu().numpy()
    out = ex.execute(x, r, bank, scores=torch.tensor(scores).cuda())
    assert out.dtype == torch.float32
    want = moe.executor(xn, routes, nb["gate_proj"], nb["up_proj"], nb["down_proj"], scores=scores,
                        group_size=group, f32=True)
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))
    gg, uu, dd = ex.execute(x, r, bank, return_all=True)
    og, ou, od = moe.executor(xn, routes, nb["gate_proj"], nb["up_proj"], nb["down_proj"], group_size=group,
                              return_all=True, f32=True)
    for got, w in ((gg, og), (uu, ou), (dd, od)):
        np.testing.assert_array_equal(got.cpu().numpy().view(np.uint32), w.view(np.uint32))
    per_slot = ex.execute(x, r, bank)
    np.testing.assert_array_equal(per_slot.cpu().numpy().view(np.uint32), od.view(np.uint32))
    for kw in ({"shared_y": sy}, {"shared": sh, "shared_gate": sgate}):
        got = ex.execute(x, r, bank, scores=torch.tensor(scores).cuda(), **{k: torch.tensor(v).cuda()
                                                                             for k, v in kw.items()})
        w = moe.executor(xn, routes, nb["gate_proj"], nb["up_proj"], nb["down_proj"], scores=scores,
                         group_size=group, f32=True, **kw)
        np.testing.assert_array_equal(got.cpu().numpy().view(np.uint32), w.view(np.uint32))


def test_executor_float32_reference_unit_case(cuda_lib):
    """The reference's mixed-precision unit case (test_metal_runtime.py:516-557):
    float32 x = ((arange(256) % 31) - 15) / 64 with bfloat16 scales/biases,
    routes [[0, 2, 3]], scores [[0.2, 0.3, 0.5]]: float32 output within the
    reference's tolerance (rtol 1e-3, atol 1e-4) of its NumPy executor, and
    bit-exact to the oracle."""
    import torch

    from flashnext_b200 import MoEExecutor, synthetic
    H, I, E = 256, 128, 4
    bank = synthetic.expert_bank(E, H, I, 32, seed=516)
    x = (((np.arange(H, dtype=np.float32) % 31) - 15) / 64).reshape(1, H).astype(np.float32)
    routes = np.array([[0, 2, 3]], dtype=np.int32)
    scores = np.array([[0.2, 0.3, 0.5]], dtype=np.float32)
    got = MoEExecutor(E, H, 3).execute(x, routes, bank, scores=scores)
    assert isinstance(got, np.ndarray) and got.dtype == np.float32
    nb = _bank_np(bank)
    ref = moe.reference_execute(x, routes, nb["gate_proj"], nb["up_proj"], nb["down_proj"], scores=scores)
    np.testing.assert_allclose(got, ref, rtol=1e-3, atol=1e-4)
    want = moe.executor(x, routes, nb["gate_proj"], nb["up_proj"], nb["down_proj"], scores=scores, f32=True)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
