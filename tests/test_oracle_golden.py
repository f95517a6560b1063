"""Pin the CPU oracle against outputs of the reference's own NumPy code.

The fixtures in ``tests/golden/reference_numpy.npz`` were produced by
``tests/golden/make_golden.py`` running ``models/flashnext/metal_runtime.py``
and ``slab_pack.py`` from the reference checkout.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import bf16, moe


@pytest.mark.parametrize("group", [32, 64])
def test_restated_numpy_projection_is_bit_exact(golden, group):
    g = {k[len(f"proj_g{group}_"):]: v for k, v in golden.items() if k.startswith(f"proj_g{group}_")}
    y = moe.reference_numpy_projection(g["x"], g["routes"], g["w"], g["s"], g["b"],
                                       g["y"].shape[-1], False, group)
    np.testing.assert_array_equal(y, g["y"])


@pytest.mark.parametrize("group", [32, 64])
def test_canonical_projection_matches_reference_formula(golden, group):
    """The canonical fixed-point projection is the reference's group formula.

    The reference accumulates in float64 and rounds once; the canonical form
    rounds each group term to float32 -- agreement to float32 precision.
    """
    g = {k[len(f"proj_g{group}_"):]: v for k, v in golden.items() if k.startswith(f"proj_g{group}_")}
    codes = moe.unpack_q4(g["w"])
    for t in range(g["routes"].shape[0]):
        for s in range(g["routes"].shape[1]):
            e = int(g["routes"][t, s])
            y = moe.qmv(g["x"][t:t + 1], codes[e], g["s"][e], g["b"][e], group)[0]
            ref = g["y"][t, s]
            np.testing.assert_allclose(y, ref, rtol=2e-6, atol=2e-6 * np.abs(ref).max())


def _exec_inputs(golden):
    e = {k[len("exec_"):]: v for k, v in golden.items() if k.startswith("exec_")}
    gate = (e["gate_w"], e["gate_s"], e["gate_b"])
    up = (e["up_w"], e["up_s"], e["up_b"])
    down = (e["down_w"], e["down_s"], e["down_b"])
    return e, gate, up, down


def test_restated_reference_executor_is_bit_exact(golden):
    e, gate, up, down = _exec_inputs(golden)
    np.testing.assert_array_equal(
        moe.reference_execute(e["x"], e["routes"], gate, up, down, scores=e["scores"]), e["combined"])
    np.testing.assert_array_equal(moe.reference_execute(e["x"], e["routes"], gate, up, down), e["per_slot"])
    g_all, u_all, d_all = moe.reference_execute(e["x"], e["routes"], gate, up, down, return_all=True)
    np.testing.assert_array_equal(g_all, e["all_gate"])
    np.testing.assert_array_equal(u_all, e["all_up"])
    np.testing.assert_array_equal(d_all, e["all_down"])
    np.testing.assert_array_equal(
        moe.reference_execute(e["x"], e["routes"], gate, up, down, scores=e["scores"], shared_y=e["shared_y"]),
        e["with_shared_y"])
    np.testing.assert_array_equal(
        moe.reference_execute(e["x"], e["routes"], gate, up, down, scores=e["scores"], shared=e["shared"],
                              shared_gate=e["shared_gate"]),
        e["with_shared_parts"])


def test_bf16_executor_tracks_reference_executor(golden):
    """The bfloat16 CUDA-path semantics agree with the reference's float32 path.

    The CUDA path rounds gate/up/SwiGLU/down to bfloat16 where the Metal
    kernels do (metal_runtime.py:262-333); the reference NumPy backend keeps
    float32 throughout.  The differences are bfloat16 rounding noise: the
    north-star tolerance (max-abs 2e-2 relative to the output scale,
    mean-rel 5e-3) holds.
    """
    e, gate, up, down = _exec_inputs(golden)
    ours = moe.executor(e["x"], e["routes"], gate, up, down, scores=e["scores"], shared_y=e["shared_y"])
    ref = e["with_shared_y"].astype(np.float64)
    err = np.abs(ours - ref)
    assert err.max() <= 2e-2 * max(1.0, np.abs(ref).max())
    assert err.mean() / np.abs(ref).mean() <= 5e-3


def test_weighted_combine_known_answer(golden):
    out = moe.weighted_combine(golden["combine_outputs"], golden["combine_routes"], golden["combine_scores"])
    np.testing.assert_array_equal(out, golden["combine_result"])
    np.testing.assert_array_equal(out, np.array([[25.75, 51.5], [192.0, 256.0]], dtype=np.float32))
    np.testing.assert_array_equal(moe.weighted_combine(golden["combine_outputs"], golden["combine_routes"],
                                                       golden["combine_scores"]), out)


@pytest.mark.parametrize("group", [32, 64])
def test_record_layout_matches_reference_slab_layout(golden, group):
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "macqwen-releases_b200"))
    from flashnext_b200.expert_table import HEADER_SIZE, record_layout

    lay = record_layout(2560, 640, group)
    assert lay.offsets == tuple(int(v) for v in golden[f"slab_g{group}_offsets"])
    assert lay.record_stride == int(golden[f"slab_g{group}_stride"])
    assert HEADER_SIZE == int(golden["slab_header"])
    if group == 32:
        assert lay.record_stride == 3_072_000
        assert lay.offsets[-1] + 102_400 == lay.record_stride


def test_golden_inputs_are_bfloat16_exact(golden):
    for key in ("exec_x", "exec_gate_s", "exec_gate_b", "proj_g32_x", "proj_g32_s"):
        v = golden[key].astype(np.float32)
        np.testing.assert_array_equal(bf16.round_f32(v), v)


def _exec32_inputs(golden):
    e, gate, up, down = _exec_inputs(golden)
    f = {k[len("exec32_"):]: v for k, v in golden.items() if k.startswith("exec32_")}
    return e, f, gate, up, down


def test_restated_reference_executor_float32_is_bit_exact(golden):
    """float32 activations through the reference NumPy executor: the
    restatement reproduces every output of the reference run bit for bit."""
    e, f, gate, up, down = _exec32_inputs(golden)
    x, r = f["x"], e["routes"]
    np.testing.assert_array_equal(moe.reference_execute(x, r, gate, up, down, scores=f["scores"]), f["combined"])
    np.testing.assert_array_equal(moe.reference_execute(x, r, gate, up, down), f["per_slot"])
    g_all, u_all, d_all = moe.reference_execute(x, r, gate, up, down, return_all=True)
    np.testing.assert_array_equal(g_all, f["all_gate"])
    np.testing.assert_array_equal(u_all, f["all_up"])
    np.testing.assert_array_equal(d_all, f["all_down"])


def test_canonical_float32_executor_matches_reference_run(golden):
    """The canonical float32 path (fixed-point projections, the float32
    SwiGLU sequence, slot-ordered float32 combine) against the reference's
    float32 run: the two differ only in float32 rounding order (the reference
    accumulates each projection in float64 and uses u * g / (1 + exp(-g))),
    so they agree to float32 precision -- relative 1e-5 of each output's scale."""
    e, f, gate, up, down = _exec32_inputs(golden)
    x, r = f["x"], e["routes"]
    cases = [
        (moe.executor(x, r, gate, up, down, scores=f["scores"], f32=True), f["combined"]),
        (moe.executor(x, r, gate, up, down, f32=True), f["per_slot"]),
        (moe.executor(x, r, gate, up, down, scores=f["scores"], shared_y=f["shared_y"], f32=True),
         f["with_shared_y"]),
        (moe.executor(x, r, gate, up, down, scores=f["scores"], shared=f["shared"], shared_gate=f["shared_gate"],
                      f32=True), f["with_shared_parts"]),
    ]
    g_all, u_all, d_all = moe.executor(x, r, gate, up, down, return_all=True, f32=True)
    cases += [(g_all, f["all_gate"]), (u_all, f["all_up"]), (d_all, f["all_down"])]
    for got, want in cases:
        assert got.dtype == np.float32 and got.shape == want.shape
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5 * np.abs(want).max())


def test_float32_swiglu_sequence():
    """The float32 SwiGLU sequence against float64 evaluation of g*sigmoid(g)*u:
    a few float32 ulps; where exp(|g|) overflows float32 the sequence gives
    sigma = 0 or 1 exactly (an absolute error below 1e-30)."""
    rng = np.random.default_rng(5)
    g = np.concatenate([rng.normal(0, 4, 4000), [0.0, -0.0, 90.0, -90.0, 1e-30]]).astype(np.float32)
    u = rng.normal(0, 1, g.shape).astype(np.float32)
    got = moe.swiglu_f32(g, u).astype(np.float64)
    gd, ud = g.astype(np.float64), u.astype(np.float64)
    want = gd / (1.0 + np.exp(-gd)) * ud
    assert np.all(np.abs(got - want) <= 4 * np.spacing(np.abs(want).astype(np.float32)).astype(np.float64) + 1e-30)
