"""Generate golden vectors by running the reference's own NumPy code.

Run with ``FLASHNEXT_REFERENCE`` set to a read-only checkout of the
reference (the variable is required):

    FLASHNEXT_REFERENCE=<checkout> python -B tests/golden/make_golden.py

It imports ``models.flashnext.metal_runtime`` and ``models.flashnext.slab_pack``
from the reference (both import with NumPy only) and records, for seeded
inputs whose values are exactly representable in bfloat16:

* ``_numpy_projection`` outputs for Q4/G32 and Q4/G64 packs
  (metal_runtime.py:955-987);
* ``MetalMoEExecutor(..., backend="reference").execute`` outputs: combined,
  per-slot and ``return_all`` forms, plus the ``shared_y`` and shared-parts
  adds (metal_runtime.py:764-941), for bfloat16-valued and for float32
  activations;
* the ``weighted_combine`` known-answer case of
  ``models/flashnext/tests/unit/test_metal_runtime.py:222-239``;
* the Q4/G32 and Q4/G64 slab record layouts (slab_pack.py:96-153).

The fixtures are committed; nothing on the GPU box reads the reference.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _reference_root() -> Path:
    root = os.environ.get("FLASHNEXT_REFERENCE")
    if not root:
        sys.exit("set FLASHNEXT_REFERENCE to a checkout of the reference repository")
    return Path(root)


def _bf16_values(a):
    a = np.asarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return u.astype(np.uint32).view(np.float32)


def _pack(codes):
    c = codes.astype(np.uint32)
    c = c.reshape(*c.shape[:-1], c.shape[-1] // 8, 8)
    return np.bitwise_or.reduce(c << (np.arange(8, dtype=np.uint32) * 4), axis=-1).astype(np.uint32)


def _projection(rng, experts, out_w, in_w, group):
    codes = rng.integers(0, 16, (experts, out_w, in_w), dtype=np.uint8)
    scales = _bf16_values(np.abs(rng.normal(0, 0.05, (experts, out_w, in_w // group))))
    biases = _bf16_values(-8 * scales + _bf16_values(rng.normal(0, 0.01, scales.shape)))
    biases = _bf16_values(biases)
    return _pack(codes), scales.astype(np.float32), biases.astype(np.float32)


def main() -> None:
    sys.path.insert(0, str(_reference_root()))
    sys.dont_write_bytecode = True
    from models.flashnext import metal_runtime as mr
    from models.flashnext import slab_pack as sp

    out = {}
    rng = np.random.default_rng(20261201)

    # 1. raw projections, G32 and G64
    for group in (32, 64):
        w, s, b = _projection(rng, 3, 48, 128, group)
        x = _bf16_values(rng.normal(0, 1, (2, 128))).astype(np.float32)
        routes = np.array([[2, 0], [1, 1]], dtype=np.uint32)
        y = mr._numpy_projection(x, routes, mr.Q4G32Projection(w, s, b), 48, False, group)
        for name, val in (("w", w), ("s", s), ("b", b), ("x", x), ("routes", routes), ("y", y)):
            out[f"proj_g{group}_{name}"] = val

    # 2. executor reference path (hidden 64, intermediate 32, 4 experts, top-3)
    hidden, inter, experts, top_k = 64, 32, 4, 3
    gate = _projection(rng, experts, inter, hidden, 32)
    up = _projection(rng, experts, inter, hidden, 32)
    down = _projection(rng, experts, hidden, inter, 32)
    x = _bf16_values(rng.normal(0, 1, (2, hidden))).astype(np.float32)
    routes = np.array([[3, 0, 1], [2, 2, 0]], dtype=np.uint32)
    scores = _bf16_values(rng.dirichlet(np.ones(top_k), size=2)).astype(np.float32)
    shared_y = _bf16_values(rng.normal(0, 0.5, (2, hidden))).astype(np.float32)
    shared = _bf16_values(rng.normal(0, 0.5, (2, hidden))).astype(np.float32)
    shared_gate = _bf16_values(rng.uniform(0, 1, (2, 1))).astype(np.float32)
    packs = {"gate_proj": gate, "up_proj": up, "down_proj": down}
    ex = mr.MetalMoEExecutor(experts, hidden, top_k, backend="reference")
    combined = ex.execute(x, routes, packs, scores=scores)
    assert ex.last_path == "reference"
    per_slot = ex.execute(x, routes, packs)
    g_all, u_all, d_all = ex.execute(x, routes, packs, return_all=True)
    with_y = ex.execute(x, routes, packs, scores=scores, shared_y=shared_y)
    with_parts = ex.execute(x, routes, packs, scores=scores, shared=shared, shared_gate=shared_gate)
    for name, val in (
        ("gate_w", gate[0]), ("gate_s", gate[1]), ("gate_b", gate[2]),
        ("up_w", up[0]), ("up_s", up[1]), ("up_b", up[2]),
        ("down_w", down[0]), ("down_s", down[1]), ("down_b", down[2]),
        ("x", x), ("routes", routes), ("scores", scores), ("shared_y", shared_y),
        ("shared", shared), ("shared_gate", shared_gate),
        ("combined", combined), ("per_slot", per_slot), ("all_gate", g_all),
        ("all_up", u_all), ("all_down", d_all), ("with_shared_y", with_y),
        ("with_shared_parts", with_parts),
    ):
        out[f"exec_{name}"] = np.asarray(val)

    # 2b. the same executor with float32 activations (production Flash-Next
    # keeps activations float32 with bfloat16 scales/biases,
    # metal_runtime.py:371-373; tests/unit/test_metal_runtime.py:516-557)
    xf = rng.normal(0, 1, (2, hidden)).astype(np.float32)
    sf = rng.dirichlet(np.ones(top_k), size=2).astype(np.float32)
    syf = rng.normal(0, 0.5, (2, hidden)).astype(np.float32)
    shf = rng.normal(0, 0.5, (2, hidden)).astype(np.float32)
    sgf = rng.uniform(0, 1, (2, 1)).astype(np.float32)
    f_combined = ex.execute(xf, routes, packs, scores=sf)
    f_per_slot = ex.execute(xf, routes, packs)
    fg, fu, fd = ex.execute(xf, routes, packs, return_all=True)
    f_with_y = ex.execute(xf, routes, packs, scores=sf, shared_y=syf)
    f_with_parts = ex.execute(xf, routes, packs, scores=sf, shared=shf, shared_gate=sgf)
    for name, val in (
        ("x", xf), ("scores", sf), ("shared_y", syf), ("shared", shf), ("shared_gate", sgf),
        ("combined", f_combined), ("per_slot", f_per_slot), ("all_gate", fg), ("all_up", fu), ("all_down", fd),
        ("with_shared_y", f_with_y), ("with_shared_parts", f_with_parts),
    ):
        out[f"exec32_{name}"] = np.asarray(val)
        assert np.asarray(val).dtype == np.float32

    # 3. weighted_combine known answer (test_metal_runtime.py:222-239)
    eo = np.array([[[1.0, 2.0], [10.0, 20.0], [100.0, 200.0]],
                   [[3.0, 4.0], [30.0, 40.0], [300.0, 400.0]]], dtype=np.float32)
    wr = np.array([[2, 0], [1, 2]], dtype=np.int32)
    ws = np.array([[0.25, 0.75], [0.4, 0.6]], dtype=np.float32)
    out["combine_outputs"] = eo
    out["combine_routes"] = wr
    out["combine_scores"] = ws
    out["combine_result"] = mr.weighted_combine(eo, wr, ws)

    # 4. slab record layouts
    for group in (32, 64):
        lay = sp.get_slab_layout(group)
        names = [name for name, _ in lay.offsets]
        out[f"slab_g{group}_offsets"] = np.array([lay.offset(*n.split(".")) for n in names], dtype=np.int64)
        out[f"slab_g{group}_stride"] = np.array(lay.record_stride, dtype=np.int64)
    out["slab_header"] = np.array(sp.HEADER_SIZE, dtype=np.int64)

    np.savez_compressed(HERE / "reference_numpy.npz", **out)
    print(f"wrote {HERE / 'reference_numpy.npz'} with {len(out)} arrays")


if __name__ == "__main__":
    main()
