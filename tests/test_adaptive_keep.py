"""Adaptive keep (threshold < 1): the oracle against the reference's own
``_keep_for_mass`` (adaptive_topk.py:43-50) through committed golden vectors,
and the keep/drop/renorm rule of adaptive_topk.py:75-261."""
from __future__ import annotations

from pathlib import Path

import numpy as np

from oracle import moe

GOLDEN = Path(__file__).resolve().parent / "golden" / "keep_for_mass.npz"


def test_keep_for_mass_matches_reference_golden():
    g = np.load(GOLDEN)
    for t, want in zip(g["thresholds"], g["keeps"]):
        got = np.array([moe.keep_for_mass(row, float(t)) for row in g["scores"]])
        np.testing.assert_array_equal(got, want)


def test_adaptive_keep_drops_to_slot_zero_with_zero_score():
    inds = np.array([[5, 9, 2, 7], [1, 3, 4, 6]], np.uint32)
    scores = np.array([[0.5, 0.25, 0.125, 0.125], [0.25, 0.25, 0.25, 0.25]], np.float32)
    ki, ks, keeps = moe.adaptive_keep(inds, scores, 0.7)
    np.testing.assert_array_equal(keeps, [2, 3])
    np.testing.assert_array_equal(ki, [[5, 9, 5, 5], [1, 3, 4, 1]])
    np.testing.assert_array_equal(ks, [[0.5, 0.25, 0, 0], [0.25, 0.25, 0.25, 0]])
    # minimum keep, and threshold >= 1 keeps everything
    _, _, keeps = moe.adaptive_keep(inds, scores, 0.1, min_keep=3)
    np.testing.assert_array_equal(keeps, [3, 3])
    ki, ks, keeps = moe.adaptive_keep(inds, scores, 1.0)
    np.testing.assert_array_equal(keeps, [4, 4])
    np.testing.assert_array_equal(ki, inds)


def test_renorm_over_kept_mass():
    from oracle import bf16

    inds = np.array([[5, 9, 2, 7]], np.uint32)
    scores = bf16.round_f32(np.array([[0.5, 0.25, 0.125, 0.125]], np.float32))
    mass = np.array([[1.0]], np.float32)
    _, ks, _ = moe.adaptive_keep(inds, scores, 0.7)
    rs, norm = moe.renorm(ks, mass, 1.0)
    np.testing.assert_array_equal(norm, [[0.75]])
    np.testing.assert_array_equal(rs[0, 2:], [0, 0])
    np.testing.assert_allclose(rs[0, :2], [2 / 3, 1 / 3], rtol=1e-2)
