"""Golden vectors for the adaptive keep from the reference's own function.

Run with ``FLASHNEXT_REFERENCE`` set to a read-only checkout of the
reference (the variable is required):

    FLASHNEXT_REFERENCE=<checkout> python -B tests/golden/make_keep_golden.py

``models/flashnext/adaptive_topk.py`` imports MLX at module level, which is
not installable here, so the script takes the source text of the pure-Python
``_keep_for_mass`` (adaptive_topk.py:43-50) from the file, executes that one
function, and records its results for seeded top-10 score rows whose values
are bfloat16 numbers in descending order (the order ``argsort(-scores)``
gives), at several thresholds.  Output: ``tests/golden/keep_for_mass.npz``.
"""
from __future__ import annotations

import ast
import os
from pathlib import Path

import numpy as np


def _reference_keep_for_mass(root: Path):
    src = (root / "models" / "flashnext" / "adaptive_topk.py").read_text()
    tree = ast.parse(src)
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "_keep_for_mass")
    namespace: dict = {}
    exec(compile(ast.Module(body=[fn], type_ignores=[]), "adaptive_topk.py", "exec"), namespace)
    return namespace["_keep_for_mass"]


def _bf16(a):
    bits = np.asarray(a, np.float32).view(np.uint32).astype(np.uint64)
    bits = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
    return bits.astype(np.uint32).view(np.float32)


def main():
    root_env = os.environ.get("FLASHNEXT_REFERENCE")
    if not root_env:
        raise SystemExit("set FLASHNEXT_REFERENCE to a checkout of the reference repository")
    root = Path(root_env)
    keep = _reference_keep_for_mass(root)
    rng = np.random.default_rng(20261202)
    rows = []
    # softmax-like top-10 rows: peaked, flat and in between
    for temp in (0.2, 0.5, 1.0, 2.0, 5.0):
        logits = rng.standard_normal((200, 512)) * temp
        p = np.exp(logits - logits.max(axis=1, keepdims=True))
        p /= p.sum(axis=1, keepdims=True)
        top = -np.sort(-p, axis=1)[:, :10]
        rows.append(_bf16(top))
    # exact ties and equal weights
    rows.append(_bf16(np.full((4, 10), 0.1)))
    scores = np.concatenate(rows).astype(np.float32)
    thresholds = np.array([0.2, 0.4, 0.5, 0.85, 0.9, 0.99], np.float64)
    keeps = np.array([[keep(row, float(t)) for row in scores.tolist()] for t in thresholds], np.int64)
    out = Path(__file__).resolve().parent / "keep_for_mass.npz"
    np.savez_compressed(out, scores=scores, thresholds=thresholds, keeps=keeps)
    print("wrote", out, scores.shape, keeps.shape)


if __name__ == "__main__":
    main()
