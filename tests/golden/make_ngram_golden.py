"""Golden vectors for the n-gram row mapping from the reference's own code.

Run with ``FLASHNEXT_REFERENCE`` set to a read-only checkout of the
reference (the variable is required):

    FLASHNEXT_REFERENCE=<checkout> python -B tests/golden/make_ngram_golden.py

``models/flashnext/ngram.py`` imports MLX at module level, which is not
installable here, so the script takes the source text of the pure-Python
pieces from the file and executes only those: ``infer_quantization``
(ngram.py:19-25) and ``StreamingShardedEmbedding.__init__``'s offset table
plus ``_groups`` (ngram.py:85-119).  For seeded shard-size lists and global
row ids -- in range, negative, past the end and at every shard boundary -- it
records the (shard, local row) that ``_groups`` picks for each id, and
``infer_quantization``'s (group_size, bits) for several packed shapes.
Output: ``tests/golden/ngram_rows.npz``.
"""
from __future__ import annotations

import ast
import os
from bisect import bisect_right
from pathlib import Path

import numpy as np


def _reference_pieces(root: Path):
    src = (root / "models" / "flashnext" / "ngram.py").read_text()
    tree = ast.parse(src)
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "infer_quantization")
    cls = next(n for n in tree.body if isinstance(n, ast.ClassDef) and n.name == "StreamingShardedEmbedding")
    keep = [n for n in cls.body if isinstance(n, ast.FunctionDef) and n.name in ("__init__", "_groups")]
    # The class without its nn.Module base, holding only the two methods.
    shim = ast.ClassDef(name="Sharded", bases=[], keywords=[], body=keep, decorator_list=[])
    namespace: dict = {"bisect_right": bisect_right, "os": os}

    class _Module:  # stands in for nn.Module's __init__ in super().__init__()
        def __init__(self):
            pass

    shim.bases = [ast.Name(id="_Module", ctx=ast.Load())]
    namespace["_Module"] = _Module
    mod = ast.Module(body=[fn, shim], type_ignores=[])
    ast.fix_missing_locations(mod)
    exec(compile(mod, "ngram.py", "exec"), namespace)
    return namespace["infer_quantization"], namespace["Sharded"]


class _ShapeStore:
    def __init__(self, shapes):
        self.shapes = shapes

    def shape(self, name):
        return self.shapes[name]


def main():
    root_env = os.environ.get("FLASHNEXT_REFERENCE")
    if not root_env:
        raise SystemExit("set FLASHNEXT_REFERENCE to a checkout of the reference repository")
    infer, sharded = _reference_pieces(Path(root_env))
    rng = np.random.default_rng(20261202)
    cases_sizes, cases_rows, cases_shard, cases_local = [], [], [], []
    for n_shards in (1, 2, 5, 128):
        sizes = rng.integers(1, 50, size=n_shards)
        emb = sharded([None] * n_shards, sizes.tolist(), 64)
        total = int(sizes.sum())
        offsets = np.concatenate([[0], np.cumsum(sizes)])
        rows = np.concatenate([rng.integers(-5, total + 5, size=200), offsets, offsets - 1,
                               [-(2 ** 40), 2 ** 40]]).astype(np.int64)
        groups = emb._groups([int(r) for r in rows])
        shard_of = np.zeros(rows.size, np.int64)
        local_of = np.zeros(rows.size, np.int64)
        for shard_index, (positions, locals_) in groups.items():
            for p, lo in zip(positions, locals_):
                shard_of[p] = shard_index
                local_of[p] = lo
        cases_sizes.append(np.pad(sizes, (0, 128 - n_shards), constant_values=-1))
        cases_rows.append(rows)
        cases_shard.append(shard_of)
        cases_local.append(local_of)
    quant = []
    for dims, bits, group in ((2048, 4, 32), (2048, 4, 64), (4096, 8, 64), (1024, 2, 32), (3072, 4, 128)):
        store = _ShapeStore({"t.weight": (10, dims * bits // 32), "t.scales": (10, dims // group)})
        quant.append((dims, dims * bits // 32, dims // group, *infer(store, "t", dims)))
    out = Path(__file__).resolve().parent / "ngram_rows.npz"
    case = np.concatenate([np.full(r.size, i, np.int64) for i, r in enumerate(cases_rows)])
    np.savez_compressed(out, sizes=np.stack(cases_sizes), case=case, rows=np.concatenate(cases_rows),
                        shard=np.concatenate(cases_shard), local=np.concatenate(cases_local),
                        quant=np.asarray(quant, np.int64))
    print(out)


if __name__ == "__main__":
    main()
