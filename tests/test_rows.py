"""Quantized embedding / n-gram row lookup (models/flashnext/ngram.py).

CPU: the oracle's row mapping and quantization inference against golden
vectors made by the reference's own ``_groups`` / ``infer_quantization``
(``tests/golden/make_ngram_golden.py``).  GPU: ``fnmoe_rows_dequantize``
bit-exact against the oracle for 2/4/8-bit tables, group sizes 32/64/128,
sharded tables with out-of-range ids, and values whose float32 evaluation
lands on a bfloat16 rounding tie.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import bf16
from oracle import rows as orows

GOLDEN = Path(__file__).resolve().parent / "golden" / "ngram_rows.npz"


def test_row_mapping_matches_reference_groups():
    d = np.load(GOLDEN)
    for c in range(d["sizes"].shape[0]):
        sizes = [int(v) for v in d["sizes"][c] if v >= 0]
        sel = d["case"] == c
        offsets = np.asarray(orows.shard_offsets(sizes))
        want = offsets[d["shard"][sel]] + d["local"][sel]
        np.testing.assert_array_equal(orows.concat_rows(d["rows"][sel], sizes), want)


def test_quantization_inference_matches_reference():
    from flashnext_b200.ngram import infer_quantization

    class Shapes:
        def __init__(self, packed, groups):
            self.s = {"t.weight": (4, packed), "t.scales": (4, groups)}

        def shape(self, name):
            return self.s[name]

    for dims, packed, groups, group_size, bits in np.load(GOLDEN)["quant"].tolist():
        assert orows.infer_quantization(packed, groups, dims) == (group_size, bits)
        assert infer_quantization(Shapes(packed, groups), "t", dims) == (group_size, bits)


def test_oracle_dequant_equals_q4_executor_rule():
    """For 4-bit rows the oracle's values equal oracle.moe.dequantize, the
    rule pinned against the reference's NumPy executor."""
    from oracle import moe
    rng = np.random.default_rng(5)
    w = rng.integers(0, 2 ** 32, size=(6, 32), dtype=np.uint64).astype(np.uint32)
    s = bf16.f32_to_bits(np.abs(rng.normal(0, 0.01, (6, 8))).astype(np.float32))
    b = bf16.f32_to_bits((-8 * bf16.bits_to_f32(s)).astype(np.float32))
    got = orows.dequantize_rows(w, s, b, np.arange(6), 4, 32)
    want = moe.dequantize(w, bf16.bits_to_f32(s), bf16.bits_to_f32(b), 32)
    np.testing.assert_array_equal(got, want)


def _table(rng, rows, dims, bits, group):
    import torch
    w = rng.integers(0, 2 ** 32, size=(rows, dims * bits // 32), dtype=np.uint64).astype(np.uint32)
    s = bf16.f32_to_bits(rng.normal(0, 0.02, (rows, dims // group)).astype(np.float32))
    bvals = -(2 ** (bits - 1)) * bf16.bits_to_f32(s) + rng.normal(0, 1e-4, s.shape).astype(np.float32)
    b = bf16.f32_to_bits(bvals.astype(np.float32))
    dev = lambda a, t: torch.from_numpy(a.view(t)).cuda()  # noqa: E731
    return (w, s, b), (dev(w, np.int32), dev(s, np.int16).view(torch.bfloat16), dev(b, np.int16).view(torch.bfloat16))


@pytest.mark.gpu
@pytest.mark.parametrize("bits,group,dims", [(4, 32, 2048), (4, 64, 1024), (8, 64, 512), (2, 32, 256),
                                             (4, 128, 384), (8, 32, 96)])
def test_rows_dequantize_bit_exact(cuda_lib, bits, group, dims):
    import torch
    from flashnext_b200.ngram import StreamingQuantizedEmbedding
    rng = np.random.default_rng(bits * 1000 + group + dims)
    host, devt = _table(rng, 37, dims, bits, group)
    emb = StreamingQuantizedEmbedding.from_arrays(*devt, dims)
    assert (emb.bits, emb.group_size) == (bits, group)
    idx = rng.integers(0, 37, size=(3, 7))
    got = emb(torch.tensor(idx).cuda())
    assert got.shape == (3, 7, dims) and got.dtype == torch.bfloat16
    want = orows.embedding_rows(*host, idx, bits, group)
    np.testing.assert_array_equal(got.cpu().view(torch.int16).numpy().view(np.uint16), want)


@pytest.mark.gpu
def test_sharded_rows_with_out_of_range_ids(cuda_lib):
    import torch
    from flashnext_b200.ngram import StreamingQuantizedEmbedding, StreamingShardedEmbedding
    rng = np.random.default_rng(11)
    sizes = [5, 1, 9, 3]
    shards, hosts = [], []
    for n in sizes:
        host, devt = _table(rng, n, 256, 4, 32)
        shards.append(StreamingQuantizedEmbedding.from_arrays(*devt, 256))
        hosts.append(host)
    emb = StreamingShardedEmbedding(shards, sizes, 256)
    total = sum(sizes)
    ids = np.array([0, 4, 5, 6, 15, 17, total - 1, total, total + 7, -1, -100, 2 ** 40], np.int64)
    got = emb(torch.tensor(ids).cuda())
    table = tuple(np.concatenate([h[i] for h in hosts]) for i in range(3))
    want = orows.embedding_rows(*table, ids, 4, 32, shard_sizes=sizes)
    np.testing.assert_array_equal(got.cpu().view(torch.int16).numpy().view(np.uint16), want)
    empty = emb(torch.zeros((0,), dtype=torch.int64).cuda())
    assert empty.shape == (0, 256)


def _tie_case():
    """A (scale, bias) pair and q for which fma(s, q, b) in float32 is a
    bfloat16 midpoint while the exact value is not (b below half a float32
    ulp of s*q), so rounding float32 to bfloat16 would round the wrong way."""
    for sbits in range(0x3F80, 0x4000):
        s = float(bf16.bits_to_f32(np.uint16(sbits)))
        for q in range(1, 16):
            v = np.float32(s * q)
            u = int(np.array(v).view(np.uint32))
            if u & 0xFFFF == 0x8000 and (u >> 16) & 1 == 0:  # tie with an even lower neighbour
                return sbits, q
    raise AssertionError("no tie case found")


@pytest.mark.gpu
def test_rows_dequantize_rounds_once_at_float32_ties(cuda_lib):
    import torch
    from flashnext_b200.ngram import rows_dequantize
    sbits, q = _tie_case()
    dims, group = 32, 32
    w = np.full((2, dims * 4 // 32), sum(q << (4 * j) for j in range(8)), np.uint32)
    s = np.full((2, 1), sbits, np.uint16)
    b = np.array([[0x3000], [0xB000]], np.uint16)  # +-2^-31: far below half a float32 ulp of s*q
    got = rows_dequantize(torch.from_numpy(w.view(np.int32)).cuda(),
                          torch.from_numpy(s.view(np.int16)).cuda().view(torch.bfloat16),
                          torch.from_numpy(b.view(np.int16)).cuda().view(torch.bfloat16),
                          torch.tensor([0, 1]).cuda(), dims, 4, group)
    want = orows.embedding_rows(w, s, b, np.array([0, 1]), 4, group)
    np.testing.assert_array_equal(got.cpu().view(torch.int16).numpy().view(np.uint16), want)
    # the exact value sits above / below the midpoint: the two rows differ by one ulp
    assert int(want[0, 0]) - int(want[1, 0]) == 1
