"""Quantized embedding / n-gram row oracle -- TEST INFRASTRUCTURE ONLY.

Restates the row lookups of ``models/flashnext/ngram.py``:

* ``infer_quantization`` (ngram.py:19-25): bits and group size from the
  packed and scale widths.
* ``StreamingShardedEmbedding._groups`` (ngram.py:106-119): a global row in
  ``[0, total)`` belongs to the shard whose offset range holds it; any other
  row goes to shard 0; the local row is clamped into its shard.
* ``StreamingQuantizedEmbedding._rows`` (ngram.py:49-60): the rows'
  ``mx.dequantize(weight, scales, biases, group_size, bits, mode="affine")``,
  ``w = s*q + b`` with value j of a uint32 word in bits ``[j*bits,
  (j+1)*bits)``; here the exact ``s*q + b`` is rounded once to bfloat16, the
  rule ``oracle.moe.dequantize`` pins for 4 bits against the reference's own
  NumPy executor.

The sharded table is held as its shards concatenated in shard order, so a
shard-local row ``l`` of shard ``k`` is row ``offsets[k] + l``.
"""
from __future__ import annotations

from bisect import bisect_right

import numpy as np

from . import bf16


def infer_quantization(packed_words: int, groups: int, dims: int) -> tuple[int, int]:
    """(group_size, bits) of a table with ``packed_words`` uint32 and
    ``groups`` scales per row of ``dims`` values (ngram.py:19-25)."""
    bits = packed_words * 32 // dims
    group_size = dims // groups
    return group_size, bits


def shard_offsets(shard_sizes) -> list[int]:
    offsets = [0]
    for size in shard_sizes:
        offsets.append(offsets[-1] + int(size))
    return offsets


def concat_rows(indices, shard_sizes) -> np.ndarray:
    """Row of the concatenated table read for each global index
    (``_groups``, ngram.py:106-119)."""
    offsets = shard_offsets(shard_sizes)
    sizes = [int(s) for s in shard_sizes]
    out = []
    for row in np.asarray(indices, np.int64).reshape(-1).tolist():
        if row < 0 or row >= offsets[-1]:
            shard, local = 0, row
        else:
            shard = bisect_right(offsets, row) - 1
            local = row - offsets[shard]
        local = min(max(local, 0), sizes[shard] - 1)
        out.append(offsets[shard] + local)
    return np.asarray(out, np.int64)


def unpack(words, bits: int) -> np.ndarray:
    """[..., W] uint32 -> [..., W * 32 / bits] values, low bits first."""
    w = np.asarray(words, np.uint32)
    per = 32 // bits
    shifts = (np.arange(per, dtype=np.uint32) * bits).astype(np.uint32)
    q = (w[..., None] >> shifts) & np.uint32((1 << bits) - 1)
    return q.reshape(*w.shape[:-1], w.shape[-1] * per)


def dequantize_rows(weight, scales, biases, rows, bits: int, group_size: int) -> np.ndarray:
    """bfloat16 bits of ``s*q + b`` (rounded once) for the given table rows."""
    rows = np.asarray(rows, np.int64)
    q = unpack(np.asarray(weight)[rows], bits).astype(np.float64)
    s = np.repeat(bf16.bits_to_f32(np.asarray(scales)[rows]).astype(np.float64), group_size, axis=-1)
    b = np.repeat(bf16.bits_to_f32(np.asarray(biases)[rows]).astype(np.float64), group_size, axis=-1)
    return bf16.f64_to_bits(s * q + b)


def embedding_rows(weight, scales, biases, indices, bits: int, group_size: int, shard_sizes=None) -> np.ndarray:
    """Looked-up rows ``[*indices.shape, dims]`` as bfloat16 bits.

    ``weight``/``scales``/``biases`` hold the whole (concatenated) table;
    ``shard_sizes`` defaults to one shard of every row."""
    idx = np.asarray(indices, np.int64)
    sizes = [int(np.asarray(weight).shape[0])] if shard_sizes is None else list(shard_sizes)
    rows = concat_rows(idx, sizes)
    out = dequantize_rows(weight, scales, biases, rows, bits, group_size)
    return out.reshape(*idx.shape, out.shape[-1])
