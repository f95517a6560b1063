"""Checkpoint loading into HBM tables (models/flashnext/loader.py, store.py,
slab_pack.py), on a synthetic safetensors checkpoint written by the test.

CPU: the safetensors reader (two shards + index), quantization inference,
and the expert table's bytes -- record layout, chosen expert order -- against
the tensors themselves.  GPU: a layer loaded with ``load_moe_block`` is
bit-exact to the oracle on the same tensors; the loaded embedding and n-gram
tables look rows up bit-exactly.
"""
from __future__ import annotations

import json
import struct

import numpy as np
import pytest

from oracle import bf16
from oracle import rows as orows

H, I, E, G = 256, 64, 6, 32
P = "language_model.model.layers.0.mlp"


def _write_safetensors(path, tensors):
    header, blobs, off = {}, [], 0
    for name, (dtype, arr) in tensors.items():
        data = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dtype, "shape": list(arr.shape), "data_offsets": [off, off + len(data)]}
        blobs.append(data)
        off += len(data)
    meta = json.dumps(header).encode()
    meta += b" " * (-len(meta) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(meta)))
        f.write(meta)
        for b in blobs:
            f.write(b)


def _q4(rng, *shape_rows_cols):
    *lead, rows, cols = shape_rows_cols
    w = rng.integers(0, 2 ** 32, size=(*lead, rows, cols // 8), dtype=np.uint64).astype(np.uint32)
    s = bf16.f32_to_bits(np.abs(rng.normal(0, 0.01, (*lead, rows, cols // G))).astype(np.float32))
    b = bf16.f32_to_bits((-8 * bf16.bits_to_f32(s)).astype(np.float32))
    return w, s, b


@pytest.fixture(scope="module")
def checkpoint(tmp_path_factory):
    d = tmp_path_factory.mktemp("ckpt")
    rng = np.random.default_rng(2026)
    t = {}
    for proj, (o, k) in (("gate_proj", (I, H)), ("up_proj", (I, H)), ("down_proj", (H, I))):
        w, s, b = _q4(rng, E, o, k)
        t[f"{P}.switch_mlp.{proj}.weight"] = ("U32", w)
        t[f"{P}.switch_mlp.{proj}.scales"] = ("BF16", s)
        t[f"{P}.switch_mlp.{proj}.biases"] = ("BF16", b)
        w, s, b = _q4(rng, o, k)
        t[f"{P}.shared_expert.{proj}.weight"] = ("U32", w)
        t[f"{P}.shared_expert.{proj}.scales"] = ("BF16", s)
        t[f"{P}.shared_expert.{proj}.biases"] = ("BF16", b)
    t[f"{P}.gate.weight"] = ("BF16", bf16.f32_to_bits(rng.normal(0, 0.02, (E, H)).astype(np.float32)))
    t[f"{P}.shared_expert_gate.weight"] = ("BF16", bf16.f32_to_bits(rng.normal(0, 0.02, (1, H)).astype(np.float32)))
    for name, rows in (("language_model.model.embed_tokens", 50), ("ngram.0", 7), ("ngram.1", 12)):
        w, s, b = _q4(rng, rows, H)
        t[f"{name}.weight"], t[f"{name}.scales"], t[f"{name}.biases"] = ("U32", w), ("BF16", s), ("BF16", b)
    names = sorted(t)
    half = len(names) // 2
    weight_map = {}
    for shard, part in (("model-00001-of-00002.safetensors", names[:half]),
                        ("model-00002-of-00002.safetensors", names[half:])):
        _write_safetensors(d / shard, {n: t[n] for n in part})
        weight_map.update({n: shard for n in part})
    (d / "model.safetensors.index.json").write_text(json.dumps({"weight_map": weight_map}))
    return d, {n: a for n, (_, a) in t.items()}


def test_store_reads_both_shards(checkpoint):
    from flashnext_b200.store import SafeTensorStore
    d, t = checkpoint
    store = SafeTensorStore(str(d))
    assert set(store.refs) == set(t)
    for name, arr in t.items():
        assert store.shape(name) == arr.shape
        np.testing.assert_array_equal(store.whole_np(name), arr)
    np.testing.assert_array_equal(store.rows_np(f"{P}.switch_mlp.up_proj.scales", [4, 0, 4]),
                                  t[f"{P}.switch_mlp.up_proj.scales"][[4, 0, 4]])


def test_quantization_inference(checkpoint):
    from flashnext_b200.loader import infer_embed_bits, infer_switch_quantization
    from flashnext_b200.store import SafeTensorStore
    store = SafeTensorStore(str(checkpoint[0]))
    assert infer_switch_quantization(store, f"{P}.switch_mlp") == (G, 4)
    assert infer_embed_bits(store) == 4


def test_expert_table_records_hold_the_checkpoint_rows(checkpoint):
    """Record r of the loaded table holds expert experts[r]'s nine parts at the
    slab layout's offsets (slab_pack.py:96-153), header first."""
    from flashnext_b200.expert_table import HEADER_MAGIC, PARTS
    from flashnext_b200.loader import host_table_bytes, load_expert_table
    from flashnext_b200.store import SafeTensorStore
    d, t = checkpoint
    store = SafeTensorStore(str(d))
    order = [3, 1, 5, 0]
    table = load_expert_table(store, 0, device="cpu", experts=order, chunk_experts=3)
    buf = table.buffer.numpy()
    assert int(buf[:4].view(np.uint32)[0]) == HEADER_MAGIC
    body = buf[table.header_size:]
    np.testing.assert_array_equal(body, host_table_bytes(store, 0, order))
    lay = table.layout
    for r, e in enumerate(order):
        for i, (proj, part) in enumerate(PARTS):
            want = np.ascontiguousarray(t[f"{P}.switch_mlp.{proj}.{part}"][e]).view(np.uint8).reshape(-1)
            start = r * lay.record_stride + lay.offsets[i]
            np.testing.assert_array_equal(body[start:start + want.size], want)


@pytest.mark.gpu
def test_loaded_block_bit_exact_to_oracle(cuda_lib, checkpoint):
    import torch
    from flashnext_b200.loader import load_moe_block
    from flashnext_b200.store import SafeTensorStore
    from oracle import moe
    d, t = checkpoint
    block = load_moe_block(SafeTensorStore(str(d)), 0, top_k=4)
    rng = np.random.default_rng(9)
    x = bf16.round_f32(rng.normal(0, 1, (5, H)).astype(np.float32))
    out = block(torch.from_numpy(x).cuda().to(torch.bfloat16))
    f = lambda n: bf16.bits_to_f32(t[n])  # noqa: E731
    bank = {proj: tuple(t[f"{P}.switch_mlp.{proj}.{part}"] if part == "weight" else f(f"{P}.switch_mlp.{proj}.{part}")
                        for part in ("weight", "scales", "biases")) for proj in ("gate_proj", "up_proj", "down_proj")}
    sh = tuple(tuple(t[f"{P}.shared_expert.{proj}.{part}"] if part == "weight" else f(f"{P}.shared_expert.{proj}.{part}")
                     for part in ("weight", "scales", "biases")) for proj in ("gate_proj", "up_proj", "down_proj"))
    ref = moe.moe_block(x, f(f"{P}.gate.weight"), 4, bank["gate_proj"], bank["up_proj"], bank["down_proj"], sh,
                        f(f"{P}.shared_expert_gate.weight"))
    got = out.float().cpu().numpy()
    np.testing.assert_array_equal(bf16.f32_to_bits(got), bf16.f32_to_bits(ref["out"]))


@pytest.mark.gpu
def test_loaded_embedding_and_ngram_tables(cuda_lib, checkpoint):
    import torch
    from flashnext_b200.loader import load_embedding, load_ngram_shards
    from flashnext_b200.store import SafeTensorStore
    d, t = checkpoint
    store = SafeTensorStore(str(d))
    emb = load_embedding(store)
    ids = np.array([[0, 49, 7], [3, 3, 12]])
    got = emb(torch.tensor(ids).cuda()).cpu().view(torch.int16).numpy().view(np.uint16)
    p = "language_model.model.embed_tokens"
    np.testing.assert_array_equal(got, orows.embedding_rows(t[f"{p}.weight"], t[f"{p}.scales"],
                                                            t[f"{p}.biases"], ids, 4, G))
    ng = load_ngram_shards(store, ["ngram.0", "ngram.1"], H)
    ids = np.array([0, 6, 7, 18, 19, -3])
    got = ng(torch.tensor(ids).cuda()).cpu().view(torch.int16).numpy().view(np.uint16)
    cat = [np.concatenate([t[f"ngram.0.{x}"], t[f"ngram.1.{x}"]]) for x in ("weight", "scales", "biases")]
    np.testing.assert_array_equal(got, orows.embedding_rows(*cat, ids, 4, G, shard_sizes=[7, 12]))
