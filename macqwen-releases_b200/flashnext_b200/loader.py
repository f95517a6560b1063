"""Fill HBM-resident tables from a safetensors checkpoint.

The reference streams a layer's routed experts from the checkpoint on every
decode step: ``_swap_experts`` (``models/flashnext/loader.py:337-361``) puts a
``StreamingSwitchGLU`` on each layer, whose reads gather expert rows
(``store.rows_into`` / ``expert_record_view``, ``store.py:537-592``) into slab
or pool records (``slab_pack.py:96-153``, ``expert_pool.py:88-145``).  On a
B200 the whole bank is resident, so loading happens once per layer:

* :func:`load_expert_table` writes a layer's experts into an
  :class:`~.expert_table.ExpertTable` -- the reference's record layout,
  addressed by bit-31 routes -- through a pinned host staging buffer filled
  with ``expert_record_view`` and copied to the device in chunks;
* :func:`load_moe_block` builds the whole :class:`~.moe_block.SparseMoEBlock`
  (router, routed experts as tiled tables, shared expert and its gate);
* :func:`load_embedding` / :func:`load_ngram_shards` load the quantized
  input-embedding and n-gram tables (``loader.py:266-295``, ``ngram.py``).

Quantization is inferred from the tensor shapes as the reference does
(``infer_switch_quantization``, ``loader.py:364-386``).  Tensor names follow
the reference checkpoint: ``language_model.model.layers.{i}.mlp.gate``,
``.switch_mlp.{gate,up,down}_proj``, ``.shared_expert.{...}``,
``.shared_expert_gate``.
"""
from __future__ import annotations

import numpy as np

from .expert_table import PARTS, ExpertTable
from .moe_block import SparseMoEBlock
from .ngram import StreamingQuantizedEmbedding, StreamingShardedEmbedding, rows_dequantize

LAYER_PREFIX = "language_model.model.layers.{index}.mlp"
EMBED_PREFIX = "language_model.model.embed_tokens"


def infer_switch_quantization(store, prefix: str) -> tuple[int, int]:
    """(group_size, bits) of an expert block from its tensor shapes
    (loader.py:364-386): ``down_proj.weight`` is [experts, hidden,
    packed_intermediate], so its second axis is the gate/up input width."""
    packed = int(store.shape(f"{prefix}.gate_proj.weight")[-1])
    groups = int(store.shape(f"{prefix}.gate_proj.scales")[-1])
    hidden = int(store.shape(f"{prefix}.down_proj.weight")[1])
    if packed <= 0 or groups <= 0 or hidden <= 0:
        raise ValueError(f"invalid switch quantization shapes at {prefix}")
    packed_bits = packed * 32
    if packed_bits % hidden or hidden % groups:
        raise ValueError(f"incompatible switch quantization shapes at {prefix}")
    return hidden // groups, packed_bits // hidden


def infer_embed_bits(store, prefix: str = EMBED_PREFIX) -> int:
    """Bits of a quantized embedding from its packed and scale widths
    (loader.py:286-294)."""
    packed = int(store.shape(f"{prefix}.weight")[-1])
    groups = int(store.shape(f"{prefix}.scales")[-1])
    for bits in (4, 8, 2, 3, 5, 6):
        logical = packed * 32 // bits
        if logical % groups == 0 and logical // groups in (32, 64, 128):
            return bits
    raise ValueError("cannot infer embedding quantization")


def _triple(store, prefix: str, device):
    return {part: store.to_device(f"{prefix}.{part}", device) for part in ("weight", "scales", "biases")}


def _dense_rows(store, name_prefix: str, device):
    """A [rows, width] matrix that may be stored dense (``.weight`` bf16) or
    affine-quantized (``.weight/.scales/.biases``); quantized ones are
    dequantised on the device with the row-lookup kernel."""
    import torch

    if f"{name_prefix}.scales" not in store.refs:
        return store.to_device(f"{name_prefix}.weight", device)
    t = _triple(store, name_prefix, device)
    rows = int(t["weight"].shape[0])
    groups = int(t["scales"].shape[-1])
    for bits in (4, 8, 2):
        dims = int(t["weight"].shape[-1]) * 32 // bits
        if dims % groups == 0 and dims // groups in (32, 64, 128):
            return rows_dequantize(t["weight"], t["scales"], t["biases"],
                                   torch.arange(rows, device=device), dims, bits, dims // groups)
    raise ValueError(f"{name_prefix}: cannot infer the quantization")


def load_experts(store, index: int, device="cuda") -> dict:
    """The layer's routed experts as {"gate_proj", "up_proj", "down_proj"} ->
    {"weight" [E,O,K/8] int32, "scales", "biases" [E,O,K/G] bf16} on ``device``."""
    prefix = f"{LAYER_PREFIX.format(index=index)}.switch_mlp"
    group, bits = infer_switch_quantization(store, prefix)
    if bits != 4:
        raise ValueError(f"{prefix}: {bits}-bit experts (only 4-bit affine experts run here)")
    return {name: _triple(store, f"{prefix}.{name}", device) for name in ("gate_proj", "up_proj", "down_proj")}


def load_expert_table(store, index: int, device="cuda", experts=None, chunk_experts: int = 64) -> ExpertTable:
    """Write the layer's experts (all, or the listed ids in order) into an
    :class:`ExpertTable`: record ``r`` holds expert ``experts[r]``.

    Each chunk of experts is assembled in a pinned host buffer through
    ``expert_record_view`` (one strided view per part) and copied to the
    device table in one transfer."""
    import torch

    prefix = f"{LAYER_PREFIX.format(index=index)}.switch_mlp"
    group, bits = infer_switch_quantization(store, prefix)
    if bits != 4:
        raise ValueError(f"{prefix}: {bits}-bit experts (only 4-bit affine experts run here)")
    n_all, inter, _ = store.shape(f"{prefix}.gate_proj.weight")
    hidden = int(store.shape(f"{prefix}.down_proj.weight")[1])
    ids = list(range(n_all)) if experts is None else [int(e) for e in experts]
    if any(not 0 <= e < n_all for e in ids):
        raise ValueError("expert id outside the checkpoint")
    table = ExpertTable(len(ids), hidden, int(inter), group, device=device)
    lay = table.layout
    stride = lay.record_stride
    staging = torch.empty(min(chunk_experts, len(ids)) * stride, dtype=torch.uint8,
                          pin_memory=torch.device(device).type == "cuda")
    host = staging.numpy()
    for c0 in range(0, len(ids), chunk_experts):
        chunk = ids[c0:c0 + chunk_experts]
        n = len(chunk)
        host[: n * stride] = 0
        for i, (proj, part) in enumerate(PARTS):
            view = store.expert_record_view(f"{prefix}.{proj}.{part}", host, n, lay.offsets[i], stride)
            view[:] = store.whole_np(f"{prefix}.{proj}.{part}")[chunk]
        base = table.header_size + c0 * stride
        table.buffer[base: base + n * stride].copy_(staging[: n * stride], non_blocking=True)
        if torch.device(device).type == "cuda":
            torch.cuda.current_stream().synchronize()  # the staging buffer is reused
    return table


def load_moe_block(store, index: int, *, top_k: int = 10, device="cuda", **kw) -> SparseMoEBlock:
    """The layer's sparse-MoE block -- router, routed experts (tiled tables
    unless ``tiled=False``), shared expert and its sigmoid gate -- resident
    on ``device``.  Extra keywords go to :class:`SparseMoEBlock`."""
    prefix = LAYER_PREFIX.format(index=index)
    group, _ = infer_switch_quantization(store, f"{prefix}.switch_mlp")
    router = _dense_rows(store, f"{prefix}.gate", device)
    experts = load_experts(store, index, device)
    shared = gate = None
    if f"{prefix}.shared_expert.gate_proj.weight" in store.refs:
        shared = {name: _triple(store, f"{prefix}.shared_expert.{name}", device)
                  for name in ("gate_proj", "up_proj", "down_proj")}
        gate = _dense_rows(store, f"{prefix}.shared_expert_gate", device)
    return SparseMoEBlock(router, experts, top_k=top_k, shared=shared, shared_expert_gate=gate,
                          group_size=group, **kw)


def load_embedding(store, prefix: str = EMBED_PREFIX, mode: str = "affine",
                   device="cuda") -> StreamingQuantizedEmbedding:
    """The quantized input embedding, resident (loader.py:266-283)."""
    dims = int(store.shape(f"{prefix}.weight")[-1]) * 32 // infer_embed_bits(store, prefix)
    return StreamingQuantizedEmbedding(store, prefix, dims, mode, device=device)


def load_ngram_shards(store, prefixes, dims: int, mode: str = "affine",
                      device="cuda") -> StreamingShardedEmbedding:
    """A sharded n-gram table (one prefix per shard, in shard order) as one
    resident table (ngram.py:82-188)."""
    shards = [StreamingQuantizedEmbedding(store, p, dims, mode, device=device) for p in prefixes]
    return StreamingShardedEmbedding(shards, [s.rows for s in shards], dims)


def host_table_bytes(store, index: int, experts=None) -> np.ndarray:
    """The records :func:`load_expert_table` writes, built on the host only
    (for checking the device table without a second code path)."""
    from .expert_table import host_records, record_layout

    prefix = f"{LAYER_PREFIX.format(index=index)}.switch_mlp"
    group, _ = infer_switch_quantization(store, prefix)
    n_all, inter, _ = store.shape(f"{prefix}.gate_proj.weight")
    hidden = int(store.shape(f"{prefix}.down_proj.weight")[1])
    ids = list(range(n_all)) if experts is None else list(experts)
    arrays = [store.whole_np(f"{prefix}.{proj}.{part}")[ids] for proj, part in PARTS]
    lay = record_layout(hidden, int(inter), group)
    return host_records(tuple(arrays[0:3]), tuple(arrays[3:6]), tuple(arrays[6:9]), lay)
