"""Benchmark configurations at full size, checked on the GPU (B200 only).

* C4: the 5,000-token prefill layer through the tcgen05 GEMMs -- routing bit
  for bit against the oracle router on every token, every token's output
  within the north-star tolerance of the exact decode path (itself bit-exact
  to the oracle), and a seeded sample of tokens against the oracle layer
  directly (a token's result does not depend on the rest of its batch).
* The tensor-core router on ragged tiles (tokens, rows and the shared gate
  row off the tile grid), bit for bit against the oracle router.
* C5: paged decode attention at the benchmark shape (16 sequences, context
  uniform in [1k, 32k], GQA 16/2, head_dim 256, page 64, a random permutation
  block table) against the attention oracle and float64 truth, at the
  reference selftest's 1.5e-2 bound (``models/qwen27b/paged_kv.py:526-567``).
* The drop-in decode API of ``paged_attention(queries, cache, scale, mask)``
  (``paged_kv.py:417``) over a ``PagedKVCache`` filled with ``append``.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import attention as attn
from oracle import bf16, moe

pytestmark = pytest.mark.gpu

TOL_MAX_ABS = 2e-2
TOL_MEAN_REL = 5e-3
SELFTEST_BOUND = 1.5e-2  # paged_kv.py:526-567


def _np(t):
    import torch

    if t.dtype == torch.bfloat16:
        return t.float().cpu().numpy()
    if t.dtype == torch.int32:
        return t.cpu().numpy().view(np.uint32)
    return t.cpu().numpy()


def assert_north_star(got, want, what=""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    err = np.abs(got - want)
    lim_max = TOL_MAX_ABS * max(1.0, np.abs(want).max())
    lim_mean = TOL_MEAN_REL * max(np.abs(want).mean(), 1e-30)
    assert err.max() <= lim_max, f"{what}: max abs {err.max():.3g} > {lim_max:.3g}"
    assert err.mean() <= lim_mean, f"{what}: mean abs {err.mean():.3g} > {lim_mean:.3g}"


def test_c4_prefill_layer_5000_tokens(cuda_lib):
    """C4: 5,000 tokens, H2048/I512/E512 top-10 Q4/G32 + shared, uniform routing."""
    import torch

    from flashnext_b200 import _lib, synthetic
    from flashnext_b200.moe_block import SparseMoEBlock
    _lib.read_device_errors()
    tokens = 5000
    L = synthetic.moe_layer(tokens, 2048, 512, 512, 10, 32, zipf=None, seed=4242)
    kw = dict(top_k=10, shared=L.shared, shared_expert_gate=L.shared_expert_gate)
    pre = SparseMoEBlock(L.router_weight, L.experts, path="prefill", **kw)
    out_p = pre(L.x).clone()
    inds_p = _np(pre.last_inds).copy()
    logits_p = _np(pre.last_logits).copy()
    del pre
    dec = SparseMoEBlock(L.router_weight, L.experts, path="decode", **kw)
    out_d = dec(L.x).clone()
    inds_d = _np(dec.last_inds).copy()
    del dec
    torch.cuda.synchronize()
    assert _lib.read_device_errors() == 0
    assert torch.isfinite(out_p.float()).all()
    # routing: all 5,000 tokens against the oracle router
    x = _np(L.x)
    w = _np(L.router_weight)
    want_inds, _, _, want_logits = moe.router(x, w, 10)
    np.testing.assert_array_equal(bf16.f32_to_bits(logits_p), bf16.f32_to_bits(want_logits))
    np.testing.assert_array_equal(inds_p, want_inds)
    np.testing.assert_array_equal(inds_d, want_inds)
    # every token of the tensor-core path against the exact decode path
    assert_north_star(_np(out_p), _np(out_d), "prefill vs decode path")
    # a seeded sample of tokens against the oracle layer itself
    rng = np.random.default_rng(4242)
    sample = np.sort(rng.choice(tokens, 256, replace=False))
    bank = {k: tuple(_np(t) for t in v) for k, v in L.experts.items()}
    sh = tuple(tuple(_np(t) for t in L.shared[k]) for k in ("gate_proj", "up_proj", "down_proj"))
    ref = moe.moe_block(x[sample], w, 10, bank["gate_proj"], bank["up_proj"], bank["down_proj"], sh,
                        _np(L.shared_expert_gate))
    np.testing.assert_array_equal(bf16.f32_to_bits(_np(out_d)[sample]), bf16.f32_to_bits(ref["out"]))
    assert_north_star(_np(out_p)[sample], ref["out"], "prefill path vs oracle sample")


def test_router_tensor_core_ragged_tiles(cuda_lib):
    """The tcgen05 router on ragged tiles: 3,900 tokens (not a multiple of the
    128-token tile), 300 experts + the shared gate row (301 rows: the last
    64-row tile one-thirteenth full, rows not a multiple of 8), H 1,024.
    Logits and top-8 bit for bit against the oracle router on every token;
    a seeded sample of tokens' outputs (which go through the shared gate's
    logit) bit for bit against the oracle layer."""
    from flashnext_b200 import synthetic
    from flashnext_b200.moe_block import SparseMoEBlock
    tokens, hidden, inter, experts, k = 3900, 1024, 64, 300, 8
    L = synthetic.moe_layer(tokens, hidden, inter, experts, k, 32, zipf=None, seed=77)
    blk = SparseMoEBlock(L.router_weight, L.experts, path="decode", top_k=k, shared=L.shared,
                         shared_expert_gate=L.shared_expert_gate)
    out = _np(blk(L.x))
    x, w = _np(L.x), _np(L.router_weight)
    want_inds, _, _, want_logits = moe.router(x, w, k)
    np.testing.assert_array_equal(bf16.f32_to_bits(_np(blk.last_logits)), bf16.f32_to_bits(want_logits))
    np.testing.assert_array_equal(_np(blk.last_inds), want_inds)
    rng = np.random.default_rng(77)
    sample = np.sort(np.concatenate([rng.choice(tokens - 60, 40, replace=False), np.arange(tokens - 60, tokens)]))
    bank = {n: tuple(_np(t) for t in v) for n, v in L.experts.items()}
    sh = tuple(tuple(_np(t) for t in L.shared[n]) for n in ("gate_proj", "up_proj", "down_proj"))
    ref = moe.moe_block(x[sample], w, k, bank["gate_proj"], bank["up_proj"], bank["down_proj"], sh,
                        _np(L.shared_expert_gate))
    np.testing.assert_array_equal(bf16.f32_to_bits(out[sample]), bf16.f32_to_bits(ref["out"]))


def _check_attention(got, P):
    q, kc, vc = _np(P.q), _np(P.k_cache), _np(P.v_cache)
    table = P.block_table.cpu().numpy()
    lens = P.context_lens.cpu().numpy()
    want = attn.paged_decode_oracle(q, kc, vc, table, lens, P.scale)
    assert_north_star(got, want, "attention vs oracle")
    page = kc.shape[1]
    hkv, d = kc.shape[2], kc.shape[3]
    for b in range(q.shape[0]):
        n = int(lens[b])
        pages = table[b, : -(-n // page)]
        k = kc[pages].reshape(-1, hkv, d)[:n]
        v = vc[pages].reshape(-1, hkv, d)[:n]
        truth = attn.dense_truth(q[b], k, v, P.scale)
        rel = np.abs(got[b] - truth).max() / np.abs(truth).max()
        assert rel < SELFTEST_BOUND, f"sequence {b} (ctx {n}): {rel:.3g}"


@pytest.mark.parametrize("seed", [500, 501])
def test_c5_paged_decode_benchmark_config(cuda_lib, seed):
    """C5: 16 sequences, ctx U[1k, 32k], GQA 16/2, head_dim 256, page 64."""
    from flashnext_b200 import synthetic
    from flashnext_b200.paged_attention import paged_decode
    P = synthetic.paged_decode_inputs(16, 16, 2, 256, 64, (1024, 32768), seed=seed)
    lens = P.context_lens.cpu().numpy()
    assert lens.min() >= 1024 and lens.max() <= 32768
    out = paged_decode(P.q, P.k_cache, P.v_cache, P.block_table, P.context_lens, P.scale)
    _check_attention(_np(out), P)


@pytest.mark.parametrize("split", [64, 256, 1024])
def test_c5_split_sizes_agree(cuda_lib, split):
    """The split-K chunking changes only the float32 merge order: all split
    sizes stay within the bound of the oracle."""
    from flashnext_b200 import synthetic
    from flashnext_b200.paged_attention import paged_decode
    P = synthetic.paged_decode_inputs(4, 16, 2, 256, 64, (1, 9000), seed=77)
    out = paged_decode(P.q, P.k_cache, P.v_cache, P.block_table, P.context_lens, P.scale, split_tokens=split)
    _check_attention(_np(out), P)


@pytest.mark.parametrize("batch,hq,hkv,d,page,ctx,split", [
    (5, 6, 2, 128, 48, (1, 200), 80),     # 3 query heads per kv head, page 48, splits not a stage multiple
    (3, 8, 1, 256, 16, (31, 33), 16),     # stages partly filled at both ends of a split
    (2, 16, 2, 256, 64, (4096, 4096), 4096),  # one split per sequence, every stage full
    (6, 4, 4, 64, 32, (1, 3000), 256),
])
def test_paged_decode_ring_edges(cuda_lib, batch, hq, hkv, d, page, ctx, split):
    """Geometry edges of the staged ring: grouped-query widths below 8, page
    sizes that do not divide a stage, splits shorter than a stage or not a
    multiple of it, one-token contexts and contexts that end a stage
    exactly."""
    from flashnext_b200 import synthetic
    from flashnext_b200.paged_attention import paged_decode
    P = synthetic.paged_decode_inputs(batch, hq, hkv, d, page, ctx, seed=batch * 31 + page)
    out = paged_decode(P.q, P.k_cache, P.v_cache, P.block_table, P.context_lens, P.scale, split_tokens=split)
    _check_attention(_np(out), P)


def test_paged_attention_api_with_cache_append(cuda_lib):
    """paged_attention(queries, cache, scale) over a PagedKVCache filled by
    append() in uneven pieces (page-crossing appends, three sequences of
    different lengths), against dense float64 attention over the same rows."""
    import torch

    from flashnext_b200.paged_attention import PagedKVCache, paged_attention
    g = torch.Generator(device="cuda")
    g.manual_seed(9)
    hq, hkv, d, page = 16, 2, 256, 64
    lens = [1, 700, 2113]
    cache = PagedKVCache(num_pages=64, page_size=page, kv_heads=hkv, head_dim=d, max_pages_per_seq=40,
                         batch=len(lens))
    rows_k, rows_v = [], []
    for b, n in enumerate(lens):
        k = torch.randn((n, hkv, d), generator=g, device="cuda").to(torch.bfloat16)
        v = torch.randn((n, hkv, d), generator=g, device="cuda").to(torch.bfloat16)
        rows_k.append(k)
        rows_v.append(v)
        pos = 0
        for piece in (1, 63, 65, 200, 10_000):
            take = min(piece, n - pos)
            if take <= 0:
                break
            cache.append(b, k[pos:pos + take], v[pos:pos + take])
            pos += take
        assert pos == n
    assert cache.context_lens.cpu().tolist() == lens
    queries = torch.randn((len(lens), hq, 1, d), generator=g, device="cuda").to(torch.bfloat16)
    scale = d ** -0.5
    out = paged_attention(queries, cache, scale)
    assert out.shape == (len(lens), hq, 1, d)
    got = _np(out)[:, :, 0, :]
    for b, n in enumerate(lens):
        truth = attn.dense_truth(_np(queries)[b, :, 0, :], _np(rows_k[b]), _np(rows_v[b]), scale)
        rel = np.abs(got[b] - truth).max() / np.abs(truth).max()
        assert rel < SELFTEST_BOUND, f"sequence {b}: {rel:.3g}"
    with pytest.raises(ValueError):
        paged_attention(queries, cache, scale, mask="causal")
    with pytest.raises(ValueError):
        paged_attention(queries.expand(-1, -1, 2, -1), cache, scale)
