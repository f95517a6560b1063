"""Properties and known answers of the CPU oracle (no GPU)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import attention as attn
from oracle import bf16, moe


def _bf(rng, shape, std=1.0):
    return bf16.round_f32((rng.standard_normal(shape) * std).astype(np.float32))


def test_pack_unpack_round_trip():
    rng = np.random.default_rng(1)
    codes = rng.integers(0, 16, (3, 5, 64), dtype=np.uint8)
    words = moe.pack_q4(codes)
    assert words.shape == (3, 5, 8)
    np.testing.assert_array_equal(moe.unpack_q4(words), codes)
    # low nibble first (metal_runtime.py:981)
    np.testing.assert_array_equal(moe.unpack_q4(np.array([0x76543210], dtype=np.uint32)), np.arange(8))


def test_dequantize_is_single_rounded_affine():
    rng = np.random.default_rng(2)
    codes = rng.integers(0, 16, (4, 64), dtype=np.uint8)
    s = bf16.round_f32(np.abs(rng.normal(0, 0.01, (4, 2))).astype(np.float32))
    b = bf16.round_f32(-8 * s)
    out = bf16.bits_to_f32(moe.dequantize(moe.pack_q4(codes), s, b, 32))
    exact = np.repeat(s, 32, 1).astype(np.float64) * codes + np.repeat(b, 32, 1)
    # b = -8 s: s*q + b = s*(q-8) is exact in float32, so both rounding rules agree
    np.testing.assert_array_equal(out, bf16.round_f32(exact.astype(np.float32)))


def test_fixed_point_limbs_are_exact():
    rng = np.random.default_rng(3)
    x = _bf(rng, (5, 128))
    x[0, :] = 0.0                        # all-zero row
    x[1, 5] = np.float32(2.0 ** -130)    # subnormal-range value
    x[2, :] = x[2, :] * np.float32(2.0 ** -120)
    emax, X = moe.fixed_point_rows(x)
    assert np.all(np.abs(X) < 2 ** 23)
    assert emax[0] == 0 and not X[0].any()
    l0, l1 = moe.limbs(X)
    assert l1.min() >= -2048 and l1.max() <= 2047 and np.abs(l0).max() <= 2048
    np.testing.assert_array_equal(4096 * l0 + l1, X.astype(np.int64))
    # every value within 2^-15 of its row maximum is represented exactly
    xr = x.astype(np.float64)
    back = np.ldexp(X, (emax - 22)[:, None].astype(np.int32))
    big = np.abs(xr) >= np.ldexp(1.0, (emax - 15)[:, None].astype(np.int32))
    np.testing.assert_array_equal(back[big], xr[big])


@pytest.mark.parametrize("group,k", [(32, 2048), (32, 512), (64, 640), (32, 32), (64, 64), (32, 96)])
def test_qmv_matches_float64(group, k):
    rng = np.random.default_rng(4)
    o = 16
    codes = rng.integers(0, 16, (o, k), dtype=np.uint8)
    s = bf16.round_f32(np.abs(rng.normal(0, 0.01, (o, k // group))).astype(np.float32))
    b = bf16.round_f32(-8 * s + bf16.round_f32(rng.normal(0, 1e-3, s.shape).astype(np.float32)))
    x = _bf(rng, (3, k))
    y = moe.qmv(x, codes, s, b, group)
    dense = np.repeat(s, group, 1).astype(np.float64) * codes + np.repeat(b, group, 1)
    ref = x.astype(np.float64) @ dense.T
    np.testing.assert_allclose(y, ref, rtol=0, atol=1e-5 * np.abs(ref).max() + 1e-30)


def _ml_bf16_swiglu(g, u):
    import ml_dtypes

    bt = ml_dtypes.bfloat16
    gb, ub = g.astype(bt), u.astype(bt)
    mag = np.abs(gb)
    ex = np.exp(mag.astype(np.float64)).astype(bt)   # exp correctly rounded to bfloat16
    den = (bt(1) + ex).astype(bt)
    small = (bt(1) / den).astype(bt)
    sig = np.where(gb < 0, small, (bt(1) - small).astype(bt)).astype(bt)
    return ((gb * sig).astype(bt) * ub).astype(bt).astype(np.float32)


@pytest.mark.parametrize("up_bits", [0x3F80, 0x3F9E])
def test_swiglu_contract_exhaustive(up_bits):
    """All 65,536 bfloat16 gate patterns (models/flashnext/tests/unit/test_swiglu_contract.py:36-50).

    The oracle's op sequence agrees bit for bit with an independent
    ml_dtypes bfloat16 evaluation of the same sequence (non-NaN results),
    and a float32 SiLU rounded once differs on some patterns, as the
    reference's contract harness reports for its fp32 candidate.
    """
    gates = bf16.bits_to_f32(np.arange(65536, dtype=np.uint32).astype(np.uint16))
    up = np.full_like(gates, bf16.bits_to_f32(np.array([up_bits], dtype=np.uint16))[0])
    ours = moe.swiglu_bf16(gates, up)
    other = _ml_bf16_swiglu(gates, up)
    finite = ~np.isnan(ours) & ~np.isnan(other)
    assert np.array_equal(np.isnan(ours), np.isnan(other))
    np.testing.assert_array_equal(bf16.f32_to_bits(ours[finite]), bf16.f32_to_bits(other[finite]))
    with np.errstate(all="ignore"):
        fp32 = bf16.round_f32((gates / (1 + np.exp(-gates)) * up).astype(np.float32))
    assert np.count_nonzero((bf16.f32_to_bits(fp32) != bf16.f32_to_bits(ours)) & finite) > 0


def test_router_dot_matches_float64():
    """The canonical router dot product differs from the exact float64 one
    only by the truncation of input bits below 2**-22 / 2**-14 of each row's
    maximum; its integer sum is exact, so byte-limb decompositions agree."""
    rng = np.random.default_rng(5)
    x = _bf(rng, (4, 2048))
    w = _bf(rng, (64, 2048), 0.02)
    got = moe.router_dot(x, w)
    ref = x.astype(np.float64) @ w.T.astype(np.float64)
    bound = 2048 * (np.abs(x).max() * np.abs(w).max() * 2.0 ** -13)
    assert np.abs(got - ref).max() < bound
    np.testing.assert_allclose(got, ref, rtol=0, atol=2e-4 * np.abs(ref).max())
    # the same integers through 3 x 2 byte limbs (the tensor-core form)
    ex, X = moe.fixed_point_bits(x, moe.ROUTER_X_BITS)
    ew, W = moe.fixed_point_bits(w, moe.ROUTER_W_BITS)
    Xi, Wi = X.astype(np.int64), W.astype(np.int64)
    xl = [Xi & 255, (Xi >> 8) & 255, Xi >> 16]
    wl = [Wi & 255, Wi >> 8]
    S = sum((xl[i] @ wl[j].T) << (8 * (i + j)) for i in range(3) for j in range(2))
    np.testing.assert_array_equal(S, Xi @ Wi.T)
    np.testing.assert_array_equal(np.ldexp(S.astype(np.float64), (ex[:, None] - 22 + ew[None, :] - 14).astype(np.int32)),
                                  got)


def test_topk_orders_by_probability_then_lower_index():
    p = np.zeros((1, 40), np.float32)
    p[0, [3, 7, 9, 20, 30]] = [0.25, 0.125, 0.25, 0.0625, 0.25]
    inds, scores, mass = moe.topk(p, 4)
    assert inds.tolist() == [[3, 9, 30, 7]]
    np.testing.assert_array_equal(scores, [[0.25, 0.25, 0.25, 0.125]])
    assert float(mass[0, 0]) == 0.875


def test_softmax_and_renorm():
    rng = np.random.default_rng(6)
    logits = _bf(rng, (8, 512), 2.0)
    p = moe.softmax_bf16(logits)
    np.testing.assert_allclose(p.sum(-1), 1.0, atol=0.02)
    inds, sc, mass = moe.topk(p, 10)
    rs, norm = moe.renorm(sc, mass, 1.0)
    np.testing.assert_array_equal(norm, mass)
    np.testing.assert_allclose(rs.sum(-1), 1.0, atol=0.03)
    assert np.all(np.diff(sc, axis=-1) <= 0)


def test_group_tokens_is_stable_counting_sort():
    keys = np.array([[3, 1], [1, 0], [3, 3]])
    counts, offsets, order = moe.group_tokens(keys, 5)
    assert counts.tolist() == [1, 2, 0, 3, 0]
    assert offsets.tolist() == [0, 1, 3, 3, 6, 6]
    assert order.tolist() == [3, 1, 2, 0, 4, 5]


@pytest.mark.parametrize("total,label", [(1000, "decode"), (256, "exact page boundary"),
                                         (300, "partial last page"), (7, "short context")])
def test_paged_attention_oracle_selftest(total, label):
    """paged_kv.selftest criterion (models/qwen27b/paged_kv.py:526-567): error vs a
    float32/float64 truth below 1.5e-2 of the truth's max magnitude."""
    rng = np.random.default_rng(total)
    n_q, n_kv, d, page = 24, 4, 256, 64
    k = rng.standard_normal((total, n_kv, d)).astype(np.float32)
    v = rng.standard_normal((total, n_kv, d)).astype(np.float32)
    q = rng.standard_normal((n_q, d)).astype(np.float32)
    truth = attn.dense_truth(q, k, v, d ** -0.5)
    pages, table = attn.to_pages(bf16.round_f32(k), bf16.round_f32(v), page, rng)
    out = attn.paged_decode_oracle(bf16.round_f32(q)[None], pages[0], pages[1], table[None],
                                   np.array([total]), d ** -0.5)[0]
    err = np.abs(out - truth).max() / np.abs(truth).max()
    assert err < 1.5e-2, (label, err)
