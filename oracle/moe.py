"""NumPy restatement of the Flash-Next sparse-MoE decode arithmetic.

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline leg of ``bench.py``; never by the product package.

Reference anchors (paths inside 1architect/macqwen-releases):

* Q4 nibble order and the affine group formula ``y = s*sum(x*q) + b*sum(x)``:
  ``models/flashnext/metal_runtime.py:955-987`` (``_numpy_projection``).
* Fused up-SwiGLU bfloat16 sequence: ``metal_runtime.py:262-285``.
* Fused down + weighted combine + shared epilogues: ``metal_runtime.py:291-336``
  and the accumulate rewrite ``:397-409``.
* ``weighted_combine``: ``metal_runtime.py:145-191``.
* Router softmax/top-k/renorm: ``models/flashnext/adaptive_topk.py:53-64,256-261``
  and ``models/flashnext/compiled.py:61-71``.
* Shared expert and sigmoid gate: ``adaptive_topk.py:263-264,288``.
* Expert grouping for ragged batches: ``models/flashnext/expert_cache.py:1790-1810``.

Canonical arithmetic.  The reference delegates the projection reduction to
MLX's ``qmv`` helpers, whose source is not present.  This oracle (and the CUDA
kernels, which implement exactly the same definition) fixes it as follows, for
one input row ``x`` of K values and one projection row with packed codes
``q`` and bfloat16 ``s``/``b`` per group of G inputs (G = 32 or 64):

1. row fixed point: ``E = floor(log2 max_i |x_i|)`` over the whole row (0 for
   an all-zero row); ``X_i = trunc(x_i * 2**(22-E))`` (integers below 2**23
   in magnitude; exact for every bfloat16 input within 2**-15 of the row
   maximum);
2. per group g: ``S_g = sum_i X_i*q_i`` and ``SX_g = sum_i X_i`` (exact
   integers, so independent of any summation order);
3. one chain from ``acc = -0.0``, groups in increasing order:
   ``acc = fma(s_g, fl(S_g), acc)``; ``acc = fma(b_g, fl(SX_g), acc)``;
4. ``y = fl(fl(acc * A) * B)`` with ``A*B = 2**(E-22)``,
   ``A = 2**max(E-22, -126)`` (``B = 1`` unless the row's largest input is
   below 2**-104).

``fl`` is float32 round-to-nearest-even and ``fma`` a float32 fused
multiply-add (one rounding).

Router dot products are exact integer sums of the token row's and the router
row's fixed points, scaled by a power of two and rounded once to bfloat16
(see ``router_dot``): independent of any summation order.  ``exp`` is correctly rounded:
to float32 in the softmax, to bfloat16 in the sigmoid.
"""
from __future__ import annotations

from functools import lru_cache

import numpy as np

from . import bf16

# --------------------------------------------------------------------------
# Q4 affine packing (metal_runtime.py:975-985)
# --------------------------------------------------------------------------


def unpack_q4(words) -> np.ndarray:
    """uint32 words [..., K/8] -> 4-bit codes [..., K], low nibble first.

    ``q = (word[k // 8] >> 4 * (k % 8)) & 15`` (metal_runtime.py:981).
    """
    w = np.asarray(words, dtype=np.uint32)
    shifts = (np.arange(8, dtype=np.uint32) * 4)
    q = (w[..., None] >> shifts) & np.uint32(15)
    return q.reshape(*w.shape[:-1], w.shape[-1] * 8).astype(np.uint8)


def pack_q4(codes) -> np.ndarray:
    """Inverse of :func:`unpack_q4` (used by fixtures and generators)."""
    c = np.asarray(codes, dtype=np.uint32)
    c = c.reshape(*c.shape[:-1], c.shape[-1] // 8, 8)
    shifts = (np.arange(8, dtype=np.uint32) * 4)
    return np.bitwise_or.reduce(c << shifts, axis=-1).astype(np.uint32)


def dequantize(words, scales, biases, group_size: int = 32) -> np.ndarray:
    """Affine Q4 dequantisation to bfloat16 bits: ``w = s*q + b`` rounded once.

    The formula is ``metal_runtime.py:984-985`` (``mx.dequantize`` call site
    ``metal_runtime.py:751-758``).  The exact real ``s*q + b`` is rounded once
    to bfloat16 (nearest even).  When ``s*q + b`` is exact in float32 (always
    when |b|/|s| < 2**12, e.g. ``b = -8*s``) this equals evaluating it in
    float32 and rounding to bfloat16.
    """
    q = unpack_q4(words).astype(np.float64)
    s = np.repeat(np.asarray(scales, np.float64), group_size, axis=-1)
    b = np.repeat(np.asarray(biases, np.float64), group_size, axis=-1)
    return bf16.f64_to_bits(s * q + b)


# --------------------------------------------------------------------------
# bfloat16 transcendental helpers
# --------------------------------------------------------------------------


@lru_cache(maxsize=1)
def exp_table() -> np.ndarray:
    """bfloat16 bits -> bfloat16 bits of exp(value), correctly rounded."""
    v = bf16.bits_to_f32(np.arange(65536, dtype=np.uint32).astype(np.uint16))
    with np.errstate(over="ignore", invalid="ignore"):
        e = np.exp(v.astype(np.float64))
    return bf16.f64_to_bits(e)


def sigmoid_bf16(g) -> np.ndarray:
    """Stable bfloat16 sigmoid, one rounding per operation.

    ``|g| -> exp -> 1+e -> 1/d -> (g<0 ? 1/d : 1-1/d)``
    (metal_runtime.py:272-281; MLX's own bfloat16 sigmoid uses this order).
    """
    g = np.asarray(g, dtype=np.float32)
    mag = np.abs(g)
    ex = bf16.bits_to_f32(exp_table()[bf16.f32_to_bits(mag)])
    den = bf16.op(np.add, np.float32(1.0), ex)
    small = bf16.op(np.divide, np.float32(1.0), den)
    return np.where(g < 0, small, bf16.op(np.subtract, np.float32(1.0), small)).astype(np.float32)


def swiglu_bf16(gate, up) -> np.ndarray:
    """``(g * sigmoid(g)) * u`` in bfloat16 arithmetic (metal_runtime.py:282).

    Equals MLX ``swiglu`` = bf16 ``silu(g) * u``
    (``models/flashnext/tests/bench/swiglu_contract.py:144-148``).
    """
    g = np.asarray(gate, dtype=np.float32)
    sg = sigmoid_bf16(g)
    return bf16.op(np.multiply, bf16.op(np.multiply, g, sg), up)


# --------------------------------------------------------------------------
# Canonical Q4 projection (metal_runtime.py:955-987 formula, fixed order)
# --------------------------------------------------------------------------


def swiglu_f32(gate, up) -> np.ndarray:
    """The fused up-SwiGLU sequence with float32 activations (the reference's
    Metal kernel instantiated with T = float, metal_runtime.py:267-285):
    |g| -> exp -> 1+e -> 1/d -> select -> g*sigma -> *u, each op rounded to
    float32; exp correctly rounded (float64 exp, one rounding)."""
    g = np.asarray(gate, dtype=np.float32)
    u = np.asarray(up, dtype=np.float32)
    with np.errstate(over="ignore", invalid="ignore"):
        mag = np.abs(g)
        ex = np.exp(mag.astype(np.float64)).astype(np.float32)
        den = (np.float32(1.0) + ex).astype(np.float32)
        small = (np.float32(1.0) / den).astype(np.float32)
        sig = np.where(g < 0, small, (np.float32(1.0) - small).astype(np.float32)).astype(np.float32)
        return ((g * sig).astype(np.float32) * u).astype(np.float32)


def fixed_point_rows(x):
    """Row fixed point of the inputs.

    Returns ``(E, X)``: ``E`` [N] the floor(log2) of each row's largest
    magnitude (0 for an all-zero row) and ``X`` [N, K] the integers
    ``trunc(x * 2**(22 - E))`` as float64 (exact, |X| < 2**23).
    """
    x = np.asarray(x, dtype=np.float64)
    nz = x != 0
    _, e = np.frexp(np.abs(x))
    e = np.where(nz, e - 1, -(1 << 20))
    emax = e.max(axis=-1)
    emax = np.where(nz.any(axis=-1), emax, 0).astype(np.int64)
    X = np.trunc(np.ldexp(x, (22 - emax)[..., None].astype(np.int32)))
    return emax, X


def limbs(X):
    """Split fixed-point integers into the two 12-bit limbs the kernels use.

    ``X = 4096*L0 + L1`` with ``L1`` in [-2048, 2047] and ``L0`` in
    [-2048, 2048]; both are exact in float16.
    """
    Xi = np.asarray(X).astype(np.int64)
    l1 = ((Xi + 2048) & 4095) - 2048
    l0 = (Xi - l1) >> 12
    return l0, l1


def fma32(a, b, c):
    """float32 fused multiply-add ``fl(a*b + c)`` with a single rounding, exactly.

    The product of two float32 values is exact in float64; the float64 sum's
    rounding error is recovered with TwoSum, and the one case where float64
    rounding can mislead the final float32 rounding -- a float64 sum that
    lands exactly on a float32 midpoint -- is resolved by the error's sign.
    """
    a64 = np.asarray(a, np.float32).astype(np.float64)
    b64 = np.asarray(b, np.float32).astype(np.float64)
    c64 = np.asarray(c, np.float32).astype(np.float64)
    with np.errstate(all="ignore"):
        p = a64 * b64
        s = p + c64
        bv = s - p
        e = (p - (s - bv)) + (c64 - bv)
        r = s.astype(np.float32)
        r64 = r.astype(np.float64)
        up = np.nextafter(r, np.float32(np.inf)).astype(np.float64)
        dn = np.nextafter(r, np.float32(-np.inf)).astype(np.float64)
        d = s - r64
        tie_up = (d > 0) & (d * 2 == up - r64)    # s halfway between r and the next float32 up
        tie_dn = (d < 0) & (-d * 2 == r64 - dn)   # s halfway between r and the next float32 down
        out = np.where(tie_up & (e > 0), up, np.where(tie_dn & (e < 0), dn, r64))
        # halfway and the error points back: r (the even neighbour) already
        # sits on the other side only if RN chose away from the true value.
        out = np.where(tie_up & (e < 0), r64, out)
        out = np.where(tie_dn & (e > 0), r64, out)
    return out.astype(np.float32)


def scale_factors(k):
    """(A, B) float32 with A*B = 2**k: A = 2**max(k, -126), B = 2**(k - max(k, -126))."""
    k = np.asarray(k).astype(np.int32)
    ka = np.maximum(k, -126)
    return np.ldexp(np.float32(1.0), ka).astype(np.float32), np.ldexp(np.float32(1.0), k - ka).astype(np.float32)





def qmv(x, codes, scales, biases, group_size: int = 32) -> np.ndarray:
    """Canonical Q4 projection rows (steps 1-4 of the module docstring).

    x      [N, K] float32 (bfloat16 values)
    codes  [O, K] uint8 nibbles
    scales, biases [O, K/G] float32 (bfloat16 values)
    returns float32 [N, O] (before the bfloat16 output rounding).
    """
    x = np.asarray(x, dtype=np.float32)
    n, k = x.shape
    o = codes.shape[0]
    gc = k // group_size
    emax, X = fixed_point_rows(x)                          # [N], [N,K]
    Xg = X.reshape(n, gc, group_size)
    qf = np.asarray(codes, np.float64).reshape(o, gc, group_size)
    # S[g, n, o]: exact integer dot products (every partial sum < 2**53).
    S = np.matmul(Xg.transpose(1, 0, 2), qf.transpose(1, 2, 0))
    fS = S.astype(np.float32)                              # [Gc, N, O]
    fSX = Xg.sum(axis=-1).astype(np.float32)               # [N, Gc]
    s = np.asarray(scales, np.float32)
    b = np.asarray(biases, np.float32)
    acc = np.full((n, o), -0.0, dtype=np.float32)
    for g in range(gc):
        acc = fma32(s[None, :, g], fS[g], acc)
        acc = fma32(b[None, :, g], fSX[:, g:g + 1], acc)
    A, B = scale_factors(emax - 22)
    with np.errstate(all="ignore"):
        u = (acc * A[:, None]).astype(np.float32)
        return (u * B[:, None]).astype(np.float32)


def expert_parts(words, scales, biases):
    """(words, scales f32, biases f32) of a projection; codes are unpacked per expert on use."""
    return (np.asarray(words), np.asarray(scales, np.float32), np.asarray(biases, np.float32))


# --------------------------------------------------------------------------
# Executor path (metal_runtime.py:764-932), canonical arithmetic
# --------------------------------------------------------------------------


def _project_pairs(rows, expert_of_row, part, group_size):
    """Project each input row with its own expert. rows [R, K] -> [R, O]."""
    words, s, b = part
    out = np.zeros((rows.shape[0], words.shape[1]), dtype=np.float32)
    for e in np.unique(expert_of_row):
        sel = np.nonzero(expert_of_row == e)[0]
        out[sel] = qmv(rows[sel], unpack_q4(words[e]), s[e], b[e], group_size)
    return out


def executor(x, routes, gate, up, down, *, scores=None, shared_y=None,
             shared=None, shared_gate=None, group_size=32, return_all=False, f32=False):
    """Gate -> up -> SwiGLU -> down -> slot-ordered combine (+ shared).

    ``gate``/``up``/``down`` are ``(words, scales, biases)`` with expert-major
    arrays (words uint32 [E, O, K/8]; scales/biases bfloat16-valued float32).
    ``routes`` [T, S] expert indices.  ``f32``: float32 activations (the
    reference's kernels instantiated with T = float): the same sequence of
    operations with every result rounded to float32 instead of bfloat16,
    float32 outputs.  Otherwise returns bfloat16-valued float32 arrays:
    ``(gate [T,S,I], up [T,S,I], down [T,S,H])`` for ``return_all``; the
    per-slot down outputs [T,S,H] when ``scores`` is None; else the combined
    [T,H] output with the requested shared epilogue
    (metal_runtime.py:315-333: per-slot bfloat16 round, float32 multiply by
    the score and add in slot order with no fused multiply-add, bfloat16
    round; then ``bf16(routed + shared_y)`` or
    ``bf16(routed + bf16(shared*shared_gate))``).
    """
    x = np.asarray(x, np.float32)
    routes = np.asarray(routes).astype(np.int64)
    t, slots = routes.shape
    gp = expert_parts(*gate)
    upp = expert_parts(*up)
    dp = expert_parts(*down)
    flat_e = routes.reshape(-1)
    xrows = np.repeat(x, slots, axis=0)
    rnd = (lambda a: np.asarray(a, np.float32)) if f32 else bf16.round_f32
    g = rnd(_project_pairs(xrows, flat_e, gp, group_size))
    u = rnd(_project_pairs(xrows, flat_e, upp, group_size))
    act = swiglu_f32(g, u) if f32 else swiglu_bf16(g, u)
    d = rnd(_project_pairs(act, flat_e, dp, group_size))
    inter = g.shape[-1]
    hidden = d.shape[-1]
    g = g.reshape(t, slots, inter)
    u = u.reshape(t, slots, inter)
    d = d.reshape(t, slots, hidden)
    if return_all:
        return g, u, d
    if scores is None:
        return d
    return combine(d, scores, shared_y=shared_y, shared=shared, shared_gate=shared_gate, f32=f32)


def combine(d, scores, *, shared_y=None, shared=None, shared_gate=None, f32=False):
    """Slot-ordered combine of per-slot outputs (metal_runtime.py:301-333):
    float32 products added in slot order (no fused multiply-add), then the
    shared add; every result rounded to bfloat16, or (``f32``) kept float32."""
    rnd = (lambda a: np.asarray(a, np.float32)) if f32 else bf16.round_f32
    d = np.asarray(d, np.float32)
    sc = np.asarray(scores, np.float32)
    t, slots, hidden = d.shape
    acc = np.zeros((t, hidden), dtype=np.float32)
    with np.errstate(all="ignore"):
        for s in range(slots):
            acc = acc + (d[:, s, :] * sc[:, s][:, None])
        routed = rnd(acc)
        if shared_y is not None:
            return rnd(routed + np.asarray(shared_y, np.float32).reshape(t, hidden))
        if shared is not None:
            comp = rnd(np.asarray(shared, np.float32).reshape(t, hidden)
                       * np.asarray(shared_gate, np.float32).reshape(t, 1))
            return rnd(routed + comp)
    return routed


def weighted_combine(expert_outputs, routes, scores) -> np.ndarray:
    """Restatement of ``weighted_combine`` (metal_runtime.py:145-191, NumPy branch).

    ``expert_outputs`` is [..., slots, hidden] or [..., experts, hidden]
    (then ``routes`` selects the slots).  Result = sum over slots of
    outputs * scores, in the NumPy dtype rules of the reference.
    """
    out = np.asarray(expert_outputs)
    routes = np.asarray(routes)
    scores = np.asarray(scores)
    if out.ndim < 2 or routes.ndim == 0:
        raise ValueError("expert_outputs and routes need at least one dimension")
    if scores.shape != routes.shape:
        raise ValueError("routes and scores must have identical shapes")
    slots = routes.shape[-1]
    if out.shape[:-1] == routes.shape:
        selected = out
    elif out.ndim == routes.ndim + 1 and out.shape[-2] >= slots:
        if routes.size and (routes.min() < 0 or routes.max() >= out.shape[-2]):
            raise ValueError("routes contain an expert outside expert_outputs")
        selected = np.take_along_axis(out, np.expand_dims(routes, -1), axis=-2)
    else:
        raise ValueError(f"expert_outputs shape {out.shape} does not match routes {routes.shape}")
    return (selected * scores[..., None]).sum(axis=-2)


# --------------------------------------------------------------------------
# The reference's own NumPy executor path, restated exactly
# --------------------------------------------------------------------------


def reference_numpy_projection(x, routes, weight, scales, biases, output_width,
                               slot_input, group_size=32) -> np.ndarray:
    """Vectorised restatement of ``_numpy_projection`` (metal_runtime.py:955-987).

    Python floats are IEEE float64: ``qsum`` and ``xsum`` accumulate in
    float64 in input order, ``result`` adds ``s*qsum`` then ``b*xsum`` per
    group in float64, and the float32 output array rounds once.
    """
    x = np.asarray(x)
    routes = np.asarray(routes).astype(np.int64)
    codes = unpack_q4(weight)
    sc = np.asarray(scales).astype(np.float64)
    bi = np.asarray(biases).astype(np.float64)
    tokens, slots = routes.shape
    k = x.shape[-1]
    gc = k // group_size
    out = np.zeros((tokens, slots, output_width), dtype=np.float32)
    for t in range(tokens):
        for s in range(slots):
            e = routes[t, s]
            src = (x[t, s] if slot_input else x[t]).astype(np.float64)
            q = codes[e, :output_width].astype(np.float64)
            result = np.zeros(output_width, dtype=np.float64)
            for g in range(gc):
                qsum = np.zeros(output_width, dtype=np.float64)
                xsum = 0.0
                for i in range(group_size):
                    kk = g * group_size + i
                    qsum = qsum + src[kk] * q[:, kk]
                    xsum = xsum + float(src[kk])
                result = result + sc[e, :output_width, g] * qsum
                result = result + bi[e, :output_width, g] * xsum
            out[t, s] = result
    return out.astype(x.dtype, copy=False)


def reference_execute(x, routes, gate, up, down, *, scores=None, shared_y=None,
                      shared=None, shared_gate=None, group_size=32, return_all=False):
    """Restatement of the reference backend of ``MetalMoEExecutor.execute``.

    ``_reference_all`` (metal_runtime.py:934-941) then ``weighted_combine``
    and the shared add (metal_runtime.py:862-870), for NumPy float32 inputs.
    """
    x = np.asarray(x)
    inter = np.asarray(gate[0]).shape[1]
    hidden = x.shape[-1]
    g = reference_numpy_projection(x, routes, *gate, inter, False, group_size)
    u = reference_numpy_projection(x, routes, *up, inter, False, group_size)
    act = u * (g / (1.0 + np.exp(-g)))
    d = reference_numpy_projection(act, routes, *down, hidden, True, group_size)
    if scores is not None and not return_all:
        d = weighted_combine(d, routes, scores)
        if shared_y is not None:
            d = d + shared_y
        elif shared is not None:
            d = d + shared_gate * shared
    return (g, u, d) if return_all else d


# --------------------------------------------------------------------------
# Router (adaptive_topk.py:53-64, compiled.py:61-71)
# --------------------------------------------------------------------------

ROUTER_LANES = 32  # lanes of the softmax's canonical float32 sum
ROUTER_X_BITS = 22  # token rows: X = trunc(x * 2**(22 - Ex)), |X| < 2**23 (the projection's fixed point)
ROUTER_W_BITS = 14  # router rows: W = trunc(w * 2**(14 - Ew)), |W| < 2**15


def fixed_point_bits(x, bits: int):
    """Row fixed point with ``bits`` fraction bits below the row's top
    exponent: ``(E, X)`` with ``X = trunc(x * 2**(bits - E))`` (float64,
    exact, |X| < 2**(bits + 1)); ``fixed_point_rows`` is the case bits = 22."""
    x = np.asarray(x, dtype=np.float64)
    nz = x != 0
    _, e = np.frexp(np.abs(x))
    e = np.where(nz, e - 1, -(1 << 20))
    emax = e.max(axis=-1)
    emax = np.where(nz.any(axis=-1), emax, 0).astype(np.int64)
    X = np.trunc(np.ldexp(x, (bits - emax)[..., None].astype(np.int32)))
    return emax, X


def router_dot(x, w) -> np.ndarray:
    """Canonical router dot products of bfloat16 rows: x [T,H], w [R,H] -> [T,R].

    The exact value of ``sum_h X[h] * W[h] * 2**(Ex - 22 + Ew - 14)`` with
    ``X``, ``W`` the row fixed points of the token row (22 fraction bits below
    its top exponent ``Ex``) and of the router row (14 bits below ``Ew``).
    The integer sum is exact in any order (|X*W| < 2**38, every partial sum
    below 2**49), so tensor-core integer MMAs on byte limbs, CUDA-core
    integer dot products and this float64 matrix product all give the same
    number; the power-of-two scale is exact.  Truncation drops only input bits
    below 2**-22 (tokens) / 2**-14 (router rows) of the row maximum.
    """
    ex, X = fixed_point_bits(x, ROUTER_X_BITS)
    ew, W = fixed_point_bits(w, ROUTER_W_BITS)
    S = np.asarray(X, np.float64) @ np.asarray(W, np.float64).T
    return np.ldexp(S, (ex[:, None] - ROUTER_X_BITS + ew[None, :] - ROUTER_W_BITS).astype(np.int32))


def router_logits(x, router_weight) -> np.ndarray:
    """BF16 router linear ``self.gate(x)`` (adaptive_topk.py:59,61): bf16
    logits, each the canonical dot product rounded once to bfloat16."""
    return bf16.bits_to_f32(bf16.f64_to_bits(router_dot(x, router_weight)))


def softmax_bf16(logits) -> np.ndarray:
    """``mx.softmax(..., precise=True)`` for bfloat16 logits, bfloat16 output.

    float32 max, ``e_i = fl(exp(l_i - max))`` correctly rounded, canonical
    32-lane sum (lane j adds e_j, e_{j+32}, ... then pairwise), ``p = fl(e/sum)``
    rounded to bfloat16.
    """
    l = np.asarray(logits, np.float32)
    t, n = l.shape
    m = l.max(axis=-1, keepdims=True)
    d = (l - m).astype(np.float32)
    ex = np.exp(d.astype(np.float64)).astype(np.float32)
    lanes = np.full((t, ROUTER_LANES), -0.0, dtype=np.float32)
    for base in range(0, n, ROUTER_LANES):
        nl = min(ROUTER_LANES, n - base)
        lanes[:, :nl] = lanes[:, :nl] + ex[:, base:base + nl]
    v = lanes
    off = ROUTER_LANES // 2
    while off >= 1:
        v = v[..., :off] + v[..., off:2 * off]
        off //= 2
    total = v[..., :1]
    return bf16.round_f32((ex / total).astype(np.float32))


def topk(probs, k):
    """Top-k of bfloat16 probabilities: larger first, ties to the lower index.

    MLX ``argpartition`` leaves the order and tie-break unspecified
    (compiled.py:63); this rule fixes both.  Returns (inds uint32 [T,k],
    scores [T,k], topk_mass [T,1]) with ``topk_mass = bf16(sum scores)`` summed
    in slot order in float32 (adaptive_topk.py:64).
    """
    p = np.asarray(probs, np.float32)
    t, n = p.shape
    bits = bf16.f32_to_bits(p).astype(np.int64)
    key = bits * 65536 + (65535 - np.arange(n))[None, :]
    order = np.argsort(-key, axis=-1, kind="stable")[:, :k]
    inds = order.astype(np.uint32)
    scores = np.take_along_axis(p, order, axis=-1)
    acc = np.zeros((t,), np.float32)
    for s in range(k):
        acc = acc + scores[:, s]
    mass = bf16.round_f32(acc)[:, None]
    return inds, scores, mass


def renorm(scores, topk_mass, blend=1.0):
    """``compiled._renorm_plain`` (compiled.py:68-71) in bfloat16 arithmetic."""
    sc = np.asarray(scores, np.float32)
    mass = np.asarray(topk_mass, np.float32).reshape(-1, 1)
    acc = np.zeros((sc.shape[0],), np.float32)
    for s in range(sc.shape[1]):
        acc = acc + sc[:, s]
    selected = bf16.round_f32(acc)[:, None]
    blend = bf16.round_f32(np.float32(blend))
    normalizer = bf16.op(np.add, mass, bf16.op(np.multiply, blend, bf16.op(np.subtract, selected, mass)))
    return bf16.op(np.divide, sc, normalizer), normalizer


def keep_for_mass(weights, threshold):
    """``_keep_for_mass`` (adaptive_topk.py:43-50): Python floats (IEEE double),
    a sequential total, then the first position whose cumulative share reaches
    the threshold."""
    ws = [float(w) for w in weights]
    total = 0.0
    for w in ws:
        total += w
    accumulated = 0.0
    for position, w in enumerate(ws):
        accumulated += w / total if total != 0.0 else float("nan")
        if accumulated >= threshold:
            return position + 1
    return len(ws)


def adaptive_keep(inds, scores, threshold, min_keep=1):
    """Adaptive keep at threshold < 1 (adaptive_topk.py:75-234 without the
    expert-cache features): the top-k slots, already in descending score order
    (ties to the lower expert, as the stable ``argsort(-scores)``), keep
    ``max(minimum, keep_for_mass)`` slots; dropped slots repeat slot 0's expert
    with score 0.  Returns (inds, scores, keeps).  Threshold >= 1 keeps all."""
    inds = np.asarray(inds)
    sc = np.asarray(scores, np.float32)
    t, k = sc.shape
    if not 0.0 < threshold < 1.0:
        return inds, sc, np.full((t,), k, np.int64)
    minimum = max(1, min(k, int(min_keep)))
    keeps = np.array([max(minimum, keep_for_mass(row, threshold)) for row in sc.tolist()], np.int64)
    active = np.arange(k)[None, :] < keeps[:, None]
    return np.where(active, inds, inds[:, :1]), np.where(active, sc, np.float32(0.0)), keeps


def router(x, router_weight, k, blend=1.0, threshold=1.0, min_keep=1):
    """Router chain: logits -> softmax -> top-k -> adaptive keep (threshold < 1)
    -> renorm over the kept mass."""
    logits = router_logits(x, router_weight)
    probs = softmax_bf16(logits)
    inds, scores, mass = topk(probs, k)
    inds, scores, _ = adaptive_keep(inds, scores, threshold, min_keep)
    rs, _ = renorm(scores, mass, blend)
    return inds, rs, mass, logits


# --------------------------------------------------------------------------
# Shared expert (adaptive_topk.py:263-264,288) and the full block
# --------------------------------------------------------------------------


def shared_expert(x, gate, up, down, gate_weight, group_size=32):
    """Returns (shared [T,H], shared_gate [T,1], shared_y [T,H]) bfloat16 values."""
    x = np.asarray(x, np.float32)
    gw, gs, gb = gate
    uw, us, ub = up
    dw, ds, db = down
    g = bf16.round_f32(qmv(x, unpack_q4(gw), gs, gb, group_size))
    u = bf16.round_f32(qmv(x, unpack_q4(uw), us, ub, group_size))
    act = swiglu_bf16(g, u)
    sh = bf16.round_f32(qmv(act, unpack_q4(dw), ds, db, group_size))
    logit = router_logits(x, np.asarray(gate_weight, np.float32).reshape(1, -1))
    sg = sigmoid_bf16(logit)
    sy = bf16.op(np.multiply, sg, sh)
    return sh, sg, sy


def moe_block(x, router_weight, k, gate, up, down, shared, shared_gate_weight,
              group_size=32, blend=1.0, threshold=1.0, min_keep=1):
    """One sparse-MoE block (adaptive_topk.py:53-292), adaptive keep when
    threshold < 1.

    Returns dict with logits, inds, scores (renormalised), mass, shared_y and
    the bfloat16 output [T, H].
    """
    inds, scores, mass, logits = router(x, router_weight, k, blend, threshold, min_keep)
    sh, sg, sy = shared_expert(x, *shared, shared_gate_weight, group_size)
    out = executor(x, inds, gate, up, down, scores=scores, shared_y=sy, group_size=group_size)
    return {"logits": logits, "inds": inds, "scores": scores, "mass": mass,
            "shared": sh, "shared_gate": sg, "shared_y": sy, "out": out}


# --------------------------------------------------------------------------
# Grouping (expert_cache.py:1790-1810: _gather_sort for ragged batches)
# --------------------------------------------------------------------------


def group_tokens(keys, n_keys):
    """Stable grouping of (token, slot) pairs by expert key.

    Returns (counts [n_keys], offsets [n_keys+1], order [T*S]) where
    ``order`` lists flattened pair indices sorted by key, ties by pair index.
    """
    flat = np.asarray(keys).reshape(-1).astype(np.int64)
    counts = np.bincount(flat, minlength=n_keys).astype(np.int64)
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    order = np.argsort(flat, kind="stable").astype(np.int64)
    return counts, offsets, order
