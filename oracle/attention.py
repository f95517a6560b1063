"""Paged decode attention oracle -- TEST INFRASTRUCTURE ONLY.

Restates ``paged_attention`` (``models/qwen27b/paged_kv.py:417-495``) for one
query token: chunks are pages of the block table in order; per chunk the
scores are computed in float32, ``m_new = max``, ``p = exp(s - m_new)``,
``l_new = sum p``, ``o_new = p @ v`` in float32, merged with
``exp(m_run - m)`` / ``exp(m_new - m)``; output ``o / l`` rounded to bfloat16.
GQA maps query head h to kv head h // (Hq / Hkv) (the reshape at
paged_kv.py:433-434).

One deliberate difference: MLX evaluates ``q @ k^T`` on bfloat16 arrays and
returns bfloat16 scores before the float32 cast (paged_kv.py:474); here the
scores stay float32, which is what the CUDA kernel computes.
"""
from __future__ import annotations

import numpy as np

from . import bf16


def dense_truth(q, k, v, scale):
    """float64 softmax attention. q [Hq, D]; k, v [T, Hkv, D] -> [Hq, D]."""
    hq = q.shape[0]
    hkv = k.shape[1]
    rep = hq // hkv
    out = np.zeros((hq, q.shape[1]))
    for h in range(hq):
        kk = k[:, h // rep, :].astype(np.float64)
        vv = v[:, h // rep, :].astype(np.float64)
        s = kk @ q[h].astype(np.float64) * scale
        w = np.exp(s - s.max())
        out[h] = (w[:, None] * vv).sum(0) / w.sum()
    return out


def to_pages(k, v, page_size, rng):
    """Scatter [T, Hkv, D] rows into randomly permuted pages; returns (pages, table)."""
    t, hkv, d = k.shape
    n = -(-t // page_size)
    perm = rng.permutation(n)
    kp = np.zeros((n, page_size, hkv, d), np.float32)
    vp = np.zeros_like(kp)
    for i in range(n):
        rows = slice(i * page_size, min(t, (i + 1) * page_size))
        kp[perm[i], : rows.stop - rows.start] = k[rows]
        vp[perm[i], : rows.stop - rows.start] = v[rows]
    return (kp, vp), perm.astype(np.int32)


def paged_decode_oracle(q, k_pages, v_pages, block_table, context_lens, scale):
    """q [B, Hq, D]; pages [P, page, Hkv, D]; block_table [B, max_pages]; -> [B, Hq, D] bf16 values."""
    q = np.asarray(q, np.float32)
    b_count, hq, d = q.shape
    page = k_pages.shape[1]
    hkv = k_pages.shape[2]
    rep = hq // hkv
    out = np.zeros((b_count, hq, d), np.float32)
    for b in range(b_count):
        ctx = int(context_lens[b])
        qs = (q[b] * np.float32(scale)).astype(np.float32).reshape(hkv, rep, d)
        m_run = l_run = o_run = None
        for pi in range(-(-ctx // page)):
            n = min(page, ctx - pi * page)
            pg = int(block_table[b, pi])
            kk = k_pages[pg, :n].astype(np.float32).transpose(1, 2, 0)   # [Hkv, D, n]
            vv = v_pages[pg, :n].astype(np.float32).transpose(1, 0, 2)   # [Hkv, n, D]
            s = np.matmul(qs, kk).astype(np.float32)                     # [Hkv, rep, n]
            m_new = s.max(-1, keepdims=True)
            p = np.exp(s - m_new).astype(np.float32)
            l_new = p.sum(-1, keepdims=True, dtype=np.float32)
            o_new = np.matmul(p, vv).astype(np.float32)                  # [Hkv, rep, D]
            if m_run is None:
                m_run, l_run, o_run = m_new, l_new, o_new
            else:
                m_cat = np.maximum(m_run, m_new)
                a = np.exp(m_run - m_cat).astype(np.float32)
                bb = np.exp(m_new - m_cat).astype(np.float32)
                l_run = a * l_run + bb * l_new
                o_run = a * o_run + bb * o_new
                m_run = m_cat
        if m_run is not None:
            out[b] = bf16.round_f32((o_run / l_run).reshape(hq, d).astype(np.float32))
    return out
