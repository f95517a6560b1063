"""The batch-1 layer as one persistent kernel (B200 only).

A one-token layer on tiled tables runs router, top-k, gate/up, down and the
combine in one cooperative launch with two grid barriers.  It must give the
oracle's bits, and the bits of the multi-launch chain (reference-layout
arrays), at every shape it accepts: the C1 layer, the C3 layer (whose
shared-memory plan reuses the gate/up ring for the down stage), group size
64, no shared expert, adaptive keep, and the interface limits.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import bf16, moe

pytestmark = pytest.mark.gpu


def _np(t):
    import torch

    if t.dtype == torch.bfloat16:
        return t.float().cpu().numpy()
    if t.dtype == torch.int32:
        return t.cpu().numpy().view(np.uint32)
    return t.cpu().numpy()


def _bits(a):
    return bf16.f32_to_bits(np.asarray(a, np.float32))


def _oracle(L, k, group, shared=True, threshold=1.0, min_keep=1):
    bank = {n: tuple(_np(t) for t in v) for n, v in L.experts.items()}
    x, w = _np(L.x), _np(L.router_weight)
    if shared:
        sh = tuple(tuple(_np(t) for t in L.shared[n]) for n in ("gate_proj", "up_proj", "down_proj"))
        return moe.moe_block(x, w, k, bank["gate_proj"], bank["up_proj"], bank["down_proj"], sh,
                             _np(L.shared_expert_gate), group_size=group, threshold=threshold, min_keep=min_keep)
    inds, scores, mass, logits = moe.router(x, w, k, threshold=threshold, min_keep=min_keep)
    out = moe.executor(x, inds, bank["gate_proj"], bank["up_proj"], bank["down_proj"], scores=scores,
                       group_size=group)
    return {"inds": inds, "scores": scores, "logits": logits, "out": out}


@pytest.mark.parametrize("hidden,inter,experts,k,group,shared,seed", [
    (2048, 512, 512, 10, 32, True, 1),     # C1
    (2048, 512, 512, 10, 32, True, 2),
    (3072, 640, 512, 10, 32, True, 3),     # C3 layer: down stage aliases the gate/up ring
    (1024, 256, 64, 8, 64, True, 4),       # group size 64
    (2048, 512, 128, 10, 32, False, 5),    # no shared expert
    (1024, 256, 1024, 16, 32, True, 6),    # 1,024 experts, top-16 (17 units)
])
def test_fused_batch1_layer_bit_exact(cuda_lib, hidden, inter, experts, k, group, shared, seed):
    import torch

    from flashnext_b200 import _lib, synthetic
    from flashnext_b200.moe_block import SparseMoEBlock
    _lib.read_device_errors()
    L = synthetic.moe_layer(1, hidden, inter, experts, k, group, seed=seed)
    kw = dict(top_k=k, group_size=group)
    if shared:
        kw.update(shared=L.shared, shared_expert_gate=L.shared_expert_gate)
    fused = SparseMoEBlock(L.router_weight, L.experts, **kw)
    assert fused.tiled is not None
    arrays = SparseMoEBlock(L.router_weight, L.experts, tiled=False, **kw)
    outs = [fused(L.x).clone() for _ in range(2)]  # two calls in a row: the barrier state restarts
    ref_out = arrays(L.x).clone()
    torch.cuda.synchronize()
    assert _lib.read_device_errors() == 0
    ref = _oracle(L, k, group, shared)
    np.testing.assert_array_equal(_np(fused.last_inds), ref["inds"])
    np.testing.assert_array_equal(_bits(_np(fused.last_logits)), _bits(ref["logits"]))
    np.testing.assert_array_equal(_bits(_np(fused.last_scores)), _bits(ref["scores"]))
    for o in outs:
        np.testing.assert_array_equal(_bits(_np(o)), _bits(ref["out"]))
        assert torch.equal(o.view(torch.int16), ref_out.view(torch.int16))


@pytest.mark.parametrize("threshold,min_keep", [(0.3, 1), (0.6, 2), (0.95, 1)])
def test_fused_batch1_adaptive_keep_bit_exact(cuda_lib, threshold, min_keep):
    from flashnext_b200 import _lib, synthetic
    from flashnext_b200.moe_block import SparseMoEBlock
    _lib.read_device_errors()
    L = synthetic.moe_layer(1, 2048, 512, 512, 10, 32, zipf=1.1, seed=40)
    block = SparseMoEBlock(L.router_weight, L.experts, top_k=10, shared=L.shared,
                           shared_expert_gate=L.shared_expert_gate, keep_threshold=threshold, min_keep=min_keep)
    out = block(L.x)
    ref = _oracle(L, 10, 32, True, threshold, min_keep)
    assert _lib.read_device_errors() == 0
    np.testing.assert_array_equal(_np(block.last_inds), ref["inds"])
    np.testing.assert_array_equal(_bits(_np(block.last_scores)), _bits(ref["scores"]))
    np.testing.assert_array_equal(_bits(_np(out)), _bits(ref["out"]))


def test_fused_batch1_layer_in_a_cuda_graph(cuda_lib):
    """Captured and replayed: eight distinct layers, as the benchmark runs them."""
    import torch

    from flashnext_b200 import _lib, synthetic
    from flashnext_b200.moe_block import SparseMoEBlock
    _lib.read_device_errors()
    blocks, xs, outs, refs = [], [], [], []
    for i in range(3):
        L = synthetic.moe_layer(1, 2048, 512, 512, 10, 32, seed=70 + i)
        b = SparseMoEBlock(L.router_weight, L.experts, top_k=10, shared=L.shared,
                           shared_expert_gate=L.shared_expert_gate)
        blocks.append(b)
        xs.append(L.x)
        outs.append(torch.empty((1, 2048), dtype=torch.bfloat16, device="cuda"))
        refs.append(b(L.x).clone())
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for b, x, o in zip(blocks, xs, outs):
                b(x, out=o)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        for o in outs:
            o.zero_()
        g.replay()
        torch.cuda.synchronize()
        for o, r in zip(outs, refs):
            assert torch.equal(o.view(torch.int16), r.view(torch.int16))
    assert _lib.read_device_errors() == 0
