"""Expert-parallel layer: dispatch / combine logic on CPU ranks (gloo).

Two (and three) spawned ranks, each with its own token batch and 1/W of the
experts, run ``ExpertParallelMoE`` with an oracle compute backend; every
rank's output must equal the single-process oracle layer on its tokens bit
for bit.  The CUDA backend runs the same orchestration in
``test_gpu_expert_parallel.py``.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

H, I, E, K, G = 64, 32, 12, 3, 32


def _model():
    from oracle import bf16

    rng = np.random.default_rng(77)

    def proj(n, o, k):
        words = rng.integers(0, 2 ** 32, (n, o, k // 8), dtype=np.uint32)
        s = bf16.round_f32(np.abs(rng.normal(0, 0.01, (n, o, k // G))).astype(np.float32))
        return words, s, bf16.round_f32(-8 * s)

    bank = {"gate_proj": proj(E, I, H), "up_proj": proj(E, I, H), "down_proj": proj(E, H, I)}
    shared = tuple(tuple(a[0] for a in t) for t in (proj(1, I, H), proj(1, I, H), proj(1, H, I)))
    w = bf16.round_f32((rng.standard_normal((E, H)) * 0.5).astype(np.float32))
    wg = bf16.round_f32((rng.standard_normal(H) * 0.05).astype(np.float32))
    return bank, shared, w, wg


def _tokens(rank):
    from oracle import bf16

    rng = np.random.default_rng(100 + rank)
    return bf16.round_f32(rng.standard_normal((5 + 2 * rank, H)).astype(np.float32))


class OracleBackend:
    """The compute steps of the layer, by the NumPy oracle (torch CPU tensors in/out)."""

    def __init__(self, bank, shared, w, wg, lo, hi):
        self.bank = {k: tuple(a[lo:hi] for a in v) for k, v in bank.items()}
        self.shared, self.w, self.wg = shared, w, wg

    @staticmethod
    def _bf(a):
        import torch

        return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16)

    def route(self, x):
        import torch

        from oracle import moe

        xn = x.float().numpy()
        inds, scores, _, _ = moe.router(xn, self.w, K)
        _, sg, _ = moe.shared_expert(xn, *self.shared, self.wg, G)
        return torch.from_numpy(inds.astype(np.int32)), self._bf(scores), self._bf(sg.reshape(-1))

    def experts(self, rows, ids):
        """Per-slot outputs [R, S, H] of received rows; id == experts per rank is the shared expert."""
        from oracle import moe

        ids = ids.numpy().astype(np.int64)
        R, S = ids.shape
        xr = rows.float().numpy()
        d = np.zeros((R, S, H), np.float32)
        per = self.bank["gate_proj"][0].shape[0]
        routed = (ids >= 0) & (ids < per)
        if routed.any():
            r, s = np.nonzero(routed)
            d[r, s] = moe.executor(xr[r], ids[r, s].reshape(-1, 1), self.bank["gate_proj"], self.bank["up_proj"],
                                   self.bank["down_proj"], group_size=G).reshape(-1, H)
        shared = ids == per
        if shared.any():
            r, s = np.nonzero(shared)
            sh, _, _ = moe.shared_expert(xr[r], *self.shared, self.wg, G)
            d[r, s] = sh
        return self._bf(d)

    def combine(self, d, inds, scores, shared, shared_gate):
        from oracle import moe

        out = moe.combine(d.float().numpy(), scores.float().numpy(), shared=shared.float().numpy(),
                          shared_gate=shared_gate.float().numpy())
        return self._bf(out)


def _worker(rank, world, port, result_dir):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "macqwen-releases_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch
    import torch.distributed as dist

    from flashnext_b200.expert_parallel import ExpertParallelMoE
    from oracle import bf16, moe

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        bank, shared, w, wg = _model()
        per = E // world
        backend = OracleBackend(bank, shared, w, wg, rank * per, (rank + 1) * per)
        layer = ExpertParallelMoE(backend, expert_count=E, hidden_size=H, top_k=K)
        x = _tokens(rank)
        got = layer(OracleBackend._bf(x)).float().numpy()
        want = moe.moe_block(x, w, K, bank["gate_proj"], bank["up_proj"], bank["down_proj"], shared, wg,
                             group_size=G)["out"]
        same = np.array_equal(bf16.f32_to_bits(got), bf16.f32_to_bits(want))
        np.save(os.path.join(result_dir, f"r{rank}.npy"), np.array([same]))
    finally:
        dist.destroy_process_group()


def _overflow_worker(rank, world, port, result_dir):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "macqwen-releases_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist

    from flashnext_b200.expert_parallel import ExpertParallelMoE

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        bank, shared, w, wg = _model()
        per = E // world
        backend = OracleBackend(bank, shared, w, wg, rank * per, (rank + 1) * per)
        layer = ExpertParallelMoE(backend, expert_count=E, hidden_size=H, top_k=K, capacity_tokens=6)
        x = _tokens(rank)  # rank 0: 5 tokens (fits), rank 1: 7 tokens (exceeds 6)
        raised = False
        try:
            layer(OracleBackend._bf(x))
        except ValueError:
            raised = True
        # the ranks are still in step: one more collective completes
        import torch
        t = torch.ones(1)
        dist.all_reduce(t)
        np.save(os.path.join(result_dir, f"o{rank}.npy"), np.array([raised, float(t[0]) == world]))
    finally:
        dist.destroy_process_group()


def test_capacity_overflow_raises_on_every_rank(tmp_path):
    """One rank routes more tokens than the fixed capacity: every rank raises
    ValueError before any exchange, and the group stays usable."""
    import torch.multiprocessing as mp

    mp.spawn(_overflow_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        raised, alive = np.load(tmp_path / f"o{r}.npy")
        assert raised, f"rank {r} did not raise"
        assert alive, f"rank {r}: the group hung or broke"


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 3])
def test_expert_parallel_matches_single_device_oracle(tmp_path, world):
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        assert bool(np.load(tmp_path / f"r{r}.npy")[0]), f"rank {r} output differs from the oracle layer"
