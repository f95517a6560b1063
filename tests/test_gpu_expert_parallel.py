"""Expert-parallel layer on 2 GPUs (NCCL): bit-identical to the one-GPU layer.

Needs two visible B200s; skipped otherwise.  Each rank holds half of the
experts (tiled), routes its own tokens, and must reproduce, bit for bit, what
``SparseMoEBlock`` (all experts on one GPU) gives for the same tokens.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, result_dir):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "macqwen-releases_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        from flashnext_b200 import synthetic
        from flashnext_b200.expert_parallel import CudaBackend, ExpertParallelMoE
        from flashnext_b200.moe_block import SparseMoEBlock

        E, H, I, K, T = 64, 2048, 512, 10, 24
        L = synthetic.moe_layer(T * world, H, I, E, K, 32, zipf=1.1, seed=313)
        x = L.x[T * rank:T * (rank + 1)].contiguous()
        per = E // world
        local = {n: tuple(t[rank * per:(rank + 1) * per].contiguous() for t in v) for n, v in L.experts.items()}
        layer = ExpertParallelMoE(CudaBackend(L.router_weight, local, L.shared, L.shared_expert_gate, top_k=K),
                                  expert_count=E, hidden_size=H, top_k=K)
        got = layer(x)
        ref = SparseMoEBlock(L.router_weight, L.experts, top_k=K, shared=L.shared,
                             shared_expert_gate=L.shared_expert_gate)(x)
        torch.cuda.synchronize()
        same = torch.equal(got.view(torch.int16), ref.view(torch.int16))
        np.save(os.path.join(result_dir, f"r{rank}.npy"), np.array([same]))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_expert_parallel_two_gpus_matches_one_gpu_layer(tmp_path):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        assert bool(np.load(tmp_path / f"r{r}.npy")[0]), f"rank {r}: expert-parallel output differs"
