"""Expert-parallel layer on 2 GPUs: bit-identical to the one-GPU layer.

Needs two visible B200s; skipped otherwise.  Each rank holds half of the
experts (tiled), routes its own tokens, and must reproduce, bit for bit, what
``SparseMoEBlock`` (all experts on one GPU) gives for the same tokens --
through the NVLink peer-memory exchange (eagerly for several steps in a row,
with a rank routing fewer tokens than the other, and replayed from a CUDA
graph) and through the all-to-all path over NCCL.
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

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    results = []
    layer = None
    graph = None
    try:
        from flashnext_b200 import _lib, synthetic
        from flashnext_b200.expert_parallel import CudaBackend, ExpertParallelMoE
        from flashnext_b200.moe_block import SparseMoEBlock

        E, H, I, K, T = 64, 2048, 512, 10, 24
        L = synthetic.moe_layer(3 * T * world, H, I, E, K, 32, zipf=1.1, seed=313)
        per = E // world
        local = {n: tuple(t[rank * per:(rank + 1) * per].contiguous() for t in v) for n, v in L.experts.items()}
        ref_block = SparseMoEBlock(L.router_weight, L.experts, top_k=K, shared=L.shared,
                                   shared_expert_gate=L.shared_expert_gate)

        def check(layer, x):
            got = layer(x)
            ref = ref_block(x)
            torch.cuda.synchronize()
            return bool(torch.equal(got.view(torch.int16), ref.view(torch.int16)))

        backend = CudaBackend(L.router_weight, local, L.shared, L.shared_expert_gate, top_k=K)
        layer = ExpertParallelMoE(backend, expert_count=E, hidden_size=H, top_k=K, capacity_tokens=T)
        assert layer.exchange is not None
        # three eager steps with different tokens; rank 1 routes fewer tokens in step 2
        for step in range(3):
            n = T if not (step == 1 and rank == 1) else T // 3
            x = L.x[(3 * rank + step) * T:(3 * rank + step) * T + n].contiguous()
            results.append(check(layer, x))
        # a captured step replayed twice
        x = L.x[(3 * rank) * T:(3 * rank + 1) * T].contiguous().clone()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph, stream=s):
                g_out = layer(x)
        torch.cuda.current_stream().wait_stream(s)
        ref = ref_block(x)
        for _ in range(2):
            g_out.zero_()
            graph.replay()
            torch.cuda.synchronize()
            results.append(bool(torch.equal(g_out.view(torch.int16), ref.view(torch.int16))))
        results.append(_lib.read_device_errors() == 0)
        # the all-to-all path over NCCL
        coll = ExpertParallelMoE(backend, expert_count=E, hidden_size=H, top_k=K, capacity_tokens=T, peer=False)
        results.append(check(coll, L.x[3 * rank * T:(3 * rank + 1) * T].contiguous()))
        np.save(os.path.join(result_dir, f"r{rank}.npy"), np.array(results))
    finally:
        torch.cuda.synchronize()
        graph = None
        if layer is not None:
            layer.close()
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
        res = np.load(tmp_path / f"r{r}.npy")
        assert res.all(), f"rank {r}: expert-parallel results {res.tolist()} (eager x3, graph x2, errors, all-to-all)"
