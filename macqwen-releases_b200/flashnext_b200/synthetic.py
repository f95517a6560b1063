"""Seeded synthetic inputs with the shapes and distributions of the benchmark configs.

There is no checkpoint or dataset on this path; every config of the
benchmark is stated as shapes and value distributions, reproduced here:

* Q4/G32 experts: packed uint32 words of uniform nibbles 0..15, bfloat16
  scales ~ |N(0, 0.01)|, biases = -8 * scale (exact in bfloat16);
* activations x ~ N(0, 1) bfloat16; router weight ~ N(0, 0.02) bfloat16;
* ragged decode: router logits biased so expert popularity follows a Zipf
  law (s = 1.1) over the experts (a shared direction ``u`` in x and a
  per-expert component along ``u`` in the router rows, see ``zipf_router``);
* paged attention: K/V ~ N(0, 1) bfloat16 pages, block tables that are a
  random permutation of the physical pages, context lengths uniform in a
  range.

Generators run on the device with a seeded ``torch.Generator`` so that
gigabyte-sized expert banks are produced in seconds.
"""
from __future__ import annotations

import math
from dataclasses import dataclass


def _torch():
    import torch

    return torch


def _gen(seed: int, device):
    torch = _torch()
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    return g


def q4_projection(experts: int, out_w: int, in_w: int, group: int = 32, *, seed: int = 0,
                  device="cuda", scale_std: float = 0.01):
    """(weight int32 [E,O,K/8], scales bf16 [E,O,K/G], biases bf16) for one projection."""
    torch = _torch()
    g = _gen(seed, device)
    shape = (experts, out_w, in_w // 8)
    # 32 random bits per word = 8 uniform nibbles.
    words = torch.randint(-(2 ** 31), 2 ** 31, shape, generator=g, device=device, dtype=torch.int64)
    weight = words.to(torch.int32)
    scales = (torch.randn((experts, out_w, in_w // group), generator=g, device=device) * scale_std).abs()
    scales = scales.to(torch.bfloat16)
    biases = (scales.float() * -8.0).to(torch.bfloat16)
    return weight, scales, biases


def expert_bank(experts: int, hidden: int, inter: int, group: int = 32, *, seed: int = 0, device="cuda"):
    """{gate_proj, up_proj, down_proj} triples for ``experts`` routed experts."""
    return {
        "gate_proj": q4_projection(experts, inter, hidden, group, seed=seed * 3 + 1, device=device),
        "up_proj": q4_projection(experts, inter, hidden, group, seed=seed * 3 + 2, device=device),
        "down_proj": q4_projection(experts, hidden, inter, group, seed=seed * 3 + 3, device=device),
    }


def shared_expert(hidden: int, inter: int, group: int = 32, *, seed: int = 0, device="cuda"):
    bank = expert_bank(1, hidden, inter, group, seed=seed + 1000, device=device)
    return {k: tuple(t[0] for t in v) for k, v in bank.items()}


def bf16_normal(shape, std: float = 1.0, *, seed: int = 0, device="cuda"):
    torch = _torch()
    g = _gen(seed, device)
    return (torch.randn(shape, generator=g, device=device) * std).to(torch.bfloat16)


# Bias scale: with x ~ N(0,1) and router rows ~ N(0, 0.02) the per-token logit
# noise is ~N(0, 0.9^2); scaling log p_e by 0.43 makes the top-10 of 64
# tokens touch ~200 distinct experts, the count that sampling 10 experts
# per token without replacement from Zipf(1.1) gives (Gumbel top-k).
ZIPF_BIAS_SCALE = 0.43


def zipf_router(tokens: int, hidden: int, experts: int, s: float = 1.1, *, seed: int = 0,
                device="cuda", strength: float = 8.0, bias_scale: float = ZIPF_BIAS_SCALE):
    """(x [T,H] bf16, W [E,H] bf16) whose top-k popularity follows Zipf(s).

    x_t = n_t + strength * u and W_e = g_e + (bias_scale * log p_e / strength) * u
    for a random unit vector u and p_e proportional to rank_e^-s (ranks a
    random permutation), so logit_e(t) ~ N(0, 0.9^2) + bias_scale * log p_e.
    """
    torch = _torch()
    g = _gen(seed, device)
    u = torch.randn(hidden, generator=g, device=device)
    u = u / u.norm()
    ranks = torch.randperm(experts, generator=g, device=device).float() + 1.0
    p = ranks.pow(-s)
    p = p / p.sum()
    n = torch.randn((tokens, hidden), generator=g, device=device)
    x = (n + strength * u).to(torch.bfloat16)
    w = torch.randn((experts, hidden), generator=g, device=device) * 0.02
    w = (w + (bias_scale * p.log() / strength)[:, None] * u[None, :]).to(torch.bfloat16)
    return x, w


@dataclass
class MoELayerInputs:
    x: object
    router_weight: object
    experts: dict
    shared: dict
    shared_expert_gate: object
    hidden: int
    inter: int
    num_experts: int
    top_k: int
    group: int


def moe_layer(tokens: int, hidden: int = 2048, inter: int = 512, num_experts: int = 512,
              top_k: int = 10, group: int = 32, *, zipf: float | None = None, seed: int = 0,
              device="cuda") -> MoELayerInputs:
    """Inputs of one qwen4_exp MoE layer (benchmark configs 1, 2 and 4)."""
    if zipf is not None:
        x, w = zipf_router(tokens, hidden, num_experts, zipf, seed=seed + 7, device=device)
    else:
        x = bf16_normal((tokens, hidden), seed=seed + 7, device=device)
        w = bf16_normal((num_experts, hidden), 0.02, seed=seed + 8, device=device)
    experts = expert_bank(num_experts, hidden, inter, group, seed=seed, device=device)
    shared = shared_expert(hidden, inter, group, seed=seed, device=device)
    wg = bf16_normal((hidden,), 0.02, seed=seed + 9, device=device)
    return MoELayerInputs(x, w, experts, shared, wg, hidden, inter, num_experts, top_k, group)


@dataclass
class PagedInputs:
    q: object
    k_cache: object
    v_cache: object
    block_table: object
    context_lens: object
    scale: float
    page_size: int


def paged_decode_inputs(batch: int = 16, q_heads: int = 16, kv_heads: int = 2, head_dim: int = 256,
                        page_size: int = 64, ctx_range=(1024, 32768), *, seed: int = 0,
                        device="cuda") -> PagedInputs:
    """Benchmark config 5: GQA 16/2, D 256, page 64, ctx ~ U[1k, 32k]."""
    torch = _torch()
    g = _gen(seed, device)
    lo, hi = ctx_range
    ctx = torch.randint(lo, hi + 1, (batch,), generator=g, device=device, dtype=torch.int64)
    max_pages = int(math.ceil(hi / page_size))
    pages_needed = ((ctx + page_size - 1) // page_size)
    total = int(pages_needed.sum())
    perm = torch.randperm(total, generator=g, device=device).to(torch.int32)
    table = torch.full((batch, max_pages), -1, dtype=torch.int32, device=device)
    start = 0
    for b in range(batch):
        n = int(pages_needed[b])
        table[b, :n] = perm[start:start + n]
        start += n
    k = (torch.randn((total, page_size, kv_heads, head_dim), generator=g, device=device)).to(torch.bfloat16)
    v = (torch.randn((total, page_size, kv_heads, head_dim), generator=g, device=device)).to(torch.bfloat16)
    q = torch.randn((batch, q_heads, head_dim), generator=g, device=device).to(torch.bfloat16)
    return PagedInputs(q, k, v, table, ctx.to(torch.int32), head_dim ** -0.5, page_size)
