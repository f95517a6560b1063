"""Host-side behaviour of the executor API (metal_runtime.py contract), no GPU.

Mirrors the checkpoint-free tests of the reference
(``models/flashnext/tests/unit/test_metal_runtime.py:18-218``).
"""
from __future__ import annotations

import os
from types import SimpleNamespace

import numpy as np
import pytest

from flashnext_b200 import MetalMoEExecutor, MoEExecutor, probe_capabilities


@pytest.mark.parametrize("kwargs", [
    {"expert_count": 0, "hidden_size": 2, "top_k": 1},
    {"expert_count": 2, "hidden_size": 0, "top_k": 1},
    {"expert_count": 2, "hidden_size": 2, "top_k": 0},
    {"expert_count": 513, "hidden_size": 2, "top_k": 1},
    {"expert_count": 2, "hidden_size": 2, "top_k": 11},
])
def test_constructor_rejects_invalid_dimensions(kwargs):
    with pytest.raises(ValueError):
        MoEExecutor(**kwargs)


def test_constructor_rejects_top_k_larger_than_expert_count():
    with pytest.raises(ValueError):
        MoEExecutor(expert_count=2, hidden_size=2, top_k=3)


def test_constructor_rejects_group_and_token_bounds():
    with pytest.raises(ValueError):
        MoEExecutor(2, 32, 1, group_size=16)
    with pytest.raises(ValueError):
        MoEExecutor(2, 32, 1, max_tokens=9)
    with pytest.raises(ValueError):
        MoEExecutor(2, 32, 1, max_width=16385)


def test_alias_keeps_the_reference_name():
    assert MetalMoEExecutor is MoEExecutor


def test_up_swiglu_flag_defaults_off_and_reads_environment():
    old = os.environ.pop("FLASHNEXT_FUSED_UP_SWIGLU", None)
    try:
        assert not MoEExecutor(2, 32, 1).fused_up_swiglu
        assert MoEExecutor(2, 32, 1, fused_up_swiglu=True).fused_up_swiglu
        os.environ["FLASHNEXT_FUSED_UP_SWIGLU"] = "1"
        assert MoEExecutor(2, 32, 1).fused_up_swiglu
    finally:
        if old is None:
            os.environ.pop("FLASHNEXT_FUSED_UP_SWIGLU", None)
        else:
            os.environ["FLASHNEXT_FUSED_UP_SWIGLU"] = old


def test_capabilities_of_injected_backends():
    caps = probe_capabilities(SimpleNamespace(available=False, supports_custom_moe=False))
    assert not caps.available and not caps.supports_custom_moe
    caps = probe_capabilities(SimpleNamespace(available=True, supports_custom_moe=True))
    assert caps.available and caps.supports_custom_moe and caps["custom_metal"]
    ref = probe_capabilities("reference")
    assert not ref.available and ref.backend == "reference"
    assert not probe_capabilities("vulkan").available


def test_unsupported_backend_fails_before_execution():
    ex = MoEExecutor(2, 2, 1, backend=SimpleNamespace(available=True, supports_custom_moe=False))
    with pytest.raises(RuntimeError, match="custom MoE"):
        ex.execute(np.zeros((1, 2), np.float32), np.zeros((1, 1), np.int32), np.ones((1, 1), np.float32))


def _packs(experts=2, hidden=32, inter=4, bad_gate=False):
    def p(o, k, words=None):
        return (np.zeros((experts, o, words if words is not None else k // 8), np.uint32),
                np.zeros((experts, o, k // 32), np.float32), np.zeros((experts, o, k // 32), np.float32))
    return {"gate_proj": p(inter, hidden, 3 if bad_gate else None), "up_proj": p(inter, hidden),
            "down_proj": p(hidden, inter if inter >= 32 else 32)}


def test_execute_rejects_a_malformed_q4_projection_pack():
    ex = MoEExecutor(2, 32, 1, backend="reference")
    with pytest.raises(ValueError, match="weight shape"):
        ex.execute(np.zeros((1, 32), np.float32), np.zeros((1, 1), np.int32), _packs(bad_gate=True))


def test_execute_rejects_a_route_with_another_token_count():
    ex = MoEExecutor(2, 32, 1, backend="reference")
    with pytest.raises(ValueError, match="same token count"):
        ex.execute(np.zeros((2, 32), np.float32), np.zeros((1, 1), np.int32), {})


def test_execute_rejects_bad_shared_arguments():
    ex = MoEExecutor(2, 32, 1, backend="reference")
    x, r = np.zeros((1, 32), np.float32), np.zeros((1, 1), np.int32)
    with pytest.raises(ValueError, match="together"):
        ex.execute(x, r, _packs(), shared=np.zeros((1, 32), np.float32))
    with pytest.raises(ValueError, match="not both"):
        ex.execute(x, r, _packs(), shared_y=np.zeros((1, 32)), shared=np.zeros((1, 32)),
                   shared_gate=np.zeros((1, 1)))
    with pytest.raises(ValueError, match="stream pack"):
        ex.execute(x, r, _packs(), stream_pack=np.zeros(16, np.uint8))


def test_execute_without_a_device_raises_instead_of_falling_back():
    ex = MoEExecutor(2, 32, 1, backend="reference")
    packs = {"gate_proj": (np.zeros((2, 32, 4), np.uint32), np.zeros((2, 32, 1), np.float32), np.zeros((2, 32, 1), np.float32)),
             "up_proj": (np.zeros((2, 32, 4), np.uint32), np.zeros((2, 32, 1), np.float32), np.zeros((2, 32, 1), np.float32)),
             "down_proj": (np.zeros((2, 32, 4), np.uint32), np.zeros((2, 32, 1), np.float32), np.zeros((2, 32, 1), np.float32))}
    with pytest.raises(RuntimeError, match="unavailable"):
        ex.execute(np.zeros((1, 32), np.float32), np.zeros((1, 1), np.int32), packs)
