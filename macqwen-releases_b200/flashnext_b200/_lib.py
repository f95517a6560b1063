"""ctypes binding of libfnmoe.so (the C ABI declared in include/fnmoe.h).

This is the reference-side binding style of ``models/flashnext/tests/bench/
metal_native.py:54-132`` (ctypes structure + argtypes + status codes + last
error string) pointed at the CUDA library.  The library is built in-tree by
``macqwen-releases_b200/build.py``; there is no fallback: if it cannot be
loaded or no sm_100 device is present, every op raises ``RuntimeError``.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libfnmoe.so"
ABI_VERSION = 4
STATIC_SCRATCH_BYTES = 16 << 20

OK = 0
ERR_NULL = -1
ERR_SHAPE = -2
ERR_UNSUPPORTED = -3
ERR_DEVICE = -4
ERR_WORKSPACE = -5
ERR_LAUNCH = -6
ERR_ABI = -7
ERR_VALUE = -8

DTYPE_BF16 = 0
DTYPE_F32 = 1

FLAG_RETURN_ALL = 0x1
FLAG_NO_COMBINE = 0x2
ROUTE_NONE = 0xFFFFFFFF  # an empty slot: skipped, its per-slot output left untouched

ERR_BAD_ROUTE = 0x1
ERR_NON_FINITE = 0x2

_vp = ctypes.c_void_p
_u32 = ctypes.c_uint32
_u64 = ctypes.c_uint64


class FnExpertTable(ctypes.Structure):
    _fields_ = [
        ("base", _vp),
        ("header_bytes", _u64),
        ("record_stride", _u64),
        ("part_offset", _u64 * 9),
        ("records", _u32),
        ("reserved", _u32),
    ]


class FnTiledExperts(ctypes.Structure):
    _fields_ = [
        ("gate_up", _vp), ("down", _vp),
        ("gate_up_record_bytes", _u64), ("down_record_bytes", _u64),
        ("records", _u32), ("has_shared", _u32),
    ]


class FnMoEArgs(ctypes.Structure):
    _fields_ = [
        ("abi_version", _u32), ("flags", _u32),
        ("x", _vp),
        ("gate_weight", _vp), ("gate_scales", _vp), ("gate_biases", _vp),
        ("up_weight", _vp), ("up_scales", _vp), ("up_biases", _vp),
        ("down_weight", _vp), ("down_scales", _vp), ("down_biases", _vp),
        ("routes", _vp), ("scores", _vp), ("output", _vp),
        ("tokens", _u32), ("slots", _u32), ("hidden_size", _u32),
        ("inter_size", _u32), ("expert_count", _u32),
        ("group_size", _u32), ("x_dtype", _u32), ("scores_dtype", _u32),
        ("reserved0", _u32),
        ("shared_y", _vp), ("shared", _vp), ("shared_gate", _vp),
        ("table", FnExpertTable),
        ("stream_table", FnExpertTable),
        ("gate_out", _vp), ("up_out", _vp), ("down_out", _vp),
        ("workspace", _vp), ("workspace_bytes", _u64),
        ("tiled", FnTiledExperts),
    ]


class FnMoELayerArgs(ctypes.Structure):
    _fields_ = [
        ("abi_version", _u32), ("top_k", _u32),
        ("x", _vp), ("router_weight", _vp),
        ("renorm_blend", ctypes.c_float),
        ("tokens", _u32), ("hidden_size", _u32), ("inter_size", _u32),
        ("expert_count", _u32), ("group_size", _u32), ("shared_inter_size", _u32),
        ("gate_weight", _vp), ("gate_scales", _vp), ("gate_biases", _vp),
        ("up_weight", _vp), ("up_scales", _vp), ("up_biases", _vp),
        ("down_weight", _vp), ("down_scales", _vp), ("down_biases", _vp),
        ("shared_gate_weight", _vp), ("shared_gate_scales", _vp), ("shared_gate_biases", _vp),
        ("shared_up_weight", _vp), ("shared_up_scales", _vp), ("shared_up_biases", _vp),
        ("shared_down_weight", _vp), ("shared_down_scales", _vp), ("shared_down_biases", _vp),
        ("shared_expert_gate", _vp),
        ("table", FnExpertTable),
        ("table_routes_of_expert", _vp),
        ("output", _vp), ("logits_out", _vp), ("inds_out", _vp), ("scores_out", _vp),
        ("workspace", _vp), ("workspace_bytes", _u64),
        ("tiled", FnTiledExperts),
        ("flags", _u32), ("reserved1", _u32),
        ("keep_threshold", ctypes.c_double), ("min_keep", _u32), ("reserved2", _u32),
    ]


LAYER_FORCE_PREFILL = 0x1
LAYER_FORCE_DECODE = 0x2
PREFILL_PAIRS = 4096


class FnTileArgs(ctypes.Structure):
    _fields_ = [
        ("abi_version", _u32), ("experts", _u32), ("hidden_size", _u32), ("inter_size", _u32),
        ("group_size", _u32), ("first_record", _u32),
        ("gate_weight", _vp), ("gate_scales", _vp), ("gate_biases", _vp),
        ("up_weight", _vp), ("up_scales", _vp), ("up_biases", _vp),
        ("down_weight", _vp), ("down_scales", _vp), ("down_biases", _vp),
        ("tiled", FnTiledExperts),
    ]


class FnPagedArgs(ctypes.Structure):
    _fields_ = [
        ("abi_version", _u32), ("batch", _u32), ("q_heads", _u32), ("kv_heads", _u32),
        ("head_dim", _u32), ("page_size", _u32), ("max_pages", _u32), ("num_pages", _u32),
        ("scale", ctypes.c_float), ("split_tokens", _u32),
        ("q", _vp), ("k_cache", _vp), ("v_cache", _vp),
        ("block_table", _vp), ("context_lens", _vp), ("out", _vp),
        ("workspace", _vp), ("workspace_bytes", _u64),
    ]


class FnRowsArgs(ctypes.Structure):
    _fields_ = [
        ("abi_version", _u32), ("dims", _u32), ("bits", _u32), ("group_size", _u32),
        ("table_rows", _u64), ("first_shard_rows", _u64), ("count", _u64),
        ("weight", _vp), ("scales", _vp), ("biases", _vp), ("indices", _vp), ("out", _vp),
    ]


EP_IPC_BYTES = 64


class FnEpConfig(ctypes.Structure):
    _fields_ = [
        ("abi_version", _u32), ("world", _u32), ("rank", _u32), ("capacity_tokens", _u32),
        ("hidden_size", _u32), ("top_k", _u32), ("experts_per_rank", _u32), ("reserved", _u32),
    ]


class FnEpWindow(ctypes.Structure):
    _fields_ = [
        ("rows", _vp), ("ids", _vp), ("slot_outputs", _vp),
        ("row_count", _u32), ("slots", _u32), ("bytes", _u64),
    ]


# Every exported symbol of include/fnmoe.h with its ctypes signature.
SIGNATURES = {
    "fnmoe_available": ([], ctypes.c_int),
    "fnmoe_get_last_error": ([ctypes.c_char_p, _u32], ctypes.c_int),
    "fnmoe_abi_version": ([], _u32),
    "fnmoe_moe_workspace_size": ([ctypes.POINTER(FnMoEArgs), ctypes.POINTER(_u64)], ctypes.c_int),
    "fnmoe_moe_execute": ([ctypes.POINTER(FnMoEArgs), _vp], ctypes.c_int),
    "fnmoe_moe_execute_static": ([ctypes.POINTER(FnMoEArgs), _vp], ctypes.c_int),
    "fnmoe_weighted_combine": ([_vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _vp], ctypes.c_int),
    "fnmoe_router_topk": ([_vp, _vp, _u32, _u32, _u32, _u32, ctypes.c_float, _vp, _vp, _vp, _vp, _vp],
                          ctypes.c_int),
    "fnmoe_router_topk_shared": ([_vp, _vp, _vp, _u32, _u32, _u32, _u32, ctypes.c_float, _vp, _vp, _vp, _vp, _vp,
                                  _vp, _vp], ctypes.c_int),
    "fnmoe_router_workspace_size": ([_u32, _u32, _u32, _u32, ctypes.POINTER(_u64)], ctypes.c_int),
    "fnmoe_router_topk_shared_ws": ([_vp, _vp, _vp, _u32, _u32, _u32, _u32, ctypes.c_float, _vp, _vp, _vp, _vp,
                                     _vp, _vp, _vp, _u64, _vp], ctypes.c_int),
    "fnmoe_combine": ([_vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _vp, _vp, _vp, _vp, _vp], ctypes.c_int),
    "fnmoe_softmax_topk": ([_vp, _u32, _u32, _u32, ctypes.c_float, _vp, _vp, _vp, _vp, _vp], ctypes.c_int),
    "fnmoe_group_tokens": ([_vp, _u32, _u32, _u32, _vp, _vp, _vp, _vp, _u64, _vp], ctypes.c_int),
    "fnmoe_moe_layer_workspace_size": ([ctypes.POINTER(FnMoELayerArgs), ctypes.POINTER(_u64)], ctypes.c_int),
    "fnmoe_moe_layer": ([ctypes.POINTER(FnMoELayerArgs), _vp], ctypes.c_int),
    "fnmoe_tiled_record_bytes": ([_u32, _u32, _u32, ctypes.POINTER(_u64), ctypes.POINTER(_u64)], ctypes.c_int),
    "fnmoe_tile_experts": ([ctypes.POINTER(FnTileArgs), _vp], ctypes.c_int),
    "fnmoe_dequantize": ([_vp, _vp, _vp, _vp, _u64, _u32, _u32, _vp], ctypes.c_int),
    "fnmoe_swiglu": ([_vp, _vp, _vp, _u64, _vp], ctypes.c_int),
    "fnmoe_paged_decode_workspace_size": ([ctypes.POINTER(FnPagedArgs), ctypes.POINTER(_u64)], ctypes.c_int),
    "fnmoe_paged_decode": ([ctypes.POINTER(FnPagedArgs), _vp], ctypes.c_int),
    "fnmoe_rows_dequantize": ([ctypes.POINTER(FnRowsArgs), _vp], ctypes.c_int),
    "fnmoe_read_device_errors": ([ctypes.POINTER(_u32), ctypes.c_int], ctypes.c_int),
    "fnmoe_profile_enable": ([ctypes.c_int], ctypes.c_int),
    "fnmoe_ep_create": ([ctypes.POINTER(FnEpConfig), ctypes.POINTER(_vp)], ctypes.c_int),
    "fnmoe_ep_ipc_handle": ([_vp, _vp], ctypes.c_int),
    "fnmoe_ep_open_peers": ([_vp, _vp], ctypes.c_int),
    "fnmoe_ep_window": ([_vp, ctypes.POINTER(FnEpWindow)], ctypes.c_int),
    "fnmoe_ep_dispatch": ([_vp, _vp, _vp, _u32, _vp], ctypes.c_int),
    "fnmoe_ep_return_combine": ([_vp, _vp, _vp, _u32, _vp, _vp], ctypes.c_int),
    "fnmoe_ep_destroy": ([_vp], ctypes.c_int),
    "fnmoe_profile_read": ([ctypes.c_char_p, _u32, ctypes.c_int], ctypes.c_int),
}

_lock = threading.Lock()
_handle: ctypes.CDLL | None = None


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Load the library once and attach signatures (no device work)."""
    global _handle
    with _lock:
        if _handle is not None and path is None:
            return _handle
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"libfnmoe.so not found at {p}; build it with "
                "`python macqwen-releases_b200/build.py` (no CPU fallback exists)"
            )
        lib = ctypes.CDLL(str(p))
        for name, (argtypes, restype) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = restype
        if lib.fnmoe_abi_version() != ABI_VERSION:
            raise RuntimeError("libfnmoe ABI version mismatch")
        if path is None:
            _handle = lib
        return lib


def last_error(lib: ctypes.CDLL | None = None) -> str:
    lib = lib or load()
    buf = ctypes.create_string_buffer(1024)
    lib.fnmoe_get_last_error(buf, len(buf))
    return buf.value.decode("utf-8", errors="replace")


def check(code: int, what: str) -> None:
    """Map a status code to the reference's exception types (metal_runtime.py)."""
    if code == OK:
        return
    msg = last_error()
    if code in (ERR_SHAPE, ERR_VALUE):
        raise ValueError(msg)
    if code == ERR_UNSUPPORTED:
        raise ValueError(msg)
    if code == ERR_NULL:
        raise TypeError(msg)
    raise RuntimeError(f"{what} failed ({code}): {msg}")


_available: dict[int, bool] = {}


def ensure_device() -> ctypes.CDLL:
    """Library handle after confirming an sm_100 device is usable.

    The first call on a device builds the library's constant tables and
    synchronises, so it must precede any CUDA graph capture.
    """
    import torch

    lib = load()
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA device unavailable: the B200 path has no CPU fallback")
    dev = torch.cuda.current_device()
    if not _available.get(dev):
        if lib.fnmoe_available() != 1:
            raise RuntimeError(f"libfnmoe unavailable: {last_error(lib)}")
        _available[dev] = True
    return lib


def read_device_errors(clear: bool = True) -> int:
    lib = ensure_device()
    flags = _u32(0)
    check(lib.fnmoe_read_device_errors(ctypes.byref(flags), 1 if clear else 0), "read_device_errors")
    return int(flags.value)


def profile_enable(on: bool = True) -> None:
    """Bracket every library kernel with CUDA events (benchmarks only)."""
    load().fnmoe_profile_enable(1 if on else 0)


def profile_read(reset: bool = True) -> dict[str, tuple[int, float]]:
    """{kernel: (launches, total device ms)} recorded since the last reset."""
    lib = load()
    buf = ctypes.create_string_buffer(1 << 16)
    check(lib.fnmoe_profile_read(buf, len(buf), 1 if reset else 0), "profile_read")
    out = {}
    for line in buf.value.decode().splitlines():
        name, count, ms = line.split()
        out[name] = (int(count), float(ms))
    return out
