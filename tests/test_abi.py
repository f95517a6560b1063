"""The C-ABI library loads, exports every declared symbol, and its structs
match the ctypes mirror (no GPU, no compute calls)."""
from __future__ import annotations

import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from flashnext_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "fnmoe.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"FNMOE_API\s+\w+\s+(fnmoe_\w+)\s*\(", text)))


def test_header_declares_the_bound_surface():
    assert set(declared_symbols()) == set(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in declared_symbols():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\b(fnmoe_\w+)\b", out))
    assert set(declared_symbols()) <= exported


def test_abi_version_and_error_channel():
    lib = _lib.load()
    assert lib.fnmoe_abi_version() == _lib.ABI_VERSION
    # argument validation runs before any device call
    need = ctypes.c_uint64(0)
    assert lib.fnmoe_moe_workspace_size(None, ctypes.byref(need)) == _lib.ERR_NULL
    assert "NULL" in _lib.last_error(lib)
    a = _lib.FnMoEArgs()
    a.abi_version = 999
    assert lib.fnmoe_moe_workspace_size(ctypes.byref(a), ctypes.byref(need)) == _lib.ERR_ABI
    assert "abi_version" in _lib.last_error(lib)


def _shapes_args(**kw):
    a = _lib.FnMoEArgs()
    a.abi_version = _lib.ABI_VERSION
    a.tokens, a.slots, a.hidden_size, a.inter_size, a.expert_count = 2, 3, 64, 32, 4
    a.group_size = 32
    dummy = 0x1000
    for f in ("x", "routes", "gate_weight", "gate_scales", "gate_biases", "up_weight", "up_scales",
              "up_biases", "down_weight", "down_scales", "down_biases", "scores", "output"):
        setattr(a, f, dummy)
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_workspace_size_and_validation_without_gpu():
    lib = _lib.load()
    need = ctypes.c_uint64(0)
    assert lib.fnmoe_moe_workspace_size(ctypes.byref(_shapes_args()), ctypes.byref(need)) == _lib.OK
    assert need.value > 0
    assert lib.fnmoe_moe_workspace_size(ctypes.byref(_shapes_args(group_size=16)), ctypes.byref(need)) == \
        _lib.ERR_UNSUPPORTED
    assert lib.fnmoe_moe_workspace_size(ctypes.byref(_shapes_args(hidden_size=48)), ctypes.byref(need)) == \
        _lib.ERR_SHAPE
    bad = _shapes_args(shared=0x2000)
    assert lib.fnmoe_moe_workspace_size(ctypes.byref(bad), ctypes.byref(need)) == _lib.ERR_VALUE
    assert "shared_gate" in _lib.last_error(lib)


def test_router_workspace_size_without_gpu():
    """The workspace router needs scratch from 64 tokens (H a multiple of 128
    up to 4096), none below; bad shapes are rejected before any device call."""
    lib = _lib.load()
    need = ctypes.c_uint64(123)
    assert lib.fnmoe_router_workspace_size(63, 2048, 512, 1, ctypes.byref(need)) == _lib.OK
    assert need.value == 0
    assert lib.fnmoe_router_workspace_size(64, 2048, 512, 1, ctypes.byref(need)) == _lib.OK
    # byte planes 3 x 64 x 2048 + 2 x 513 x 2048 at least, plus exponents
    assert need.value >= 3 * 64 * 2048 + 2 * 513 * 2048 + 4 * (64 + 513)
    assert lib.fnmoe_router_workspace_size(64, 2056, 512, 1, ctypes.byref(need)) == _lib.OK
    assert need.value == 0  # H not a multiple of 128: the GEMV path
    assert lib.fnmoe_router_workspace_size(64, 2050, 512, 1, ctypes.byref(need)) == _lib.ERR_SHAPE
    assert lib.fnmoe_router_workspace_size(64, 2048, 2048, 1, ctypes.byref(need)) == _lib.ERR_SHAPE
    # the workspace router refuses a missing or short workspace before any device call
    fake = [ctypes.c_void_p(256 * (i + 1)) for i in range(9)]
    args = (fake[0], fake[1], fake[2], 64, 2048, 512, 10, ctypes.c_float(1.0), *fake[3:9])
    assert lib.fnmoe_router_topk_shared_ws(*args, None, 0, None) == _lib.ERR_WORKSPACE
    assert lib.fnmoe_router_topk_shared_ws(*args, fake[0], 1024, None) == _lib.ERR_WORKSPACE
    assert "workspace" in _lib.last_error(lib)
    assert lib.fnmoe_router_topk_shared_ws(fake[0], None, fake[2], 64, 2048, 512, 10, ctypes.c_float(1.0),
                                           *fake[3:9], None, 0, None) == _lib.ERR_NULL


C_PROBE = r"""
#include <stdio.h>
#include <stddef.h>
#include "fnmoe.h"
int main(void) {
  printf("FnExpertTable %zu\n", sizeof(FnExpertTable));
  printf("FnMoEArgs %zu %zu %zu %zu %zu\n", sizeof(FnMoEArgs), offsetof(FnMoEArgs, tokens),
         offsetof(FnMoEArgs, table), offsetof(FnMoEArgs, stream_table), offsetof(FnMoEArgs, workspace));
  printf("FnMoELayerArgs %zu %zu %zu\n", sizeof(FnMoELayerArgs), offsetof(FnMoELayerArgs, table),
         offsetof(FnMoELayerArgs, workspace));
  printf("FnPagedArgs %zu %zu\n", sizeof(FnPagedArgs), offsetof(FnPagedArgs, q));
  printf("FnTiledExperts %zu %zu\n", sizeof(FnTiledExperts), offsetof(FnTiledExperts, records));
  printf("FnTileArgs %zu %zu %zu\n", sizeof(FnTileArgs), offsetof(FnTileArgs, gate_weight),
         offsetof(FnTileArgs, tiled));
  printf("LayerTiled %zu\n", offsetof(FnMoELayerArgs, tiled));
  printf("LayerKeep %zu %zu\n", offsetof(FnMoELayerArgs, keep_threshold), offsetof(FnMoELayerArgs, min_keep));
  printf("FnRowsArgs %zu %zu %zu\n", sizeof(FnRowsArgs), offsetof(FnRowsArgs, table_rows),
         offsetof(FnRowsArgs, weight));
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_struct_layout_matches_c_compiler(tmp_path):
    src = tmp_path / "probe.c"
    src.write_text(C_PROBE)
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    lines = dict(line.split(" ", 1) for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                                check=True).stdout.strip().splitlines())
    s = ctypes.sizeof
    assert int(lines["FnExpertTable"]) == s(_lib.FnExpertTable)
    got = [int(v) for v in lines["FnMoEArgs"].split()]
    assert got == [s(_lib.FnMoEArgs), _lib.FnMoEArgs.tokens.offset, _lib.FnMoEArgs.table.offset,
                   _lib.FnMoEArgs.stream_table.offset, _lib.FnMoEArgs.workspace.offset]
    got = [int(v) for v in lines["FnMoELayerArgs"].split()]
    assert got == [s(_lib.FnMoELayerArgs), _lib.FnMoELayerArgs.table.offset, _lib.FnMoELayerArgs.workspace.offset]
    got = [int(v) for v in lines["FnPagedArgs"].split()]
    assert got == [s(_lib.FnPagedArgs), _lib.FnPagedArgs.q.offset]
    got = [int(v) for v in lines["FnTiledExperts"].split()]
    assert got == [s(_lib.FnTiledExperts), _lib.FnTiledExperts.records.offset]
    got = [int(v) for v in lines["FnTileArgs"].split()]
    assert got == [s(_lib.FnTileArgs), _lib.FnTileArgs.gate_weight.offset, _lib.FnTileArgs.tiled.offset]
    assert int(lines["LayerTiled"]) == _lib.FnMoELayerArgs.tiled.offset
    got = [int(v) for v in lines["LayerKeep"].split()]
    assert got == [_lib.FnMoELayerArgs.keep_threshold.offset, _lib.FnMoELayerArgs.min_keep.offset]
    got = [int(v) for v in lines["FnRowsArgs"].split()]
    assert got == [s(_lib.FnRowsArgs), _lib.FnRowsArgs.table_rows.offset, _lib.FnRowsArgs.weight.offset]


def test_rows_dequantize_validates_before_any_device_call():
    """Argument checks of the row lookup run on the host: a bad bit width,
    group size, shape or alignment is an error code, never a launch."""
    lib = _lib.load()
    a = _lib.FnRowsArgs()
    a.abi_version = _lib.ABI_VERSION
    a.dims, a.bits, a.group_size = 256, 4, 32
    a.table_rows, a.first_shard_rows, a.count = 10, 10, 3
    a.weight, a.scales, a.biases, a.indices, a.out = 0x1000, 0x2000, 0x3000, 0x4000, 0x5000
    for field, value, code in (("bits", 3, _lib.ERR_UNSUPPORTED), ("group_size", 16, _lib.ERR_UNSUPPORTED),
                               ("dims", 48, _lib.ERR_SHAPE), ("first_shard_rows", 11, _lib.ERR_SHAPE),
                               ("out", 0x5008, _lib.ERR_VALUE), ("indices", None, _lib.ERR_NULL)):
        b = _lib.FnRowsArgs.from_buffer_copy(a)
        setattr(b, field, value)
        assert lib.fnmoe_rows_dequantize(ctypes.byref(b), None) == code, field
    b = _lib.FnRowsArgs.from_buffer_copy(a)
    b.count = 0
    assert lib.fnmoe_rows_dequantize(ctypes.byref(b), None) == _lib.OK  # nothing to do
    b.abi_version = 3
    assert lib.fnmoe_rows_dequantize(ctypes.byref(b), None) == _lib.ERR_ABI


def test_tiled_record_bytes_without_gpu():
    """Record sizes of the tiled tables: one 2560-byte chunk per (row group,
    128-byte block); gate/up groups hold 8 gate + 8 up rows, down groups 16 rows."""
    lib = _lib.load()
    gu, dn = ctypes.c_uint64(0), ctypes.c_uint64(0)
    assert lib.fnmoe_tiled_record_bytes(2048, 512, 32, ctypes.byref(gu), ctypes.byref(dn)) == _lib.OK
    assert gu.value == (512 // 8) * (1024 // 128) * 2560 == 2 * (512 * 1024 + 2 * 512 * 64 * 2)
    assert dn.value == (2048 // 16) * (256 // 128) * 2560 == 2048 * 256 + 2 * 2048 * 16 * 2
    # H3072 / I640: the down rows (320 bytes) end in a partial block
    assert lib.fnmoe_tiled_record_bytes(3072, 640, 32, ctypes.byref(gu), ctypes.byref(dn)) == _lib.OK
    assert gu.value == 80 * 12 * 2560 and dn.value == 192 * 3 * 2560
    assert lib.fnmoe_tiled_record_bytes(2048, 100, 32, ctypes.byref(gu), ctypes.byref(dn)) == _lib.ERR_SHAPE
