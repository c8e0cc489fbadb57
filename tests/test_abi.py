"""CPU: the C-ABI library builds for sm_100a, loads, exports every declared symbol and rejects
bad arguments before touching the GPU."""

import ctypes
import re
from pathlib import Path

import pytest

from kernel_optim_b200 import _lib
from kernel_optim_b200.build import build

HEADER = Path(__file__).resolve().parents[1] / "include" / "kopt.h"


@pytest.fixture(scope="module")
def lib():
    build()
    return _lib.lib()


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kopt_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert names, "no declarations parsed"
    for n in names:
        assert hasattr(lib, n), f"{n} declared in kopt.h but not exported"
    assert set(names) == set(_lib.EXPORTED)


def test_abi_version_and_strerror(lib):
    assert lib.kopt_abi_version() == 2
    assert lib.kopt_strerror(0) == b"ok"
    assert b"argument" in lib.kopt_strerror(_lib.KOPT_ERR_ARG)
    assert lib.kopt_strerror(999) == b"unknown kopt status"


def test_struct_layouts_match_header():
    # kopt_kv_cache: 2 pointers, 2 int64, 2 int32, pointer, 2 int32 -> 56 bytes on LP64
    assert ctypes.sizeof(_lib.KvCache) == 56
    assert ctypes.sizeof(_lib.Plan) == 56
    # kopt_gather: 8 + 8 pointers, pointer, 2 int32, 2 int64 -> 160 bytes
    assert ctypes.sizeof(_lib.Gather) == 160
    # kopt_gemv_plan: 10 int32, int64 -> 48 bytes
    assert ctypes.sizeof(_lib.GemvPlan) == 48
    # kopt_gemv_fuse: 2 pointers, int32, float, pointer -> 32 bytes
    assert ctypes.sizeof(_lib.GemvFuse) == 32


@pytest.mark.parametrize("args", [
    (0, 16, 1, 32, 8, 64, 4097, 0),     # head_dim 64 unsupported
    (0, 16, 1, 24, 8, 128, 4097, 0),    # group != 4
    (0, 0, 1, 32, 8, 128, 4097, 0),     # empty batch
    (0, 257, 1, 32, 8, 128, 4097, 0),   # batch above the plan limit
    (0, 16, 9, 32, 8, 128, 4097, 0),    # more than 8 query tokens per sequence
    (0, 16, 0, 32, 8, 128, 4097, 0),    # no query token
    (0, 16, 1, 32, 8, 128, 0, 0),       # no capacity
])
def test_plan_rejects_bad_shapes(lib, args):
    plan = _lib.Plan()
    assert lib.kopt_decode_attn_plan(*args, ctypes.byref(plan)) == _lib.KOPT_ERR_ARG


def test_launchers_reject_null_arguments(lib):
    plan = _lib.Plan()
    cache = _lib.KvCache()
    assert lib.kopt_decode_attn(None, None, None, None, None, None, 1.0, None) == _lib.KOPT_ERR_ARG
    assert lib.kopt_decode_attn(ctypes.byref(plan), None, ctypes.byref(cache), None, None, None,
                                1.0, None) == _lib.KOPT_ERR_ARG
    assert lib.kopt_decode_attn_fused(ctypes.byref(plan), None, None, None, None, None, 0,
                                      ctypes.byref(cache), None, None, None, None, 1.0, 1e-6,
                                      None) == _lib.KOPT_ERR_ARG
    assert lib.kopt_qk_norm_rope(None, None, None, None, None, 1, None, None, ctypes.byref(cache),
                                 1, 1, 32, 8, 128, 1e-6, None, 0, None) == _lib.KOPT_ERR_ARG
    assert lib.kopt_workspace_init(None, None, None) == _lib.KOPT_ERR_ARG
    err = ctypes.c_int(0)
    assert lib.kopt_read_error(None, None, ctypes.byref(err), None) == _lib.KOPT_ERR_ARG


@pytest.mark.parametrize("args", [
    (0, 0, 64, 64, 1, 0),       # no rows
    (0, 65, 64, 64, 1, 0),      # more rows than the kernel's 64
    (0, 8, 100, 64, 1, 0),      # N not a multiple of 16 (16-column output segments)
    (0, 8, 48, 64, 3, 0),       # SWIGLU N not a multiple of 64 (gate/up tile halves)
    (0, 8, 64, 60, 1, 0),       # K not a multiple of 8 (TMA row stride)
    (0, 8, 64, 64, 5, 0),       # unknown epilogue
    (0, 8, 64, 64, 1, -1),      # negative split
])
def test_gemv_plan_rejects_bad_shapes(lib, args):
    plan = _lib.GemvPlan()
    assert lib.kopt_gemv_plan_make(*args, ctypes.byref(plan)) == _lib.KOPT_ERR_ARG


def test_gemv_rejects_null_arguments(lib):
    plan = _lib.GemvPlan()
    assert lib.kopt_gemv(None, None, None, None, None, None) == _lib.KOPT_ERR_ARG
    assert lib.kopt_gemv(ctypes.byref(plan), None, None, None, None, None) == _lib.KOPT_ERR_ARG
    assert lib.kopt_gemv_fused(ctypes.byref(plan), None, None, None, None, None, None) == _lib.KOPT_ERR_ARG
    err = ctypes.c_int(0)
    assert lib.kopt_gemv_read_error(None, None, ctypes.byref(err), None) == _lib.KOPT_ERR_ARG


def _hand_plan(B=4, nkv=8, grid=148, max_len=2048, T=1):
    """A T = 1 plan filled by hand the way kopt_decode_attn_plan fills it (no GPU needed):
    max_units = grid + ceil(pages / 32) + B * nkv, and the workspace layout of decode_attn.cu
    (256-byte header, counters, (m, l) pairs and 4 x 128 fp32 partials per unit slot)."""
    plan = _lib.Plan()
    pages = B * nkv * ((max_len + 15) // 16)
    plan.B, plan.T, plan.nkv, plan.grid, plan.max_len = B, T, nkv, grid, max_len
    plan.max_units = grid + (pages + 31) // 32 + B * nkv
    plan.ctas_per_sm, plan.device, plan.static_pct = 1, 0, 100
    plan.ws_bytes = _ws_bytes(B, nkv, plan.max_units)
    return plan


def _ws_bytes(B, nkv, units, rows=4):
    a256 = lambda x: (x + 255) & ~255
    return 256 + a256(B * nkv * 4) + a256(units * rows * 8) + units * rows * 128 * 4


def _noalloc(lib, plan):
    cache = _lib.KvCache()
    return lib.kopt_decode_attn_fused_noalloc(ctypes.byref(plan), None, None, None, None, None, 1,
                                              ctypes.byref(cache), None, None, None, 1.0, 1e-6,
                                              None, None)


def test_noalloc_rejects_edited_plans_before_queuing_anything(lib):
    """The allocation-free entry point clears part of its built-in buffer before the launch; a
    plan whose fields disagree must be turned away before that (and before any CUDA call, which is
    why this runs without a GPU)."""
    plan = _hand_plan()
    plan.B = 64                      # batch edited, slots and workspace left as they were
    assert _noalloc(lib, plan) == _lib.KOPT_ERR_ARG
    plan = _hand_plan()
    plan.max_units *= 4              # more slots than ws_bytes pays for
    assert _noalloc(lib, plan) == _lib.KOPT_ERR_WORKSPACE
    plan = _hand_plan()
    plan.T = 2                       # the fused prologue appends one token per sequence
    assert _noalloc(lib, plan) == _lib.KOPT_ERR_ARG
    plan = _hand_plan()
    plan.grid = 4 * plan.grid        # more CTAs than the unit slots were sized for
    assert _noalloc(lib, plan) == _lib.KOPT_ERR_ARG
    big = _hand_plan(B=4, max_len=131072)   # consistent, but above the 8 MiB buffer
    assert big.ws_bytes > 8 << 20
    assert _noalloc(lib, big) == _lib.KOPT_ERR_SCRATCH


def test_workspace_launchers_reject_inconsistent_plans(lib):
    """The same consistency check guards the entry points that take a caller's workspace: an
    edited grid would index unit slots past the end of the workspace."""
    # Host addresses stand in for device buffers: the plan check must turn the call away before
    # anything reaches the device (only an inconsistent plan is ever passed with them, so nothing
    # is launched on a machine with a GPU either).
    buf = ctypes.create_string_buffer(1024)
    base = (ctypes.addressof(buf) + 255) & ~255
    cache = _lib.KvCache()
    cache.k = cache.v = base
    cache.cap = 16
    plan = _hand_plan()
    plan.grid = 4 * plan.grid
    assert lib.kopt_decode_attn(ctypes.byref(plan), base, ctypes.byref(cache), base, base,
                                base, 1.0, None) == _lib.KOPT_ERR_ARG
    plan = _hand_plan()
    plan.max_units -= 1              # one slot short of what the grid and the batch need
    assert lib.kopt_decode_attn(ctypes.byref(plan), base, ctypes.byref(cache), base, base,
                                base, 1.0, None) == _lib.KOPT_ERR_ARG
