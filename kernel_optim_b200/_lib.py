"""ctypes binding of libkopt.so (the C ABI declared in include/kopt.h).

The library is built in-tree by kernel_optim_b200/build.py. There is no fallback: if the library is
missing or fails to load, every entry point raises KoptError.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libkopt.so"

KOPT_OK = 0
KOPT_ERR_ARG = 1
KOPT_ERR_CUDA = 2
KOPT_ERR_WORKSPACE = 3
KOPT_ERR_SCRATCH = 4

PLAN_OVERLAP_PREV = 1

DEV_ERR_PAGE = 1
DEV_ERR_LEN = 2
DEV_ERR_TIMEOUT = 4
DEV_ERR_ROPE = 8
DEV_ERR_PLAN = 16

#: every symbol include/kopt.h declares
EXPORTED = (
    "kopt_abi_version",
    "kopt_strerror",
    "kopt_decode_attn_plan",
    "kopt_workspace_init",
    "kopt_read_error",
    "kopt_decode_attn",
    "kopt_qk_norm_rope",
    "kopt_decode_attn_fused",
    "kopt_decode_attn_fused_noalloc",
    "kopt_prefill_attn",
    "kopt_decode_attn_fused_gather",
    "kopt_ipc_alloc",
    "kopt_ipc_free",
    "kopt_ipc_get_handle",
    "kopt_ipc_open",
    "kopt_ipc_close",
    "kopt_add_rms_norm",
    "kopt_silu_mul",
    "kopt_gemv_plan_make",
    "kopt_gemv",
    "kopt_gemv_fused",
    "kopt_row_sumsq",
    "kopt_gemv_read_error",
)

GEMV_F32, GEMV_BF16, GEMV_RESID, GEMV_SWIGLU, GEMV_ARGMAX = 0, 1, 2, 3, 4
GEMV_OVERLAP_PREV = 1

IPC_HANDLE_BYTES = 64
MAX_RANKS = 8


class KoptError(RuntimeError):
    """A kopt entry point returned a non-zero status, or the library is unavailable."""


class KvCache(ctypes.Structure):
    """Mirror of struct kopt_kv_cache."""

    _fields_ = [
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("stride_b", ctypes.c_int64),
        ("stride_h", ctypes.c_int64),
        ("cap", ctypes.c_int32),
        ("num_pages", ctypes.c_int32),
        ("block_table", ctypes.c_void_p),
        ("bt_stride", ctypes.c_int32),
        ("page_size", ctypes.c_int32),
    ]


class Plan(ctypes.Structure):
    """Mirror of struct kopt_plan."""

    _fields_ = [
        ("B", ctypes.c_int32),
        ("T", ctypes.c_int32),
        ("nkv", ctypes.c_int32),
        ("grid", ctypes.c_int32),
        ("ctas_per_sm", ctypes.c_int32),
        ("tile_tokens", ctypes.c_int32),
        ("max_units", ctypes.c_int32),
        ("device", ctypes.c_int32),
        ("max_len", ctypes.c_int32),
        ("chunk_tokens", ctypes.c_int32),
        ("static_pct", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("ws_bytes", ctypes.c_int64),
    ]


class Gather(ctypes.Structure):
    """Mirror of struct kopt_gather."""

    _fields_ = [
        ("out", ctypes.c_void_p * MAX_RANKS),
        ("flags", ctypes.c_void_p * MAX_RANKS),
        ("epoch", ctypes.c_void_p),
        ("rank", ctypes.c_int32),
        ("world", ctypes.c_int32),
        ("row_elems", ctypes.c_int64),
        ("wait_ns", ctypes.c_int64),
    ]


class GemvPlan(ctypes.Structure):
    """Mirror of struct kopt_gemv_plan."""

    _fields_ = [
        ("device", ctypes.c_int32),
        ("M", ctypes.c_int32),
        ("N", ctypes.c_int32),
        ("K", ctypes.c_int32),
        ("epi", ctypes.c_int32),
        ("units_per_cta", ctypes.c_int32),
        ("tiles", ctypes.c_int32),
        ("grid", ctypes.c_int32),
        ("ctas_per_sm", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("ws_bytes", ctypes.c_int64),
    ]


class GemvFuse(ctypes.Structure):
    """Mirror of struct kopt_gemv_fuse."""

    _fields_ = [
        ("norm_weight", ctypes.c_void_p),
        ("ss_in", ctypes.c_void_p),
        ("ss_tiles", ctypes.c_int32),
        ("eps", ctypes.c_float),
        ("ss_out", ctypes.c_void_p),
    ]


_lock = threading.Lock()
_lib = None

_vp, _i32, _i64, _f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
_SIGS = {
    "kopt_abi_version": (_i32, []),
    "kopt_strerror": (ctypes.c_char_p, [_i32]),
    "kopt_decode_attn_plan": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
                                     ctypes.POINTER(Plan)]),
    "kopt_workspace_init": (_i32, [ctypes.POINTER(Plan), _vp, _vp]),
    "kopt_read_error": (_i32, [ctypes.POINTER(Plan), _vp, ctypes.POINTER(ctypes.c_int), _vp]),
    "kopt_decode_attn": (_i32, [ctypes.POINTER(Plan), _vp, ctypes.POINTER(KvCache), _vp, _vp, _vp,
                                _f32, _vp]),
    "kopt_qk_norm_rope": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _vp, _vp, ctypes.POINTER(KvCache),
                                 _i32, _i32, _i32, _i32, _i32, _f32, _vp, _i32, _vp]),
    "kopt_decode_attn_fused": (_i32, [ctypes.POINTER(Plan), _vp, _vp, _vp, _vp, _vp, _i32,
                                      ctypes.POINTER(KvCache), _vp, _vp, _vp, _vp, _f32, _f32, _vp]),
    "kopt_prefill_attn": (_i32, [_vp, ctypes.POINTER(KvCache), _vp, _i32, _i32, _i32, _i32, _i32,
                                 ctypes.c_float, _vp, _i32, _vp]),
    "kopt_decode_attn_fused_noalloc": (_i32, [ctypes.POINTER(Plan), _vp, _vp, _vp, _vp, _vp, _i32,
                                              ctypes.POINTER(KvCache), _vp, _vp, _vp, _f32, _f32,
                                              _vp, _vp]),
    "kopt_decode_attn_fused_gather": (_i32, [ctypes.POINTER(Plan), _vp, _vp, _vp, _vp, _vp, _i32,
                                             ctypes.POINTER(KvCache), _vp, ctypes.POINTER(Gather),
                                             _vp, _vp, _f32, _f32, _vp]),
    "kopt_ipc_alloc": (_i32, [_i32, _i64, ctypes.POINTER(_vp)]),
    "kopt_ipc_free": (_i32, [_i32, _vp]),
    "kopt_ipc_get_handle": (_i32, [_vp, _vp]),
    "kopt_ipc_open": (_i32, [_i32, _vp, ctypes.POINTER(_vp)]),
    "kopt_ipc_close": (_i32, [_i32, _vp]),
    "kopt_add_rms_norm": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _f32, _vp]),
    "kopt_silu_mul": (_i32, [_vp, _vp, _i32, _i32, _vp]),
    "kopt_gemv_plan_make": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32, ctypes.POINTER(GemvPlan)]),
    "kopt_gemv": (_i32, [ctypes.POINTER(GemvPlan), _vp, _vp, _vp, _vp, _vp]),
    "kopt_gemv_fused": (_i32, [ctypes.POINTER(GemvPlan), _vp, _vp, _vp, _vp,
                               ctypes.POINTER(GemvFuse), _vp]),
    "kopt_row_sumsq": (_i32, [_vp, _i32, _i32, _vp, _vp]),
    "kopt_gemv_read_error": (_i32, [ctypes.POINTER(GemvPlan), _vp, ctypes.POINTER(ctypes.c_int),
                                    _vp]),
}


def lib() -> ctypes.CDLL:
    """Load libkopt.so once and declare every signature. Raises KoptError if it is unavailable."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise KoptError(
                    f"{LIB_PATH.name} is not built: run `python -m kernel_optim_b200.build` "
                    "(or __graft_entry__.build()); there is no CPU fallback")
            try:
                handle = ctypes.CDLL(str(LIB_PATH))
            except OSError as e:  # pragma: no cover - depends on the host
                raise KoptError(f"cannot load {LIB_PATH}: {e}") from e
            for name, (res, args) in _SIGS.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    if rc != KOPT_OK:
        msg = lib().kopt_strerror(rc).decode()
        raise KoptError(f"{what} failed: status {rc} ({msg})")


def dev_error_text(bits: int) -> str:
    names = []
    if bits & DEV_ERR_PAGE:
        names.append("block-table page id out of range")
    if bits & DEV_ERR_LEN:
        names.append("position outside the cache capacity (clamped)")
    if bits & DEV_ERR_TIMEOUT:
        names.append("a bounded wait timed out (a copy that did not land, or a peer that did "
                     "not raise its gather flag)")
    if bits & DEV_ERR_ROPE:
        names.append("position outside the RoPE table (clamped)")
    if bits & DEV_ERR_PLAN:
        names.append("internal work-split invariant violated")
    return ", ".join(names) or "none"
