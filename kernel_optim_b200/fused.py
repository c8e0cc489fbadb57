"""Drop-in attention step for the Qwen3-4B engine, backed by the sm_100a library.

Same names, arguments and semantics as the reference's kernel wrappers in
GodRishUniverse/kernel_optim engine/kernels/fused.py:

* ``DecodeAttention(B, T, cap, nq, nkv, d, device, target_ctas=...)`` (fused.py:204-219) owns the
  split scratch, allocated once, so ``__call__`` allocates nothing and is CUDA-graph capturable.
* ``DecodeAttention.__call__(q, k_cache, v_cache, pos, out)`` (fused.py:221-234): q/out
  ``[B*T, nq*d]`` bf16 contiguous; k/v one layer ``[B, nkv, cap, d]`` with any batch/head strides
  and token stride d; pos ``[B]`` int32 on the device, the new K/V already written at pos[b].
* ``qk_norm_rope(qkv, q_w, k_w, cos, sin, pos, q_out, k_cache, v_cache, T, eps, nq, nkv, d)``
  (fused.py:99-106): per-head RMSNorm + RoPE, K/V appended to the cache.

Launches go to the current torch stream of the tensors' device. No Triton, no CPU path: when the
library is not built, construction raises KoptError.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import KoptError, KvCache, Plan, check

BF16 = torch.bfloat16


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _require_cuda(t: torch.Tensor, name: str, dtype=BF16) -> None:
    if not t.is_cuda:
        raise KoptError(f"{name} must be a CUDA tensor (this library has no CPU path)")
    if t.dtype != dtype:
        raise KoptError(f"{name} must be {dtype}, got {t.dtype}")


def contiguous_cache(k_cache: torch.Tensor, v_cache: torch.Tensor) -> KvCache:
    """Descriptor of one layer's contiguous cache [B, nkv, cap, d] (token stride d)."""
    _require_cuda(k_cache, "k_cache")
    _require_cuda(v_cache, "v_cache")
    if k_cache.dim() != 4 or k_cache.shape != v_cache.shape or k_cache.stride() != v_cache.stride():
        raise KoptError("k_cache/v_cache must be matching [B, nkv, cap, d] views")
    d = k_cache.shape[3]
    if k_cache.stride(3) != 1 or k_cache.stride(2) != d:
        raise KoptError("cache token stride must be d and element stride 1")
    c = KvCache()
    c.k, c.v = k_cache.data_ptr(), v_cache.data_ptr()
    c.stride_b, c.stride_h = k_cache.stride(0), k_cache.stride(1)
    c.cap = k_cache.shape[2]
    c.num_pages, c.block_table, c.bt_stride, c.page_size = 0, None, 0, 16
    return c


class DecodeAttention:
    """Preallocated split-K attention for T query tokens per sequence, fixed (B, T, cap).

    Mirrors engine/kernels/fused.py:204-234. The split of each sequence's keys is decided on the
    device from the live position at every call (splits never cover unused capacity), and the
    cross-split merge happens inside the same launch.
    """

    def __init__(self, B, T, cap, nq, nkv, d, device, target_ctas=None):
        self.B, self.T, self.cap, self.nq, self.nkv, self.d = B, T, cap, nq, nkv, d
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise KoptError("DecodeAttention needs a CUDA device (no CPU path)")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.plan = Plan()
        check(_lib.lib().kopt_decode_attn_plan(self.device.index, B, T, nq, nkv, d, cap,
                                               int(target_ctas or 0), ctypes.byref(self.plan)),
              "kopt_decode_attn_plan")
        self.ws = torch.empty(self.plan.ws_bytes, dtype=torch.uint8, device=self.device)
        check(_lib.lib().kopt_workspace_init(ctypes.byref(self.plan), _ptr(self.ws),
                                             _stream(self.device)), "kopt_workspace_init")
        self.scale = d ** -0.5

    def __call__(self, q, k_cache, v_cache, pos, out):
        """q: [B*T, NQ*D]; k/v_cache: [B, NKV, cap, D]; pos: [B] int32; out: [B*T, NQ*D]."""
        _require_cuda(q, "q")
        _require_cuda(out, "out")
        _require_cuda(pos, "pos", torch.int32)
        rows = self.B * self.T
        if q.shape != (rows, self.nq * self.d) or out.shape != q.shape:
            raise KoptError(f"q/out must be [{rows}, {self.nq * self.d}]")
        if not (q.is_contiguous() and out.is_contiguous() and pos.is_contiguous()):
            raise KoptError("q, out and pos must be contiguous")
        if k_cache.shape[0] != self.B or k_cache.shape[1] != self.nkv or k_cache.shape[3] != self.d:
            raise KoptError("k_cache must be [B, nkv, cap, d] for this plan")
        cache = contiguous_cache(k_cache, v_cache)
        check(_lib.lib().kopt_decode_attn(ctypes.byref(self.plan), _ptr(q), ctypes.byref(cache),
                                          _ptr(pos), _ptr(out), _ptr(self.ws),
                                          ctypes.c_float(self.scale), _stream(q.device)),
              "kopt_decode_attn")

    def read_error(self) -> int:
        """Device error bits since the last read (synchronises the current stream)."""
        err = ctypes.c_int(0)
        check(_lib.lib().kopt_read_error(ctypes.byref(self.plan), _ptr(self.ws), ctypes.byref(err),
                                         _stream(self.device)), "kopt_read_error")
        return err.value


class _DevErr:
    """Per-device int32 error word for the standalone prologue kernel."""

    _words: dict[int, torch.Tensor] = {}

    @classmethod
    def get(cls, device: torch.device) -> torch.Tensor:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        w = cls._words.get(idx)
        if w is None:
            # a normal tensor even when first asked for under torch.inference_mode (the engine's
            # generate), so that callers outside it can still clear it in place
            with torch.inference_mode(False):
                w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
            cls._words[idx] = w
        return w


def qk_norm_rope_error(device) -> int:
    """Read and clear the prologue's device error bits (synchronises)."""
    w = _DevErr.get(torch.device(device))
    v = int(w.item())
    w.zero_()
    return v


def qk_norm_rope(qkv, q_w, k_w, cos, sin, pos, q_out, k_cache, v_cache, T, eps, nq, nkv, d):
    """Per-head q/k RMSNorm + RoPE; q to q_out, K/V appended at pos[b] + m % T.

    Mirrors engine/kernels/fused.py:99-106 (k_cache/v_cache: one layer, [B, NKV, cap, D]).
    """
    for t, n in ((qkv, "qkv"), (q_w, "q_w"), (k_w, "k_w"), (cos, "cos"), (sin, "sin"),
                 (q_out, "q_out")):
        _require_cuda(t, n)
        if not t.is_contiguous():
            raise KoptError(f"{n} must be contiguous")
    _require_cuda(pos, "pos", torch.int32)
    M = qkv.shape[0]
    if M % T or qkv.shape[1] != (nq + 2 * nkv) * d or q_out.shape != (M, nq * d):
        raise KoptError("qkv must be [B*T, (nq + 2 nkv) d] and q_out [B*T, nq d]")
    if cos.shape != sin.shape or cos.shape[1] != d:
        raise KoptError("cos/sin must be [n, d]")
    cache = contiguous_cache(k_cache, v_cache)
    dev = qkv.device
    err = _DevErr.get(dev)
    check(_lib.lib().kopt_qk_norm_rope(_ptr(qkv), _ptr(q_w), _ptr(k_w), _ptr(cos), _ptr(sin),
                                       cos.shape[0], _ptr(pos), _ptr(q_out), ctypes.byref(cache),
                                       M // T, T, nq, nkv, d, ctypes.c_float(eps), _ptr(err),
                                       dev.index, _stream(dev)), "kopt_qk_norm_rope")


def add_rms_norm(res, delta, weight, out, eps):
    """out = rmsnorm(res + delta) * weight; res <- res + delta (rounded to bf16) when delta is
    given. Rows contiguous [M, N] bf16. Mirrors engine/kernels/fused.py:39-46."""
    _require_cuda(res, "res")
    _require_cuda(weight, "weight")
    _require_cuda(out, "out")
    if delta is not None:
        _require_cuda(delta, "delta")
    M, N = res.shape
    if out.shape != res.shape or weight.shape != (N,) or (delta is not None and delta.shape != res.shape):
        raise KoptError("add_rms_norm: res/delta/out must be [M, N] and weight [N]")
    for t in (res, weight, out) + ((delta,) if delta is not None else ()):
        if not t.is_contiguous():
            raise KoptError("add_rms_norm: tensors must be contiguous")
    check(_lib.lib().kopt_add_rms_norm(_ptr(res), _ptr(delta), _ptr(weight), _ptr(out), M, N,
                                       ctypes.c_float(eps), _stream(res.device)), "kopt_add_rms_norm")


def silu_mul(gu, out):
    """out = bf16(bf16(silu(gate)) * up) with gate = gu[:, :I], up = gu[:, I:]; gu [M, 2I], out
    [M, I] bf16. Mirrors engine/kernels/fused.py:123-127."""
    _require_cuda(gu, "gu")
    _require_cuda(out, "out")
    M, two_i = gu.shape
    if two_i % 2 or out.shape != (M, two_i // 2) or not gu.is_contiguous() or not out.is_contiguous():
        raise KoptError("silu_mul: gu must be [M, 2I] and out [M, I], contiguous")
    check(_lib.lib().kopt_silu_mul(_ptr(gu), _ptr(out), M, two_i // 2, _stream(gu.device)),
          "kopt_silu_mul")
