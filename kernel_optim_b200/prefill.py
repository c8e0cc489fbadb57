"""Causal GQA attention over a prompt (the prefill) on the tcgen05 kernel (kopt_prefill_attn).

Replaces the reference's prefill attention, ``F.scaled_dot_product_attention(q, k, v,
is_causal=True)`` with GQA (GodRishUniverse/kernel_optim engine/engine.py:376-377). The prompt's
K/V are read from the cache, where the prologue (``kopt_qk_norm_rope`` with pos = 0 and T = S)
writes them, so they are never materialised in a separate [B, nkv, S, d] tensor.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import KoptError, check
from .fused import _DevErr, _ptr, _require_cuda, _stream, contiguous_cache


def prefill_attention(q: torch.Tensor, cache, layer: int, out: torch.Tensor, B: int, S: int,
                      nq: int, nkv: int, d: int = 128, scale: float | None = None) -> None:
    """out[b*S + s, h] = causal softmax attention of q[b*S + s, h] over keys 0 .. s of kv head h/4.

    q, out: [B*S, nq*d] bf16 contiguous; cache: a PagedKVCache (layer ``layer``) or a (k, v) pair
    of one-layer contiguous views [B, nkv, cap, d] holding the prompt at positions 0 .. S-1.
    Device error bits go to the prologue's error word (``fused.qk_norm_rope_error``)."""
    _require_cuda(q, "q")
    _require_cuda(out, "out")
    if q.shape != (B * S, nq * d) or out.shape != q.shape or not q.is_contiguous() or not out.is_contiguous():
        raise KoptError("q and out must be contiguous [B*S, nq*d]")
    desc = contiguous_cache(*cache) if isinstance(cache, tuple) else cache.descriptor(layer)
    dev = q.device
    err = _DevErr.get(dev)
    sc = d ** -0.5 if scale is None else scale
    check(_lib.lib().kopt_prefill_attn(_ptr(q), ctypes.byref(desc), _ptr(out), B, S, nq, nkv, d,
                                       ctypes.c_float(sc), _ptr(err), dev.index, _stream(dev)),
          "kopt_prefill_attn")
