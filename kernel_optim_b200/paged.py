"""Paged KV cache and the fused paged decode-attention step.

The reference keeps a contiguous cache ``[L, B, NKV, cap, D]`` sized to the longest run
(engine/engine.py:184-187). Here each layer owns a page pool ``[num_pages, NKV, 16, D]`` bf16: one
16-token page of one kv head is 4 KiB contiguous, which is exactly one ``cp.async.bulk`` copy in the
kernel. A block table ``[B, max_pages]`` int32 maps sequence b's page j (tokens 16j..16j+15) to a
pool page; pages of one sequence need not be contiguous or ordered.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import KoptError, KvCache, Plan, check
from .fused import _DevErr, _ptr, _require_cuda, _stream, contiguous_cache

PAGE = 16


class PagedKVCache:
    """Page pools for all layers plus one block table shared by the layers.

    ``k[i]`` / ``v[i]`` are layer i's pools ``[num_pages, nkv, 16, d]``. ``block_table`` is
    ``[B, max_pages]`` int32 on the device.
    """

    def __init__(self, n_layers, num_pages, nkv, d, B, max_len, device, dtype=torch.bfloat16):
        self.n_layers, self.num_pages, self.nkv, self.d = n_layers, num_pages, nkv, d
        self.B, self.max_len = B, max_len
        self.max_pages = (max_len + PAGE - 1) // PAGE
        self.device = torch.device(device)
        self.k = torch.zeros(n_layers, num_pages, nkv, PAGE, d, dtype=dtype, device=self.device)
        self.v = torch.zeros_like(self.k)
        self.block_table = torch.full((B, self.max_pages), -1, dtype=torch.int32, device=self.device)

    @property
    def capacity(self) -> int:
        """Keys per sequence the block table can address (max_pages * 16)."""
        return self.max_pages * PAGE

    # ------------------------------------------------------------------ page assignment
    def assign_pages(self, table: torch.Tensor) -> None:
        """Install a block table [B, max_pages] (entries in [0, num_pages), or -1 if unused)."""
        if table.shape != (self.B, self.max_pages):
            raise KoptError(f"block table must be [{self.B}, {self.max_pages}]")
        t = table.to(torch.int32)
        used = t[t >= 0]
        if used.numel() and (int(used.max()) >= self.num_pages):
            raise KoptError("block table references a page outside the pool")
        if used.numel() != torch.unique(used).numel():
            raise KoptError("block table maps two slots to the same page")
        self.block_table.copy_(t)

    def assign_sequential(self, lengths) -> None:
        """Give each sequence ceil(len/16) fresh pages, in order."""
        table = torch.full((self.B, self.max_pages), -1, dtype=torch.int32)
        nxt = 0
        for b, L in enumerate(lengths):
            n = (int(L) + PAGE - 1) // PAGE
            table[b, :n] = torch.arange(nxt, nxt + n, dtype=torch.int32)
            nxt += n
        if nxt > self.num_pages:
            raise KoptError(f"{nxt} pages needed, pool has {self.num_pages}")
        self.assign_pages(table)

    def assign_permuted(self, lengths, generator: torch.Generator) -> None:
        """Pages drawn as a random permutation of the pool (the ragged-config layout)."""
        need = [(int(L) + PAGE - 1) // PAGE for L in lengths]
        total = sum(need)
        if total > self.num_pages:
            raise KoptError(f"{total} pages needed, pool has {self.num_pages}")
        perm = torch.randperm(self.num_pages, generator=generator)[:total].to(torch.int32)
        table = torch.full((self.B, self.max_pages), -1, dtype=torch.int32)
        o = 0
        for b, n in enumerate(need):
            table[b, :n] = perm[o:o + n]
            o += n
        self.assign_pages(table)

    # --------------------------------------------------------------------- data movement
    def _slots(self, B: int, S: int):
        t = torch.arange(S, device=self.device)
        pid = self.block_table[:B, t // PAGE].long()           # [B, S]
        row = (t % PAGE).expand(B, S)
        if bool((pid < 0).any()):
            raise KoptError("block table has no page for some prefill position")
        return pid.reshape(-1), row.reshape(-1)

    def write_prefix(self, layer: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Scatter contiguous K/V [B, nkv, S, d] (positions 0..S-1) into layer's pages."""
        B, H, S, D = k.shape
        pid, row = self._slots(B, S)
        self.k[layer][pid, :, row] = k.permute(0, 2, 1, 3).reshape(B * S, H, D).to(self.k.dtype)
        self.v[layer][pid, :, row] = v.permute(0, 2, 1, 3).reshape(B * S, H, D).to(self.v.dtype)

    def gather(self, layer: int, b: int, L: int):
        """Contiguous copy of sequence b's first L tokens: (k, v) each [nkv, L, d]."""
        t = torch.arange(L, device=self.device)
        pid = self.block_table[b, t // PAGE].long()
        row = t % PAGE
        return (self.k[layer][pid, :, row].permute(1, 0, 2).contiguous(),
                self.v[layer][pid, :, row].permute(1, 0, 2).contiguous())

    def descriptor(self, layer: int) -> KvCache:
        c = KvCache()
        c.k, c.v = self.k[layer].data_ptr(), self.v[layer].data_ptr()
        c.stride_b = c.stride_h = 0
        c.cap = self.capacity
        c.num_pages = self.num_pages
        c.block_table = self.block_table.data_ptr()
        c.bt_stride = self.block_table.stride(0)
        c.page_size = PAGE
        return c


class PagedDecodeAttention:
    """The engine's attention step over a paged cache, one launch per layer.

    ``__call__`` = the reference's ``qk_norm_rope`` (fused.py:99) followed by ``attn1``
    (fused.py:221) as engine/engine.py:328-330 calls them: the q/k RMSNorm + RoPE prologue, the new
    token's K/V appended at pos[b], and split-K attention over keys 0..pos[b].
    """

    def __init__(self, B, nq, nkv, d, device, max_len, target_ctas=None, eps=1e-6,
                 overlap_prev=False, T=1):
        """max_len: the largest cache capacity (keys per sequence) any call will pass.
        overlap_prev: launch with programmatic dependent launch (KOPT_PLAN_OVERLAP_PREV), so that
        each call's work split and first page copies overlap the end of the kernel before it on
        the stream. Only valid when that kernel writes neither pos, the block table, nor the cache
        rows below pos of the call: a QKV projection GEMM, or an attention call of another layer.
        T: query tokens per sequence; T > 1 (up to 8) is the verify step, through ``attend`` only
        (the fused ``__call__`` appends one token per sequence)."""
        self.B, self.nq, self.nkv, self.d, self.eps = B, nq, nkv, d, eps
        self.max_len = max_len
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise KoptError("PagedDecodeAttention needs a CUDA device (no CPU path)")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.plan = Plan()
        self.T = T
        check(_lib.lib().kopt_decode_attn_plan(self.device.index, B, T, nq, nkv, d, max_len,
                                               int(target_ctas or 0), ctypes.byref(self.plan)),
              "kopt_decode_attn_plan")
        if overlap_prev:
            self.plan.flags |= _lib.PLAN_OVERLAP_PREV
        self.ws = torch.empty(self.plan.ws_bytes, dtype=torch.uint8, device=self.device)
        check(_lib.lib().kopt_workspace_init(ctypes.byref(self.plan), _ptr(self.ws),
                                             _stream(self.device)), "kopt_workspace_init")
        self.scale = d ** -0.5

    @staticmethod
    def _cache(cache, layer: int) -> KvCache:
        """Descriptor for layer `layer` of a PagedKVCache, or for a contiguous (k, v) pair of
        one-layer views [B, nkv, cap, d] (then `layer` is ignored). Built per call: the launcher
        copies it into the kernel parameters, so nothing refers to it after the call."""
        if isinstance(cache, tuple):
            return contiguous_cache(*cache)
        return cache.descriptor(layer)

    def __call__(self, qkv, q_norm_w, k_norm_w, cos, sin, cache, layer, pos, out, q_out=None):
        """qkv [B, (nq+2nkv)d]; pos [B] int32 = position of the new token; out [B, nq d].
        cache: a PagedKVCache (with `layer`) or a contiguous (k_cache, v_cache) layer pair."""
        for t, n in ((qkv, "qkv"), (q_norm_w, "q_norm_w"), (k_norm_w, "k_norm_w"), (cos, "cos"),
                     (sin, "sin"), (out, "out")):
            _require_cuda(t, n)
        _require_cuda(pos, "pos", torch.int32)
        if qkv.shape != (self.B, (self.nq + 2 * self.nkv) * self.d) or out.shape != (self.B, self.nq * self.d):
            raise KoptError("qkv must be [B, (nq+2nkv)d] and out [B, nq d]")
        check(_lib.lib().kopt_decode_attn_fused(
            ctypes.byref(self.plan), _ptr(qkv), _ptr(q_norm_w), _ptr(k_norm_w), _ptr(cos),
            _ptr(sin), cos.shape[0], ctypes.byref(self._cache(cache, layer)), _ptr(pos), _ptr(out),
            _ptr(q_out), _ptr(self.ws), ctypes.c_float(self.scale), ctypes.c_float(self.eps),
            _stream(qkv.device)), "kopt_decode_attn_fused")

    def attend(self, q, cache, layer, pos, out):
        """Attention only (K/V already appended at pos[b] .. pos[b] + T - 1): q/out
        [B*T, nq d], rows b * T + t; query t sees keys 0 .. pos[b] + t (T > 1: verify)."""
        _require_cuda(q, "q")
        _require_cuda(out, "out")
        _require_cuda(pos, "pos", torch.int32)
        check(_lib.lib().kopt_decode_attn(ctypes.byref(self.plan), _ptr(q),
                                          ctypes.byref(self._cache(cache, layer)), _ptr(pos),
                                          _ptr(out), _ptr(self.ws), ctypes.c_float(self.scale),
                                          _stream(q.device)), "kopt_decode_attn")

    def read_error(self) -> int:
        err = ctypes.c_int(0)
        check(_lib.lib().kopt_read_error(ctypes.byref(self.plan), _ptr(self.ws), ctypes.byref(err),
                                         _stream(self.device)), "kopt_read_error")
        return err.value


def qk_norm_rope_paged(qkv, q_w, k_w, cos, sin, pos, q_out, cache: PagedKVCache, layer, T, eps,
                       nq, nkv, d):
    """The prologue alone over a paged cache (K/V appended at pos[b] + m % T)."""
    M = qkv.shape[0]
    dev = qkv.device
    err = _DevErr.get(dev)
    desc = cache.descriptor(layer)
    check(_lib.lib().kopt_qk_norm_rope(_ptr(qkv), _ptr(q_w), _ptr(k_w), _ptr(cos), _ptr(sin),
                                       cos.shape[0], _ptr(pos), _ptr(q_out), ctypes.byref(desc),
                                       M // T, T, nq, nkv, d, ctypes.c_float(eps), _ptr(err),
                                       dev.index, _stream(dev)), "kopt_qk_norm_rope")
