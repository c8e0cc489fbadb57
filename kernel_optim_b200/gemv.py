"""Decode-step projections (skinny GEMMs) on the sm_100a library.

Same names and call shape as the reference's ``Gemv`` (GodRishUniverse/kernel_optim
engine/kernels/gemv.py:109-150): ``Gemv(M, N, K, epi, norm, allow_split, eps)`` builds one
projection of the decode batch, ``__call__(x, w, y, nw, ss, h, ss_out)`` runs it and ``tune(weights,
deadline)`` picks the launch configuration by GPU time inside a CUDA graph.

y[M, N] = x[M, K] . w[N, K]^T with fp32 sums and one epilogue (gemv.py:86-105):

* ``EPI_F32``    y float [M, N], the sums (no atomics: split partials are added in split order);
* ``EPI_BF16``   y bf16 [M, N] = bf16(sum);
* ``EPI_RESID``  h bf16 [M, N] updated in place: h = bf16(h + bf16(sum));
* ``EPI_SWIGLU`` w = [gate; up] of [2N, K]; y bf16 [M, N] = bf16(bf16(silu(bf16 g)) * bf16 u);
* ``EPI_ARGMAX`` y int64 [M]: per row the index of the largest bf16(sum), the first one on ties —
  the LM head and greedy pick of the reference's decode step (engine.py:263 logits, then argmax)
  in one kernel that never writes the logits.

``norm=True`` normalises x first, bf16(nw * bf16(x * rstd)) with rstd = rsqrt(mean(x^2) + eps)
(gemv.py:66-79). By default a row kernel (``kopt_add_rms_norm``) writes the normalised rows once
and the projection reads them: on B200 that is faster than normalising inside the projection. With
``fuse_norm=True`` the kernel does it itself (``kopt_gemv_fused``): four warps rewrite each x tile
in shared memory between its TMA copy and the MMAs, rstd from ``ss``, the row sums of squares the
RESID projection before wrote into its ``ss_out`` — float32 ``[T, M]``, one partial per weight tile
of that projection (``Gemv.ss_tiles``), added in tile order, so nothing depends on timing where the
reference adds them with atomics; a ``[M]`` tensor of whole sums works too; without ``ss`` a row
kernel (``kopt_row_sumsq``, the reference's ``embed_ss``) computes them first.

The kernel splits K wherever a tile's chunks fall to several CTAs, for every epilogue (their fp32
partials are added in CTA order), so ``allow_split`` is accepted for the signature and does not
restrict the split.

Launches go to the current torch stream of the tensors' device; a missing library raises KoptError.
"""

from __future__ import annotations

import ctypes
import time

import torch

from . import _lib
from ._lib import GemvFuse, GemvPlan, KoptError, check
from .fused import _ptr, _require_cuda, _stream, add_rms_norm

EPI_F32, EPI_BF16, EPI_RESID, EPI_SWIGLU, EPI_ARGMAX = (
    _lib.GEMV_F32, _lib.GEMV_BF16, _lib.GEMV_RESID, _lib.GEMV_SWIGLU, _lib.GEMV_ARGMAX)


class Gemv:
    """One fused projection of M rows; owns its workspace, so calls allocate nothing and can be
    captured in a CUDA graph. ``ctas`` = 0 launches one resident wave of persistent CTAs, each
    streaming an equal run of (weight tile, K chunk) units; a positive value sets the CTA count.
    ``overlap_prev`` launches with programmatic dependent launch (weight tiles stream while the
    kernel before it on the stream drains)."""

    def __init__(self, M, N, K, epi, norm=False, allow_split=False, eps=1e-6, device=None,
                 ctas=0, overlap_prev=False, fuse_norm=False):
        self.M, self.N, self.K, self.epi, self.norm, self.eps = M, N, K, epi, norm, eps
        self.allow_split = allow_split
        dev = torch.device(device) if device is not None else torch.device("cuda")
        self.device = dev if dev.index is not None else torch.device("cuda", torch.cuda.current_device())
        self.overlap_prev = overlap_prev
        self._plans: dict[int, tuple[GemvPlan, torch.Tensor]] = {}
        self._ss = None   # row sums of squares of x, when the caller gives none
        self.fuse_norm = fuse_norm
        self._xn = (torch.empty(M, K, dtype=torch.bfloat16, device=self.device)
                    if norm and not fuse_norm else None)
        self.cfg = self._plan(ctas).grid

    def _plan(self, ctas: int) -> GemvPlan:
        """Plan (and workspace) for a requested CTA count; cached under the request and under the
        grid it resolves to, which is what ``cfg`` holds."""
        if ctas in self._plans:
            return self._plans[ctas][0]
        plan = GemvPlan()
        check(_lib.lib().kopt_gemv_plan_make(self.device.index, self.M, self.N, self.K, self.epi,
                                             ctas, ctypes.byref(plan)), "kopt_gemv_plan_make")
        plan.flags = _lib.GEMV_OVERLAP_PREV if self.overlap_prev else 0
        if plan.grid in self._plans:
            self._plans[ctas] = self._plans[plan.grid]
            return self._plans[ctas][0]
        ws = torch.zeros(plan.ws_bytes, dtype=torch.uint8, device=self.device)
        self._plans[ctas] = (plan, ws)
        self._plans[plan.grid] = (plan, ws)
        return plan

    @property
    def grid(self) -> int:
        return self.cfg

    @property
    def ss_tiles(self) -> int:
        """Rows of the ``ss_out`` partials a RESID call writes: one per weight tile."""
        return self._plan(self.cfg).tiles

    def __call__(self, x, w, y=None, nw=None, ss=None, h=None, ss_out=None, cfg=None):
        key = self.cfg if cfg is None else cfg
        plan = self._plan(key)
        ws = self._plans[key][1]
        M, N, K = self.M, self.N, self.K
        _require_cuda(x, "x")
        _require_cuda(w, "w")
        rows = 2 * N if self.epi == EPI_SWIGLU else N
        if x.shape != (M, K) or w.shape != (rows, K) or not x.is_contiguous() or not w.is_contiguous():
            raise KoptError(f"Gemv: x must be [{M}, {K}] and w [{rows}, {K}], contiguous")
        if self.epi == EPI_RESID:
            out = h
            if out is None:
                raise KoptError("Gemv(EPI_RESID) needs h")
        else:
            out = y
            if out is None:
                raise KoptError("Gemv needs y")
        if self.epi == EPI_ARGMAX:
            _require_cuda(out, "y", torch.int64)
            if out.shape != (M,) or not out.is_contiguous():
                raise KoptError(f"Gemv(EPI_ARGMAX): y must be int64 [{M}]")
        else:
            _require_cuda(out, "y", torch.float32 if self.epi == EPI_F32 else torch.bfloat16)
            if out.shape != (M, N) or not out.is_contiguous():
                raise KoptError(f"Gemv: output must be [{M}, {N}] contiguous")
        fuse = None
        if self.norm and not self.fuse_norm:
            if nw is None:
                raise KoptError("Gemv(norm=True) needs nw")
            add_rms_norm(x, None, nw, self._xn, self.eps)
            x = self._xn
        if (self.norm and self.fuse_norm) or ss_out is not None:
            fuse = GemvFuse()
            fuse.eps = self.eps
            if self.norm and self.fuse_norm:
                if nw is None:
                    raise KoptError("Gemv(norm=True) needs nw")
                _require_cuda(nw, "nw")
                if nw.shape != (K,) or not nw.is_contiguous():
                    raise KoptError(f"Gemv: nw must be [{K}] contiguous")
                fuse.norm_weight = nw.data_ptr()
                if ss is None:   # no residual projection wrote them: one row pass first
                    if self._ss is None:
                        self._ss = torch.empty(1, M, dtype=torch.float32, device=self.device)
                    check(_lib.lib().kopt_row_sumsq(_ptr(x), M, K, _ptr(self._ss), _stream(x.device)),
                          "kopt_row_sumsq")
                    ss = self._ss
                if ss is not None:
                    _require_cuda(ss, "ss", torch.float32)
                    if ss.numel() % M or not ss.is_contiguous() or ss.shape[-1] != M:
                        raise KoptError(f"Gemv: ss must be float32 [T, {M}] (or [{M}]) contiguous")
                    fuse.ss_in = ss.data_ptr()
                    fuse.ss_tiles = ss.numel() // M
            if ss_out is not None:
                if self.epi != EPI_RESID:
                    raise KoptError("Gemv: ss_out is written by EPI_RESID only")
                _require_cuda(ss_out, "ss_out", torch.float32)
                if ss_out.shape != (plan.tiles, M) or not ss_out.is_contiguous():
                    raise KoptError(f"Gemv: ss_out must be float32 [{plan.tiles}, {M}] contiguous")
                fuse.ss_out = ss_out.data_ptr()
        check(_lib.lib().kopt_gemv_fused(ctypes.byref(plan), _ptr(x), _ptr(w), _ptr(out), _ptr(ws),
                                         ctypes.byref(fuse) if fuse is not None else None,
                                         _stream(x.device)), "kopt_gemv_fused")

    def read_error(self) -> int:
        """KOPT_DEV_ERR_* bits of past calls (synchronises); clears them."""
        plan, ws = self._plans[self.cfg]
        err = ctypes.c_int(0)
        check(_lib.lib().kopt_gemv_read_error(ctypes.byref(plan), _ptr(ws), ctypes.byref(err),
                                              _stream(self.device)), "kopt_gemv_read_error")
        return err.value

    def candidates(self) -> list[int]:
        """Grid sizes worth timing: the library's one resident wave first, then fractions of it."""
        auto = self._plan(0)
        # the device's SM count: auto.grid is clipped to the unit count for small projections
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        out = [auto.grid] + [self._plan(c).grid for c in (sms, 3 * sms // 2, 3 * sms) if c > 0]
        return list(dict.fromkeys(out))

    def tune(self, weights, deadline):
        """Pick the grid by GPU time: one call per real layer weight (cold, as in a decode step),
        captured in a CUDA graph; stops trying new candidates after ``deadline``
        (time.monotonic()), keeping the best so far. Mirrors gemv.py:152-199."""
        dev = weights[0].device
        M, N, K = self.M, self.N, self.K
        x = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
        if self.epi == EPI_ARGMAX:
            y = torch.zeros(M, device=dev, dtype=torch.int64)
        else:
            y = torch.zeros(M, N, device=dev,
                            dtype=torch.float32 if self.epi == EPI_F32 else torch.bfloat16)
        nw = torch.ones(K, device=dev, dtype=torch.bfloat16)
        h = torch.zeros(M, N, device=dev, dtype=torch.bfloat16)
        best = None
        for cfg in self.candidates():
            if time.monotonic() > deadline:
                break
            self(x, weights[0], y, nw, None, h, None, cfg=cfg)
            torch.cuda.synchronize(dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for wt in weights:
                    self(x, wt, y, nw, None, h, None, cfg=cfg)
            g.replay()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            g.replay()
            g.replay()
            b.record()
            torch.cuda.synchronize(dev)
            t = a.elapsed_time(b)
            del g
            if best is None or t < best[0]:
                best = (t, cfg)
        if best is not None:
            self.cfg = self._plan(best[1]).grid
            self.us = best[0] / (2 * len(weights)) * 1e3
        return self.cfg
