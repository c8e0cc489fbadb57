"""GPU: the allocation-free entry point against the workspace entry point, through the C ABI.

kopt_decode_attn_fused_noalloc serves callers that cannot allocate device memory for the split
scratch (an engine that owns the whole memory budget, an allocator frozen after start-up, a plugin
host with no device allocator at the call site); its scratch is an 8 MiB buffer built into the
library. This file is collected last on purpose and runs alone as well as after the other tests.
"""

import ctypes

import pytest
import torch

from kernel_optim_b200 import _lib
from kernel_optim_b200.fused import _ptr, _stream
from kernel_optim_b200.paged import PagedDecodeAttention, PagedKVCache
from kernel_optim_b200.workloads import rope_tables
from oracle.attention import compare, decode_attn_fp32
from oracle.prologue import qk_norm_rope_ref

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
NQ, NKV, D = 32, 8, 128
MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _inputs():
    g = torch.Generator(device=DEV).manual_seed(77)
    lens = [1500, 640, 33, 1]             # cached keys before the appended one
    B, max_len = len(lens), max(lens) + 1
    cache = PagedKVCache(1, sum((L + 16) // 16 for L in lens) + 4, NKV, D, B, max_len, DEV)
    cache.assign_permuted([L + 1 for L in lens], torch.Generator().manual_seed(3))
    cache.k.normal_(generator=g)
    cache.v.normal_(generator=g)
    qkv = torch.randn(B, (NQ + 2 * NKV) * D, generator=g, device=DEV).to(torch.bfloat16)
    w = (1 + 0.2 * torch.randn(D, generator=g, device=DEV)).to(torch.bfloat16)
    cos, sin = rope_tables(max_len, DEV)
    pos = torch.tensor(lens, dtype=torch.int32, device=DEV)
    return B, cache, qkv, w, cos, sin, pos


def _noalloc(attn, cache, qkv, w, cos, sin, pos, out, err):
    desc = cache.descriptor(0)
    return _lib.lib().kopt_decode_attn_fused_noalloc(
        ctypes.byref(attn.plan), _ptr(qkv), _ptr(w), _ptr(w), _ptr(cos), _ptr(sin), cos.shape[0],
        ctypes.byref(desc), _ptr(pos), _ptr(out), None, ctypes.c_float(attn.scale),
        ctypes.c_float(attn.eps), _ptr(err), _stream(DEV))


def _oracle(B, cache, qkv, w, cos, sin, pos):
    """fp32 SDPA over the cached keys plus the appended token (restated prologue, CPU)."""
    lens = pos.tolist()
    q, k_new, v_new, _ = qk_norm_rope_ref(qkv, w, w, cos, sin, pos, 1, NQ, NKV, 1e-6)
    kk = torch.zeros(B, NKV, max(lens) + 1, D, dtype=torch.bfloat16)
    vv = torch.zeros_like(kk)
    for b, L in enumerate(lens):
        kb, vb = cache.gather(0, b, L)
        kk[b, :, :L], vv[b, :, :L] = kb.cpu(), vb.cpu()
        kk[b, :, L], vv[b, :, L] = k_new[b], v_new[b]
    return decode_attn_fp32(q.view(B, NQ, D), kk, vv, [L + 1 for L in lens])


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    """Same plan, same kernel, same split of the keys, merges in a fixed slot order: the outputs
    must be identical bit for bit on both calls, so that counters or partials left in the shared
    buffer by the first call cannot hide behind a tolerance. Both are also checked against the
    fp32 oracle within the north-star tolerance (max-abs 2e-2, mean-abs 2e-3)."""
    B, cache, qkv, w, cos, sin, pos = _inputs()
    ref32 = _oracle(B, cache, qkv, w, cos, sin, pos)
    attn = PagedDecodeAttention(B, NQ, NKV, D, DEV, cache.capacity)
    assert attn.plan.ws_bytes <= 8 << 20
    ref = torch.empty(B, NQ * D, dtype=torch.bfloat16, device=DEV)
    attn(qkv, w, w, cos, sin, cache, 0, pos, ref)
    torch.cuda.synchronize()
    assert attn.read_error() == 0
    mx, mean = compare(ref.view(B, NQ, D), ref32)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, f"workspace entry point: max-abs {mx} mean-abs {mean}"
    err = torch.full((1,), -1, dtype=torch.int32, device=DEV)
    for call in range(2):   # the shared buffer keeps the first call's contents for the second
        out = torch.full_like(ref, float("nan"))
        _lib.check(_noalloc(attn, cache, qkv, w, cos, sin, pos, out, err),
                   "kopt_decode_attn_fused_noalloc")
        torch.cuda.synchronize()
        assert int(err.item()) == 0, f"call {call}: device error bits {int(err.item())}"
        assert torch.equal(out, ref), f"call {call}: differs from the workspace entry point"
        mx, mean = compare(out.view(B, NQ, D), ref32)
        assert mx <= MAX_ABS and mean <= MEAN_ABS, f"call {call}: max-abs {mx} mean-abs {mean}"


def test_noalloc_rejects_plans_beyond_the_builtin_scratch():
    attn = PagedDecodeAttention(4, NQ, NKV, D, DEV, 131072)
    assert attn.plan.ws_bytes > 8 << 20
    B, cache, qkv, w, cos, sin, pos = _inputs()
    out = torch.empty(B, NQ * D, dtype=torch.bfloat16, device=DEV)
    rc = _noalloc(attn, cache, qkv, w, cos, sin, pos, out, None)
    assert rc == _lib.KOPT_ERR_SCRATCH
    assert b"8 MiB" in _lib.lib().kopt_strerror(rc)
