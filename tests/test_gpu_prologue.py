"""GPU: the QK-norm + RoPE + KV-append prologue, bit for bit against the restatement and within
rare single-rounding flips of Transformers (golden fixture)."""

import pytest
import torch

from golden_io import bits, load
from kernel_optim_b200.fused import qk_norm_rope, qk_norm_rope_error
from kernel_optim_b200.paged import PAGE, PagedKVCache, qk_norm_rope_paged
from kernel_optim_b200.workloads import rope_tables
from oracle.prologue import qk_norm_rope_ref

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
NQ, NKV, D, EPS = 32, 8, 128, 1e-6


def test_golden_prologue_paged():
    """Positions 0 .. 131071 with T = 3 tokens per sequence, written through a paged cache that
    holds only the pages those positions touch."""
    z = load("prologue")
    T = int(z["T"])
    qkv, q_w, k_w = bits(z["qkv"]).to(DEV), bits(z["q_w"]).to(DEV), bits(z["k_w"]).to(DEV)
    pos = torch.from_numpy(z["pos"]).to(DEV)
    positions = torch.from_numpy(z["positions"])
    B = pos.numel()
    cos, sin = rope_tables(131072, DEV)
    cache = PagedKVCache(1, 2 * B, NKV, D, B, 131072, DEV)
    table = torch.full((B, cache.max_pages), -1, dtype=torch.int32)
    nxt = 0
    for b in range(B):
        for p in sorted({int(positions[b * T + t]) // PAGE for t in range(T)}):
            table[b, p] = nxt
            nxt += 1
    cache.assign_pages(table)
    q_out = torch.empty(B * T, NQ * D, dtype=torch.bfloat16, device=DEV)
    qk_norm_rope_paged(qkv, q_w, k_w, cos, sin, pos, q_out, cache, 0, T, EPS, NQ, NKV, D)
    torch.cuda.synchronize()
    assert qk_norm_rope_error(DEV) == 0
    rq, rk, rv, _ = qk_norm_rope_ref(qkv, q_w, k_w, cos, sin, pos, T, NQ, NKV, EPS)
    assert torch.equal(q_out.cpu(), rq)
    for m in range(B * T):
        b, p = m // T, int(positions[m])
        pid = int(table[b, p // PAGE])
        assert torch.equal(cache.k[0, pid, :, p % PAGE].cpu(), rk[m]), m
        assert torch.equal(cache.v[0, pid, :, p % PAGE].cpu(), rv[m]), m
    # against Transformers: identical except rare single-rounding flips
    gq = bits(z["q"])
    assert (q_out.cpu().view(torch.int16) != gq.view(torch.int16)).float().mean() < 2e-3


@pytest.mark.parametrize("T", [1, 2])
def test_contiguous_drop_in(T):
    g = torch.Generator(device=DEV).manual_seed(21 + T)
    B, cap = 5, 300
    qkv = torch.randn(B * T, (NQ + 2 * NKV) * D, generator=g, device=DEV).to(torch.bfloat16)
    q_w = (1 + 0.3 * torch.randn(D, generator=g, device=DEV)).to(torch.bfloat16)
    k_w = (1 + 0.3 * torch.randn(D, generator=g, device=DEV)).to(torch.bfloat16)
    pos = torch.tensor([0, 7, 16, 150, 297], dtype=torch.int32, device=DEV)
    cos, sin = rope_tables(cap, DEV)
    kc = torch.zeros(B, NKV, cap, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    q_out = torch.empty(B * T, NQ * D, dtype=torch.bfloat16, device=DEV)
    qk_norm_rope(qkv, q_w, k_w, cos, sin, pos, q_out, kc, vc, T, EPS, NQ, NKV, D)
    torch.cuda.synchronize()
    assert qk_norm_rope_error(DEV) == 0
    rq, rk, rv, positions = qk_norm_rope_ref(qkv, q_w, k_w, cos, sin, pos, T, NQ, NKV, EPS)
    assert torch.equal(q_out.cpu(), rq)
    written = torch.zeros(B, cap, dtype=torch.bool)
    for m in range(B * T):
        b, p = m // T, int(positions[m])
        written[b, p] = True
        assert torch.equal(kc[b, :, p].cpu(), rk[m])
        assert torch.equal(vc[b, :, p].cpu(), rv[m])
    untouched = ~written
    assert not kc.cpu().permute(0, 2, 1, 3)[untouched].any()   # nothing else written


def test_position_beyond_cache_is_clamped_and_reported():
    """pos + T past the capacity is caught by the kernel's bounds check (recorded, clamped)."""
    B, cap = 1, 32
    qkv = torch.randn(B, (NQ + 2 * NKV) * D, device=DEV).to(torch.bfloat16)
    w = torch.ones(D, dtype=torch.bfloat16, device=DEV)
    cos, sin = rope_tables(64, DEV)
    kc = torch.zeros(B, NKV, cap, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    q_out = torch.empty(B, NQ * D, dtype=torch.bfloat16, device=DEV)
    qk_norm_rope(qkv, w, w, cos, sin, torch.tensor([40], dtype=torch.int32, device=DEV), q_out, kc,
                 vc, 1, EPS, NQ, NKV, D)
    torch.cuda.synchronize()
    assert qk_norm_rope_error(DEV) & 2
