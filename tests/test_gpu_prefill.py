"""GPU: the tcgen05 prefill attention (kopt_prefill_attn) against fp32 SDPA.

Causal GQA attention of B prompts of S tokens, 32 query / 8 kv heads, d = 128: the kernel's bf16
output against torch's fp32 scaled_dot_product_attention (is_causal, the kv heads repeated) on the
same bf16 inputs, within the north-star tolerance (max-abs 2e-2, mean-abs 2e-3). Sizes cover one
token, tiles cut inside (S not a multiple of 128 or of the 16-token page), one and several query
tiles, contiguous caches and paged caches with a random page permutation. The engine-level check
(the prompt's K/V written into the pages by the prologue, then this kernel) is in
tests/test_gpu_engine.py.
"""

import pytest
import torch

from kernel_optim_b200.fused import qk_norm_rope_error
from kernel_optim_b200.paged import PagedKVCache
from kernel_optim_b200.prefill import prefill_attention

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
NQ, NKV, D = 32, 8, 128
MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def sdpa_fp32(q, k, v, B, S):
    """q [B*S, nq*d]; k/v [B, nkv, S, d] -> [B*S, nq*d] fp32, causal."""
    qh = q.view(B, S, NQ, D).transpose(1, 2).float()
    kh = k.float().repeat_interleave(NQ // NKV, dim=1)
    vh = v.float().repeat_interleave(NQ // NKV, dim=1)
    o = torch.nn.functional.scaled_dot_product_attention(qh, kh, vh, is_causal=True, scale=D ** -0.5)
    return o.transpose(1, 2).reshape(B * S, NQ * D)


def check(out, ref):
    d = (out.float() - ref).abs()
    assert torch.isfinite(out.float()).all()
    mx, mean = float(d.max()), float(d.mean())
    assert mx <= MAX_ABS and mean <= MEAN_ABS, f"max-abs {mx:.3e} mean-abs {mean:.3e}"


SIZES = [(1, 1), (2, 5), (1, 128), (3, 129), (2, 300), (1, 1024), (4, 777)]


@pytest.mark.parametrize("B,S", SIZES)
def test_contiguous_cache(B, S):
    g = torch.Generator(device=DEV).manual_seed(B * 1000 + S)
    cap = S + 19
    q = torch.randn(B * S, NQ * D, generator=g, device=DEV).to(torch.bfloat16)
    k = torch.randn(B, NKV, cap, D, generator=g, device=DEV).to(torch.bfloat16)
    v = torch.randn(B, NKV, cap, D, generator=g, device=DEV).to(torch.bfloat16)
    k[:, :, S:] = float("nan")   # past the prompt: never attended, never multiplied in
    v[:, :, S:] = float("nan")
    out = torch.full_like(q, float("nan"))
    prefill_attention(q, (k, v), 0, out, B, S, NQ, NKV)
    torch.cuda.synchronize()
    assert qk_norm_rope_error(DEV) == 0
    check(out, sdpa_fp32(q, k[:, :, :S], v[:, :, :S], B, S))


@pytest.mark.parametrize("B,S", SIZES)
def test_paged_cache_permuted_pages(B, S):
    g = torch.Generator(device=DEV).manual_seed(B * 7 + S)
    pages = B * ((S + 15) // 16) + 3
    cache = PagedKVCache(2, pages, NKV, D, B, S, DEV)
    cache.assign_permuted([S] * B, torch.Generator().manual_seed(S))
    cache.k.normal_(generator=g)
    cache.v.normal_(generator=g)
    q = torch.randn(B * S, NQ * D, generator=g, device=DEV).to(torch.bfloat16)
    out = torch.full_like(q, float("nan"))
    prefill_attention(q, cache, 1, out, B, S, NQ, NKV)
    torch.cuda.synchronize()
    assert qk_norm_rope_error(DEV) == 0
    kk = torch.stack([cache.gather(1, b, S)[0] for b in range(B)])
    vv = torch.stack([cache.gather(1, b, S)[1] for b in range(B)])
    check(out, sdpa_fp32(q, kk, vv, B, S))


def test_repeated_calls_are_bit_identical():
    g = torch.Generator(device=DEV).manual_seed(5)
    B, S = 2, 640
    q = torch.randn(B * S, NQ * D, generator=g, device=DEV).to(torch.bfloat16)
    k = torch.randn(B, NKV, S, D, generator=g, device=DEV).to(torch.bfloat16)
    v = torch.randn(B, NKV, S, D, generator=g, device=DEV).to(torch.bfloat16)
    outs = []
    for _ in range(3):
        out = torch.empty_like(q)
        prefill_attention(q, (k, v), 0, out, B, S, NQ, NKV)
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
