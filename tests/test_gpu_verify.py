"""GPU parity of verify attention: T query tokens per sequence, causal among themselves
(engine/kernels/fused.py:130-185 with T > 1, as engine.py:403-415 verifies K = T - 1 drafts),
through the C ABI (kopt_decode_attn with a plan of T > 1).

Tolerance as for decode: bf16 outputs within max-abs 2e-2 and mean-abs 2e-3 of the fp32 oracle
(oracle/attention.py: verify_attn_fp32). Paged and contiguous layouts of the same data, same plan,
agree bit for bit.
"""

import pytest
import torch

from kernel_optim_b200 import KoptError
from kernel_optim_b200.fused import DecodeAttention
from kernel_optim_b200.paged import PAGE, PagedDecodeAttention, PagedKVCache
from oracle.attention import compare, verify_attn_fp32

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
NQ, NKV, D = 32, 8, 128
MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _case(B, T, cap, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    q = torch.randn(B * T, NQ * D, generator=g, device=DEV).to(torch.bfloat16)
    k = torch.randn(B, NKV, cap, D, generator=g, device=DEV).to(torch.bfloat16)
    v = torch.randn(B, NKV, cap, D, generator=g, device=DEV).to(torch.bfloat16)
    return q, k, v


def _run(B, T, pos, cap, seed=0, target_ctas=None):
    q, k, v = _case(B, T, cap, seed)
    attn = DecodeAttention(B, T, cap, NQ, NKV, D, DEV, target_ctas=target_ctas)
    out = torch.full_like(q, float("nan"))
    attn(q, k, v, torch.tensor(pos, dtype=torch.int32, device=DEV), out)
    torch.cuda.synchronize()
    assert attn.read_error() == 0
    ref = verify_attn_fp32(q.view(B * T, NQ, D), k, v, pos, T)
    mx, mean = compare(out.view(B * T, NQ, D).cpu(), ref)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, f"T={T}: max-abs {mx:.3e} mean-abs {mean:.3e}"
    return attn, out


@pytest.mark.parametrize("T", [2, 3, 4, 5, 7, 8])
def test_verify_matches_oracle(T):
    """Ragged positions, including pos 0 (the block sees only its own keys) and lengths that
    end mid-page."""
    pos = [0, 37, 300, 2047]
    _run(len(pos), T, pos, max(pos) + T + 9, seed=T)


@pytest.mark.parametrize("target_ctas", [1, 100000])
def test_verify_one_split_and_many_splits(target_ctas):
    """One split (outputs stored directly) and as many splits as the capacity allows (most of
    them empty for the short sequences, merged by the last)."""
    attn, _ = _run(3, 5, [3, 700, 4100], 4200, seed=7, target_ctas=target_ctas)
    nsplit = attn.plan.grid // (3 * NKV)
    assert (nsplit == 1) == (target_ctas == 1)


def test_verify_repeated_calls_are_identical():
    B, T, pos, cap = 2, 7, [100, 1000], 1100
    q, k, v = _case(B, T, cap, 3)
    attn = DecodeAttention(B, T, cap, NQ, NKV, D, DEV)
    p = torch.tensor(pos, dtype=torch.int32, device=DEV)
    outs = []
    for _ in range(3):
        out = torch.empty_like(q)
        attn(q, k, v, p, out)
        outs.append(out)
    torch.cuda.synchronize()
    assert attn.read_error() == 0
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])


@pytest.mark.parametrize("T", [3, 5])
def test_verify_paged_matches_contiguous_bitwise(T):
    B, pos = 3, [15, 500, 1601]
    lens = [p_ + T for p_ in pos]
    cap = 1616
    q, k, v = _case(B, T, cap, 5)
    cache = PagedKVCache(1, sum((L + PAGE - 1) // PAGE for L in lens) + 4, NKV, D, B, cap, DEV)
    cache.assign_permuted(lens, torch.Generator().manual_seed(9))
    for b, L in enumerate(lens):
        t = torch.arange(L, device=DEV)
        pid = cache.block_table[b, t // PAGE].long()
        cache.k[0][pid, :, t % PAGE] = k[b, :, :L].permute(1, 0, 2)
        cache.v[0][pid, :, t % PAGE] = v[b, :, :L].permute(1, 0, 2)
    p = torch.tensor(pos, dtype=torch.int32, device=DEV)
    paged = PagedDecodeAttention(B, NQ, NKV, D, DEV, cache.capacity, T=T)
    out_p = torch.empty_like(q)
    paged.attend(q, cache, 0, p, out_p)
    contig = DecodeAttention(B, T, cache.capacity, NQ, NKV, D, DEV)
    kc = torch.zeros(B, NKV, cache.capacity, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    kc[:, :, :cap], vc[:, :, :cap] = k, v
    out_c = torch.empty_like(q)
    contig(q, kc, vc, p, out_c)
    torch.cuda.synchronize()
    assert paged.read_error() == 0 and contig.read_error() == 0
    assert paged.plan.grid == contig.plan.grid
    assert torch.equal(out_p, out_c)
    ref = verify_attn_fp32(q.view(B * T, NQ, D), k, v, pos, T)
    mx, mean = compare(out_p.view(B * T, NQ, D).cpu(), ref)
    assert mx <= MAX_ABS and mean <= MEAN_ABS


def test_verify_rejects_bad_plans_and_the_fused_entry():
    with pytest.raises(KoptError):
        DecodeAttention(2, 9, 128, NQ, NKV, D, DEV)   # more than 8 query tokens
    attn = PagedDecodeAttention(2, NQ, NKV, D, DEV, 64, T=3)
    z = torch.zeros(2, (NQ + 2 * NKV) * D, dtype=torch.bfloat16, device=DEV)
    w = torch.ones(D, dtype=torch.bfloat16, device=DEV)
    cache = PagedKVCache(1, 8, NKV, D, 2, 64, DEV)
    cache.assign_sequential([64, 64])
    with pytest.raises(KoptError):   # the fused prologue appends one token per sequence
        attn(z, w, w, w.view(1, D).expand(64, D).contiguous(), w.view(1, D).expand(64, D).contiguous(),
             cache, 0, torch.zeros(2, dtype=torch.int32, device=DEV),
             torch.empty(2, NQ * D, dtype=torch.bfloat16, device=DEV))
