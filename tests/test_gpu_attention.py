"""GPU parity of the sm_100a decode attention against the fp32 SDPA oracle, through the C ABI.

Tolerance (north star): bf16 output within max-abs 2e-2 and mean-abs 2e-3 of fp32 SDPA.
Bit-exact checks: the appended K/V and roped q against the restatement; paged vs contiguous and
page-permuted layouts against each other (same plan, same arithmetic).
"""

import pytest
import torch
import torch.nn.functional as F

from golden_io import attention_case
from kernel_optim_b200 import KoptError
from kernel_optim_b200.fused import DecodeAttention
from kernel_optim_b200.paged import PAGE, PagedDecodeAttention, PagedKVCache
from kernel_optim_b200.workloads import build_case
from oracle.attention import compare, decode_attn_fp32
from oracle.prologue import qk_norm_rope_ref

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
NQ, NKV, D = 32, 8, 128
MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def within(got, ref, what=""):
    mx, mean = compare(got.reshape(ref.shape), ref)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, f"{what}: max-abs {mx:.3e} mean-abs {mean:.3e}"
    return mx, mean


def run_contiguous(q, k, v, lens, target_ctas=None):
    B, cap = len(lens), k.shape[2]
    attn = DecodeAttention(B, 1, cap, NQ, NKV, D, DEV, target_ctas=target_ctas)
    qd = q.reshape(B, NQ * D).to(DEV).contiguous()
    out = torch.empty_like(qd)
    pos = torch.tensor(lens, dtype=torch.int32, device=DEV) - 1
    attn(qd, k.to(DEV), v.to(DEV), pos, out)
    torch.cuda.synchronize()
    assert attn.read_error() == 0
    return out.cpu()


@pytest.mark.parametrize("name", ["c1", "ragged"])
def test_golden_contiguous(name):
    q, k, v, lens, out_gqa, out_rep = attention_case(name)
    got = run_contiguous(q, k, v, lens)
    within(got, out_gqa, name)
    within(got, out_rep, name + " repeat_kv")


def test_golden_paged_matches_contiguous_bitwise():
    q, k, v, lens, out_gqa, _ = attention_case("ragged")
    B = len(lens)
    cache = PagedKVCache(1, sum((L + PAGE - 1) // PAGE for L in lens) + 3, NKV, D, B, max(lens), DEV)
    cache.assign_permuted(lens, torch.Generator().manual_seed(5))
    for b, L in enumerate(lens):
        t = torch.arange(L, device=DEV)
        pid = cache.block_table[b, t // PAGE].long()
        cache.k[0][pid, :, t % PAGE] = k[b, :, :L].to(DEV).permute(1, 0, 2)
        cache.v[0][pid, :, t % PAGE] = v[b, :, :L].to(DEV).permute(1, 0, 2)
    attn = PagedDecodeAttention(B, NQ, NKV, D, DEV, cache.capacity)
    qd = q.reshape(B, NQ * D).to(DEV).contiguous()
    out = torch.empty_like(qd)
    attn.attend(qd, cache, 0, torch.tensor(lens, dtype=torch.int32, device=DEV) - 1, out)
    torch.cuda.synchronize()
    assert attn.read_error() == 0
    within(out.cpu(), out_gqa, "paged")
    assert torch.equal(out.cpu(), run_contiguous(q, k, v, lens))


def test_strided_cache_views():
    """k_cache[i] views of 5-D caches with batch-major and head-major layouts (arbitrary strides,
    as engine.py:395 passes self.k_cache[i])."""
    g = torch.Generator(device=DEV).manual_seed(3)
    lens = [5, 130, 77]
    B, cap, L = len(lens), 136, 2
    q = torch.randn(B, NQ, D, generator=g, device=DEV).to(torch.bfloat16)
    kb = torch.randn(L, B, NKV, cap, D, generator=g, device=DEV).to(torch.bfloat16)
    vb = torch.randn(L, B, NKV, cap, D, generator=g, device=DEV).to(torch.bfloat16)
    kh = kb.permute(0, 2, 1, 3, 4).contiguous().permute(0, 2, 1, 3, 4)   # head-major storage
    vh = vb.permute(0, 2, 1, 3, 4).contiguous().permute(0, 2, 1, 3, 4)
    ref = decode_attn_fp32(q.cpu(), kb[1].cpu(), vb[1].cpu(), lens)
    attn = DecodeAttention(B, 1, cap, NQ, NKV, D, DEV)
    pos = torch.tensor(lens, dtype=torch.int32, device=DEV) - 1
    qd = q.reshape(B, -1).contiguous()
    o1, o2 = torch.empty_like(qd), torch.empty_like(qd)
    attn(qd, kb[1], vb[1], pos, o1)
    attn(qd, kh[1], vh[1], pos, o2)
    torch.cuda.synchronize()
    within(o1.cpu(), ref, "batch-major")
    assert torch.equal(o1, o2)


LENGTHS = [1, 2, 15, 16, 17, 31, 63, 64, 65, 127, 128, 129, 500, 1000, 2049, 4097]


@pytest.mark.parametrize("target_ctas", [None, 8, 37, 1000])
def test_lengths_and_split_plans(target_ctas):
    """Every boundary around the 16-token page and 64-token tile, one-wave and multi-wave plans."""
    g = torch.Generator().manual_seed(11)
    B, cap = len(LENGTHS), max(LENGTHS)
    q = torch.randn(B, NQ, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, NKV, cap, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, NKV, cap, D, generator=g).to(torch.bfloat16)
    ref = decode_attn_fp32(q, k, v, LENGTHS)
    got = run_contiguous(q, k, v, LENGTHS, target_ctas)
    for b, L in enumerate(LENGTHS):
        within(got[b], ref[b], f"L={L} target_ctas={target_ctas}")


@pytest.mark.parametrize("B", [32, 37])
def test_whole_pair_pieces_when_pairs_outnumber_ctas(B):
    """Equal lengths and more (sequence, kv head) pairs than CTAs (c5's decode step: 256 pairs):
    each CTA takes whole pairs, nothing is split or merged; B = 37 fills all 148 CTAs."""
    g = torch.Generator().manual_seed(12)
    L = 1153
    q = torch.randn(B, NQ, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, NKV, L, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, NKV, L, D, generator=g).to(torch.bfloat16)
    ref = decode_attn_fp32(q, k, v, [L] * B)
    got = run_contiguous(q, k, v, [L] * B)
    within(got, ref, f"B={B} L={L}")


def test_repeated_calls_bitwise_identical():
    """The split counters are reset by the merging CTA, so replays see a clean workspace."""
    g = torch.Generator().manual_seed(12)
    lens = [4097] * 4 + [300] * 4
    B, cap = len(lens), max(lens)
    q = torch.randn(B, NQ, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, NKV, cap, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, NKV, cap, D, generator=g).to(torch.bfloat16)
    attn = DecodeAttention(B, 1, cap, NQ, NKV, D, DEV)
    qd, kd, vd = q.reshape(B, -1).to(DEV), k.to(DEV), v.to(DEV)
    pos = torch.tensor(lens, dtype=torch.int32, device=DEV) - 1
    outs = []
    for _ in range(3):
        o = torch.empty_like(qd)
        attn(qd, kd, vd, pos, o)
        outs.append(o)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    within(outs[0].cpu(), decode_attn_fp32(q, k, v, lens))


def _fused_reference(case, cache_k_ctx, cache_v_ctx):
    """Oracle for a fused step: restated prologue, then fp32 SDPA over cached + appended keys."""
    t = case.tensors
    q, k_new, v_new, _ = qk_norm_rope_ref(t["qkv"], t["q_norm_w"], t["k_norm_w"], t["cos"],
                                          t["sin"], t["pos"], 1, case.nq, case.nkv, 1e-6)
    B = case.B
    cap = max(case.keys)
    kk = torch.zeros(B, case.nkv, cap, D, dtype=torch.bfloat16)
    vv = torch.zeros_like(kk)
    for b, L in enumerate(case.cached):
        kk[b, :, :L] = cache_k_ctx[b]
        vv[b, :, :L] = cache_v_ctx[b]
        kk[b, :, L] = k_new[b]
        vv[b, :, L] = v_new[b]
    return q, k_new, v_new, decode_attn_fp32(q.view(B, case.nq, D), kk, vv, case.keys)


def test_c2_fused_paged_full_size():
    case = build_case("c2", DEV, seed=0, paged=True)
    t, cache = case.tensors, case.tensors["cache"]
    B = case.B
    ctx = [cache.gather(0, b, L) for b, L in enumerate(case.cached)]
    ref_q, k_new, v_new, ref_out = _fused_reference(case, [c[0].cpu() for c in ctx],
                                                    [c[1].cpu() for c in ctx])
    attn = PagedDecodeAttention(B, NQ, NKV, D, DEV, cache.capacity)
    out = torch.empty(B, NQ * D, dtype=torch.bfloat16, device=DEV)
    q_out = torch.empty_like(out)
    attn(t["qkv"], t["q_norm_w"], t["k_norm_w"], t["cos"], t["sin"], cache, 0, t["pos"], out, q_out)
    torch.cuda.synchronize()
    assert attn.read_error() == 0
    mx, mean = within(out.cpu(), ref_out, "c2 fused")
    assert torch.equal(q_out.cpu(), ref_q)
    for b, L in enumerate(case.cached):
        kb, vb = cache.gather(0, b, L + 1)
        assert torch.equal(kb[:, L].cpu(), k_new[b]), f"appended K differs (b={b})"
        assert torch.equal(vb[:, L].cpu(), v_new[b]), f"appended V differs (b={b})"
        assert torch.equal(kb[:, :L].cpu(), ctx[b][0].cpu())   # nothing else written


def test_c2_fused_contiguous_equals_paged():
    pc = build_case("c2", DEV, seed=1, paged=True)
    cc = build_case("c2", DEV, seed=1, paged=False)
    B = pc.B
    outs = []
    for case in (pc, cc):
        t = case.tensors
        out = torch.empty(B, NQ * D, dtype=torch.bfloat16, device=DEV)
        cache = t["cache"] if "cache" in t else (t["k_cache"][0], t["v_cache"][0])
        a = PagedDecodeAttention(B, NQ, NKV, D, DEV, max(case.keys) + 16)
        a(t["qkv"], t["q_norm_w"], t["k_norm_w"], t["cos"], t["sin"], cache, 0, t["pos"], out)
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])


def test_c3_ragged_paged_full_size():
    case = build_case("c3", DEV, seed=0, paged=True)
    t, cache = case.tensors, case.tensors["cache"]
    B = case.B
    q, k_new, v_new, _ = qk_norm_rope_ref(t["qkv"], t["q_norm_w"], t["k_norm_w"], t["cos"],
                                          t["sin"], t["pos"], 1, NQ, NKV, 1e-6)
    attn = PagedDecodeAttention(B, NQ, NKV, D, DEV, cache.capacity)
    out = torch.empty(B, NQ * D, dtype=torch.bfloat16, device=DEV)
    attn(t["qkv"], t["q_norm_w"], t["k_norm_w"], t["cos"], t["sin"], cache, 0, t["pos"], out)
    torch.cuda.synchronize()
    assert attn.read_error() == 0
    qg = q.view(B, NQ, D).to(DEV)
    for b in range(0, B, 7):   # torch fp32 reference on the GPU for every 7th sequence
        L = case.keys[b]
        kb, vb = cache.gather(0, b, L)
        assert torch.equal(kb[:, L - 1].cpu(), k_new[b]) and torch.equal(vb[:, L - 1].cpu(), v_new[b])
        ref = F.scaled_dot_product_attention(qg[b:b + 1].float().unsqueeze(2), kb[None].float(),
                                             vb[None].float(), scale=D ** -0.5, enable_gqa=True)
        within(out[b].cpu(), ref[0, :, 0].cpu(), f"c3 b={b} L={L}")


def test_c4_long_context_full_size():
    case = build_case("c4", DEV, seed=0, paged=False)
    t = case.tensors
    B = case.B
    a = PagedDecodeAttention(B, NQ, NKV, D, DEV, t["k_cache"].shape[3])
    out = torch.empty(B, NQ * D, dtype=torch.bfloat16, device=DEV)
    q_out = torch.empty_like(out)
    a(t["qkv"], t["q_norm_w"], t["k_norm_w"], t["cos"], t["sin"],
      (t["k_cache"][0], t["v_cache"][0]), 0, t["pos"], out, q_out)
    torch.cuda.synchronize()
    assert a.read_error() == 0
    for b in range(B):
        L = case.keys[b]
        ref = F.scaled_dot_product_attention(
            q_out[b].view(1, NQ, 1, D).float(), t["k_cache"][0, b:b + 1, :, :L].float(),
            t["v_cache"][0, b:b + 1, :, :L].float(), scale=D ** -0.5, enable_gqa=True)
        within(out[b].cpu(), ref[0, :, 0].cpu(), f"c4 b={b}")


def test_graph_capture_and_replay():
    """The fused paged step captured once in a CUDA graph and replayed at advancing positions
    matches eager launches (addresses fixed, positions read from device memory)."""
    g = torch.Generator(device=DEV).manual_seed(9)
    B, L0, steps = 6, 200, 5
    max_len = L0 + steps + 1
    case_cache = PagedKVCache(1, B * ((max_len + 15) // 16), NKV, D, B, max_len, DEV)
    case_cache.assign_sequential([max_len] * B)
    case_cache.k.normal_(generator=g)
    case_cache.v.normal_(generator=g)
    snap_k, snap_v = case_cache.k.clone(), case_cache.v.clone()
    from kernel_optim_b200.workloads import rope_tables
    cos, sin = rope_tables(max_len, DEV)
    w = torch.ones(D, dtype=torch.bfloat16, device=DEV)
    qkv = torch.randn(B, (NQ + 2 * NKV) * D, generator=g, device=DEV).to(torch.bfloat16)
    pos = torch.full((B,), L0, dtype=torch.int32, device=DEV)
    out = torch.empty(B, NQ * D, dtype=torch.bfloat16, device=DEV)
    attn = PagedDecodeAttention(B, NQ, NKV, D, DEV, case_cache.capacity)
    eager = []
    for s in range(steps):
        pos.fill_(L0 + s)
        attn(qkv, w, w, cos, sin, case_cache, 0, pos, out)
        eager.append(out.clone())
    case_cache.k.copy_(snap_k)
    case_cache.v.copy_(snap_v)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        attn(qkv, w, w, cos, sin, case_cache, 0, pos, out)
    torch.cuda.current_stream().wait_stream(side)
    case_cache.k.copy_(snap_k)
    case_cache.v.copy_(snap_v)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        attn(qkv, w, w, cos, sin, case_cache, 0, pos, out)
    for s in range(steps):
        pos.fill_(L0 + s)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager[s]), f"replay step {s} differs from eager"
    assert attn.read_error() == 0


def test_bad_page_id_is_reported_not_faulted():
    """A block-table entry outside the pool is caught by the kernel's own bounds check: the copy
    is skipped, KOPT_DEV_ERR_PAGE is recorded and the launch completes."""
    B, L = 2, 40
    cache = PagedKVCache(1, 8, NKV, D, B, 64, DEV)
    cache.assign_sequential([L, L])
    cache.block_table[1, 1] = 1000           # outside [0, 8): never dereferenced
    attn = PagedDecodeAttention(B, NQ, NKV, D, DEV, cache.capacity)
    q = torch.randn(B, NQ * D, device=DEV).to(torch.bfloat16)
    out = torch.empty_like(q)
    attn.attend(q, cache, 0, torch.tensor([L - 1, L - 1], dtype=torch.int32, device=DEV), out)
    torch.cuda.synchronize()
    assert attn.read_error() & 1
    assert attn.read_error() == 0            # read clears the word


def test_rejects_cpu_tensors_and_bad_shapes():
    attn = DecodeAttention(2, 1, 64, NQ, NKV, D, DEV)
    q = torch.zeros(2, NQ * D, dtype=torch.bfloat16)
    k = torch.zeros(2, NKV, 64, D, dtype=torch.bfloat16)
    pos = torch.zeros(2, dtype=torch.int32)
    with pytest.raises(KoptError):
        attn(q, k, k, pos, q)
    with pytest.raises(KoptError):
        attn(q.to(DEV)[:, :100], k.to(DEV), k.to(DEV), pos.to(DEV), q.to(DEV))


def test_overlapped_launches_match_plain():
    """KOPT_PLAN_OVERLAP_PREV: back-to-back calls over different layers (each call's split and
    first page copies issued while the previous call finishes) and the same calls behind a QKV
    GEMM inside a CUDA graph. The flag also shortens the last CTAs' pieces, so the split differs
    from a plain launch: outputs match plain launches within the bf16 tolerance and are
    bit-identical from one overlapped call to the next, eager or graphed."""
    from kernel_optim_b200.workloads import build_case
    layers = 4
    case = build_case("c2", DEV, seed=3, paged=True, layers=layers)
    t = case.tensors
    cache = t["cache"]
    args = (t["q_norm_w"], t["k_norm_w"], t["cos"], t["sin"], cache)
    plain = PagedDecodeAttention(case.B, NQ, NKV, D, DEV, cache.capacity)
    over = PagedDecodeAttention(case.B, NQ, NKV, D, DEV, cache.capacity, overlap_prev=True)
    g = torch.Generator(device=DEV).manual_seed(4)
    x = torch.randn(case.B, 512, generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn((NQ + 2 * NKV) * D, 512, generator=g, device=DEV) / 16).to(torch.bfloat16)
    qkv = torch.mm(x, w.t())
    ref = []
    for layer in range(layers):
        out = torch.empty(case.B, NQ * D, dtype=torch.bfloat16, device=DEV)
        plain(qkv, *args, layer, t["pos"], out)
        ref.append(out)
    outs = [torch.empty_like(ref[0]) for _ in range(layers)]
    first = None
    for rep in range(3):
        for layer in range(layers):
            over(qkv, *args, layer, t["pos"], outs[layer])
        torch.cuda.synchronize()
        if first is None:
            first = [o.clone() for o in outs]
            for layer in range(layers):
                d = (first[layer].float() - ref[layer].float()).abs()
                assert float(d.max()) <= MAX_ABS and float(d.mean()) <= MEAN_ABS, f"layer {layer}"
        for layer in range(layers):
            assert torch.equal(outs[layer], first[layer]), f"rep {rep} layer {layer}"
    # GEMM -> attention pairs in a graph: the attention overlaps the GEMM that produces its qkv
    qkv_g = torch.empty_like(qkv)
    for o in outs:
        o.zero_()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        torch.mm(x, w.t(), out=qkv_g)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for layer in range(layers):
            torch.mm(x, w.t(), out=qkv_g)
            over(qkv_g, *args, layer, t["pos"], outs[layer])
    for _ in range(2):
        graph.replay()
        torch.cuda.synchronize()
        for layer in range(layers):
            assert torch.equal(outs[layer], first[layer]), f"graph layer {layer}"
    assert plain.read_error() == 0 and over.read_error() == 0
