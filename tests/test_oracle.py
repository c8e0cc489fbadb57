"""CPU: the oracle against the golden fixtures written from the reference's native path."""

import numpy as np
import torch

from golden_io import attention_case, bits, load
from oracle.attention import compare, decode_attn_fp32, reference_plan, reference_split_k
from oracle.bf16 import bf16r, bits_to_f32, f32_to_bits
from oracle.prologue import norm_rope_rows, qk_norm_rope_ref, rope_tables, transformers_prologue

NQ, NKV, D, EPS = 32, 8, 128, 1e-6
MAX_ABS, MEAN_ABS = 2e-2, 2e-3   # north-star tolerance on bf16 outputs vs fp32 SDPA


def test_bf16_rounding_matches_torch():
    x = torch.randn(100000) * torch.logspace(-30, 30, 100000)
    ours = bits_to_f32(f32_to_bits(x.numpy()))
    ref = x.to(torch.bfloat16).float().numpy()
    assert np.array_equal(ours, ref)
    assert np.array_equal(bf16r(x.numpy()), ref)


def test_rope_tables_match_golden():
    z = load("rope")
    cos, sin = rope_tables(131073)
    idx = torch.from_numpy(z["idx"])
    assert torch.equal(cos[idx], bits(z["cos"]))
    assert torch.equal(sin[idx], bits(z["sin"]))


def test_transformers_prologue_reproduces_golden():
    z = load("prologue")
    cos, sin = rope_tables(131072)
    q, k, v = transformers_prologue(bits(z["qkv"]), bits(z["q_w"]), bits(z["k_w"]), cos, sin,
                                    torch.from_numpy(z["positions"]), NQ, NKV, EPS)
    assert torch.equal(q, bits(z["q"]))
    assert torch.equal(k, bits(z["k"]))
    assert torch.equal(v, bits(z["v"]))


def _ulp_diff(a: torch.Tensor, b: torch.Tensor):
    """Elements that differ and their distance in bf16 ulps of the reference value."""
    af, bf = a.float(), b.float()
    diff = (af - bf).abs()
    ulp = torch.where(bf == 0, torch.full_like(bf, 2.0 ** -133),
                      2.0 ** (torch.floor(torch.log2(bf.abs())) - 7))
    return int((a.view(torch.int16) != b.view(torch.int16)).sum()), float((diff / ulp).max())


def test_prologue_restatement_vs_transformers():
    """The restatement (fixed summation order) agrees with Transformers bit for bit except for
    rare one-rounding flips when the two sums of squares differ in the last fp32 bit."""
    z = load("prologue")
    T = int(z["T"])
    cos, sin = rope_tables(131072)
    q, k, v, positions = qk_norm_rope_ref(bits(z["qkv"]), bits(z["q_w"]), bits(z["k_w"]), cos,
                                          sin, torch.from_numpy(z["pos"]), T, NQ, NKV, EPS)
    assert np.array_equal(positions.numpy(), z["positions"])
    assert torch.equal(v, bits(z["v"]))
    nq_bad, q_ulp = _ulp_diff(q, bits(z["q"]))
    nk_bad, k_ulp = _ulp_diff(k, bits(z["k"]))
    assert (nq_bad + nk_bad) <= 2e-3 * (q.numel() + k.numel())
    assert q_ulp <= 8 and k_ulp <= 8


def test_prologue_rows_known_answer():
    """Hand-checkable case: x = 1 everywhere, unit weights, position 0 (cos 1, sin 0) -> y = 1."""
    x = np.ones((2, D), np.float32)
    y = norm_rope_rows(x, np.ones(D, np.float32), np.ones((2, D), np.float32),
                       np.zeros((2, D), np.float32), 1e-6)
    assert np.array_equal(y, np.ones((2, D), np.float32))


def test_fp32_oracle_reproduces_golden():
    for name in ("c1", "ragged"):
        q, k, v, lens, out_gqa, out_rep = attention_case(name)
        out = decode_attn_fp32(q, k, v, lens)
        assert torch.allclose(out, out_gqa, atol=1e-6, rtol=0)
        # repeat_kv (pinned Transformers) and enable_gqa (installed) forms agree
        assert torch.allclose(out_gqa, out_rep, atol=1e-6, rtol=0)


def test_reference_split_k_restatement_within_tolerance():
    """The reference's own algorithm (capacity split plan, bf16 p) is inside the north-star
    tolerance of the fp32 oracle, on C1 and on the ragged batch."""
    for name in ("c1", "ragged"):
        q, k, v, lens, out_gqa, _ = attention_case(name)
        pos = torch.tensor(lens) - 1
        got = reference_split_k(q, k, v, pos, cap=k.shape[2])
        mx, mean = compare(got, out_gqa)
        assert mx <= MAX_ABS and mean <= MEAN_ABS, (name, mx, mean)


def test_reference_plan_matches_fused_py():
    # fused.py:211-214 at the shapes the survey tabulates
    assert reference_plan(4097, 16, 8) == (3, 1408)
    assert reference_plan(131073, 4, 8) == (9, 14592)
    assert reference_plan(512, 1, 8) == (4, 128)


def test_verify_oracle_matches_masked_restatement():
    """The verify oracle (one single-token SDPA per query token) against one masked SDPA per
    sequence: two independent statements of 'query t sees keys 0 .. pos + t'."""
    from oracle.attention import verify_attn_fp32, verify_attn_masked_fp32
    g = torch.Generator().manual_seed(11)
    B, T, nq, nkv = 3, 5, 32, 8
    pos = [0, 9, 40]
    cap = max(pos) + T
    q = torch.randn(B * T, nq, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(B, nkv, cap, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(B, nkv, cap, 128, generator=g).to(torch.bfloat16)
    a = verify_attn_fp32(q, k, v, pos, T)
    b = verify_attn_masked_fp32(q, k, v, pos, T)
    assert torch.allclose(a, b, atol=1e-5, rtol=1e-5)


def test_epilogue_restatement_matches_transformers():
    """The decode-step epilogues restated (oracle/epilogue.py) against Transformers' own modules:
    Qwen3RMSNorm after a bf16 residual add, and Qwen3MLP's act_fn(gate) * up."""
    from transformers import Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm
    from oracle.epilogue import add_rms_norm_ref, silu_mul_ref
    g = torch.Generator().manual_seed(4)
    M, N, I = 5, 256, 96
    res = torch.randn(M, N, generator=g).to(torch.bfloat16)
    delta = torch.randn(M, N, generator=g).to(torch.bfloat16)
    norm = Qwen3RMSNorm(N, eps=1e-6)
    with torch.no_grad():
        norm.weight.copy_((1 + 0.1 * torch.randn(N, generator=g)).to(torch.float32))
    norm = norm.to(torch.bfloat16)
    new_res, y = add_rms_norm_ref(res, delta, norm.weight.data, 1e-6)
    want_res = res + delta
    assert torch.equal(new_res, want_res)
    assert torch.equal(y, norm(want_res))
    gu = torch.randn(M, 2 * I, generator=g).to(torch.bfloat16)
    act = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
    assert torch.equal(silu_mul_ref(gu), act)
    del Qwen3Config


def test_gemv_restatement_matches_transformers_layers():
    """gemv_ref's epilogues against the modules they replace, on CPU in bf16: Qwen3MLP's
    down(act_fn(gate(x)) * up(x)) with the residual add of Qwen3DecoderLayer, and the LM head's
    greedy argmax. Only fp32 summation order differs (Transformers' bf16 Linear vs one fp32
    matmul), so a bf16 rounding may flip in a few elements, by one ulp."""
    from transformers import Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import Qwen3MLP
    from oracle.epilogue import GEMV_ARGMAX, GEMV_BF16, GEMV_RESID, GEMV_SWIGLU, gemv_ref
    g = torch.Generator().manual_seed(6)
    M, H, I, V = 6, 256, 512, 1000 - 1000 % 64
    cfg = Qwen3Config(hidden_size=H, intermediate_size=I, hidden_act="silu")
    mlp = Qwen3MLP(cfg).to(torch.bfloat16)
    with torch.no_grad():
        for lin in (mlp.gate_proj, mlp.up_proj, mlp.down_proj):
            lin.weight.copy_(torch.randn(lin.weight.shape, generator=g) * lin.weight.shape[1] ** -0.5)
    x = torch.randn(M, H, generator=g).to(torch.bfloat16)
    h = torch.randn(M, H, generator=g).to(torch.bfloat16)
    with torch.no_grad():
        act_want = mlp.act_fn(mlp.gate_proj(x)) * mlp.up_proj(x)
        h_want = h + mlp.down_proj(act_want)
    gu = torch.cat([mlp.gate_proj.weight, mlp.up_proj.weight], 0)
    act = gemv_ref(x, gu.data, GEMV_SWIGLU)
    h_new = gemv_ref(act_want, mlp.down_proj.weight.data, GEMV_RESID, h)

    def close(a, b, frac):
        d = (a.float() - b.float()).abs()
        assert bool((d <= (a.float().abs() + b.float().abs()) * 2.0 ** -7 + 1e-6).all())
        assert float((d > 0).float().mean()) <= frac
    close(act, act_want, 0.03)
    close(h_new, h_want, 0.03)
    lm = torch.randn(V, H, generator=g).to(torch.bfloat16) * H ** -0.5
    logits = gemv_ref(x, lm, GEMV_BF16)
    want = torch.nn.functional.linear(x, lm).argmax(dim=-1)
    got = gemv_ref(x, lm, GEMV_ARGMAX)
    assert bool((logits.float().gather(1, got[:, None]) >= logits.float().gather(1, want[:, None]) - 1e-2).all())
    # ties: the first index among equal bf16 logits, as torch.argmax
    w = torch.zeros(128, 4, dtype=torch.bfloat16)
    w[[9, 40, 77]] = 1.0
    assert gemv_ref(torch.ones(2, 4, dtype=torch.bfloat16), w, GEMV_ARGMAX).tolist() == [9, 9]
