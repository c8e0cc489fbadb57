"""Write the golden fixtures in tests/golden/ from the reference's native path.

Run from the repository root:  python tests/golden/make_golden.py

The reference (GodRishUniverse/kernel_optim) has no test vectors for decode attention and its
Triton kernels need a GPU. What it is judged against is Transformers' Qwen3 path
(QWEN_ENGINE_CONTRACT.md:105-123): Qwen3RMSNorm + Qwen3RotaryEmbedding + apply_rotary_pos_emb for
the prologue, torch scaled_dot_product_attention for attention. This script evaluates exactly those
on seeded inputs (CPU, installed Transformers and torch) and stores inputs and outputs as bf16/fp32
arrays, so that the oracle restatement and the GPU kernels can be checked against them without
re-running Transformers.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle.bf16 import torch_to_bits  # noqa: E402
from oracle.prologue import rope_tables, transformers_prologue  # noqa: E402

OUT = Path(__file__).resolve().parent
NQ, NKV, D, EPS = 32, 8, 128, 1e-6


def prologue_fixture():
    g = torch.Generator().manual_seed(1234)
    M, T = 24, 3                      # 8 sequences x 3 tokens (exercises pos[b] + m % T)
    qkv = torch.randn(M, (NQ + 2 * NKV) * D, generator=g).to(torch.bfloat16)
    q_w = (1 + 0.25 * torch.randn(D, generator=g)).to(torch.bfloat16)
    k_w = (1 + 0.25 * torch.randn(D, generator=g)).to(torch.bfloat16)
    pos = torch.tensor([0, 1, 15, 16, 511, 4096, 70000, 131069], dtype=torch.int32)
    cos, sin = rope_tables(131072)
    positions = pos.long()[torch.arange(M) // T] + torch.arange(M) % T
    q, k, v = transformers_prologue(qkv, q_w, k_w, cos, sin, positions, NQ, NKV, EPS)
    np.savez_compressed(
        OUT / "prologue.npz", T=T, qkv=torch_to_bits(qkv), q_w=torch_to_bits(q_w),
        k_w=torch_to_bits(k_w), pos=pos.numpy(), cos_rows=torch_to_bits(cos[positions]),
        sin_rows=torch_to_bits(sin[positions]), positions=positions.numpy(),
        q=torch_to_bits(q), k=torch_to_bits(k), v=torch_to_bits(v))


def rope_fixture():
    cos, sin = rope_tables(131073)
    idx = np.array([0, 1, 2, 63, 64, 511, 512, 4095, 4096, 32767, 65536, 131071, 131072])
    np.savez_compressed(OUT / "rope.npz", idx=idx, cos=torch_to_bits(cos[idx]),
                        sin=torch_to_bits(sin[idx]))


def attention_fixture():
    """C1 (B=1, 512 keys) plus a ragged batch, fp32 SDPA on bf16 inputs, both SDPA forms.
    K/V are stored packed: the live tokens of every sequence, concatenated along the token axis."""
    g = torch.Generator().manual_seed(4321)
    cases = {}
    for name, lens in (("c1", [512]), ("ragged", [1, 15, 16, 17, 33, 64, 65, 40])):
        B = len(lens)
        q = torch.randn(B, NQ, D, generator=g).to(torch.bfloat16)
        ks = [torch.randn(NKV, L, D, generator=g).to(torch.bfloat16) for L in lens]
        vs = [torch.randn(NKV, L, D, generator=g).to(torch.bfloat16) for L in lens]
        out_gqa = torch.empty(B, NQ, D)
        out_rep = torch.empty(B, NQ, D)
        for b in range(B):
            qb = q[b:b + 1].float().unsqueeze(2)
            kb, vb = ks[b].float().unsqueeze(0), vs[b].float().unsqueeze(0)
            out_gqa[b] = F.scaled_dot_product_attention(qb, kb, vb, scale=D ** -0.5,
                                                        enable_gqa=True)[0, :, 0]
            # Transformers' repeat_kv form (the pinned 4.51.3 sdpa path)
            kr, vr = kb.repeat_interleave(NQ // NKV, 1), vb.repeat_interleave(NQ // NKV, 1)
            out_rep[b] = F.scaled_dot_product_attention(qb, kr, vr, scale=D ** -0.5)[0, :, 0]
        cases[name] = dict(lens=np.array(lens), q=torch_to_bits(q),
                           k=torch_to_bits(torch.cat(ks, 1)), v=torch_to_bits(torch.cat(vs, 1)),
                           out_gqa=out_gqa.numpy(), out_rep=out_rep.numpy())
    np.savez_compressed(OUT / "attention.npz",
                        **{f"{n}_{key}": val for n, c in cases.items() for key, val in c.items()})


if __name__ == "__main__":
    prologue_fixture()
    rope_fixture()
    attention_fixture()
    for f in sorted(OUT.glob("*.npz")):
        print(f.name, f.stat().st_size)
