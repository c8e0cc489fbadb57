"""CPU restatement of the decode-step epilogues (test infrastructure; nothing in the product
imports it).

add_rms_norm follows engine/kernels/fused.py:16-37 (Transformers' Qwen3RMSNorm after the residual
add of Qwen3DecoderLayer); silu_mul follows fused.py:111-120 (Qwen3MLP's act_fn(gate) * up). All
arithmetic in fp32, rounded to bf16 where the reference rounds.
"""

from __future__ import annotations

import torch



def bf16r(t: torch.Tensor) -> torch.Tensor:
    """Round fp32 to bf16 (round to nearest even) and back."""
    return t.to(torch.bfloat16).float()


def add_rms_norm_ref(res: torch.Tensor, delta: torch.Tensor | None, weight: torch.Tensor, eps: float):
    """-> (new residual bf16, normed bf16)."""
    x = res.float()
    if delta is not None:
        x = bf16r(x + delta.float())                       # hidden = residual + hidden (bf16)
    var = (x * x).mean(-1, keepdim=True)
    normed = bf16r(x * torch.rsqrt(var + eps))             # hidden_states.to(input_dtype)
    y = bf16r(weight.float() * normed)                     # weight * hidden_states
    return x.to(torch.bfloat16), y.to(torch.bfloat16)


def silu_mul_ref(gu: torch.Tensor) -> torch.Tensor:
    I = gu.shape[1] // 2
    g, u = gu[:, :I].float(), gu[:, I:].float()
    s = bf16r(g / (1.0 + torch.exp(-g)))                   # act_fn(gate) in bf16
    return bf16r(s * u).to(torch.bfloat16)                 # * up, rounded
