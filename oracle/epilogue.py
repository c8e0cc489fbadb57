"""CPU restatement of the decode-step epilogues (test infrastructure; nothing in the product
imports it).

add_rms_norm follows engine/kernels/fused.py:16-37 (Transformers' Qwen3RMSNorm after the residual
add of Qwen3DecoderLayer); silu_mul follows fused.py:111-120 (Qwen3MLP's act_fn(gate) * up);
gemv_ref follows the epilogues of engine/kernels/gemv.py:86-105. All arithmetic in fp32, rounded to
bf16 where the reference rounds.
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


GEMV_F32, GEMV_BF16, GEMV_RESID, GEMV_SWIGLU, GEMV_ARGMAX = 0, 1, 2, 3, 4


def gemv_epilogue_ref(acc: torch.Tensor, epi: int, h: torch.Tensor | None = None) -> torch.Tensor:
    """The epilogues of gemv.py:86-105 applied to fp32 sums acc [M, N] ([M, 2N] gate|up for
    SWIGLU): acc (F32), bf16(acc) (BF16), bf16(h + bf16(acc)) (RESID, gemv.py:95-97),
    bf16(bf16(silu(bf16 g)) * bf16 u) (SWIGLU, gemv.py:101-105), or the int64 index of each row's
    largest bf16(acc), the first one among equal values (ARGMAX: engine.py:263's bf16 logits,
    then the greedy argmax)."""
    if epi == GEMV_F32:
        return acc
    if epi == GEMV_BF16:
        return acc.to(torch.bfloat16)
    if epi == GEMV_RESID:
        return bf16r(h.float() + bf16r(acc)).to(torch.bfloat16)
    if epi == GEMV_ARGMAX:
        logits = bf16r(acc)
        top = logits.max(dim=1, keepdim=True).values
        cols = torch.arange(logits.shape[1]).expand_as(logits)
        return torch.where(logits == top, cols, logits.shape[1]).min(dim=1).values
    n = acc.shape[1] // 2
    g, u = bf16r(acc[:, :n]), bf16r(acc[:, n:])
    s = bf16r(g / (1.0 + torch.exp(-g)))
    return bf16r(s * u).to(torch.bfloat16)


def gemv_ref(x: torch.Tensor, w: torch.Tensor, epi: int, h: torch.Tensor | None = None) -> torch.Tensor:
    """x [M, K], w [N, K] ([2N, K] gate|up for SWIGLU), bf16 -> gemv_epilogue_ref of the fp32
    sums x . w^T."""
    return gemv_epilogue_ref(x.float() @ w.float().t(), epi, h)
