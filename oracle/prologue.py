"""QK-norm + RoPE + KV append, restated on the CPU (test infrastructure; see oracle/__init__.py).

Restates GodRishUniverse/kernel_optim engine/kernels/fused.py:54-96 (_qk_norm_rope_kernel):
for token row m (sequence b = m // T, position pos[b] + m % T) and head h of
qkv[M, (nq + 2 nkv) * 128]:
  q/k heads:  rstd = 1 / sqrt(sum(x^2) / 128 + eps)                 (fused.py:79)
              xn   = bf16(w * bf16(x * rstd))                         (fused.py:80-81)
              rh   = [-xn[64:], xn[:64]]                              (fused.py:82)
              y    = bf16(bf16(xn * cos[pos]) + bf16(rh * sin[pos]))  (fused.py:83-87)
              q -> q_out[m, h*128] (fused.py:88-89); k -> cache[b, h-nq, pos] (fused.py:90-92)
  v heads:    copied unchanged to cache[b, h-nq-nkv, pos]            (fused.py:93-96)

The reference reduces sum(x^2) with tl.sum, whose order is Triton's choice, and Transformers
(the native path, installed modeling_qwen3.py Qwen3RMSNorm) uses torch's CPU or CUDA reduction.
Neither order is fixed across platforms, so this restatement fixes one: per lane l (dims 4l..4l+3)
((x0^2 + x1^2) + x2^2) + x3^2, then an xor butterfly over 32 lanes with offsets 16, 8, 4, 2, 1.
The sm_100a kernel uses exactly this order, so kernel == restatement bit for bit; restatement vs
Transformers agrees to within one bf16 ulp on rare elements (tests measure the rate).
"""

from __future__ import annotations

import numpy as np
import torch

from .bf16 import bf16r, bits_to_f32, f32_to_bits, torch_to_bits

D = 128


def norm_rope_rows(x: np.ndarray, w: np.ndarray, cos: np.ndarray, sin: np.ndarray,
                   eps: float) -> np.ndarray:
    """x [R, 128] fp32 (bf16 values), w [128], cos/sin [R, 128] -> y [R, 128] fp32 (bf16 values)."""
    x = np.asarray(x, np.float32)
    sq = x * x
    lanes = sq.reshape(-1, 32, 4)
    acc = ((lanes[:, :, 0] + lanes[:, :, 1]) + lanes[:, :, 2]) + lanes[:, :, 3]
    idx = np.arange(32)
    for off in (16, 8, 4, 2, 1):
        acc = acc + acc[:, idx ^ off]
    var = acc[:, 0] * np.float32(1.0 / D)
    rstd = np.float32(1.0) / np.sqrt(var + np.float32(eps))
    xs = bf16r(x * rstd[:, None])
    xn = bf16r(np.asarray(w, np.float32)[None, :] * xs)
    rh = np.concatenate([-xn[:, D // 2:], xn[:, : D // 2]], axis=1)
    return bf16r(bf16r(xn * cos) + bf16r(rh * sin))


def qk_norm_rope_ref(qkv: torch.Tensor, q_w: torch.Tensor, k_w: torch.Tensor, cos: torch.Tensor,
                     sin: torch.Tensor, pos, T: int, nq: int, nkv: int, eps: float):
    """Restatement of fused.py:54-106 on bf16 torch tensors (any device; computed on CPU).

    Returns (q_out [M, nq*128], k_new [M, nkv, 128], v_new [M, nkv, 128]) as bf16 CPU tensors and
    positions [M] int64 (where row m's K/V go in the cache).
    """
    qkv_b = torch_to_bits(qkv)
    M = qkv_b.shape[0]
    pos = np.asarray(torch.as_tensor(pos).cpu(), dtype=np.int64)
    positions = pos[np.arange(M) // T] + np.arange(M) % T
    x = bits_to_f32(qkv_b).reshape(M, nq + 2 * nkv, D)
    cos_f = bits_to_f32(torch_to_bits(cos))[positions]           # [M, 128]
    sin_f = bits_to_f32(torch_to_bits(sin))[positions]
    qwf = bits_to_f32(torch_to_bits(q_w))
    kwf = bits_to_f32(torch_to_bits(k_w))
    q = norm_rope_rows(x[:, :nq].reshape(-1, D), qwf, np.repeat(cos_f, nq, 0),
                       np.repeat(sin_f, nq, 0), eps).reshape(M, nq * D)
    k = norm_rope_rows(x[:, nq:nq + nkv].reshape(-1, D), kwf, np.repeat(cos_f, nkv, 0),
                       np.repeat(sin_f, nkv, 0), eps).reshape(M, nkv, D)
    v = x[:, nq + nkv:]
    to_t = lambda a: torch.from_numpy(f32_to_bits(a).view(np.int16)).view(torch.bfloat16)
    return to_t(q), to_t(k), to_t(np.ascontiguousarray(v)), torch.from_numpy(positions)


# ------------------------------------------------------------------ the native path (Transformers)
def _qwen3_config(theta: float = 5e6, eps: float = 1e-6, nq: int = 32, nkv: int = 8):
    from transformers import Qwen3Config
    return Qwen3Config(hidden_size=2560, num_attention_heads=nq, num_key_value_heads=nkv,
                       head_dim=D, rope_theta=theta, rms_norm_eps=eps, max_position_embeddings=262144,
                       num_hidden_layers=1, intermediate_size=64, vocab_size=64)


def rope_tables(n: int, theta: float = 5e6):
    """cos/sin [n, 128] bf16 exactly as the reference builds them (engine/engine.py:164-171):
    Transformers' Qwen3RotaryEmbedding evaluated on positions 0..n-1 with a bf16 dummy."""
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding
    rot = Qwen3RotaryEmbedding(_qwen3_config(theta))
    dummy = torch.empty(1, dtype=torch.bfloat16)
    cos, sin = rot(dummy, torch.arange(n).unsqueeze(0))
    return cos[0].contiguous(), sin[0].contiguous()


def transformers_prologue(qkv: torch.Tensor, q_w: torch.Tensor, k_w: torch.Tensor,
                          cos: torch.Tensor, sin: torch.Tensor, positions, nq: int, nkv: int,
                          eps: float):
    """The native path on CPU: Qwen3RMSNorm (q_norm / k_norm) then apply_rotary_pos_emb, the way
    Qwen3Attention.forward applies them (installed modeling_qwen3.py). Returns (q, k, v) bf16 with
    q [M, nq*128], k/v [M, nkv, 128]."""
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm, apply_rotary_pos_emb
    M = qkv.shape[0]
    x = qkv.detach().cpu().view(M, nq + 2 * nkv, D)
    qn = Qwen3RMSNorm(D, eps=eps).to(torch.bfloat16)
    kn = Qwen3RMSNorm(D, eps=eps).to(torch.bfloat16)
    with torch.no_grad():
        qn.weight.copy_(q_w.cpu())
        kn.weight.copy_(k_w.cpu())
        q = qn(x[:, :nq]).unsqueeze(2)                 # [M, nq, 1, D]
        k = kn(x[:, nq:nq + nkv]).unsqueeze(2)
        positions = torch.as_tensor(positions).long()
        c = cos.cpu()[positions].unsqueeze(1)          # [M, 1, D] -> unsqueeze_dim=1 in apply
        s = sin.cpu()[positions].unsqueeze(1)
        q, k = apply_rotary_pos_emb(q, k, c, s, unsqueeze_dim=1)
    return (q.reshape(M, nq * D).contiguous(), k.reshape(M, nkv, D).contiguous(),
            x[:, nq + nkv:].contiguous())
