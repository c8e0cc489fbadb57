"""The reference's CPU path for one decode-attention step (test infrastructure / timed baseline).

The reference engine has no CPU implementation of this path (engine/engine.py:34 hard-codes
cuda:0). Its declared native path -- what its judge runs and what the engine must match -- is
Transformers' Qwen3Attention with attn_implementation="sdpa": per-head q_norm / k_norm
(Qwen3RMSNorm), apply_rotary_pos_emb, the KV-cache update at the new position, then
sdpa_attention_forward. In the pinned Transformers 4.51.3 that last step expands K/V with repeat_kv
before torch.nn.functional.scaled_dot_product_attention (engine/engine.py:97-99 describes this);
the installed 5.5.0 passes enable_gqa=True instead when there is no mask. Both forms are here; the
CPU baseline reports the pinned (repeat_kv) form and records the other in its sample text.
"""

from __future__ import annotations

import os
import time

import torch
import torch.nn.functional as F

D = 128


class CpuDecodeStep:
    """One decode-attention step of B sequences on the CPU, Transformers' way, on bf16 tensors."""

    def __init__(self, qkv, q_w, k_w, cos, sin, pos, k_ctx, v_ctx, nq, nkv, eps=1e-6,
                 form="repeat_kv"):
        from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm, apply_rotary_pos_emb, repeat_kv
        self._apply, self._repeat = apply_rotary_pos_emb, repeat_kv
        self.B, self.nq, self.nkv, self.form = qkv.shape[0], nq, nkv, form
        self.qkv = qkv.cpu()
        self.q_norm = Qwen3RMSNorm(D, eps).to(torch.bfloat16)
        self.k_norm = Qwen3RMSNorm(D, eps).to(torch.bfloat16)
        with torch.no_grad():
            self.q_norm.weight.copy_(q_w.cpu())
            self.k_norm.weight.copy_(k_w.cpu())
        self.pos = [int(p) for p in pos.cpu().tolist()]
        cap = max(self.pos) + 1
        self.k = torch.zeros(self.B, nkv, cap, D, dtype=torch.bfloat16)
        self.v = torch.zeros_like(self.k)
        for b, p in enumerate(self.pos):
            self.k[b, :, :p] = k_ctx[b][:, :p].cpu()
            self.v[b, :, :p] = v_ctx[b][:, :p].cpu()
        self.cos, self.sin = cos.cpu(), sin.cpu()

    @torch.no_grad()
    def __call__(self) -> torch.Tensor:
        B, nq, nkv = self.B, self.nq, self.nkv
        x = self.qkv.view(B, nq + 2 * nkv, D)
        q = self.q_norm(x[:, :nq]).unsqueeze(2)              # [B, nq, 1, D]
        k = self.k_norm(x[:, nq:nq + nkv]).unsqueeze(2)      # [B, nkv, 1, D]
        v = x[:, nq + nkv:].unsqueeze(2)
        out = torch.empty(B, nq, D, dtype=torch.bfloat16)
        for b, p in enumerate(self.pos):
            c = self.cos[p].view(1, 1, D)
            s = self.sin[p].view(1, 1, D)
            qb, kb = self._apply(q[b:b + 1], k[b:b + 1], c, s)
            self.k[b, :, p] = kb[0, :, 0]
            self.v[b, :, p] = v[b, :, 0]
            keys, vals = self.k[b:b + 1, :, :p + 1], self.v[b:b + 1, :, :p + 1]
            if self.form == "repeat_kv":
                keys, vals = self._repeat(keys, nq // nkv), self._repeat(vals, nq // nkv)
                o = F.scaled_dot_product_attention(qb, keys, vals, scale=D ** -0.5)
            else:
                o = F.scaled_dot_product_attention(qb, keys, vals, scale=D ** -0.5, enable_gqa=True)
            out[b] = o[0, :, 0]
        return out


def time_steps(step: CpuDecodeStep, steps: int, warmup: int) -> float:
    """Seconds for `steps` calls after `warmup` untimed calls (all host threads)."""
    torch.set_num_threads(os.cpu_count() or 1)
    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    return time.perf_counter() - t0
