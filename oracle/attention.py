"""Decode-attention oracles (test infrastructure; see oracle/__init__.py).

* decode_attn_fp32: the north-star oracle. torch scaled_dot_product_attention in fp32 on the CPU
  over keys 0..L_b-1 of each sequence, GQA (query head h reads kv head h // 4), scale 128^-0.5.
  The bf16 kernel output must lie within max-abs 2e-2 / mean-abs 2e-3 of it.
* reference_split_k: a numpy restatement of the reference's own algorithm,
  GodRishUniverse/kernel_optim engine/kernels/fused.py:138-234 -- the capacity-based split plan
  (fused.py:211-214), 64-key blocks with online softmax and p rounded to bf16 before p.v
  (fused.py:168-180), un-normalised partials (fused.py:182-185) and the LSE combine
  (fused.py:188-201). Small sizes only.
* gather_pages: paged pool + block table -> contiguous K/V.
"""

from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

from .bf16 import bf16r

D = 128


def decode_attn_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, lens) -> torch.Tensor:
    """q [B, nq, D]; k/v [B, nkv, >=max(lens), D]; lens [B] keys per sequence -> [B, nq, D] fp32."""
    B, nq, _ = q.shape
    out = torch.empty(B, nq, D, dtype=torch.float32)
    lens = [int(x) for x in torch.as_tensor(lens).cpu().tolist()]
    for b in range(B):
        L = lens[b]
        qb = q[b:b + 1].float().cpu().unsqueeze(2)                  # [1, nq, 1, D]
        kb = k[b:b + 1, :, :L].float().cpu()
        vb = v[b:b + 1, :, :L].float().cpu()
        o = F.scaled_dot_product_attention(qb, kb, vb, scale=D ** -0.5, enable_gqa=True)
        out[b] = o[0, :, 0]
    return out


def verify_attn_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, pos, T: int) -> torch.Tensor:
    """T query tokens per sequence, causal among themselves (engine/kernels/fused.py:130-185 with
    T > 1; rows laid out b * T + t as fused.py:137): query t of sequence b sees keys
    0 .. pos[b] + t. q [B*T, nq, D] -> [B*T, nq, D] fp32, one single-token oracle call per t."""
    B = len(pos)
    pos = [int(x) for x in torch.as_tensor(pos).cpu().tolist()]
    out = torch.empty(B * T, q.shape[1], D, dtype=torch.float32)
    qv = q.view(B, T, q.shape[1], D)
    for t in range(T):
        out.view(B, T, q.shape[1], D)[:, t] = decode_attn_fp32(qv[:, t], k, v, [p + t + 1 for p in pos])
    return out


def verify_attn_masked_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, pos, T: int) -> torch.Tensor:
    """The same in one SDPA call per sequence with an explicit boolean mask (query t may attend
    key i iff i <= pos[b] + t): an independent restatement to check verify_attn_fp32 against."""
    B = len(pos)
    pos = [int(x) for x in torch.as_tensor(pos).cpu().tolist()]
    nq = q.shape[1]
    out = torch.empty(B * T, nq, D, dtype=torch.float32)
    for b in range(B):
        L = pos[b] + T
        qb = q[b * T:(b + 1) * T].float().cpu().permute(1, 0, 2).unsqueeze(0)   # [1, nq, T, D]
        kb = k[b:b + 1, :, :L].float().cpu()
        vb = v[b:b + 1, :, :L].float().cpu()
        mask = torch.arange(L)[None, :] <= (pos[b] + torch.arange(T))[:, None]   # [T, L]
        o = F.scaled_dot_product_attention(qb, kb, vb, attn_mask=mask, scale=D ** -0.5, enable_gqa=True)
        out[b * T:(b + 1) * T] = o[0].permute(1, 0, 2)
    return out


def gather_pages(pool: torch.Tensor, table: torch.Tensor, b: int, L: int) -> torch.Tensor:
    """pool [num_pages, nkv, 16, D], table [B, max_pages] -> [nkv, L, D] for sequence b."""
    t = torch.arange(L)
    pid = table[b].cpu().long()[t // 16]
    return pool.cpu()[pid, :, t % 16].permute(1, 0, 2).contiguous()


def reference_plan(cap: int, B: int, nkv: int, target_ctas: int = 264, block_n: int = 64):
    """fused.py:211-214: NSPLIT and chunk from the capacity."""
    max_split = max(1, math.ceil(cap / 128))
    nsplit = max(1, min(max_split, math.ceil(target_ctas / (B * nkv))))
    chunk = math.ceil(math.ceil(cap / nsplit) / block_n) * block_n
    return math.ceil(cap / chunk), chunk


def reference_split_k(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, pos, cap: int,
                      target_ctas: int = 264, block_n: int = 64) -> torch.Tensor:
    """The reference's decode attention for T = 1, restated: q [B, nq, D] bf16; k/v
    [B, nkv, cap, D] bf16; pos [B] (keys 0..pos[b]). Returns bf16 [B, nq, D]."""
    B, nq, _ = q.shape
    nkv = k.shape[1]
    group = nq // nkv
    nsplit, chunk = reference_plan(cap, B, nkv, target_ctas, block_n)
    scale = np.float32(D ** -0.5)
    qf = q.float().cpu().numpy()
    kf = k.float().cpu().numpy()
    vf = v.float().cpu().numpy()
    pos = [int(x) for x in torch.as_tensor(pos).cpu().tolist()]
    out = np.empty((B, nq, D), np.float32)
    for b in range(B):
        p0 = pos[b]
        for kh in range(nkv):
            qr = qf[b, kh * group:(kh + 1) * group]                    # [4, D]
            parts = []
            for split in range(nsplit):
                start, end = split * chunk, min(split * chunk + chunk, p0 + 1)
                m = np.full(group, -1.0e30, np.float32)
                l = np.zeros(group, np.float32)
                acc = np.zeros((group, D), np.float32)
                for s0 in range(start, end, block_n):
                    idx = np.arange(s0, min(s0 + block_n, end))
                    s = (qr @ kf[b, kh, idx].T) * scale                # [4, n]
                    s = np.where(idx[None, :] <= p0, s, -np.inf).astype(np.float32)
                    m_new = np.maximum(m, s.max(axis=1))
                    alpha = np.exp(m - m_new).astype(np.float32)
                    p = np.exp(s - m_new[:, None]).astype(np.float32)
                    l = l * alpha + p.sum(axis=1)
                    acc = acc * alpha[:, None] + bf16r(p) @ vf[b, kh, idx]
                    m = m_new
                parts.append((m, l, acc))
            ms = np.stack([p_[0] for p_ in parts])                      # [S, 4]
            ls = np.stack([p_[1] for p_ in parts])
            os_ = np.stack([p_[2] for p_ in parts])                     # [S, 4, D]
            M = ms.max(axis=0)
            w = np.exp(ms - M[None]).astype(np.float32)
            L = (w * ls).sum(axis=0)
            out[b, kh * group:(kh + 1) * group] = (os_ * w[:, :, None]).sum(axis=0) / L[:, None]
    return torch.from_numpy(out).to(torch.bfloat16)


def compare(got: torch.Tensor, ref: torch.Tensor) -> tuple[float, float]:
    """(max-abs, mean-abs) of got - ref in fp32."""
    d = (got.float().cpu() - ref.float().cpu()).abs()
    return float(d.max()), float(d.mean())
