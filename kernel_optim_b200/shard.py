"""KV-head sharding of the decode-attention step across G ranks (one GPU each).

Rank r owns kv heads [r*nkv/G, (r+1)*nkv/G) and their 4*nkv/G query heads: its rows of the q, k and
v projection weights, its slice of the KV cache and its share of the attention work. After
attention every rank holds [B, (nq/G)*128]; one all-gather over the group rebuilds the full
[B, nq*128] in head order, because rank-major order of contiguous head blocks is head order. o_proj,
the MLP, the LM head and argmax are then replicated, so every rank produces the same tokens.
"""

from __future__ import annotations

import torch

from .comm import collective


def head_range(nkv: int, rank: int, world: int) -> tuple[int, int]:
    """kv heads [h0, h1) of `rank`."""
    if nkv % world:
        raise ValueError(f"{nkv} kv heads do not shard over {world} ranks")
    per = nkv // world
    return rank * per, (rank + 1) * per


def shard_qkv_weight(q_w: torch.Tensor, k_w: torch.Tensor, v_w: torch.Tensor, nkv: int, rank: int,
                     world: int, d: int = 128, group: int = 4) -> torch.Tensor:
    """This rank's fused QKV weight [(4 + 2) * (nkv/G) * d, hidden]: its query heads, then its k
    heads, then its v heads (the layout the fused attention step reads)."""
    h0, h1 = head_range(nkv, rank, world)
    return torch.cat([q_w[h0 * group * d:h1 * group * d], k_w[h0 * d:h1 * d], v_w[h0 * d:h1 * d]],
                     0).contiguous()


def gather_heads(local: torch.Tensor, out: torch.Tensor, group=None, watch=None) -> torch.Tensor:
    """All-gather [B, heads_l*d] from every rank into `out` [G, B, heads_l*d]; returns the
    [B, G*heads_l*d] head-ordered view. A failed or timed-out all-gather aborts the group and
    raises comm.CollectiveError (recorded in `watch`, a comm.PeerWatch, when given)."""
    G, B, W = out.shape
    collective(torch.distributed.all_gather_into_tensor, out.view(G * B, W), local.contiguous(),
               group=group, watch=watch, what="all-gather of the head outputs")
    return out.permute(1, 0, 2).reshape(B, G * W)
