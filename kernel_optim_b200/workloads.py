"""Seeded synthetic inputs for the decode-attention configurations, and their algorithmic bytes.

The reference quotes no dataset for this path; the BASELINE configurations name shapes and value
distributions, which these generators reproduce with fixed seeds:

  c1  B=1,  512 cached keys, q/K/V N(0,1) bf16, attention only (no append), keys 0..511.
  c2  B=16, 4096 cached keys + 1 appended (pos 4096); raw q/k/v of the new token N(0,1) go through
      per-head RMSNorm (unit weights, eps 1e-6) and RoPE (theta 5e6) at position 4096.
  c3  B=64, cached lengths ~ U[1024, 32768] (seeded), 16-token pages, block table = random
      permutation of the pool, prologue fused.
  c4  B=4, 131071 cached + 1 appended = 131072 keys per sequence, prologue fused.
  c5  end-to-end engine (kernel_optim_b200.engine), not built here.
  v3, v5, v7  verify (T = 3, 5, 7 query tokens per sequence, causal among themselves; the draft
      lengths engine.py:48-56 picks for B <= 32, 16, 4): c2's shape, B=16, 4096 cached keys + the T
      new ones already in the cache, roped q [B*T, nq*128] N(0,1).

Algorithmic bytes of one call (the roofline numerator):
  sum_b keys_b * nkv * 128 * 2 B * 2 (K and V)  +  B * nq * 128 * 2 (out write)
  + unfused: B * T * nq * 128 * 2 (q read; T query tokens per sequence, out likewise)
  + fused:   B * (nq + 2 nkv) * 128 * 2 (qkv read) + B * 2 * nkv * 128 * 2 (K/V append write)
Page-table reads and split scratch are overhead, not counted.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from .paged import PAGE, PagedKVCache

D = 128
NQ, NKV = 32, 8
EPS = 1e-6
THETA = 5e6


def rope_tables(n: int, device, theta: float = THETA):
    """cos/sin [n, 128] bf16 from Transformers' Qwen3RotaryEmbedding, exactly as the reference
    engine builds its tables (engine/engine.py:164-171)."""
    from transformers import Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding
    cfg = Qwen3Config(hidden_size=NQ * D, num_attention_heads=NQ, num_key_value_heads=NKV,
                      head_dim=D, rope_theta=theta, max_position_embeddings=max(n, 32768),
                      num_hidden_layers=1, intermediate_size=64, vocab_size=64)
    rot = Qwen3RotaryEmbedding(cfg)
    dummy = torch.empty(1, dtype=torch.bfloat16)
    cos, sin = rot(dummy, torch.arange(n).unsqueeze(0))
    return cos[0].contiguous().to(device), sin[0].contiguous().to(device)


@dataclass
class Case:
    name: str
    B: int
    cached: list[int]            # tokens already in the cache per sequence
    fused: bool                  # new token appended through the prologue
    nq: int = NQ
    nkv: int = NKV
    T: int = 1                   # query tokens per sequence (verify when > 1)
    tensors: dict = field(default_factory=dict)

    @property
    def keys(self) -> list[int]:
        """Keys attended per sequence."""
        return [c + 1 for c in self.cached] if self.fused else list(self.cached)

    def algorithmic_bytes(self) -> int:
        kv = sum(self.keys) * self.nkv * D * 2 * 2
        out = self.B * self.T * self.nq * D * 2
        if self.fused:
            extra = self.B * (self.nq + 2 * self.nkv) * D * 2 + self.B * 2 * self.nkv * D * 2
        else:
            extra = self.B * self.T * self.nq * D * 2
        return kv + out + extra


def case_shape(name: str, seed: int = 0, batch_scale: int = 1, kv_shard: int = 1) -> Case:
    """Shapes and lengths of a configuration. batch_scale multiplies B (weak scaling);
    kv_shard divides the kv heads (KV-head sharding across ranks)."""
    g = torch.Generator().manual_seed(seed + 1000)
    nkv = NKV // kv_shard
    if name == "c1":
        return Case("c1", 1 * batch_scale, [512] * batch_scale, False, NQ // kv_shard, nkv)
    if name == "c2":
        B = 16 * batch_scale
        return Case("c2", B, [4096] * B, True, NQ // kv_shard, nkv)
    if name == "c3":
        B = 64 * batch_scale
        lens = torch.randint(1024, 32769, (B,), generator=g).tolist()
        return Case("c3", B, lens, True, NQ // kv_shard, nkv)
    if name == "c4":
        B = 4 * batch_scale
        return Case("c4", B, [131071] * B, True, NQ // kv_shard, nkv)
    if name in ("v3", "v5", "v7"):
        T = int(name[1])
        B = 16 * batch_scale
        return Case(name, B, [4096 + T] * B, False, NQ // kv_shard, nkv, T)
    raise ValueError(f"unknown decode-attention config {name!r}")


def build_case(name: str, device, seed: int = 0, paged: bool = True, batch_scale: int = 1,
               kv_shard: int = 1, kv_rank: int = 0, layers: int = 1) -> Case:
    """Materialise a configuration on `device` (seeded). For kv_shard > 1 the tensors are rank
    kv_rank's slice: its kv heads, their query heads and its part of the cache, drawn from the same
    global stream so every rank's slice is a slice of the unsharded inputs."""
    case = case_shape(name, seed, batch_scale, kv_shard)
    dev = torch.device(device)
    B, nq_l, nkv_l = case.B, case.nq, case.nkv
    h0 = kv_rank * nkv_l
    gen = torch.Generator(device=dev).manual_seed(seed)
    bf = torch.bfloat16
    max_keys = max(case.keys)
    t = case.tensors
    if case.fused:
        # full qkv row for the global heads, then this rank's slice [q heads | k heads | v heads]
        full = torch.randn(B, (NQ + 2 * NKV) * D, generator=gen, device=dev, dtype=torch.float32).to(bf)
        q = full[:, h0 * 4 * D:(h0 + nkv_l) * 4 * D]
        k = full[:, (NQ + h0) * D:(NQ + h0 + nkv_l) * D]
        v = full[:, (NQ + NKV + h0) * D:(NQ + NKV + h0 + nkv_l) * D]
        t["qkv"] = torch.cat([q, k, v], 1).contiguous()
        t["q_norm_w"] = torch.ones(D, dtype=bf, device=dev)
        t["k_norm_w"] = torch.ones(D, dtype=bf, device=dev)
        t["cos"], t["sin"] = rope_tables(max_keys, dev)
    else:
        full = torch.randn(B * case.T, NQ * D, generator=gen, device=dev, dtype=torch.float32).to(bf)
        t["q"] = full[:, h0 * 4 * D:(h0 + nkv_l) * 4 * D].contiguous()
    t["pos"] = torch.tensor([c if case.fused else c - case.T for c in case.cached], dtype=torch.int32,
                            device=dev)
    if paged:
        n_pages = sum((k_ + PAGE - 1) // PAGE for k_ in case.keys)
        cache = PagedKVCache(layers, n_pages, nkv_l, D, B, max_keys, dev)
        cache.assign_permuted(case.keys, torch.Generator().manual_seed(seed + 7))
        for layer in range(layers):
            _fill_pages(cache, layer, case, gen, h0)
        t["cache"] = cache
    else:
        kc = torch.zeros(layers, B, nkv_l, max_keys, D, dtype=bf, device=dev)
        vc = torch.zeros_like(kc)
        for layer in range(layers):
            for b in range(B):
                L = case.cached[b]
                kk = torch.randn(NKV, L, D, generator=gen, device=dev, dtype=torch.float32)
                vv = torch.randn(NKV, L, D, generator=gen, device=dev, dtype=torch.float32)
                kc[layer, b, :, :L] = kk[h0:h0 + nkv_l].to(bf)
                vc[layer, b, :, :L] = vv[h0:h0 + nkv_l].to(bf)
        t["k_cache"], t["v_cache"] = kc, vc
    return case


def _fill_pages(cache: PagedKVCache, layer: int, case: Case, gen, h0: int) -> None:
    """Cached tokens N(0,1), written sequence by sequence in the same stream order as the
    contiguous layout uses, so paged and contiguous builds of one seed hold identical values."""
    bf = torch.bfloat16
    nkv_l = case.nkv
    dev = cache.device
    for b in range(case.B):
        L = case.cached[b]
        kk = torch.randn(NKV, L, D, generator=gen, device=dev, dtype=torch.float32)
        vv = torch.randn(NKV, L, D, generator=gen, device=dev, dtype=torch.float32)
        t = torch.arange(L, device=dev)
        pid = cache.block_table[b, t // PAGE].long()
        row = t % PAGE
        cache.k[layer][pid, :, row] = kk[h0:h0 + nkv_l].to(bf).permute(1, 0, 2)
        cache.v[layer][pid, :, row] = vv[h0:h0 + nkv_l].to(bf).permute(1, 0, 2)
