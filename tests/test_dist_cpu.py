"""CPU, 2 gloo ranks: the KV-head sharding glue of the multi-GPU step (kernel_optim_b200/shard.py).

Each rank projects qkv with its shard of the fused QKV weight, runs attention for its kv heads
(here the CPU oracle stands in for the kernel) and all-gathers the head outputs; the result must be
the unsharded attention output, identically on every rank.
"""

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kernel_optim_b200.shard import gather_heads, head_range, shard_qkv_weight
from oracle.attention import decode_attn_fp32

NQ, NKV, D, H = 32, 8, 128, 64


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    g = torch.Generator().manual_seed(0)
    B, L = 3, 40
    x = torch.randn(B, H, generator=g)
    wq = torch.randn(NQ * D, H, generator=g) / 8
    wk = torch.randn(NKV * D, H, generator=g) / 8
    wv = torch.randn(NKV * D, H, generator=g) / 8
    k = torch.randn(B, NKV, L, D, generator=g)
    v = torch.randn(B, NKV, L, D, generator=g)
    lens = [40, 17, 1]
    return x, wq, wk, wv, k, v, lens


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, wq, wk, wv, k, v, lens = _inputs()
        B = x.shape[0]
        h0, h1 = head_range(NKV, rank, world)
        w = shard_qkv_weight(wq, wk, wv, NKV, rank, world, D)
        qkv = x @ w.t()                                    # this rank's [q heads | k heads | v heads]
        nq_l = (h1 - h0) * 4
        qh = qkv[:, :nq_l * D].reshape(B, nq_l, D)
        # the projected k/v of this rank's heads equal the matching rows of the full projection
        assert torch.allclose(qkv[:, nq_l * D:(nq_l + (h1 - h0)) * D], (x @ wk.t())[:, h0 * D:h1 * D])
        local = decode_attn_fp32(qh, k[:, h0:h1], v[:, h0:h1], lens).reshape(B, -1)
        out = gather_heads(local, torch.empty(world, B, local.shape[1]))
        q.put((rank, out.numpy()))   # by value: a queued tensor's shared memory dies with its sender
    finally:
        dist.destroy_process_group()


def test_kv_head_shard_and_gather_reproduce_unsharded_attention():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        results = {r: torch.from_numpy(a) for r, a in (q.get(timeout=120) for _ in range(world))}
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    x, wq, wk, wv, k, v, lens = _inputs()
    B = x.shape[0]
    full = decode_attn_fp32((x @ wq.t()).reshape(B, NQ, D), k, v, lens).reshape(B, -1)
    for r in range(world):
        assert torch.equal(results[r], results[0])
    assert torch.allclose(results[0], full, atol=1e-5)
