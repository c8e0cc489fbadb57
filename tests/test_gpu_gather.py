"""GPU: the decode-attention step with its all-gather fused over NVLink (kernel_optim_b200/gather.py).

Rank r of G runs attention for its kv heads (KV-head sharding) through
kopt_decode_attn_fused_gather; its rows land in every rank's gathered buffer. Checks:

* the gathered buffer is identical on every rank, and rank r's columns are bit-identical to what
  the plain fused entry point writes for the same rank-local inputs (same plan, same arithmetic);
* the gathered rows match the unsharded single-GPU step within the bf16 tolerance;
* the same holds when the calls are captured in a CUDA graph (odd number of calls, slot rotation)
  and replayed, and no wait runs out (error bits stay 0).

World 1 runs in-process on one GPU (the kernel's last CTA raises its own flag and finds it up).
World 2 runs as two processes on two GPUs and is skipped with fewer GPUs.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
MAX_ABS, MEAN_ABS = 2e-2, 2e-3
LAYERS = 3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_run(rank, world, dev):
    """Eager calls, then a graph of LAYERS calls replayed twice. Returns (gathered rows per eager
    call, per replay and call, rank-local rows of the plain entry point per call, error bits)."""
    from kernel_optim_b200.gather import PeerGather, slot_of
    from kernel_optim_b200.paged import PagedDecodeAttention
    from kernel_optim_b200.workloads import build_case

    case = build_case("c2", dev, seed=0, paged=True, kv_shard=world, kv_rank=rank, layers=LAYERS)
    t = case.tensors
    B, nq_l, nkv_l = case.B, case.nq, case.nkv
    cache = t["cache"]
    attn = PagedDecodeAttention(B, nq_l, nkv_l, 128, dev, cache.capacity)
    pg = PeerGather(B, world * nq_l * 128, dev)
    args = (t["qkv"], t["q_norm_w"], t["k_norm_w"], t["cos"], t["sin"], cache)
    try:
        local = []
        for layer in range(LAYERS):
            out = torch.empty(B, nq_l * 128, dtype=torch.bfloat16, device=dev)
            attn(*args, layer, t["pos"], out)
            local.append(out)
        eager = []
        for layer in range(LAYERS):
            g = pg.attend(attn, *args, layer, t["pos"], slot_of(layer, LAYERS))
            eager.append(g.clone())
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        snaps = [torch.empty(B, world * nq_l * 128, dtype=torch.bfloat16, device=dev)
                 for _ in range(LAYERS)]
        with torch.cuda.graph(graph):
            for layer in range(LAYERS):
                g = pg.attend(attn, *args, layer, t["pos"], slot_of(layer, LAYERS))
                snaps[layer].copy_(g)
        graphed = []
        for _ in range(2):
            graph.replay()
            graphed.append([x.clone() for x in snaps])
        torch.cuda.synchronize(dev)
        err = attn.read_error()
        del graph
        return ([x.cpu() for x in eager], [[x.cpu() for x in r] for r in graphed],
                [x.cpu() for x in local], err)
    finally:
        pg.close()


def _np(x):
    """bf16 tensor -> int16 array: pickled by value, unlike a tensor sent through a queue (whose
    shared-memory handle dies with the sending process)."""
    return x.view(torch.int16).numpy()


def _tensor(a):
    return torch.from_numpy(a).view(torch.bfloat16)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        eager, graphed, local, err = _rank_run(rank, world, torch.device("cuda", rank))
        q.put((rank, ([_np(x) for x in eager], [[_np(x) for x in r] for r in graphed],
                      [_np(x) for x in local], err)))
    except Exception as e:  # surfaced by the parent
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def _unsharded(dev):
    from kernel_optim_b200.paged import PagedDecodeAttention
    from kernel_optim_b200.workloads import build_case
    case = build_case("c2", dev, seed=0, paged=True, layers=LAYERS)
    t = case.tensors
    attn = PagedDecodeAttention(case.B, case.nq, case.nkv, 128, dev, t["cache"].capacity)
    outs = []
    for layer in range(LAYERS):
        out = torch.empty(case.B, case.nq * 128, dtype=torch.bfloat16, device=dev)
        attn(t["qkv"], t["q_norm_w"], t["k_norm_w"], t["cos"], t["sin"], t["cache"], layer, t["pos"],
             out)
        outs.append(out.cpu())
    torch.cuda.synchronize(dev)
    assert attn.read_error() == 0
    return outs


def _check(results, world, full):
    W = results[0][2][0].shape[1]
    for r in range(world):
        eager, graphed, _, err = results[r]
        assert err == 0, f"rank {r}: device error bits {err}"
        assert eager[0].shape[1] == world * W
        for layer in range(LAYERS):
            ref = torch.cat([results[w][2][layer] for w in range(world)], 1)
            assert torch.equal(eager[layer], ref), f"rank {r} layer {layer}: eager gather differs"
            for rep in graphed:
                assert torch.equal(rep[layer], ref), f"rank {r} layer {layer}: graph replay differs"
            d = (eager[layer].float() - full[layer].float()).abs()
            assert float(d.max()) <= MAX_ABS and float(d.mean()) <= MEAN_ABS


def test_fused_gather_world1_matches_plain_step():
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()))
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        res = _rank_run(0, 1, torch.device("cuda:0"))
    finally:
        dist.destroy_process_group()
    _check({0: res}, 1, _unsharded(torch.device("cuda:0")))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_gather_two_ranks_over_nvlink():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        results = dict(q.get(timeout=300) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert not isinstance(results[r], str), f"rank {r}: {results[r]}"
    assert all(p.exitcode == 0 for p in procs)
    results = {r: ([_tensor(a) for a in e], [[_tensor(a) for a in x] for x in g],
                   [_tensor(a) for a in lo], err) for r, (e, g, lo, err) in results.items()}
    _check(results, world, _unsharded(torch.device("cuda:0")))


def test_gather_flag_wait_runs_out_on_one_gpu():
    """The fused gather's bounded flag wait, made to run out on purpose without a second GPU: a
    world-2 descriptor whose "peer" buffers are a second local allocation that no kernel ever
    signals. The call must complete, set KOPT_DEV_ERR_TIMEOUT (and nothing else), still store this
    rank's rows into both buffers and raise its flag in both flag arrays; after the error word is
    read and cleared, a world-1 call on the same workspace is correct again. While the timeout bit
    is still unread, a further call (bound 1 s) raises its flags but does not wait: it ends in far
    less than its bound. Nothing hangs: the waits are bounded at 5 ms and 1 s (the descriptor's
    wait_ns)."""
    import ctypes

    from kernel_optim_b200 import _lib
    from kernel_optim_b200.fused import _ptr, _stream
    from kernel_optim_b200.paged import PagedDecodeAttention
    from kernel_optim_b200.workloads import build_case

    dev = torch.device("cuda:0")
    case = build_case("c2", dev, seed=5, paged=True, kv_shard=2, kv_rank=0, layers=1)
    t = case.tensors
    B, nq_l, nkv_l = case.B, case.nq, case.nkv
    cache = t["cache"]
    attn = PagedDecodeAttention(B, nq_l, nkv_l, 128, dev, cache.capacity)
    args = (t["qkv"], t["q_norm_w"], t["k_norm_w"], t["cos"], t["sin"], cache)
    plain = torch.empty(B, nq_l * 128, dtype=torch.bfloat16, device=dev)
    attn(*args, 0, t["pos"], plain)
    torch.cuda.synchronize(dev)
    assert attn.read_error() == 0
    row = 2 * nq_l * 128
    outs = [torch.zeros(B, row, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    flags = [torch.zeros(64, dtype=torch.int32, device=dev) for _ in range(2)]
    epoch = torch.zeros(64, dtype=torch.int32, device=dev)

    def call(world, wait_ns):
        g = _lib.Gather()
        for w in range(world):
            g.out[w], g.flags[w] = outs[w].data_ptr(), flags[w].data_ptr()
        g.epoch, g.rank, g.world, g.row_elems, g.wait_ns = epoch.data_ptr(), 0, world, row, wait_ns
        _lib.check(_lib.lib().kopt_decode_attn_fused_gather(
            ctypes.byref(attn.plan), _ptr(t["qkv"]), _ptr(t["q_norm_w"]), _ptr(t["k_norm_w"]),
            _ptr(t["cos"]), _ptr(t["sin"]), t["cos"].shape[0], ctypes.byref(attn._cache(cache, 0)),
            _ptr(t["pos"]), ctypes.byref(g), None, _ptr(attn.ws), ctypes.c_float(attn.scale),
            ctypes.c_float(attn.eps), _stream(dev)), "kopt_decode_attn_fused_gather")

    call(2, 5_000_000)
    torch.cuda.synchronize(dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record()
    call(2, 1_000_000_000)   # the unread timeout bit: flags raised, no second wait
    ev[1].record()
    torch.cuda.synchronize(dev)
    assert ev[0].elapsed_time(ev[1]) < 100.0, f"{ev[0].elapsed_time(ev[1]):.1f} ms"
    assert attn.read_error() == _lib.DEV_ERR_TIMEOUT   # read_error also clears the word
    for w in range(2):
        assert torch.equal(outs[w][:, : nq_l * 128], plain), f"rows missing in buffer {w}"
        assert int(flags[w][0]) == 2, f"flag not raised in array {w}"
    assert int(flags[0][1]) == 0 and int(epoch[0]) == 2
    outs[0].zero_()
    flags[0].zero_()
    epoch.zero_()
    call(1, 0)   # default bound; its own flag is the only one it waits for
    torch.cuda.synchronize(dev)
    assert attn.read_error() == 0
    assert torch.equal(outs[0][:, : nq_l * 128], plain)
