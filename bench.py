#!/usr/bin/env python
"""Benchmark of the decode-attention hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c2]

A step is one decode-attention call of the engine (the fused QK-norm/RoPE/KV-append prologue plus
split-K GQA attention over the paged cache) for one batch. The default workload is BASELINE config
c2 (B=16, 4096 cached keys + 1 appended, 32 query / 8 kv heads, d=128) per GPU. For N > 1 the kv
heads are sharded 8/N per GPU and the batch grows to 16N (weak scaling: per-GPU work fixed), and
each step all-gathers the head outputs, as the engine does before o_proj: by default inside the
attention kernel, which stores its rows into every rank's buffer over NVLink and ends with a
bounded wait for the peers' flags (kernel_optim_b200/gather.py); `--gather nccl` uses an NCCL
all-gather after the kernel instead.

value: whole-job algorithmic bytes / device time (TB/s), inputs resident in HBM, back-to-back
launches timed with CUDA events on the launching stream, max over ranks. Each step reads a different
layer's cache (`--layers` caches in rotation, together far larger than the 126 MB L2).
e2e: the same metric through the public call with host buffers: each step copies the new token's
qkv and positions from pinned host memory, runs the step and copies the output back.
--impl reference: the reference's CPU path (Transformers' q/k norm + RoPE + sdpa, oracle/cpu_path.py)
on the same config, rank 0 only.

Other workloads: c3/c4 (longer contexts), v3/v5/v7 (the T > 1 verify step), c5 (the engine end to
end, tokens/s), p5 (the projections of one decode step on the skinny-GEMM kernel, TB/s) and f5
(the prefill attention of c5's prompts on the tcgen05 kernel, TFLOP/s).

The c2 line also carries `c4_strong`: config c4 (B=4, 131072 keys) strong-scaled over the N GPUs,
each keeping 8/N kv heads of every sequence, with the head outputs all-gathered in the kernel; its
`value` is the whole job's algorithmic bytes per call over the device time (max over ranks).
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode-attn achieved HBM TB/s (% of peak), us/call; Qwen3-4B decode tokens/s"
PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
TRAFFIC_FILE = ROOT / "profiles" / "ncu_traffic.json"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["c2", "c3", "c4", "c5", "v3", "v5", "v7", "p5", "f5"],
                    default="c2",
                    help="c2-c4: one decode-attention call per step; c5: the engine end to end")
    ap.add_argument("--layers", type=int, default=8, help="layer caches rotated across steps")
    ap.add_argument("--layout", choices=["paged", "contiguous"], default="paged")
    ap.add_argument("--gather", choices=["fused", "nccl"], default="fused",
                    help="N > 1: all-gather fused into the attention kernel (NVLink stores) or NCCL")
    ap.add_argument("--no-overlap", action="store_true",
                    help="launch without programmatic dependent launch (each call waits for the "
                         "previous kernel before it starts)")
    ap.add_argument("--p5-layers", type=int, default=36,
                    help="p5: transformer layers in the step (36 = Qwen3-4B; fewer for a small "
                         "profiling case)")
    ap.add_argument("--prefill", choices=["native", "transformers"], default="native",
                    help="c5: prefill on the row kernels + SDPA, or the Transformers forward")
    ap.add_argument("--no-gemv", action="store_true",
                    help="c5: cuBLAS GEMMs + separate SwiGLU / residual kernels instead of the "
                         "tcgen05 skinny-GEMM projections with fused epilogues (kopt_gemv)")
    ap.add_argument("--spec", action="store_true",
                    help="c5: speculative decoding (n-gram drafts + the T > 1 verify step), as the "
                         "reference's ENGINE_SPEC=1 (which this flag stands for; the variable works too)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-strong", action="store_true",
                    help="c2: skip the extra c4 strong-scaling measurement (key c4_strong)")
    ap.add_argument("--soak-ms", type=float, default=600.0,
                    help="untimed launches before the timed region, for the clock samples")
    return ap.parse_args()


# ----------------------------------------------------------------------------------- plumbing
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_dist(world, local):
    """NCCL group with a bounded timeout on every collective (kernel_optim_b200.comm)."""
    if world > 1:
        import torch.distributed as dist

        from kernel_optim_b200.comm import init_group
        torch.cuda.set_device(local)
        init_group("nccl", timeout_s=120, device=torch.device("cuda", local))
        return dist
    return None


def max_over_ranks(dist, x: float) -> float:
    if dist is None:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def tensor_peak():
    """Dense bf16 tensor peak: the measured cuBLAS burst figure (a kernel timed alone)."""
    try:
        p = json.loads(PEAKS_FILE.read_text())
        return float(p["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops, cuBLAS burst)"
    except Exception:
        return 1590.0, "fallback 1.59 PFLOP/s (no MEASURED_PEAKS.json)"


def peaks():
    try:
        p = json.loads(PEAKS_FILE.read_text())
        return float(p["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, torch copy_ burst)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback 6.65 TB/s (no MEASURED_PEAKS.json)"


def ncu_traffic(key: str):
    try:
        return json.loads(TRAFFIC_FILE.read_text()).get(key)
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples every 50 ms for this process's GPU."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.proc = None
        try:
            uuid = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", uuid, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, pw, reasons = [], [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                mx.append(float(f[1]))
                pw.append(float(f[2]))
            except ValueError:
                continue
            for n, val in zip(names, f[4:8]):
                if val.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "samples": len(sm),
                "power_w_max": max(pw), "reasons": sorted(reasons)}


# ------------------------------------------------------------------------------- our arm
class StepLauncher:
    """Prebuilt C-ABI arguments for every layer, so a step costs one ctypes call."""

    def __init__(self, case, attn, layers, out, qkv=None, pos=None, gather=None):
        from kernel_optim_b200 import _lib
        from kernel_optim_b200.fused import _ptr, contiguous_cache
        L = _lib.lib()
        self.gather = gather
        self.slot = 0
        self.verify = not case.fused   # T query tokens (v3/v5/v7): attention only
        if self.verify:
            self.fn = L.kopt_decode_attn
            self.dst = [_ptr(out)] * 2
        elif gather is None:
            self.fn = L.kopt_decode_attn_fused
            self.dst = [_ptr(out)] * 2
        else:
            self.fn = L.kopt_decode_attn_fused_gather
            self.dst = [ctypes.byref(gather.descriptor(s)) for s in range(2)]
        self.check = _lib.check
        t = case.tensors
        pos = t["pos"] if pos is None else pos
        if "cache" in t:
            self.descs = [t["cache"].descriptor(i) for i in range(layers)]
        else:
            self.descs = [contiguous_cache(t["k_cache"][i], t["v_cache"][i]) for i in range(layers)]
        self.pos = _ptr(pos)
        if self.verify:
            self.common = (ctypes.byref(attn.plan), _ptr(t["q"] if qkv is None else qkv))
            self.tail = (_ptr(attn.ws), ctypes.c_float(attn.scale))
        else:
            qkv = t["qkv"] if qkv is None else qkv
            self.common = (ctypes.byref(attn.plan), _ptr(qkv), _ptr(t["q_norm_w"]),
                           _ptr(t["k_norm_w"]), _ptr(t["cos"]), _ptr(t["sin"]), t["cos"].shape[0])
            self.tail = (None, _ptr(attn.ws), ctypes.c_float(attn.scale), ctypes.c_float(attn.eps))
        self.stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        self.layers = layers

    def result(self, out):
        """The buffer holding the last step's (gathered) output."""
        return out if self.gather is None else self.gather.out[self.slot]

    def __call__(self, step: int):
        if self.gather is not None:
            self.slot = self.gather.next_slot()
        rc = self.fn(*self.common, ctypes.byref(self.descs[step % self.layers]), self.pos,
                     self.dst[self.slot], *self.tail, self.stream)
        if rc:
            self.check(rc, "kopt_decode_attn_fused")


def run_ours(args):
    from kernel_optim_b200.comm import collective
    from kernel_optim_b200.paged import PagedDecodeAttention
    from kernel_optim_b200.workloads import build_case
    world, rank, local = dist_env()
    dist = init_dist(world, local)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    n = world
    case = build_case(args.workload, dev, seed=0, paged=args.layout == "paged", batch_scale=n,
                      kv_shard=n, kv_rank=rank, layers=args.layers)
    t = case.tensors
    B = case.B
    cap = t["cache"].capacity if "cache" in t else t["k_cache"].shape[3]
    # consecutive calls read different layers' caches, so each may overlap the previous one
    attn = PagedDecodeAttention(B, case.nq, case.nkv, 128, dev, cap, overlap_prev=not args.no_overlap,
                                T=case.T)
    out = torch.empty(B * case.T, case.nq * 128, dtype=torch.bfloat16, device=dev)
    fused_gather = n > 1 and args.gather == "fused" and case.T == 1   # the gather is T = 1 only
    nccl_gather = n > 1 and not fused_gather
    gathered = (torch.empty(n, B * case.T, case.nq * 128, dtype=torch.bfloat16, device=dev)
                if nccl_gather else None)
    pg = None
    if fused_gather:
        from kernel_optim_b200.gather import PeerGather
        pg = PeerGather(B, n * case.nq * 128, dev)
    launch = StepLauncher(case, attn, args.layers, out)          # attention alone (roofline)
    step_launch = StepLauncher(case, attn, args.layers, out, gather=pg) if pg else launch
    bytes_rank = case.algorithmic_bytes()
    bytes_job = bytes_rank * n

    def step(i):
        step_launch(i)
        if nccl_gather:
            collective(dist.all_gather_into_tensor, gathered.view(-1, gathered.shape[-1]), out,
                       what="all-gather of the head outputs")

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    err = attn.read_error()
    if err:
        raise RuntimeError(f"device error word {err} after warm-up")

    # soak: untimed launches so the clock samples see the GPU under this load. Every rank runs the
    # same number of steps (each step is a collective), sized from a short timed probe.
    n_soak = 0
    if args.soak_ms > 0:
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record()
        for i in range(8):
            step(i)
        p1.record()
        torch.cuda.synchronize()
        n_soak = int(max_over_ranks(dist, args.soak_ms / max(p0.elapsed_time(p1) / 8, 1e-3)))
    sampler = ClockSampler(local)
    for i in range(n_soak):
        step(i)
        if i % 64 == 63:
            torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.profiler.start()       # ncu --profile-from-start off captures the timed region only
    ev0.record()
    for i in range(args.steps):
        step(i)
    ev1.record()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    clocks = sampler.stop()
    if dist is not None:
        dist.barrier()
    ms = max_over_ranks(dist, ev0.elapsed_time(ev1))
    ms_step = ms / args.steps
    value_tbs = bytes_job / (ms_step * 1e-3) / 1e12

    # kernel-only duration (no collective) for the roofline, same stream, back-to-back launches
    torch.cuda.synchronize()
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k0.record()
    for i in range(args.steps):
        launch(i)
    k1.record()
    torch.cuda.synchronize()
    kern_ms = max_over_ranks(dist, k0.elapsed_time(k1)) / args.steps
    err = attn.read_error()
    if err:
        raise RuntimeError(f"device error word {err} after the timed region")

    peak, peak_src = peaks()
    achieved = bytes_rank / (kern_ms * 1e-3) / 1e9
    traffic = ncu_traffic(args.workload)
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "frac_of_8TBs_nominal": round(achieved / 8000, 4),
                "traffic": traffic, "peak_source": peak_src,
                "kernel": ("decode_attn_kernel<PAGED=1,FUSED=1>" if case.fused else
                           (f"verify_tc_kernel<PAGED=1> (T={case.T}, tcgen05)" if case.T > 4
                            else f"verify_attn_kernel<PAGED=1> (T={case.T})")),
                "kernel_us": round(kern_ms * 1e3, 2),
                "algorithmic_bytes_per_launch": bytes_rank}

    e2e = None if args.no_e2e else run_e2e(args, case, attn, out, gathered, pg, dist, bytes_job)
    strong = None
    if args.workload == "c2" and not args.no_strong and args.layout == "paged":
        strong = run_strong_c4(args, dist, n, rank, dev)
    cpu = None
    if n == 1 and rank == 0 and not args.no_cpu_baseline and args.layout == "paged" and case.fused:
        cpu = cpu_baseline(case, bytes_rank)

    line = {
        "metric": METRIC, "value": round(value_tbs, 4), "unit": "TB/s", "n_gpus": n,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
        "us_per_call": round(ms_step * 1e3, 2), "pct_of_peak": round(100 * value_tbs * 1e3 / (peak * n), 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) bf16 cache and new-token q/k/v, unit norm weights, "
                "Transformers Qwen3 RoPE tables (theta 5e6)",
        "config": {
            "workload": f"{args.workload} per GPU" + (f", weak-scaled x{n}" if n > 1 else ""),
            "B": B, "keys_per_seq": (max(case.keys) if len(set(case.keys)) == 1 else "ragged"),
            "q_heads_per_gpu": case.nq, "kv_heads_per_gpu": case.nkv, "head_dim": 128,
            "paged": args.layout == "paged", "page_size": 16, "layers_rotated": args.layers,
            "parallelism": (f"kv-head shard x{n} + all-gather fused into the kernel (NVLink stores)"
                            if fused_gather else f"kv-head shard x{n} + NCCL all-gather"
                            if n > 1 else "single GPU"),
            "l2": f"inputs larger than L2: {args.layers} layer caches of "
                  f"{bytes_rank / 1e6:.0f} MB read in rotation, one per step",
            "launch": "back-to-back C-ABI calls on one stream" + (
                "" if args.no_overlap else ", programmatic dependent launch (each call's split "
                "and first page copies overlap the previous call's end)"),
        },
        "roofline": roofline,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": args.steps,
        "clocks": clocks,
    }
    if strong is not None:
        line["c4_strong"] = strong
    if rank == 0:
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_strong_c4(args, dist, n, rank, dev):
    """Config c4 strong-scaled over the N ranks: B = 4 sequences of 131072 keys in total, rank r
    keeping kv heads [r 8/N, (r+1) 8/N) of every sequence (and their query heads), the head outputs
    all-gathered inside the kernel over NVLink (N > 1). Back-to-back calls over two layer caches,
    CUDA events on the launching stream, max over ranks; value = the job's algorithmic bytes
    (2 GiB of K/V per call, whatever N) over that time."""
    from kernel_optim_b200.comm import collective
    from kernel_optim_b200.paged import PagedDecodeAttention
    from kernel_optim_b200.workloads import build_case
    layers = 2
    case = build_case("c4", dev, seed=0, paged=True, batch_scale=1, kv_shard=n, kv_rank=rank,
                      layers=layers)
    t = case.tensors
    attn = PagedDecodeAttention(case.B, case.nq, case.nkv, 128, dev, t["cache"].capacity,
                                overlap_prev=not args.no_overlap)
    out = torch.empty(case.B, case.nq * 128, dtype=torch.bfloat16, device=dev)
    pg = None
    if n > 1:
        from kernel_optim_b200.gather import PeerGather
        pg = PeerGather(case.B, n * case.nq * 128, dev)
    try:
        launch = StepLauncher(case, attn, layers, out, gather=pg)
        steps = max(4, min(args.steps, 40))
        for i in range(max(args.warmup, 3)):
            launch(i)
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(steps):
            launch(i)
        e1.record()
        torch.cuda.synchronize()
        ms = max_over_ranks(dist, e0.elapsed_time(e1)) / steps
        err = attn.read_error()
        if err:
            raise RuntimeError(f"device error word {err} in the c4 strong-scaling run")
        bytes_job = case.algorithmic_bytes() * n
        return {"workload": "c4 strong-scaled: B=4 sequences of 131072 keys in total, kv heads "
                            "sharded 8/N per GPU, head outputs all-gathered in the kernel",
                "kv_heads_per_gpu": case.nkv, "us_per_call": round(ms * 1e3, 2),
                "value": round(bytes_job / (ms * 1e-3) / 1e12, 4), "unit": "TB/s",
                "steps": steps, "algorithmic_bytes_per_call": bytes_job}
    finally:
        if pg is not None:
            if dist is not None:
                dist.barrier()
            pg.close()


def run_e2e(args, case, attn, out, gathered, pg, dist, bytes_job):
    """Same steps through host buffers, pipelined the way a server runs them: each step's qkv and
    positions are copied from pinned host memory on an H2D stream one step ahead, and each step's
    (gathered) output is copied back on a D2H stream while the steps after it compute; four device
    buffers of each, every step's copies inside the timed region. The host orders the compute
    stream against the copies (it waits for a step's input copy, and for the copy-out of the
    buffer's previous step, before it queues the step): a stream wait on another stream's event
    that has not completed when the launch is queued costs the launch its programmatic overlap
    with the call before it (measured on c2: 52.5-55 against 47.2-48 us per call)."""
    from kernel_optim_b200.comm import collective
    t = case.tensors
    dev = out.device
    NB = 4
    src = t["qkv"] if case.fused else t["q"]   # the step's per-token input
    qkv_b = src.numel() * 2
    host_in = torch.empty(qkv_b + t["pos"].numel() * 4, dtype=torch.uint8, pin_memory=True)
    host_in[:qkv_b].view(torch.bfloat16).copy_(src.reshape(-1).cpu())
    host_in[qkv_b:].view(torch.int32).copy_(t["pos"].cpu())
    dev_in = [torch.empty_like(host_in, device=dev) for _ in range(NB)]
    outs = [out] + [torch.empty_like(out) for _ in range(NB - 1)]
    gath = ([gathered] + [torch.empty_like(gathered) for _ in range(NB - 1)]
            if gathered is not None else None)
    launchers = [StepLauncher(case, attn, args.layers, outs[j],
                              qkv=dev_in[j][:qkv_b].view(torch.bfloat16).view(src.shape),
                              pos=dev_in[j][qkv_b:].view(torch.int32), gather=pg)
                 for j in range(NB)]
    res0 = gath[0] if gath is not None else pg.out[0] if pg is not None else out
    out_h = [torch.empty(res0.shape, dtype=res0.dtype, pin_memory=True) for _ in range(NB)]
    # fused gather: the gathered rows land in one of two slots that the peers write again two
    # steps later, so each step's rows are first copied to a buffer of its own on the device
    snap = [torch.empty_like(res0) for _ in range(NB)] if pg is not None else None
    compute = torch.cuda.current_stream(dev)
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    in_ready = [torch.cuda.Event() for _ in range(NB)]
    done = [torch.cuda.Event() for _ in range(NB)]      # step's kernel(s) finished with its buffers
    out_free = [torch.cuda.Event() for _ in range(NB)]  # step's output copied to the host

    def copy_in(k, start):
        """Queue step k's input copy: after the step that last used its buffer, or the clock."""
        j = k % NB
        with torch.cuda.stream(h2d):
            h2d.wait_event(done[j] if k >= NB else start)
            dev_in[j].copy_(host_in, non_blocking=True)
            in_ready[j].record(h2d)

    def run(n, start):
        copy_in(0, start)
        for i in range(n):
            j = i % NB
            if i + 1 < n:
                copy_in(i + 1, start)
            in_ready[j].synchronize()
            if i >= NB:
                out_free[j].synchronize()
            launchers[j](i)
            if gath is not None:
                collective(dist.all_gather_into_tensor, gath[j].view(-1, gath[j].shape[-1]), outs[j],
                           what="all-gather of the head outputs")
            res = gath[j] if gath is not None else launchers[j].result(outs[j])
            if snap is not None:
                # before the next step raises its flags, so before any peer writes this slot again
                snap[j].copy_(res, non_blocking=True)
                res = snap[j]
            done[j].record(compute)
            with torch.cuda.stream(d2h):
                d2h.wait_event(done[j])
                out_h[j].copy_(res, non_blocking=True)
                out_free[j].record(d2h)
        compute.wait_stream(h2d)
        compute.wait_stream(d2h)

    w0 = torch.cuda.Event()
    w0.record(compute)
    run(max(args.warmup, NB + 1), w0)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(compute)                                  # no copy starts before the clock
    run(args.steps, e0)
    e1.record(compute)
    torch.cuda.synchronize()
    ms = max_over_ranks(dist, e0.elapsed_time(e1)) / args.steps
    return {"value": round(bytes_job / (ms * 1e-3) / 1e12, 4), "unit": "TB/s",
            "us_per_call": round(ms * 1e3, 2),
            "h2d_bytes_per_step": host_in.numel(), "d2h_bytes_per_step": out_h[0].numel() * 2,
            "pipeline": "input copy one step ahead, output copy while later steps compute "
                        "(4 buffers; the host orders the compute stream against the copies)"}


# --------------------------------------------------------------------------- CPU reference
def _cpu_step_for(case, form):
    from oracle.cpu_path import CpuDecodeStep
    t = case.tensors
    cache = t["cache"]
    k_ctx, v_ctx = [], []
    for b, L in enumerate(case.cached):
        kb, vb = cache.gather(0, b, L)
        k_ctx.append(kb.cpu())
        v_ctx.append(vb.cpu())
    return CpuDecodeStep(t["qkv"], t["q_norm_w"], t["k_norm_w"], t["cos"][: max(case.keys)],
                         t["sin"][: max(case.keys)], t["pos"], k_ctx, v_ctx, case.nq, case.nkv,
                         form=form)


def cpu_baseline(case, bytes_step):
    """The reference's CPU path on the full step, bounded to a few seconds per form."""
    from oracle.cpu_path import time_steps
    res = {}
    for form, reps in (("repeat_kv", 10), ("enable_gqa", 30)):
        st = _cpu_step_for(case, form)
        secs = time_steps(st, reps, 2)
        res[form] = secs / reps
    per = res["repeat_kv"]
    return {"value": round(bytes_step / per / 1e12, 6), "unit": "TB/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": (f"full {case.name} step (B={case.B}) on the host: Transformers Qwen3RMSNorm + "
                       f"apply_rotary_pos_emb + cache write + sdpa; repeat_kv form (pinned "
                       f"Transformers 4.51.3) {per * 1e3:.1f} ms/step x10; enable_gqa form (installed "
                       f"5.5.0) {res['enable_gqa'] * 1e3:.1f} ms/step x30")}


def run_reference(args):
    world, rank, local = dist_env()
    if rank != 0:
        return
    from kernel_optim_b200.workloads import build_case
    from oracle.cpu_path import time_steps
    dev = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    n = world
    case = build_case(args.workload, dev, seed=0, paged=True, batch_scale=n, kv_shard=1, layers=1)
    st = _cpu_step_for(case, "repeat_kv")
    secs = time_steps(st, args.steps, args.warmup)
    per = secs / args.steps
    bytes_step = case.algorithmic_bytes()
    v = bytes_step / per / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": round(v, 6), "unit": "TB/s", "n_gpus": n,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per * 1e3, 3),
        "us_per_call": round(per * 1e6, 1), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (same seeded inputs as ours)",
        "config": {"workload": f"{args.workload} per GPU" + (f", weak-scaled x{n}" if n > 1 else ""),
                   "B": case.B, "keys_per_seq": max(case.keys), "q_heads": case.nq,
                   "kv_heads": case.nkv, "head_dim": 128},
        "cpu_baseline": {"value": round(v, 6), "unit": "TB/s", "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": f"full {case.name} step per timed step on the host: Transformers "
                                   "Qwen3 q/k norm + RoPE + cache write + repeat_kv sdpa"},
        "e2e": {"value": round(v, 6), "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------- p5: a decode step's projections
P5_METRIC = "decode-step projections achieved HBM TB/s (kopt_gemv, Qwen3-4B, B=32)"


def run_proj(args):
    """Workload p5: the projections of one Qwen3-4B decode step at B = 32 rows, on the skinny-GEMM
    kernel with the reference's epilogues (engine.py:259-263): per layer QKV (bf16 out), o_proj
    (residual add), gate|up (SwiGLU) and down_proj (residual add), 36 layers with their own
    weights, then the LM head with the greedy argmax (the RMSNorm row kernels between them, as in
    the engine, are not part of this workload). Random weights (std 0.02, seeded), random
    inputs; the step is one CUDA graph of its 145 launches, replayed; consecutive launches overlap
    by programmatic dependent launch. value: weight + activation bytes per step / device time.
    N > 1: independent replicas (the projections are replicated in the sharded engine)."""
    from kernel_optim_b200.checkpoint import QWEN3_4B
    from kernel_optim_b200.gemv import EPI_ARGMAX, EPI_BF16, EPI_RESID, EPI_SWIGLU, Gemv
    world, rank, local = dist_env()
    dist = init_dist(world, local)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    B, H, I, V, L = 32, QWEN3_4B["hidden"], QWEN3_4B["intermediate"], QWEN3_4B["vocab"], args.p5_layers
    NQKV, NATT = 32 * 128 + 2 * 8 * 128, 32 * 128
    bf = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(*shape, std=0.02):
        return (torch.randn(*shape, generator=g, device=dev) * std).to(bf)

    W = [dict(qkv=rnd(NQKV, H), o=rnd(H, NATT), gu=rnd(2 * I, H), down=rnd(H, I)) for _ in range(L)]
    lm = rnd(V, H)
    xn, attn = rnd(B, H, std=1.0), rnd(B, NATT, std=1.0)
    h = rnd(B, H, std=1.0)
    qkv = torch.empty(B, NQKV, dtype=bf, device=dev)
    act = torch.empty(B, I, dtype=bf, device=dev)
    ids = torch.empty(B, dtype=torch.int64, device=dev)
    ov = not args.no_overlap
    G = dict(qkv=Gemv(B, NQKV, H, EPI_BF16, device=dev, overlap_prev=ov),
             o=Gemv(B, H, NATT, EPI_RESID, device=dev, overlap_prev=ov),
             gu=Gemv(B, I, H, EPI_SWIGLU, device=dev, overlap_prev=ov),
             down=Gemv(B, H, I, EPI_RESID, device=dev, overlap_prev=ov),
             lm=Gemv(B, V, H, EPI_ARGMAX, device=dev, overlap_prev=ov))
    launches = 4 * L + 1

    def step(x=xn):
        for w in W:
            G["qkv"](x, w["qkv"], qkv)
            G["o"](attn, w["o"], h=h)
            G["gu"](x, w["gu"], act)
            G["down"](act, w["down"], h=h)
        G["lm"](x, lm, ids)

    wbytes = sum(t.numel() * 2 for w in W for t in w.values()) + lm.numel() * 2
    # activations: x read once per weight tile would be an L2 effect; count each input row block
    # once per projection and every output (h read and written by the residual epilogues)
    abytes = L * (B * H * 2 * 2 + B * NATT * 2 + B * I * 2 * 2 + B * NQKV * 2 + 4 * B * H * 2) + B * H * 2 + B * 8
    bytes_step = wbytes + abytes

    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(max(1, args.warmup)):
            step()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(max(3, args.warmup)):
        graph.replay()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    t_end = time.perf_counter() + args.soak_ms / 1e3
    while time.perf_counter() < t_end:
        graph.replay()
        torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms_step = max_over_ranks(dist, e0.elapsed_time(e1)) / args.steps
    errs = {k: op.read_error() for k, op in G.items()}
    if any(errs.values()):
        raise RuntimeError(f"device error words {errs}")
    value = world * bytes_step / (ms_step * 1e-3) / 1e12
    peak, peak_src = peaks()
    achieved = bytes_step / (ms_step * 1e-3) / 1e9
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": ncu_traffic("p5"),
                "peak_source": peak_src,
                "kernel": f"gemv_kernel<MT=2, EPI> (every launch of the step: {launches} per step)",
                "algorithmic_bytes_per_step": bytes_step, "weight_bytes_per_step": wbytes}

    e2e = None
    if not args.no_e2e:
        # through the public call (Gemv.__call__, eager): the step's input rows come from pinned
        # host memory, the token ids go back to it, both inside the timed region
        host_x = torch.empty(B, H, dtype=bf, pin_memory=True)
        host_x.copy_(xn.cpu())
        host_ids = torch.empty(B, dtype=torch.int64, pin_memory=True)
        x_dev = torch.empty_like(xn)
        for _ in range(2):
            x_dev.copy_(host_x, non_blocking=True)
            step(x_dev)
            host_ids.copy_(ids, non_blocking=True)
        torch.cuda.synchronize()
        n_e2e = max(1, min(args.steps, 10))
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        for _ in range(n_e2e):
            x_dev.copy_(host_x, non_blocking=True)
            step(x_dev)
            host_ids.copy_(ids, non_blocking=True)
        a1.record()
        torch.cuda.synchronize()
        ms_e2e = max_over_ranks(dist, a0.elapsed_time(a1)) / n_e2e
        e2e = {"value": round(world * bytes_step / (ms_e2e * 1e-3) / 1e12, 4), "unit": "TB/s",
               "ms_per_step": round(ms_e2e, 3), "h2d_bytes_per_step": B * H * 2,
               "d2h_bytes_per_step": B * 8, "steps": n_e2e,
               "path": f"eager Gemv.__call__ per projection ({launches} C-ABI calls per step)"}
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        from oracle.epilogue import GEMV_BF16, GEMV_RESID, GEMV_SWIGLU, gemv_ref
        w0 = {k: v.cpu() for k, v in W[0].items()}
        xc, ac, hc = xn.cpu(), attn.cpu(), h.cpu()
        t0 = time.perf_counter()
        reps = 0
        while reps < 1 or time.perf_counter() - t0 < 10.0:
            gemv_ref(xc, w0["qkv"], GEMV_BF16)
            gemv_ref(ac, w0["o"], GEMV_RESID, hc)
            a_c = gemv_ref(xc, w0["gu"], GEMV_SWIGLU)
            gemv_ref(a_c, w0["down"], GEMV_RESID, hc)
            reps += 1
        secs = (time.perf_counter() - t0) / reps
        lbytes = sum(t.numel() * 2 for t in w0.values())
        cpu = {"value": round(lbytes / secs / 1e12, 6), "unit": "TB/s", "cores": torch.get_num_threads(),
               "kind": "port",
               "sample": f"one layer's four projections with their epilogues (oracle/epilogue.py "
                         f"gemv_ref, fp32 torch on the host) x{reps}, {secs * 1e3:.1f} ms per layer"}
    line = {
        "metric": P5_METRIC, "value": round(value, 4), "unit": "TB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0, 0.02^2) bf16 weights of Qwen3-4B's shapes, N(0,1) inputs",
        "config": {"workload": "p5 decode-step projections", "B": B, "layers": L,
                   "shapes": {"qkv": [NQKV, H], "o": [H, NATT], "gate_up": [2 * I, H],
                              "down": [H, I], "lm_head": [V, H]},
                   "parallelism": "replicas" if world > 1 else "single GPU",
                   "l2": f"inputs larger than L2: {wbytes / 1e9:.2f} GB of weights per step",
                   "launch": "one CUDA graph per step" + ("" if args.no_overlap else
                             ", programmatic dependent launch between projections"),
                   "grids": {k: op.grid for k, op in G.items()}},
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": launches * args.steps, "clocks": clocks,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    del graph
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------ f5: prefill attention (tcgen05)
F5_METRIC = "prefill attention TFLOP/s (causal GQA, c5 prompts), us/call"


def run_prefill(args):
    """Workload f5: the attention of config c5's prefill, one call per layer: B = 32 prompts of
    S = 1024 tokens, 32 query / 8 kv heads, d = 128, causal, on the tcgen05 kernel
    (kopt_prefill_attn) over a paged cache (random page permutation) as the engine's prefill runs
    it; four layers' q and K/V rotated (1.6 GB, far above L2). value: algorithmic FLOPs per call,
    4 d per (query, key) pair with key <= query (S (S + 1) / 2 pairs per sequence and query
    head: Q K^T and P V), over the device time. torch SDPA (its fastest backend for these
    shapes, enable_gqa) on the same inputs is timed beside it as the library reference."""
    from kernel_optim_b200.fused import qk_norm_rope_error
    from kernel_optim_b200.paged import PagedKVCache
    from kernel_optim_b200.prefill import prefill_attention
    world, rank, local = dist_env()
    dist = init_dist(world, local)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    B, S, NQ, NKV, D, L = 32, 1024, 32, 8, 128, 4
    bf = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(0)
    cache = PagedKVCache(L, B * S // 16, NKV, D, B, S, dev)
    cache.assign_permuted([S] * B, torch.Generator().manual_seed(1))
    cache.k.normal_(generator=g)
    cache.v.normal_(generator=g)
    qs = [torch.randn(B * S, NQ * D, generator=g, device=dev).to(bf) for _ in range(L)]
    out = torch.empty(B * S, NQ * D, dtype=bf, device=dev)
    flops = B * NQ * 4 * D * S * (S + 1) // 2

    def step(i):
        prefill_attention(qs[i % L], cache, i % L, out, B, S, NQ, NKV, D)

    def timed(fn, n):
        for i in range(max(3, args.warmup)):
            fn(i)
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(n):
            fn(i)
        e1.record()
        torch.cuda.synchronize()
        return max_over_ranks(dist, e0.elapsed_time(e1)) / n

    sampler = ClockSampler(local)
    t_end = time.perf_counter() + args.soak_ms / 1e3
    i = 0
    while time.perf_counter() < t_end:
        step(i)
        i += 1
        if i % 16 == 0:
            torch.cuda.synchronize()
    ms = timed(step, args.steps)
    clocks = sampler.stop()
    err = qk_norm_rope_error(dev)
    if err:
        raise RuntimeError(f"device error word {err}")
    # the library reference on the same inputs: contiguous [B, H, S, D] views for SDPA
    kk = [torch.stack([cache.gather(j, b, S)[0] for b in range(B)]) for j in range(L)]
    vv = [torch.stack([cache.gather(j, b, S)[1] for b in range(B)]) for j in range(L)]
    qh = [q.view(B, S, NQ, D).transpose(1, 2) for q in qs]

    def sdpa(i):
        torch.nn.functional.scaled_dot_product_attention(qh[i % L], kk[i % L], vv[i % L],
                                                         is_causal=True, enable_gqa=True)
    ms_sdpa = timed(sdpa, max(4, args.steps // 2))
    bf16_peak, peak_src = tensor_peak()
    achieved = flops / (ms * 1e-3) / 1e12
    roofline = {"bound": "tensor", "achieved": round(achieved, 1), "peak": bf16_peak,
                "unit": "TFLOP/s", "frac": round(achieved / bf16_peak, 4), "traffic": ncu_traffic("f5"),
                "peak_source": peak_src, "kernel": "prefill_attn_kernel<PAGED=1>",
                "kernel_us": round(ms * 1e3, 2), "algorithmic_flops_per_launch": flops}

    e2e = None
    if not args.no_e2e:
        # through the public call with host buffers: q from pinned memory in, the output back
        host_q = torch.empty(B * S, NQ * D, dtype=bf, pin_memory=True)
        host_q.copy_(qs[0].cpu())
        host_o = torch.empty_like(host_q, pin_memory=True)
        n_e2e = max(2, min(args.steps, 6))

        def e2e_step(i):
            qs[0].copy_(host_q, non_blocking=True)
            prefill_attention(qs[0], cache, 0, out, B, S, NQ, NKV, D)
            host_o.copy_(out, non_blocking=True)
        ms_e2e = timed(e2e_step, n_e2e)
        e2e = {"value": round(world * flops / (ms_e2e * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
               "us_per_call": round(ms_e2e * 1e3, 1), "h2d_bytes_per_step": host_q.numel() * 2,
               "d2h_bytes_per_step": host_o.numel() * 2, "steps": n_e2e}
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        # the reference's CPU path for the same attention (torch SDPA, causal, GQA) on one sequence
        qc, kc, vc = qh[0][:1].cpu(), kk[0][:1].cpu(), vv[0][:1].cpu()
        t0 = time.perf_counter()
        reps = 0
        while reps < 1 or time.perf_counter() - t0 < 10.0:
            torch.nn.functional.scaled_dot_product_attention(qc, kc, vc, is_causal=True, enable_gqa=True)
            reps += 1
        secs = (time.perf_counter() - t0) / reps
        cpu = {"value": round(flops / B / secs / 1e12, 5), "unit": "TFLOP/s",
               "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"one of the 32 sequences (bf16 torch SDPA, causal, enable_gqa, host) x{reps}, "
                         f"{secs * 1e3:.1f} ms per sequence"}
    line = {
        "metric": F5_METRIC, "value": round(world * achieved, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "us_per_call": round(ms * 1e3, 1), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) bf16 q and K/V cache, paged with a random page permutation",
        "config": {"workload": "f5 prefill attention (c5 prompts)", "B": B, "S": S, "q_heads": NQ,
                   "kv_heads": NKV, "head_dim": D, "causal": True, "paged": True, "layers_rotated": L,
                   "parallelism": "replicas" if world > 1 else "single GPU",
                   "l2": f"inputs larger than L2: {L} layers' q and K/V in rotation"},
        "roofline": roofline,
        "library_reference": {"impl": "torch.nn.functional.scaled_dot_product_attention (enable_gqa, "
                                      "is_causal) on contiguous copies", "us_per_call": round(ms_sdpa * 1e3, 1),
                              "value": round(flops / (ms_sdpa * 1e-3) / 1e12, 2), "unit": "TFLOP/s"},
        "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": args.steps, "clocks": clocks,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


# --------------------------------------------------------------------------- c5: the engine
def engine_launches(eng, N):
    """This library's kernels launched by one generate() of N tokens (without speculation, whose
    count depends on the drafts): the native prefill's five per layer (two norms, the q/k norm +
    RoPE prologue, the prefill attention, SwiGLU) and its final norm, four with the sharded
    prefill (SDPA attends), none with the Transformers prefill; then N - 1 decode steps of six per
    layer with the skinny-GEMM projections (two norms, QKV, attention, gate|up, down_proj) and the
    final norm and LM head, or four per layer with cuBLAS projections (two norms, attention,
    SwiGLU) and the final norm."""
    if eng.K:
        return None
    L = eng.n_layers
    if eng.prefill != "native":
        pre = 0
    else:
        pre = (5 if eng.world == 1 else 4) * L + 1
    step = 6 * L + 2 if eng.gemv is not None and "lm" in eng.gemv else \
        (6 * L + 1 if eng.gemv is not None else 4 * L + 1)
    return pre + (N - 1) * step


def run_engine(args):
    """BASELINE config c5: random-init Qwen3-4B (std 0.02, seeded), B=32 prompts of 1024 uniform
    ids, 256 new tokens, CUDA-graph decode; KV heads sharded over the torchrun ranks. One step =
    one generate() call; tokens/s = B * new tokens / device time of the call (prefill included),
    and decode_tokens_s from the replays alone."""
    from kernel_optim_b200.checkpoint import QWEN3_4B, random_model
    from kernel_optim_b200.engine import Engine
    world, rank, local = dist_env()
    dist = init_dist(world, local)
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    B, S, N = 32, 1024, 256
    model = random_model(QWEN3_4B["layers"], QWEN3_4B["hidden"], QWEN3_4B["intermediate"],
                         QWEN3_4B["vocab"], seed=0, device=dev)
    eng = Engine.from_model(model, dev, group=dist.group.WORLD if dist is not None else None,
                            overlap=not args.no_overlap, gemv=not args.no_gemv,
                            prefill=args.prefill, spec=True if args.spec else None)
    g = torch.Generator().manual_seed(5)
    prompts = torch.randint(0, QWEN3_4B["vocab"], (B, S), generator=g).tolist()
    for _ in range(max(1, args.warmup)):
        list(eng.generate(prompts, N))
    steps = max(1, args.steps)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    t0 = time.perf_counter()
    for _ in range(steps):
        toks = list(eng.generate(prompts, N))
    e1.record()
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) / steps
    ms = max_over_ranks(dist, e0.elapsed_time(e1)) / steps
    # decode-only: graph replays back to back (buffers are inference tensors made by generate)
    with torch.inference_mode():
        eng.pos.fill_(S)
        d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        d0.record()
        for _ in range(N):
            eng.graph.replay()
        d1.record()
        torch.cuda.synchronize()
    step_ms = max_over_ranks(dist, d0.elapsed_time(d1)) / N
    err = eng.read_error()
    line = {
        "metric": "Qwen3-4B decode tokens/s", "value": round(B * N / (ms * 1e-3), 1),
        "unit": "tokens/s", "n_gpus": world, "steps": steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: random-init Qwen3-4B (std 0.02, seed 0), uniform random prompt ids",
        "config": {"workload": "c5 engine generate", "B": B, "prompt": S, "new_tokens": N,
                   "overlap_prev": not args.no_overlap,
                   "projections": "cuBLAS" if eng.gemv is None else
                                  "kopt_gemv (fused epilogues) for qkv, gate|up, down, lm_head; cuBLAS o_proj",
                   "prefill": args.prefill,
                   "parallelism": (f"kv-head shard x{world}, all-gather fused into the attention "
                                   "kernel (NVLink stores)" if world > 1 else "single GPU")},
        "decode_tokens_s": round(B / (step_ms * 1e-3), 1), "decode_step_ms": round(step_ms, 4),
        "wall_s_per_generate": round(wall, 3), "device_error_bits": err,
        "gpu_launches": (None if engine_launches(eng, N) is None
                         else engine_launches(eng, N) * steps),
        "tokens_sample": toks[0][:4],
    }
    if eng.K:
        line["speculative"] = {"draft_tokens": eng.K, "verify_steps_last_generate": eng.spec_steps,
                               "one_token_step_ms": round(eng.step_ms, 4),
                               "verify_step_ms": round(eng.verify_ms, 4),
                               "breakeven_tokens_per_verify": round(eng.breakeven, 3)}
    if rank == 0:
        print(json.dumps(line), flush=True)
    eng.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse_args()
    if args.workload == "p5" and args.impl == "ours":
        run_proj(args)
    elif args.workload == "f5" and args.impl == "ours":
        run_prefill(args)
    elif args.workload == "f5":
        if dist_env()[1] == 0:
            print(json.dumps({"impl": "reference", "unavailable": (
                "the reference arm times the headline decode step (c2); the prefill attention's "
                "CPU reference is timed in the f5 line's cpu_baseline")}), flush=True)
    elif args.workload == "p5":
        if dist_env()[1] == 0:
            print(json.dumps({"impl": "reference", "unavailable": (
                "the reference arm times the headline decode step (c2); the projections have no "
                "separate CPU arm (their oracle is timed in the p5 line's cpu_baseline)")}), flush=True)
    elif args.workload == "c5" and args.impl == "ours":
        run_engine(args)
    elif args.workload == "c5":
        if dist_env()[1] == 0:
            print(json.dumps({"impl": "reference", "unavailable": (
                "c5 runs a random-init Qwen3-4B end to end; its CPU prefill of 32 x 1024 tokens "
                "alone is ~260 TFLOP, hours on the host cores; the reference arm times c2")}),
                flush=True)
    elif args.impl == "reference" and args.workload.startswith("v"):
        if dist_env()[1] == 0:
            print(json.dumps({"impl": "reference", "unavailable": (
                "the reference arm times the headline decode step (c2); the verify workloads "
                "have no separate CPU arm")}), flush=True)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
