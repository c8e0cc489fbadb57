"""GPU: the engine end to end on a small random-init Qwen3 (3 layers, hidden 512, vocab 4096;
head_dim 128, 32 query / 8 kv heads), as extra checks beside the full-shape greedy parity test
(tests/test_gpu_qwen3_4b_greedy.py): the engine's options, generation state, the sharded engine on
two GPUs and the prefill's K/V, on a model small enough to run each variant in seconds.

Judged the way the reference's judge judges (QWEN_ENGINE_CONTRACT.md, "The quality rule"): the
emitted tokens are replayed through native Transformers Qwen3 (sdpa), teacher-forced, and every
emitted token must be the native argmax at its position or within 2.0 logits of it.
"""

import pytest
import torch

from kernel_optim_b200.checkpoint import random_qwen3
from kernel_optim_b200.engine import Engine

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TIE_MARGIN = 2.0


def replay_margins(model, prompts, generated):
    """Teacher-forced native replay: (max logit - logit of the emitted token) per output step, and
    whether the emitted token is the native argmax."""
    seq = torch.cat([prompts, generated[:, :-1]], 1).to(DEV)
    with torch.no_grad():
        logits = model(input_ids=seq).logits.float()
    S = prompts.shape[1]
    lg = logits[:, S - 1:]                                   # positions that produced each output
    chosen = lg.gather(-1, generated.to(DEV).unsqueeze(-1)).squeeze(-1)
    return (lg.max(-1).values - chosen).cpu(), (lg.argmax(-1).cpu() == generated)


@pytest.fixture(scope="module")
def small_model(tmp_path_factory):
    path = tmp_path_factory.mktemp("qwen3_small")
    random_qwen3(path, layers=3, hidden=512, intermediate=1024, vocab=4096, seed=0)
    return path


@pytest.mark.parametrize("gemv,prefill", [(False, "native"), (True, "native"), (True, "transformers")],
                         ids=["cublas", "kopt_gemv", "kopt_gemv-transformers_prefill"])
def test_generate_passes_the_reference_quality_rule(small_model, gemv, prefill):
    """Both projection paths (cuBLAS GEMMs with the epilogue kernels; the skinny-GEMM kernel with
    residual / SwiGLU / LM-head argmax epilogues) and both prefills (the row kernels + SDPA; the
    Transformers forward)."""
    eng = Engine(str(small_model), DEV, gemv=gemv, prefill=prefill)
    g = torch.Generator().manual_seed(1)
    B, S, N = 4, 96, 64
    prompts = torch.randint(0, 4096, (B, S), generator=g)
    steps = list(eng.generate(prompts.tolist(), N))
    assert (eng.gemv is not None) == gemv
    assert len(steps) == N and all(len(s) == B for s in steps)
    assert eng.read_error() == 0
    generated = torch.tensor(steps).t()                      # [B, N]
    margins, exact = replay_margins(eng.model, prompts, generated)
    assert float(margins.max()) <= TIE_MARGIN, f"max margin {float(margins.max()):.3f}"
    assert float(exact.float().mean()) >= 0.9, f"argmax agreement {float(exact.float().mean()):.3f}"


@pytest.mark.parametrize("B,min_advance,gemv", [(2, "0", False), (4, "0", False), (8, "100", False),
                                                (4, "0", True)],
                         ids=["B2-always", "B4-always", "B8-falls-back", "B4-always-kopt_gemv"])
def test_speculative_generate(small_model, monkeypatch, B, min_advance, gemv):
    """The speculative path (n-gram drafts, the T = K + 1 verify step on the verify attention,
    acceptance, per-sequence positions; spec.py): the tokens pass the quality rule, and they equal
    the non-speculative engine's on the same cuBLAS projections except at near-ties (both are
    greedy over the same model). ENGINE_MIN_ADVANCE 0 speculates to the end; 100 falls back to
    the one-token graph at the first break-even check. With the skinny-GEMM projections the
    one-token step runs on them and the verify step on cuBLAS."""
    monkeypatch.setenv("ENGINE_MIN_ADVANCE", min_advance)
    g = torch.Generator().manual_seed(4)
    S, N = 48, 40
    prompts = torch.randint(0, 4096, (B, S), generator=g)
    eng = Engine(str(small_model), DEV, gemv=gemv, spec=True)
    steps = list(eng.generate(prompts.tolist(), N))
    assert eng.K == {2: 6, 4: 6, 8: 4}[B]
    assert len(steps) == N and all(len(s) == B for s in steps)
    assert eng.read_error() == 0 and eng.attnk.read_error() == 0
    assert eng.spec_steps >= 1
    if min_advance == "100":
        assert eng.spec_steps <= 8           # one window at most, then the one-token graph
    generated = torch.tensor(steps).t()
    margins, exact = replay_margins(eng.model, prompts, generated)
    assert float(margins.max()) <= TIE_MARGIN, f"max margin {float(margins.max()):.3f}"
    assert float(exact.float().mean()) >= 0.9, f"argmax agreement {float(exact.float().mean()):.3f}"
    plain = torch.tensor(list(Engine(str(small_model), DEV, gemv=gemv, spec=False)
                              .generate(prompts.tolist(), N))).t()
    same = (plain == generated).all(1).float().mean()
    assert float(same) >= 0.5, f"{float(same):.2f} of the sequences identical to the plain engine's"


def test_two_generations_do_not_share_state(small_model):
    """Two consecutive generate calls with different prompts (OPTIMIZATION_GUIDE.md: reset
    prompt-dependent state); the second must equal a fresh engine's output."""
    g = torch.Generator().manual_seed(2)
    p1 = torch.randint(0, 4096, (2, 40), generator=g).tolist()
    p2 = torch.randint(0, 4096, (2, 40), generator=g).tolist()
    eng = Engine(str(small_model), DEV)
    list(eng.generate(p1, 16))
    second = list(eng.generate(p2, 16))
    fresh = list(Engine(str(small_model), DEV).generate(p2, 16))
    assert second == fresh


def _engine_worker(rank, world, port, path, prompts, n, q):
    import os

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        eng = Engine(path, f"cuda:{rank}", group=dist.group.WORLD)
        steps = list(eng.generate(prompts, n))
        err = eng.read_error()
        eng.close()
        q.put((rank, (steps, err)))
    except Exception as e:  # surfaced by the parent
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_kv_head_sharded_engine_on_two_gpus(small_model):
    """Two ranks, 4 kv heads each, attention with the fused NVLink all-gather: both ranks emit the
    same tokens, and they pass the quality rule against the native model."""
    import socket

    import torch.multiprocessing as mp
    from transformers import AutoModelForCausalLM
    g = torch.Generator().manual_seed(3)
    B, S, N = 4, 64, 32
    prompts = torch.randint(0, 4096, (B, S), generator=g)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_engine_worker, args=(r, 2, port, str(small_model), prompts.tolist(),
                                                      N, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = dict(q.get(timeout=300) for _ in range(2))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(2):
        assert not isinstance(res[r], str), f"rank {r}: {res[r]}"
        assert res[r][1] == 0, f"rank {r}: device error bits {res[r][1]}"
    assert res[0][0] == res[1][0]
    model = AutoModelForCausalLM.from_pretrained(str(small_model), dtype=torch.bfloat16,
                                                 attn_implementation="sdpa").to(DEV).eval()
    generated = torch.tensor(res[0][0]).t()
    margins, exact = replay_margins(model, prompts, generated)
    assert float(margins.max()) <= TIE_MARGIN, f"max margin {float(margins.max()):.3f}"
    assert float(exact.float().mean()) >= 0.9, f"argmax agreement {float(exact.float().mean()):.3f}"


def test_native_prefill_matches_transformers_prefill(small_model):
    """The native prefill writes the same K/V into the pages as the Transformers forward and picks
    the same first token. Same computation in the same cast order; the fused QKV GEMM and the
    attention may sum in another order than the per-module calls, so a bf16 value can round the
    other way and the difference grows through the residual stream: mean-abs within 0.5% and
    max-abs within 2% of the values' scale (a bf16 step is 0.4-0.8%)."""
    g = torch.Generator().manual_seed(3)
    B, S = 4, 96
    prompts = torch.randint(0, 4096, (B, S), generator=g)
    engs = [Engine(str(small_model), DEV, prefill=p) for p in ("native", "transformers")]
    firsts = [next(iter(e.generate(prompts.tolist(), 2))) for e in engs]
    assert firsts[0] == firsts[1]
    for layer in range(3):
        for b in range(B):
            ka, va = engs[0].cache.gather(layer, b, S)
            kb, vb = engs[1].cache.gather(layer, b, S)
            for x, y in ((ka, kb), (va, vb)):
                d = (x.float() - y.float()).abs()
                assert float(d.max()) <= 2e-2 * float(y.float().abs().max()) + 1e-3
                assert float(d.mean()) <= 5e-3 * float(y.float().abs().mean()) + 1e-4
