"""GPU: greedy decoding of the full-shape random-init Qwen3-4B against the native model.

The model is the one BASELINE config c5 names: 36 layers, hidden 2560, 32 query / 8 kv heads of
dim 128, SwiGLU 9728, vocab 151936, tied embeddings, RMSNorm eps 1e-6 with per-head QK-norm,
RoPE theta 5e6, Transformers' initialisation (normal, std 0.02) from a seed, bf16. Prompts are
1024 token ids drawn uniformly over the vocabulary; 64 greedy steps.

The oracle is the reference's declared native path, the one its judge replays
(QWEN_ENGINE_CONTRACT.md, "The quality rule"): Transformers Qwen3ForCausalLM with sdpa attention
on the same GPU, in two forms:

* native greedy decoding, free-running with its own KV cache (the loop of
  OPTIMIZATION_GUIDE.md:322-363), which gives native's own token sequence;
* a teacher-forced replay of a token sequence through one full forward, which gives the native
  logits at every position given that prefix.

Checks, for the engine on both projection paths (tcgen05 skinny GEMMs with fused epilogues, the
default; cuBLAS GEMMs with the epilogue kernels) and, on the default path, both prefills (the
engine's own row kernels; the Transformers forward, bit-identical to native's prefill):

1. the reference's quality rule, tightened: every emitted token is the native argmax at its
   position (replayed on the engine's own prefix), or within NEAR_TIE = 0.25 logits of it (the
   judge allows 2.0);
2. token identity with native greedy: the engine's 64 tokens equal native's, step for step, up to
   the first position where native's own replayed top-2 logits are within NEAR_TIE of each other;
   a flip anywhere else fails. Each divergence is reported with the native margin there;
3. the same rule between the two projection paths.

Why not identity over all 64 steps: this random-init model's logits are nearly flat (median top-2
margin about 0.16 logits, most positions within 0.25), and native is not consistent with itself
at that resolution: its own cached decode leaves the argmax of its own full-forward replay at
about one position in ten, by up to 0.19 logits (measured and printed by this test). Two bf16
computations that sum in different orders cannot agree on ties that native itself breaks both
ways; NEAR_TIE bounds the flips to those.
"""

from __future__ import annotations

import pytest
import torch

from kernel_optim_b200.checkpoint import QWEN3_4B, random_model
from kernel_optim_b200.engine import Engine

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
S, N = 1024, 64
TIE_MARGIN = 2.0     # the reference judge's tieMarginLogits
# Native's own cached decode departs from its replayed argmax by up to ~0.19 logits on this
# model; a logit in [4, 8) has a bf16 step of 1/32. Flips are accepted only at native top-2
# margins this small, and emitted tokens must lie this close to the replayed argmax.
NEAR_TIE = 0.25


@pytest.fixture(scope="module")
def qwen3_4b():
    model = random_model(**QWEN3_4B, seed=0, device=DEV)
    yield model
    del model
    torch.cuda.empty_cache()


@torch.inference_mode()
def native_greedy(model, prompts: torch.Tensor, n: int) -> torch.Tensor:
    """Native free-running greedy decode: prefill, then one cached step per token. [B, n]."""
    out = model(input_ids=prompts, use_cache=True, logits_to_keep=1)
    past = out.past_key_values
    tok = out.logits[:, -1].argmax(-1)
    toks = [tok]
    for _ in range(n - 1):
        out = model(input_ids=tok[:, None], past_key_values=past, use_cache=True)
        past = out.past_key_values
        tok = out.logits[:, -1].argmax(-1)
        toks.append(tok)
    return torch.stack(toks, 1)


@torch.inference_mode()
def replay_logits(model, prompts: torch.Tensor, generated: torch.Tensor) -> torch.Tensor:
    """Teacher-forced native logits [B, n, V] (fp32) at the positions that produce each token."""
    seq = torch.cat([prompts, generated[:, :-1]], 1)
    hid = model.model(input_ids=seq).last_hidden_state[:, prompts.shape[1] - 1:]
    return model.lm_head(hid).float()


def first_divergence(a: torch.Tensor, b: torch.Tensor) -> list[int]:
    """Per row, the first step where a and b differ (len if never)."""
    out = []
    for x, y in zip(a.tolist(), b.tolist()):
        j = next((i for i, (u, v) in enumerate(zip(x, y)) if u != v), len(x))
        out.append(j)
    return out


def check_identity(name, ours, ref, logits, report):
    """Rule 2: identical up to a near tie of native's replayed logits at the first flip."""
    div = first_divergence(ours, ref)
    for b, j in enumerate(div):
        if j == ours.shape[1]:
            report.append(f"{name} seq {b}: identical over {ours.shape[1]} steps")
            continue
        lg = logits[b, j]
        top2 = lg.topk(2).values
        margin = float(top2[0] - top2[1])
        gap = float(lg.max() - lg[ours[b, j]])
        report.append(f"{name} seq {b}: identical for {j} steps; at step {j} native top-2 margin "
                      f"{margin:.4f}, emitted token {gap:.4f} below native's argmax")
        assert margin <= NEAR_TIE, (
            f"{name}: sequence {b} leaves native greedy at step {j} where native's top-2 margin "
            f"is {margin:.3f} (> {NEAR_TIE}): not a near tie")


@pytest.mark.parametrize("B", [4, 32])
def test_full_shape_greedy_matches_native(qwen3_4b, B, capsys):
    g = torch.Generator().manual_seed(100 + B)
    prompts = torch.randint(0, QWEN3_4B["vocab"], (B, S), generator=g).to(DEV)
    native = native_greedy(qwen3_4b, prompts, N)
    nat_logits = replay_logits(qwen3_4b, prompts, native)
    report = []
    try:
        _run_checks(qwen3_4b, B, prompts, native, nat_logits, report)
    finally:
        with capsys.disabled():
            tag = f"\n[B={B}] "
            print(tag + tag.join(report))


def _run_checks(qwen3_4b, B, prompts, native, nat_logits, report):
    top2 = nat_logits.topk(2, dim=-1).values
    m2 = (top2[..., 0] - top2[..., 1]).flatten()
    report.append(f"native replayed top-2 margins: min {float(m2.min()):.4f}, median "
                  f"{float(m2.median()):.4f}, {int((m2 <= NEAR_TIE).sum())} of {m2.numel()} "
                  f"within {NEAR_TIE}")
    # native's own cached decode against its replay (the judge's calibration of the tie margin)
    nat_gap = nat_logits.max(-1).values - nat_logits.gather(-1, native.unsqueeze(-1)).squeeze(-1)
    report.append(f"native cached decode vs its own replay: {int((nat_gap > 0).sum())} of "
                  f"{nat_gap.numel()} tokens not the replay argmax, max {float(nat_gap.max()):.4f}")
    emitted = {}
    for gemv, prefill in ((True, "native"), (False, "native"), (True, "transformers")):
        name = ("kopt_gemv" if gemv else "cublas") + ("" if prefill == "native" else "+tf_prefill")
        eng = Engine.from_model(qwen3_4b, DEV, gemv=gemv, prefill=prefill)
        steps = list(eng.generate(prompts.tolist(), N))
        assert eng.read_error() == 0
        assert (eng.gemv is not None) == gemv
        ours = torch.tensor(steps, device=DEV).t()
        emitted[name] = ours
        eng.close()
        del eng
        torch.cuda.empty_cache()
        # rule 1: the judge's quality rule, replayed on our own prefix
        lg = replay_logits(qwen3_4b, prompts, ours)
        gap = lg.max(-1).values - lg.gather(-1, ours.unsqueeze(-1)).squeeze(-1)
        report.append(f"{name}: {int((gap > 0).sum())} of {gap.numel()} tokens not the replay "
                      f"argmax, max {float(gap.max()):.4f} logits below it")
        assert float(gap.max()) <= TIE_MARGIN, f"{name}: a token {float(gap.max()):.3f} below argmax"
        assert float(gap.max()) <= NEAR_TIE, f"{name}: a token {float(gap.max()):.3f} below argmax"
        # rule 2: identity with native greedy up to a genuine near tie
        check_identity(name, ours, native, nat_logits, report)
    # rule 3: the two projection paths against each other (margins from the first's replay)
    a, b = emitted["kopt_gemv"], emitted["cublas"]
    lg = replay_logits(qwen3_4b, prompts, a)
    check_identity("kopt_gemv vs cublas", b, a, lg, report)
