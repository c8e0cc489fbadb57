"""GPU: the decode-step projections (kopt_gemv through kernel_optim_b200.gemv.Gemv) against the
fp32 restatement of the reference's epilogues (oracle/epilogue.py gemv_ref, gemv.py:86-105).

The kernel and the oracle add the same products in different orders, so their fp32 sums differ by
at most a few units of 2^-24 * sum|x||w|; the tests allow 2^-20 * sum|x||w| (tol). Every check is
then exact up to that slack: the F32 sums are within tol of the oracle's, and each bf16 output
lies between the epilogue evaluated at sum - tol and at sum + tol (rounding to bf16, the residual
add and the product are monotone; for SwiGLU the four corners of the gate/up interval bound it).
Repeated calls, CUDA-graph replays and programmatically overlapped launches are bit-identical
(the split partials are added in split order, whichever CTA finishes last).
"""

import pytest
import torch

from kernel_optim_b200 import KoptError
from kernel_optim_b200.fused import add_rms_norm
from kernel_optim_b200.gemv import EPI_ARGMAX, EPI_BF16, EPI_F32, EPI_RESID, EPI_SWIGLU, Gemv
from oracle.epilogue import add_rms_norm_ref, gemv_epilogue_ref, gemv_ref

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _inputs(M, N, K, epi, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    rows = 2 * N if epi == EPI_SWIGLU else N
    x = torch.randn(M, K, generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn(rows, K, generator=g, device=DEV) * (2.0 / K ** 0.5)).to(torch.bfloat16)
    h = torch.randn(M, N, generator=g, device=DEV).to(torch.bfloat16)
    return x, w, h


def _out(M, N, epi):
    return torch.zeros(M, N, device=DEV, dtype=torch.float32 if epi == EPI_F32 else torch.bfloat16)


def _run(op, x, w, h, epi):
    y = _out(op.M, op.N, epi)
    hh = h.clone()
    op(x, w, y, h=hh)
    torch.cuda.synchronize()
    return hh if epi == EPI_RESID else y


def _epi(acc, h, epi):
    return gemv_epilogue_ref(acc, epi, h).float()


def _check(got, x, w, h, epi):
    xf, wf = x.cpu().float(), w.cpu().float()
    acc = xf @ wf.t()
    tol = (xf.abs() @ wf.abs().t()) * 2.0 ** -20
    g = got.float().cpu()
    if epi == EPI_F32:
        d = (g - acc).abs()
        assert bool((d <= tol).all()), f"max excess {float((d - tol).max())}"
        return
    hh = None if h is None else h.cpu()
    if epi == EPI_SWIGLU:
        n = acc.shape[1] // 2
        corners = []
        for sg in (-1, 1):
            for su in (-1, 1):
                a = acc.clone()
                a[:, :n] += sg * tol[:, :n]
                a[:, n:] += su * tol[:, n:]
                corners.append(_epi(a, hh, epi))
        lo = torch.stack(corners).min(0).values
        hi = torch.stack(corners).max(0).values
    else:
        lo, hi = _epi(acc - tol, hh, epi), _epi(acc + tol, hh, epi)
    ok = (g >= lo) & (g <= hi)
    if not bool(ok.all()):
        i = int(torch.nonzero(~ok.flatten())[0])
        raise AssertionError(f"epi {epi}: {int((~ok).sum())} outputs outside their rounding interval, "
                             f"first: got {float(g.flatten()[i])} not in [{float(lo.flatten()[i])}, "
                             f"{float(hi.flatten()[i])}]")


# Qwen3-4B decode shapes at batch 32 (qkv, o, gate|up, down) and edge cases: one row, rows not a
# multiple of 16, 64 rows, K not a multiple of the 64-wide chunk, a single tile, N not a multiple
# of the 128-row weight tile (the last tile's rows past N are read as zero and not stored).
CASES = [
    (32, 6144, 2560, EPI_BF16),
    (32, 2560, 4096, EPI_RESID),
    (32, 9728, 2560, EPI_SWIGLU),
    (32, 2560, 9728, EPI_RESID),
    (1, 256, 128, EPI_BF16),
    (5, 64, 64, EPI_F32),
    (17, 128, 200, EPI_BF16),
    (64, 192, 512, EPI_F32),
    (64, 128, 1024, EPI_SWIGLU),
    (3, 64, 136, EPI_SWIGLU),
    (9, 336, 512, EPI_RESID),
    (16, 512, 2048, EPI_RESID),
]


@pytest.mark.parametrize("M,N,K,epi", CASES)
def test_gemv_matches_oracle(M, N, K, epi):
    x, w, h = _inputs(M, N, K, epi, seed=M * 7 + N + K + epi)
    op = Gemv(M, N, K, epi, device=DEV)
    got = _run(op, x, w, h, epi)
    _check(got, x, w, h, epi)
    assert op.read_error() == 0


@pytest.mark.parametrize("ctas", [1, 2, 3, 7, 64, 296, 0])
@pytest.mark.parametrize("epi", [EPI_F32, EPI_BF16, EPI_RESID, EPI_SWIGLU])
def test_every_grid_size(ctas, epi):
    """From one CTA streaming everything to one CTA per unit: tiles whole in a CTA, split over
    two or many CTAs, and runs that start and end mid-tile."""
    M, N, K = 24, 256, 4096
    x, w, h = _inputs(M, N, K, epi, seed=ctas + 10 * epi)
    op = Gemv(M, N, K, epi, device=DEV, ctas=ctas)
    if ctas:
        assert 1 <= op.grid <= ctas
    a = _run(op, x, w, h, epi)
    _check(a, x, w, h, epi)
    b = _run(op, x, w, h, epi)        # the arrival counters were re-armed by the first call
    assert torch.equal(a, b)


def test_multi_wave_grid_is_exact():
    """More CTAs than fit at once (later CTAs start as earlier ones leave), many tiles split."""
    M, N, K = 32, 19456, 2560
    x, w, h = _inputs(M, N, K, EPI_F32, seed=3)
    op = Gemv(M, N, K, EPI_F32, device=DEV, ctas=1216)
    for _ in range(5):
        _check(_run(op, x, w, h, EPI_F32), x, w, h, EPI_F32)


def test_graph_replay_and_overlap_are_bit_identical():
    M, N, K = 32, 2560, 9728
    x, w, h = _inputs(M, N, K, EPI_RESID, seed=5)
    plain = Gemv(M, N, K, EPI_RESID, device=DEV)
    want = _run(plain, x, w, h, EPI_RESID)
    ov = Gemv(M, N, K, EPI_RESID, device=DEV, overlap_prev=True)
    hh = h.clone()
    s = torch.cuda.Stream(DEV)
    with torch.cuda.stream(s):
        torch.mm(x[:, :2560], x[:, :2560].t())   # a kernel for the launch to overlap
        ov(x, w, None, h=hh)
    torch.cuda.synchronize()
    assert torch.equal(hh, want)
    # three chained in-place updates in one graph = three eager calls
    g = torch.cuda.CUDAGraph()
    hg = h.clone()
    with torch.cuda.graph(g):
        for _ in range(3):
            ov(x, w, None, h=hg)
    he = h.clone()
    for _ in range(3):
        plain(x, w, None, h=he)
    hg.copy_(h)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(hg, he)
    del g


@pytest.mark.parametrize("M,K,with_ss", [(32, 2560, False), (32, 2560, True), (5, 1024, True),
                                          (64, 512, False), (16, 200, False)])
@pytest.mark.parametrize("fuse", [True, False], ids=["in_kernel", "row_kernel"])
def test_fused_norm(M, K, with_ss, fuse):
    """norm=True, in the kernel (fuse_norm) or by the row kernel first: x normalised, bf16(nw * bf16(x * rstd)) with rstd from the
    given per-tile sums of squares or from x itself. Against the oracle's normalised rows, whose
    rstd adds the squares in another fp32 order: a normalised value may round to the neighbouring
    bf16 where it sits on a rounding boundary, so the check is the attention tolerance (max-abs
    2e-2 and mean-abs 2e-3 relative to the outputs' scale) plus near-total agreement."""
    N = 640
    x, w, _ = _inputs(M, N, K, EPI_BF16, seed=K + M)
    nw = (1 + 0.1 * torch.randn(K, device=DEV)).to(torch.bfloat16)
    op = Gemv(M, N, K, EPI_BF16, norm=True, fuse_norm=fuse, device=DEV)
    y = _out(M, N, EPI_BF16)
    ss = None
    if with_ss:   # three "tiles" of partial sums, as a residual projection would write them
        xf = x.float()
        cut = [0, K // 3, 2 * K // 3, K]
        ss = torch.stack([(xf[:, a:b] ** 2).sum(1) for a, b in zip(cut, cut[1:])]).contiguous()
    op(x, w, y, nw=nw, ss=ss)
    torch.cuda.synchronize()
    _, want_xn = add_rms_norm_ref(x.cpu(), None, nw.cpu(), 1e-6)
    ref = gemv_ref(want_xn, w.cpu(), EPI_BF16).float()
    d = (y.cpu().float() - ref).abs()
    scale = ref.abs().mean()
    assert float(d.max()) <= 2e-2 * float(ref.abs().max()), f"max diff {float(d.max())}"
    assert float(d.mean()) <= 2e-3 * float(scale), f"mean diff {float(d.mean())}"
    assert float((d <= ref.abs() * 2.0 ** -7 + 1e-6).float().mean()) >= 0.97
    assert op.read_error() == 0


def test_resid_sums_of_squares():
    """EPI_RESID with ss_out: per (tile, row) the sum of squares of the new bf16 h over the tile's
    columns, and a norm=True projection fed with them equals one that sums x itself."""
    M, N, K = 32, 2560, 4096
    x, w, h = _inputs(M, N, K, EPI_RESID, seed=21)
    op = Gemv(M, N, K, EPI_RESID, device=DEV)
    ss = torch.full((op.ss_tiles, M), float("nan"), device=DEV)
    hh = h.clone()
    op(x, w, None, h=hh, ss_out=ss)
    torch.cuda.synchronize()
    _check(hh, x, w, h, EPI_RESID)
    hf = hh.cpu().float()
    want = torch.stack([(hf[:, 128 * t:128 * (t + 1)] ** 2).sum(1) for t in range(op.ss_tiles)])
    torch.testing.assert_close(ss.cpu(), want, rtol=1e-5, atol=1e-5)
    nw = (1 + 0.1 * torch.randn(N, device=DEV)).to(torch.bfloat16)
    w2 = (torch.randn(512, N, device=DEV) * N ** -0.5).to(torch.bfloat16)
    nxt = Gemv(M, 512, N, EPI_BF16, norm=True, fuse_norm=True, device=DEV)
    a, b = _out(M, 512, EPI_BF16), _out(M, 512, EPI_BF16)
    nxt(hh, w2, a, nw=nw, ss=ss)
    nxt(hh, w2, b, nw=nw)
    torch.cuda.synchronize()
    d = (a.float() - b.float()).abs()
    assert float(d.max()) <= 2e-2 * float(b.float().abs().max())
    assert float((a == b).float().mean()) >= 0.97


def test_tune_picks_a_listed_grid():
    M, N, K = 32, 2560, 4096
    ws = [torch.randn(N, K, device=DEV).to(torch.bfloat16) for _ in range(3)]
    op = Gemv(M, N, K, EPI_BF16, device=DEV)
    import time
    cfg = op.tune(ws, time.monotonic() + 30)
    assert cfg in op.candidates() and op.us > 0
    x, _, h = _inputs(M, N, K, EPI_BF16, seed=1)
    _check(_run(op, x, ws[0], h, EPI_BF16), x, ws[0], h, EPI_BF16)


def test_bad_arguments_raise():
    with pytest.raises(KoptError):
        Gemv(65, 64, 64, EPI_BF16, device=DEV)
    with pytest.raises(KoptError):
        Gemv(4, 100, 64, EPI_BF16, device=DEV)
    op = Gemv(4, 64, 64, EPI_BF16, device=DEV)
    x = torch.zeros(4, 64, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(KoptError):
        op(x, torch.zeros(32, 64, dtype=torch.bfloat16, device=DEV), _out(4, 64, EPI_BF16))
    with pytest.raises(KoptError):
        op(x, torch.zeros(64, 64, dtype=torch.bfloat16, device=DEV), _out(4, 64, EPI_F32))


@pytest.mark.parametrize("M,N,K,ctas", [(32, 151936, 2560, 0), (1, 4096, 256, 0), (7, 640, 1024, 5),
                                        (64, 1024, 512, 1)])
def test_argmax_epilogue(M, N, K, ctas):
    """The LM head's greedy pick: the kernel's index must hold the row's largest bf16 logit of the
    oracle (a flipped rounding can only swap indices whose logits are one bf16 ulp apart), and
    equal the oracle's first-index pick in nearly every row."""
    x, w, _ = _inputs(M, N, K, EPI_BF16, seed=N + M)
    op = Gemv(M, N, K, EPI_ARGMAX, device=DEV, ctas=ctas)
    ids = torch.full((M,), -1, dtype=torch.int64, device=DEV)
    for _ in range(2):                       # the keys are re-armed by the first call
        op(x, w, ids)
        torch.cuda.synchronize()
        want = gemv_ref(x.cpu(), w.cpu(), EPI_ARGMAX)
        logits = (x.cpu().float() @ w.cpu().float().t()).to(torch.bfloat16).float()
        got = ids.cpu()
        assert bool(((got >= 0) & (got < N)).all())
        top = logits.max(dim=1).values
        picked = logits.gather(1, got.unsqueeze(1)).squeeze(1)
        assert bool((top - picked <= top.abs() * 2.0 ** -7 + 1e-30).all())
        assert float((got == want).float().mean()) >= 0.9


def test_argmax_ties_take_the_first_index():
    M, N, K = 4, 512, 64
    x = torch.ones(M, K, dtype=torch.bfloat16, device=DEV)
    w = torch.zeros(N, K, dtype=torch.bfloat16, device=DEV)
    w[[70, 300, 301, 499]] = 1.0              # equal logits at four columns of different tiles
    ids = torch.empty(M, dtype=torch.int64, device=DEV)
    Gemv(M, N, K, EPI_ARGMAX, device=DEV)(x, w, ids)
    torch.cuda.synchronize()
    assert ids.tolist() == [70] * M
    w.zero_()                                  # all logits +0 / -0: column 0
    w[5, 0] = -0.0
    Gemv(M, N, K, EPI_ARGMAX, device=DEV)(x, w, ids)
    torch.cuda.synchronize()
    assert ids.tolist() == [0] * M


@pytest.mark.parametrize("N,K,epi", [(6144, 2560, EPI_BF16), (2560, 9728, EPI_RESID),
                                     (9728, 2560, EPI_SWIGLU), (151936, 2560, EPI_ARGMAX)])
def test_plan_matches_host_mirror(N, K, epi):
    """kopt_gemv_plan_make's split equals the host restatement that tests/test_gemv_plan.py checks."""
    from kernel_optim_b200.gemv_plan import gemv_split
    sms = torch.cuda.get_device_properties(DEV).multi_processor_count
    op = Gemv(32, N, K, epi, device=DEV)
    plan = op._plans[op.grid][0]
    want = gemv_split(N, K, swiglu=epi == EPI_SWIGLU, ctas=sms * plan.ctas_per_sm)
    assert (plan.tiles, plan.units_per_cta, plan.grid) == (want.tiles, want.per, want.grid)
