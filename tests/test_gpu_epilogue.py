"""GPU: the decode-step epilogue kernels (kopt_add_rms_norm, kopt_silu_mul) against the CPU
restatement of the reference's cast order (oracle/epilogue.py, itself checked bit for bit against
Transformers' Qwen3RMSNorm and Qwen3MLP on CPU).

The residual update is bit-exact. The normed rows and the SwiGLU product may differ from the CPU
restatement by one bf16 rounding where the fp32 value sits on a rounding boundary (the kernel sums
the squares in another order, and rsqrtf / expf are not the CPU's): at most one bf16 ulp, in
under 1% of the elements.
"""

import pytest
import torch

from kernel_optim_b200 import KoptError
from kernel_optim_b200.fused import add_rms_norm, silu_mul
from oracle.epilogue import add_rms_norm_ref, silu_mul_ref

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _ulp_check(got, ref, frac=0.01):
    g, r = got.float().cpu(), ref.float().cpu()
    diff = (g - r).abs()
    ulp = r.abs().clamp_min(1e-30) * 2.0 ** -7      # one bf16 ulp is at most |x| * 2^-7
    assert bool((diff <= ulp + 1e-30).all()), f"max diff {float(diff.max())}"
    mism = float((diff > 0).float().mean())
    assert mism <= frac, f"{mism:.4f} of the elements differ"


@pytest.mark.parametrize("M,N", [(32, 2560), (3, 256), (1, 4096)])
@pytest.mark.parametrize("with_delta", [True, False])
def test_add_rms_norm(M, N, with_delta):
    g = torch.Generator(device=DEV).manual_seed(M + N)
    res = torch.randn(M, N, generator=g, device=DEV).to(torch.bfloat16)
    delta = torch.randn(M, N, generator=g, device=DEV).to(torch.bfloat16) if with_delta else None
    w = (1 + 0.1 * torch.randn(N, generator=g, device=DEV)).to(torch.bfloat16)
    want_res, want_y = add_rms_norm_ref(res.cpu(), None if delta is None else delta.cpu(), w.cpu(), 1e-6)
    out = torch.empty_like(res)
    add_rms_norm(res, delta, w, out, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(res.cpu(), want_res)
    _ulp_check(out, want_y)


@pytest.mark.parametrize("M,I", [(32, 9728), (2, 64)])
def test_silu_mul(M, I):
    g = torch.Generator(device=DEV).manual_seed(I)
    gu = (3 * torch.randn(M, 2 * I, generator=g, device=DEV)).to(torch.bfloat16)
    out = torch.empty(M, I, dtype=torch.bfloat16, device=DEV)
    silu_mul(gu, out)
    torch.cuda.synchronize()
    _ulp_check(out, silu_mul_ref(gu.cpu()), frac=0.001)
    # and against torch's own GPU ops, which the Transformers module runs
    ref = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
    _ulp_check(out, ref, frac=0.001)


def test_epilogues_reject_bad_shapes():
    x = torch.zeros(2, 12, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(KoptError):
        add_rms_norm(x, None, torch.ones(12, dtype=torch.bfloat16, device=DEV), x.clone(), 1e-6)
    with pytest.raises(KoptError):
        silu_mul(torch.zeros(2, 10, dtype=torch.bfloat16, device=DEV),
                 torch.zeros(2, 5, dtype=torch.bfloat16, device=DEV))
