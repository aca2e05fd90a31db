"""RMSNorm and SwiGLU row kernels (forward and backward) against autograd of the reference formulas
(GPU)."""

import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ops():
    from orthrus_training_b200 import ops

    return ops


@pytest.mark.parametrize("dtype,d", [(torch.float32, 1024), (torch.float32, 64), (torch.bfloat16, 1024),
                                     (torch.bfloat16, 128), (torch.bfloat16, 256), (torch.bfloat16, 768),
                                     (torch.bfloat16, 2048)])
def test_rmsnorm_forward_backward(dtype, d):
    g = torch.Generator().manual_seed(d)
    x = (torch.randn(333, d, generator=g) * 3).to(dtype)
    w = (1 + 0.1 * torch.randn(d, generator=g)).to(dtype)
    dy = torch.randn(333, d, generator=g).to(dtype)
    y, rstd = _ops().rms_norm(x.to(DEV), w.to(DEV), 1e-6, want_rstd=True)
    dx = _ops().rms_norm_backward(x.to(DEV), w.to(DEV), rstd, dy.to(DEV))
    xr = x.float().clone().requires_grad_(True)
    ref = O.rms_norm(xr, w.float(), 1e-6)
    ref.backward(dy.float())
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert (y.float().cpu() - ref.detach()).abs().max().item() <= tol * max(1.0, ref.abs().max().item())
    assert (dx.float().cpu() - xr.grad).abs().max().item() <= tol * max(1.0, xr.grad.abs().max().item())


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_swiglu_forward_backward(dtype):
    g = torch.Generator().manual_seed(7)
    gu = (torch.randn(257, 2 * 384, generator=g) * 2).to(dtype)
    dout = torch.randn(257, 384, generator=g).to(dtype)
    out = _ops().silu_mul(gu.to(DEV))
    dgu = _ops().silu_mul_backward(gu.to(DEV), dout.to(DEV))
    r = gu.float().clone().requires_grad_(True)
    ref = torch.nn.functional.silu(r[:, :384]) * r[:, 384:]
    ref.backward(dout.float())
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert (out.float().cpu() - ref.detach()).abs().max().item() <= tol * max(1.0, ref.abs().max().item())
    assert (dgu.float().cpu() - r.grad).abs().max().item() <= tol * max(1.0, r.grad.abs().max().item())
