"""Core front on the GPU: RMSNorm forms against the oracle."""
from __future__ import annotations

import pytest
import torch

from koemi_5hom_b200.cuda_kernels.core import fused_rmsnorm_silu, gated_rmsnorm_silu, rms_norm
from oracle import ops

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (2e-5, 2e-5), torch.bfloat16: (1.6e-2, 1e-2), torch.float16: (2e-3, 2e-3)}


def _xw(rows, hidden, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, hidden, generator=g) * 2.0
    w = 1.0 + 0.02 * torch.randn(hidden, generator=g)
    return x.to(dtype), w.to(dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(32, 512), (13, 96), (7, 100), (5, 4096), (3, 2048), (65, 1), (9, 8200)])
def test_rmsnorm_silu_matches_oracle(dtype, shape, cuda):
    x, w = _xw(*shape, dtype, seed=shape[1])
    y = fused_rmsnorm_silu(x.to(cuda), w.to(cuda))
    expected, _ = ops.rmsnorm_silu(x, w)
    rtol, atol = TOL[dtype]
    torch.testing.assert_close(y.cpu().double(), expected.to(dtype).double(), rtol=rtol, atol=atol)


def test_rmsnorm_silu_golden(golden_ops, cuda):
    g = golden_ops["rmsnorm"]
    y = fused_rmsnorm_silu(g["x"].to(cuda), g["w"].to(cuda))
    torch.testing.assert_close(y.cpu(), g["silu_y"], rtol=2e-5, atol=2e-5)
    torch.testing.assert_close(rms_norm(g["x"].to(cuda), g["w"].to(cuda)).cpu(), g["y"], rtol=1e-5, atol=1e-5)


def test_rmsnorm_silu_backward_matches_oracle(cuda):
    x, w = _xw(37, 200, torch.float32, seed=1)
    gy = torch.randn(37, 200, generator=torch.Generator().manual_seed(2))
    xd, wd = x.to(cuda).requires_grad_(True), w.to(cuda).requires_grad_(True)
    fused_rmsnorm_silu(xd, wd).backward(gy.to(cuda))
    gx, gw = ops.rmsnorm_silu_grads(x, w, gy)
    torch.testing.assert_close(xd.grad.cpu().double(), gx, rtol=3e-4, atol=3e-4)
    torch.testing.assert_close(wd.grad.cpu().double(), gw, rtol=3e-4, atol=3e-4)


def test_rmsnorm_silu_backward_is_deterministic(cuda):
    x, w = _xw(3000, 256, torch.float32, seed=3)
    gy = torch.randn(3000, 256).to(cuda)
    grads = []
    for _ in range(2):
        wd = w.to(cuda).requires_grad_(True)
        fused_rmsnorm_silu(x.to(cuda), wd).backward(gy)
        grads.append(wd.grad.clone())
    assert torch.equal(grads[0], grads[1])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_gated_form_config3_rows(dtype, cuda):
    """Config 3 shape (65536 x 2048 bf16): sampled rows against the oracle."""
    g = torch.Generator().manual_seed(3)
    rows = 65536 if dtype == torch.bfloat16 else 4096
    x = torch.randn(rows, 2048, generator=g).to(dtype)
    gate = torch.randn(rows, 2048, generator=g).to(dtype)
    w = (1.0 + 0.02 * torch.randn(2048, generator=g)).to(dtype)
    y = gated_rmsnorm_silu(x.to(cuda), gate.to(cuda), w.to(cuda))
    pick = torch.tensor([0, 1, 777, rows // 2, rows - 1])
    expected = ops.gated_rmsnorm_silu(x[pick], gate[pick], w)
    rtol, atol = TOL[dtype]
    torch.testing.assert_close(y[pick].cpu().double(), expected.to(dtype).double(), rtol=rtol, atol=atol)


def test_plain_norm_with_residual_keep_and_cast(cuda):
    g = torch.Generator().manual_seed(4)
    x = torch.randn(20, 256, generator=g)
    r = torch.randn(20, 256, generator=g)
    w = 1.0 + 0.1 * torch.randn(256, generator=g)
    keep = torch.rand(20, generator=g) > 0.3
    y = rms_norm(x.to(cuda), w.to(cuda), residual=r.to(cuda), keep=keep.to(cuda))
    expected = torch.where(keep.unsqueeze(-1), ops.rms_norm(x + r, w).float(), x)
    torch.testing.assert_close(y.cpu(), expected, rtol=1e-5, atol=1e-5)
    yb = rms_norm(x.to(cuda), w.to(cuda), out_dtype=torch.bfloat16)
    assert yb.dtype == torch.bfloat16
    torch.testing.assert_close(yb.cpu().float(), ops.rms_norm(x, w).bfloat16().float(), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("shape", [(5003, 2048), (4741, 1024), (9000, 520)])
def test_streamed_rows_match_oracle(dtype, shape, cuda):
    """Row counts large enough for the persistent bulk-copy kernel, including
    a ragged last group of rows; every row is checked for both the SiLU front
    (with its inv_rms output) and the gated form."""
    rows, hidden = shape
    if dtype == torch.float32 and hidden > 1024:
        hidden = 1024
    g = torch.Generator().manual_seed(rows)
    x = (torch.randn(rows, hidden, generator=g) * 2.0).to(dtype)
    gate = torch.randn(rows, hidden, generator=g).to(dtype)
    w = (1.0 + 0.02 * torch.randn(hidden, generator=g)).to(dtype)
    rtol, atol = TOL[dtype]
    y = fused_rmsnorm_silu(x.to(cuda), w.to(cuda))
    expected, _ = ops.rmsnorm_silu(x, w)
    torch.testing.assert_close(y.cpu().double(), expected.to(dtype).double(), rtol=rtol, atol=atol)
    yg = gated_rmsnorm_silu(x.to(cuda), gate.to(cuda), w.to(cuda))
    torch.testing.assert_close(yg.cpu().double(), ops.gated_rmsnorm_silu(x, gate, w).to(dtype).double(),
                               rtol=rtol, atol=atol)


def test_streamed_rows_return_inv_rms(cuda):
    from koemi_5hom_b200.cuda_kernels import _ops
    g = torch.Generator().manual_seed(8)
    x = torch.randn(6000, 2048, generator=g).bfloat16()
    w = torch.ones(2048).bfloat16()
    y, inv = _ops.rmsnorm_silu_forward(x.to(cuda), w.to(cuda), 1e-6)
    expected = torch.rsqrt(x.double().pow(2).mean(-1) + 1e-6)
    torch.testing.assert_close(inv.cpu().double(), expected, rtol=1e-5, atol=1e-6)
