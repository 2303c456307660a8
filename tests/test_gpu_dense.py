"""Dense front on the GPU: scan parity with the oracle (fp32 <= 1e-5 relative)."""
from __future__ import annotations

import pytest
import torch

from koemi_5hom_b200.cuda_kernels.dense import dense_affine_scan
from oracle import ops

pytestmark = pytest.mark.gpu

TOL = {torch.float64: (1e-10, 1e-10), torch.float32: (1e-5, 1e-5), torch.bfloat16: (1.6e-2, 1e-2),
       torch.float16: (2e-3, 2e-3)}


def _inputs(batch, length, features, dtype, seed, broadcast=False):
    g = torch.Generator().manual_seed(seed)
    a_shape = (batch, length, 1) if broadcast else (batch, length, features)
    a = torch.sigmoid(torch.randn(a_shape, generator=g))
    b = torch.randn(batch, length, features, generator=g)
    h0 = torch.randn(batch, features, generator=g)
    return a.to(dtype), b.to(dtype), h0.to(dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16, torch.float64])
@pytest.mark.parametrize("shape", [(3, 37, 24), (2, 300, 40), (1, 1000, 33), (4, 5, 64), (2, 129, 8), (5, 64, 32)])
def test_scan_matches_oracle(dtype, shape, cuda):
    a, b, h0 = _inputs(*shape, dtype, seed=sum(shape))
    got = dense_affine_scan(a.to(cuda), b.to(cuda), h0.to(cuda))
    expected = ops.affine_scan(a, b, h0)
    rtol, atol = TOL[dtype]
    assert got.dtype == dtype
    torch.testing.assert_close(got.cpu().double(), expected.to(dtype).double(), rtol=rtol, atol=atol)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_scan_broadcast_retention_and_zero_initial(dtype, cuda):
    a, b, _ = _inputs(3, 200, 48, dtype, seed=3, broadcast=True)
    got = dense_affine_scan(a.to(cuda), b.to(cuda))
    rtol, atol = TOL[dtype]
    torch.testing.assert_close(got.cpu().double(), ops.affine_scan(a, b).to(dtype).double(), rtol=rtol, atol=atol)


def test_scan_golden_fixture(golden_ops, cuda):
    g = golden_ops["scan"]
    got = dense_affine_scan(g["a"].to(cuda), g["b"].to(cuda), g["h0"].to(cuda))
    torch.testing.assert_close(got.cpu(), g["h"], rtol=1e-5, atol=1e-5)
    gb = golden_ops["scan_broadcast"]
    torch.testing.assert_close(dense_affine_scan(gb["a"].to(cuda), gb["b"].to(cuda)).cpu(), gb["h"], rtol=1e-5, atol=1e-5)


def test_scan_decode_step_shape(cuda):
    """T = 1 at B = 256, D = 2048: one fused step, h = a*h0 + b."""
    a, b, h0 = _inputs(256, 1, 2048, torch.bfloat16, seed=9)
    got = dense_affine_scan(a.to(cuda), b.to(cuda), h0.to(cuda)).cpu().float()
    torch.testing.assert_close(got, (a.float() * h0.float().unsqueeze(1) + b.float()).bfloat16().float(),
                               rtol=1.6e-2, atol=1e-2)


def test_scan_baseline_config_lanes_and_linearity(cuda):
    """Config 2 (B=8, T=4096, D=1024 bf16, a=sigmoid(N(0,1)), b~N(0,1), h0=0):
    sampled lanes against the fp64 oracle, and linearity in h0."""
    g = torch.Generator(device="cpu").manual_seed(2)
    a = torch.sigmoid(torch.randn(8, 4096, 1024, generator=g)).bfloat16().to(cuda)
    b = torch.randn(8, 4096, 1024, generator=g).bfloat16().to(cuda)
    h = dense_affine_scan(a, b)
    lanes = [(0, 0), (3, 517), (7, 1023), (5, 64)]
    for bi, f in lanes:
        expected = ops.affine_scan(a[bi:bi + 1, :, f:f + 1].cpu(), b[bi:bi + 1, :, f:f + 1].cpu())
        torch.testing.assert_close(h[bi, :, f].cpu().double(), expected[0, :, 0].bfloat16().double(),
                                   rtol=1.6e-2, atol=1e-2)
    h0 = torch.randn(8, 1024, generator=g).to(cuda)
    a32, b32 = a.float(), b.float()
    with_h0 = dense_affine_scan(a32, b32, h0)
    without = dense_affine_scan(a32, b32)
    decay = torch.cumprod(a32, dim=1)
    torch.testing.assert_close(with_h0, without + decay * h0.unsqueeze(1), rtol=1e-4, atol=1e-5)


def test_scan_gradients_match_oracle(cuda):
    a, b, h0 = _inputs(2, 70, 16, torch.float32, seed=4)
    grad = torch.randn(2, 70, 16, generator=torch.Generator().manual_seed(5))
    ad, bd, hd = (t.to(cuda).requires_grad_(True) for t in (a, b, h0))
    dense_affine_scan(ad, bd, hd).backward(grad.to(cuda))
    ga, gb, gh = ops.affine_scan_grads(a, b, h0, grad)
    torch.testing.assert_close(ad.grad.cpu().double(), ga, rtol=2e-5, atol=2e-5)
    torch.testing.assert_close(bd.grad.cpu().double(), gb, rtol=2e-5, atol=2e-5)
    torch.testing.assert_close(hd.grad.cpu().double(), gh, rtol=2e-5, atol=2e-5)


def test_scan_broadcast_gradient_reduces_to_retention_shape(cuda):
    a, b, h0 = _inputs(2, 30, 8, torch.float32, seed=6, broadcast=True)
    ad = a.to(cuda).requires_grad_(True)
    dense_affine_scan(ad, b.to(cuda), h0.to(cuda)).sum().backward()
    ga, _, _ = ops.affine_scan_grads(a, b, h0, torch.ones(2, 30, 8))
    torch.testing.assert_close(ad.grad.cpu().double(), ga.sum(-1, keepdim=True), rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(2, 1500, 72), (3, 2049, 128), (1, 513, 8), (4, 300, 200)])
def test_segmented_scan_ragged_segments(dtype, shape, cuda):
    """Several look-back segments, a ragged last segment and a ragged last
    feature tile, against the fp64 oracle."""
    a, b, h0 = _inputs(*shape, dtype, seed=sum(shape) + 1)
    got = dense_affine_scan(a.to(cuda), b.to(cuda), h0.to(cuda))
    rtol, atol = TOL[dtype]
    torch.testing.assert_close(got.cpu().double(), ops.affine_scan(a, b, h0).to(dtype).double(),
                               rtol=rtol, atol=atol)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_segmented_scan_broadcast_retention(dtype, cuda):
    a, b, h0 = _inputs(3, 1100, 64, dtype, seed=21, broadcast=True)
    got = dense_affine_scan(a.to(cuda), b.to(cuda), h0.to(cuda))
    rtol, atol = TOL[dtype]
    torch.testing.assert_close(got.cpu().double(), ops.affine_scan(a, b, h0).to(dtype).double(),
                               rtol=rtol, atol=atol)


@pytest.mark.parametrize("broadcast", [False, True])
def test_segmented_and_chunked_kernels_agree(broadcast, cuda):
    """The C-ABI call with a workspace (segments + look-back) and without one
    (one walker per lane group) give the same fp32 states within 1e-5."""
    from koemi_5hom_b200 import _native
    from koemi_5hom_b200._native import call, ptr
    a, b, h0 = (t.to(cuda) for t in _inputs(2, 3000, 96, torch.float32, seed=31, broadcast=broadcast))
    lib = _native.library()
    size = lib.koemi_dense_affine_scan_workspace(2, 3000, 96, _native.F32)
    assert size > 0
    workspace = torch.empty(size, dtype=torch.uint8, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    outs = []
    for ws, nbytes in ((workspace, size), (None, 0)):
        out = torch.empty_like(b)
        call("koemi_dense_affine_scan_forward", ptr(a), ptr(b), ptr(h0), ptr(out), 2, 3000, 96, int(broadcast),
             _native.F32, ptr(ws), nbytes, stream)
        outs.append(out)
    torch.testing.assert_close(outs[0], outs[1], rtol=1e-5, atol=1e-5)
    # A workspace one byte short is not used: the call falls back to the walker.
    out = torch.empty_like(b)
    call("koemi_dense_affine_scan_forward", ptr(a), ptr(b), ptr(h0), ptr(out), 2, 3000, 96, int(broadcast),
         _native.F32, ptr(workspace), size - 1, stream)
    torch.testing.assert_close(out, outs[1], rtol=0, atol=0)


def test_segmented_scan_many_tiles_linearity(cuda):
    """B=64, T=4096, D=512 bf16 (32768 tiles): sampled lanes against the oracle
    and h0-linearity of the fp32 path at the same size."""
    g = torch.Generator(device="cpu").manual_seed(12)
    a = torch.sigmoid(torch.randn(64, 4096, 512, generator=g)).to(cuda)
    b = torch.randn(64, 4096, 512, generator=g).to(cuda)
    h0 = torch.randn(64, 512, generator=g).to(cuda)
    hb = dense_affine_scan(a.bfloat16(), b.bfloat16())
    for bi, f in [(0, 0), (63, 511), (17, 300), (40, 64)]:
        expected = ops.affine_scan(a[bi:bi + 1, :, f:f + 1].bfloat16().cpu(), b[bi:bi + 1, :, f:f + 1].bfloat16().cpu())
        torch.testing.assert_close(hb[bi, :, f].cpu().double(), expected[0, :, 0].bfloat16().double(),
                                   rtol=1.6e-2, atol=1e-2)
    with_h0 = dense_affine_scan(a, b, h0)
    without = dense_affine_scan(a, b)
    torch.testing.assert_close(with_h0, without + torch.cumprod(a, dim=1) * h0.unsqueeze(1), rtol=1e-4, atol=1e-5)
