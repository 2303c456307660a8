"""Operand builders of the prefill window path (koemi_window_pack_rows,
koemi_window_slot_operands) against the same layouts built with torch copies:
fp32 -> bf16/f16 conversion rounds to nearest even in both, so bit-exact."""
from __future__ import annotations

import pytest
import torch

from koemi_5hom_b200.cuda_kernels import _ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("rows,widths,extra", [(300, (64, 128, 8, 4), 4), (7, (2048, 2048, 2048, 2048), 4),
                                               (5, (12, 0, 40), 4), (70000, (16,), 4), (33, (8, 12, 2048), 2)])
def test_pack_rows_matches_torch(rows, widths, extra, dtype, cuda):
    g = torch.Generator(device=cuda).manual_seed(rows + len(widths))
    sources = []
    for i, w in enumerate(widths):
        # row strides beyond the width; extra = 2 gives even strides that are
        # not multiples of 4 (8-byte loads), like the associative projection's
        wide = torch.randn(rows, w + extra * (i + 1), generator=g, device=cuda)
        sources.append(wide[:, :w] if i % 2 == 0 else wide[:, extra * (i + 1):])
    total = sum(widths)
    out = torch.full((rows, total + 8), 7.0, dtype=dtype, device=cuda)
    _ops.pack_rows(out, sources)
    expected = torch.cat(sources, dim=1).to(dtype)
    assert torch.equal(out[:, :total], expected)
    assert bool((out[:, total:] == 7).all())  # the row padding is untouched


def test_pack_rows_builds_the_shifted_prior(cuda):
    g = torch.Generator(device=cuda).manual_seed(3)
    batch, length, d = 6, 9, 256
    state = torch.randn(batch, 2 * d, generator=g, device=cuda)[:, :d]
    h = torch.randn(batch, length, d, generator=g, device=cuda)
    prior = torch.empty(batch, length, d, dtype=torch.bfloat16, device=cuda)
    _ops.pack_rows(prior.view(batch, length * d), [state, h.reshape(batch, length * d)[:, :(length - 1) * d]])
    expected = torch.cat((state.unsqueeze(1), h[:, :-1]), dim=1).bfloat16()
    assert torch.equal(prior, expected)
    one = torch.empty(batch, 1, d, dtype=torch.bfloat16, device=cuda)  # a one-position window
    _ops.pack_rows(one.view(batch, d), [state, h[:, :1].reshape(batch, d)[:, :0]])
    assert torch.equal(one[:, 0], state.bfloat16())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("batch,carried,length,width,padded", [(3, 128, 128, 256, 256), (2, 0, 40, 72, 40),
                                                               (4, 17, 30, 64, 56), (1, 128, 1, 2048, 136)])
def test_slot_operands_match_torch(batch, carried, length, width, padded, dtype, cuda):
    g = torch.Generator(device=cuda).manual_seed(batch * 1000 + carried + length)
    ring = torch.randn(batch, carried + 5, width, generator=g, device=cuda)[:, 5:]  # a ring-tail view
    ring_values = torch.randn(batch, carried + 5, width, generator=g, device=cuda)[:, 5:]
    keys = torch.randn(batch, length, width, generator=g, device=cuda)
    values = torch.randn(batch, length, width, generator=g, device=cuda)
    stacked, transposed = _ops.window_slot_operands(ring, ring_values, keys, values, padded, dtype)
    slots = carried + length
    expect_keys = torch.zeros(batch, padded, width, dtype=dtype, device=cuda)
    expect_keys[:, :slots] = torch.cat((ring, keys), dim=1).to(dtype)
    expect_values = torch.zeros(batch, width, padded, dtype=dtype, device=cuda)
    expect_values[:, :, :slots] = torch.cat((ring_values, values), dim=1).transpose(1, 2).to(dtype)
    assert torch.equal(stacked, expect_keys)
    assert torch.equal(transposed, expect_values)


@pytest.mark.parametrize("rows,features", [(300, 64), (70000, 8), (5, 6)])
def test_bounded_gates_vector_and_scalar_paths_agree(rows, features, cuda):
    """The window path's bounded gates (network.py:305-310): retention =
    lo + (hi - lo) sigmoid(a), increment = (1 - retention) tanh(c), padded rows
    (1, 0). The 16-byte kernel and the per-element kernel (taken for a
    misaligned view) give the same bits; both within fp32 rounding of fp64."""
    g = torch.Generator(device=cuda).manual_seed(rows + features)
    backing = torch.randn(rows * 2 * features + 1, generator=g, device=cuda) * 3
    misaligned = backing[1:].view(rows, 2 * features)
    aligned = misaligned.clone()
    valid = torch.rand(rows, generator=g, device=cuda) > 0.2
    lo, hi = 0.05, 0.995
    ret_v, inc_v = _ops.bounded_gates(aligned, valid, lo, hi)
    ret_s, inc_s = _ops.bounded_gates(misaligned, valid, lo, hi)
    assert torch.equal(ret_v, ret_s) and torch.equal(inc_v, inc_s)
    a, c = aligned.double()[:, :features], aligned.double()[:, features:]
    ret = torch.where(valid[:, None], lo + (hi - lo) * torch.sigmoid(a), 1.0)
    inc = torch.where(valid[:, None], (1 - ret) * torch.tanh(c), 0.0)
    torch.testing.assert_close(ret_v.double(), ret, rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(inc_v.double(), inc, rtol=1e-5, atol=1e-6)
