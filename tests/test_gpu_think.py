"""Think front on the GPU: fused surprise and salient admission vs the oracle."""
from __future__ import annotations

import pytest
import torch

from koemi_5hom_b200.cuda_kernels.think import causal_surprise, salient_admission
from oracle import ops

pytestmark = pytest.mark.gpu


def _case(batch, length, width, vocab, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    prior = torch.randn(batch, length, width, generator=g).to(dtype)
    weight = (torch.randn(vocab, width, generator=g) * width ** -0.5).to(dtype)
    bias = (torch.randn(vocab, generator=g) * 0.1).to(dtype)
    targets = torch.randint(0, vocab, (batch, length), generator=g)
    valid = torch.rand(batch, length, generator=g) > 0.2
    return prior, weight, bias, targets, valid


@pytest.mark.parametrize("shape", [(4, 64, 128, 1024), (2, 256, 256, 256), (3, 10, 32, 299), (1, 7, 2048, 5000),
                                   (2, 3, 16, 2)])
def test_surprise_fp32_matches_oracle(shape, cuda):
    prior, weight, bias, targets, valid = _case(*shape, torch.float32, seed=shape[3])
    got = causal_surprise(*(t.to(cuda) for t in (prior, weight, bias, targets, valid)))
    expected = ops.causal_surprise(prior, weight, bias, targets, valid)
    assert got.dtype == torch.float32
    torch.testing.assert_close(got.cpu().double(), expected, rtol=2e-5, atol=2e-6)
    assert bool((got.cpu()[~valid] == 0).all())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_surprise_16bit_matches_oracle(dtype, cuda):
    prior, weight, bias, targets, valid = _case(4, 33, 256, 3000, dtype, seed=7)
    got = causal_surprise(*(t.to(cuda) for t in (prior, weight, bias, targets, valid)))
    expected = ops.causal_surprise(prior, weight, bias, targets, valid)  # on the rounded inputs
    assert got.dtype == dtype
    torch.testing.assert_close(got.cpu().double(), expected.to(dtype).double(), rtol=1.6e-2, atol=4e-3)


def test_surprise_golden_fixture(golden_ops, cuda):
    g = golden_ops["surprise"]
    keep = [i for i in range(g["head_weight"].shape[0]) if i != 256]
    target = torch.where(g["target"] > 256, g["target"] - 1, g["target"])
    got = causal_surprise(g["prior"].to(cuda), g["head_weight"][keep].contiguous().to(cuda),
                          g["head_bias"][keep].contiguous().to(cuda), target.to(cuda), g["valid"].to(cuda))
    torch.testing.assert_close(got.cpu(), g["surprise"], rtol=2e-5, atol=2e-6)


def test_surprise_empty_sequence(cuda):
    prior, weight, bias, targets, valid = _case(2, 0, 16, 10, torch.float32, seed=1)
    out = causal_surprise(*(t.to(cuda) for t in (prior, weight, bias, targets, valid)))
    assert out.shape == (2, 0)


def test_surprise_rejects_out_of_range_targets(cuda):
    prior, weight, bias, targets, valid = _case(1, 4, 16, 10, torch.float32, seed=1)
    targets[0, 2] = 10
    from koemi_5hom_b200.cuda_kernels.think import CudaThinkValidationError
    with pytest.raises(CudaThinkValidationError, match=r"target_ids must be in \[0, 10\)"):
        causal_surprise(*(t.to(cuda) for t in (prior, weight, bias, targets, valid)))


@pytest.mark.parametrize("shape,dtype", [((2, 5, 16, 40), torch.float32), ((3, 50, 256, 3000), torch.float32),
                                         ((4, 64, 256, 3000), torch.bfloat16), ((2, 40, 128, 999), torch.float16),
                                         ((2, 128, 2048, 5000), torch.bfloat16)])
def test_surprise_backward_matches_autograd_oracle(shape, dtype, cuda):
    """The native backward (dlogits kernel: FMA tiles for fp32, tcgen05 for
    16-bit; fp32 contractions) against fp64 autograd through the oracle's
    formula on the same (rounded) inputs and a random upstream gradient.
    fp32: the reference's own tolerance (tests/cuda/test_think_cuda.py:120,
    2e-3); 16-bit: the gradients are rounded to the input dtype, so the gate
    is 2e-2 of each gradient's largest magnitude."""
    prior, weight, bias, targets, valid = _case(*shape, dtype, seed=shape[3])
    upstream = torch.randn(shape[0], shape[1], generator=torch.Generator().manual_seed(9)).to(dtype)
    ins = [t.to(cuda).requires_grad_(True) for t in (prior, weight, bias)]
    causal_surprise(*ins, targets.to(cuda), valid.to(cuda)).backward(upstream.to(cuda))
    ref = [t.double().requires_grad_(True) for t in (prior, weight, bias)]
    ops.causal_surprise(*ref, targets, valid).backward(upstream.double())
    for mine, theirs in zip(ins, ref):
        got = mine.grad.cpu().double()
        assert mine.grad.dtype == dtype
        if dtype == torch.float32:
            torch.testing.assert_close(got, theirs.grad, rtol=2e-3, atol=2e-5)
        else:
            assert (got - theirs.grad).abs().max() <= 2e-2 * theirs.grad.abs().max()


@pytest.mark.parametrize("name", ["grow", "compact", "long"])
def test_salient_admission_golden(golden_ops, name, cuda):
    g = golden_ops["salient_tail"][name]
    surprise = g["admission"].float()  # admitted where surprise 1 > 0.5
    valid = torch.ones_like(g["admission"])
    k, v, ok, adm = salient_admission(*(t.to(cuda) for t in (g["carried_keys"], g["carried_values"],
                                                            g["carried_valid"], g["keys"], g["values"], surprise,
                                                            valid)), 0.5, g["capacity"])
    assert torch.equal(adm.cpu(), g["admission"])
    expected = ops.salient_tail(g["carried_keys"], g["carried_values"], g["carried_valid"], g["keys"], g["values"],
                                g["admission"], g["capacity"])
    assert torch.equal(ok.cpu(), expected[2])
    assert torch.equal(k.cpu(), expected[0]) and torch.equal(v.cpu(), expected[1])
    for (mk, mv), (rk, rv) in zip(ops.admitted_sequence(k.cpu(), v.cpu(), ok.cpu()),
                                  ops.admitted_sequence(g["out_keys"], g["out_values"], g["out_valid"])):
        assert torch.equal(mk, rk) and torch.equal(mv, rv)


@pytest.mark.parametrize("carried,length,capacity", [(128, 1, 128), (0, 128, 128), (128, 128, 128), (32, 300, 32),
                                                     (5, 0, 8)])
def test_salient_admission_matches_oracle(carried, length, capacity, cuda):
    g = torch.Generator().manual_seed(carried + length)
    batch, width = 3, 24
    ck, cv = torch.randn(batch, carried, width, generator=g), torch.randn(batch, carried, width, generator=g)
    cvalid = torch.rand(batch, carried, generator=g) > 0.5
    keys, values = torch.randn(batch, length, width, generator=g), torch.randn(batch, length, width, generator=g)
    surprise = torch.rand(batch, length, generator=g)
    valid = torch.rand(batch, length, generator=g) > 0.1
    k, v, ok, adm = salient_admission(*(t.to(cuda) for t in (ck, cv, cvalid, keys, values, surprise, valid)),
                                      0.6, capacity)
    admission = valid & (surprise > 0.6)
    expected = ops.salient_tail(ck, cv, cvalid, keys, values, admission, capacity)
    assert torch.equal(adm.cpu(), admission)
    assert torch.equal(ok.cpu(), expected[2])
    assert torch.equal(k.cpu(), expected[0]) and torch.equal(v.cpu(), expected[1])


def test_surprise_accepts_strided_targets(cuda):
    """A window slice of the ids (ids[:, a:b]) is not contiguous; the op must
    read it by value, not by raw pointer."""
    prior, weight, bias, targets, valid = _case(2, 40, 32, 256, torch.float32, seed=9)
    wide = torch.randint(0, 256, (2, 100), generator=torch.Generator().manual_seed(3))
    wide[:, 30:70] = targets
    strided = wide.to(cuda)[:, 30:70]
    assert not strided.is_contiguous()
    from koemi_5hom_b200.cuda_kernels import _ops
    got = _ops.causal_surprise_forward(prior.to(cuda), weight.to(cuda), bias.to(cuda), strided, valid.to(cuda),
                                       torch.float32)
    torch.testing.assert_close(got.cpu().double(), ops.causal_surprise(prior, weight, bias, targets, valid),
                               rtol=2e-5, atol=2e-6)


def test_surprise_tensor_core_decode_shape(cuda):
    """Config-5 decode: 256 rows x d=2048 against the 32767-entry content head
    (bf16 operands, fp32 accumulate); sampled rows vs the fp64 oracle."""
    g = torch.Generator().manual_seed(12)
    prior = torch.randn(1, 256, 2048, generator=g).bfloat16()
    weight = (torch.randn(32767, 2048, generator=g) * 0.02).bfloat16()
    bias = (torch.randn(32767, generator=g) * 0.002).bfloat16()
    targets = torch.randint(0, 32767, (1, 256), generator=g)
    valid = torch.ones(1, 256, dtype=torch.bool)
    got = causal_surprise(*(t.to(cuda) for t in (prior, weight, bias, targets, valid)))
    pick = [0, 1, 127, 128, 200, 255]
    expected = ops.causal_surprise(prior[:, pick], weight, bias, targets[:, pick], valid[:, pick])
    torch.testing.assert_close(got[:, pick].cpu().double(), expected.bfloat16().double(), rtol=1.6e-2, atol=4e-3)


@pytest.mark.parametrize("blocks,batch,width,vocab,dtype", [(3, 100, 256, 1000, torch.bfloat16),
                                                            (2, 37, 128, 300, torch.float16),
                                                            (24, 32, 2048, 32768, torch.bfloat16)])
def test_merged_head_pass_gives_logits_and_next_surprise(blocks, batch, width, vocab, dtype, cuda):
    """The decode step's merged head pass against the oracle: the logits rows
    equal row W^T + b over the full head, and the surprise finished from the
    prior rows' partials once the tokens are known equals causal_surprise over
    the content head (PAD column removed, targets remapped). Row counts that
    are not multiples of 32 put prior rows and logits rows in one warp."""
    from koemi_5hom_b200 import _native
    pad = 256
    g = torch.Generator().manual_seed(vocab + batch)
    lse_rows = blocks * batch
    rows = torch.randn(lse_rows + batch, width, generator=g).to(dtype)
    weight = (torch.randn(vocab, width, generator=g) * width ** -0.5).to(dtype)
    bias = (torch.randn(vocab, generator=g) * 0.1).to(dtype)
    tokens = torch.randint(0, vocab, (batch,), generator=g)
    tokens[::7] = pad  # invalid streams score 0
    valid = tokens != pad
    d_rows, d_w, d_b = rows.to(cuda), weight.to(cuda), bias.to(cuda)
    lib = _native.library()
    slices = lib.koemi_think_head_pass_slices(vocab)
    partials = torch.empty(slices, lse_rows, 3, device=cuda)
    logits = torch.empty(batch, vocab, device=cuda)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    code = _native.dtype_code(dtype)
    _native.call("koemi_think_head_pass", d_rows.data_ptr(), lse_rows, batch, width, d_w.data_ptr(), d_b.data_ptr(),
                 vocab, pad, partials.data_ptr(), logits.data_ptr(), code, stream)
    surprise = torch.empty(lse_rows, device=cuda)
    d_tokens, d_valid = tokens.to(cuda), valid.to(cuda)
    _native.call("koemi_think_surprise_from_partials", d_rows.data_ptr(), d_w.data_ptr(), d_b.data_ptr(),
                 d_tokens.data_ptr(), d_valid.data_ptr(), partials.data_ptr(), slices, lse_rows, batch, width, vocab,
                 pad, code, surprise.data_ptr(), stream)
    torch.cuda.synchronize()
    expected_logits = rows[lse_rows:].double() @ weight.double().T + bias.double()
    torch.testing.assert_close(logits.cpu().double(), expected_logits, rtol=1e-5, atol=1e-4)
    keep = [i for i in range(vocab) if i != pad]
    content = torch.where(tokens > pad, tokens - 1, tokens).repeat(blocks)
    expected = ops.causal_surprise(rows[:lse_rows], weight[keep], bias[keep], content, valid.repeat(blocks))
    torch.testing.assert_close(surprise.cpu().double(), expected, rtol=1e-5, atol=2e-6)
    assert bool((surprise.cpu()[~valid.repeat(blocks)] == 0).all())
