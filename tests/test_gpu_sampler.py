"""Native greedy sampler against TokenSampler's torch formula
(fast_decode.py:40-87: PAD filled with -inf, then argmax)."""
from __future__ import annotations

import pytest
import torch

from koemi_5hom_b200 import _native
from koemi_5hom_b200.cuda_kernels import _ops
from koemi_5hom_b200.model.settings import PAD_TOKEN_ID

pytestmark = pytest.mark.gpu


def _torch_greedy(logits: torch.Tensor, pad: int) -> torch.Tensor:
    return logits.float().index_fill(-1, torch.tensor([pad], device=logits.device), float("-inf")).argmax(
        dim=-1, keepdim=True)


@pytest.mark.parametrize("rows,vocab", [(256, 32768), (3, 257), (17, 1001), (1, 5)])
def test_greedy_matches_masked_argmax(rows, vocab, cuda):
    g = torch.Generator(device=cuda).manual_seed(rows + vocab)
    logits = torch.randn(rows, vocab, generator=g, device=cuda)
    pad = PAD_TOKEN_ID if vocab > PAD_TOKEN_ID else vocab - 1
    assert torch.equal(_ops.greedy_tokens(logits, pad), _torch_greedy(logits, pad))


def test_greedy_ties_infinities_nan_and_pad(cuda):
    vocab = 1000
    logits = torch.randn(8, vocab, device=cuda)
    logits[0, [5, 700, 999]] = 50.0              # ties: first index
    logits[1, PAD_TOKEN_ID] = 1e9                 # PAD is never chosen
    logits[2] = float("-inf")                     # all -inf: index 0 (first)
    logits[3, [10, 20]] = float("nan")            # NaN ranks first, first NaN wins
    logits[4, 900:] = float("inf")                # +inf ties
    logits[5] = 0.0                               # all equal
    logits[6, PAD_TOKEN_ID] = float("nan")        # a masked NaN is -inf
    got = _ops.greedy_tokens(logits, PAD_TOKEN_ID)
    assert torch.equal(got, _torch_greedy(logits, PAD_TOKEN_ID))
    assert got[0, 0] == 5 and got[1, 0] != PAD_TOKEN_ID and got[3, 0] == 10 and got[4, 0] == 900


def test_greedy_row_stride_through_the_c_abi(cuda):
    wide = torch.randn(9, 1100, device=cuda)
    logits = wide[:, 3:1003]  # rows 1100 floats apart, first element not 16-byte aligned
    out = torch.empty(9, dtype=torch.int64, device=cuda)
    _native.call("koemi_sampler_greedy", wide.data_ptr() + 12, 9, 1000, 1100, PAD_TOKEN_ID, out.data_ptr(),
                 torch.cuda.current_stream().cuda_stream)
    assert torch.equal(out.unsqueeze(1), _torch_greedy(logits, PAD_TOKEN_ID))


@pytest.mark.parametrize("rows,vocab,temperature,top_k", [(256, 32768, 0.8, None), (7, 1000, 1.3, 50),
                                                          (33, 300, 0.5, None)])
def test_temperature_sampler_matches_oracle(rows, vocab, temperature, top_k, cuda):
    """The native Gumbel-max sampler draws the oracle's tokens for the same
    (seed, stream, step): the random stream is restated bit for bit; only the
    logarithms differ in the last bits, so rows whose two best perturbed
    scores lie within 1e-4 are left out."""
    import numpy as np
    from koemi_5hom_b200.runtime import SamplingPolicy, TokenSampler
    from oracle import ops
    g = torch.Generator().manual_seed(rows * vocab)
    logits = torch.randn(rows, vocab, generator=g) * 3.0
    logits[0, :5] = float("nan")
    sampler = TokenSampler(SamplingPolicy(temperature=temperature, top_k=top_k), cuda, stream_seed=1234,
                           stream_offset=40)
    for step in range(3):
        got = sampler(logits.to(cuda)).cpu().squeeze(1).numpy()
        thresholds = None
        if top_k is not None:
            masked = logits.clone()
            masked[:, PAD_TOKEN_ID] = float("-inf")
            thresholds = torch.topk(masked, top_k, dim=-1).values[:, -1].numpy()
        ids, scores = ops.gumbel_sample(logits.numpy(), temperature, 1234, 40, step, PAD_TOKEN_ID, thresholds)
        best2 = np.sort(np.where(np.isfinite(scores), scores, -1e30), axis=1)[:, -2:]
        decided = (best2[:, 1] - best2[:, 0]) > 1e-4
        assert decided.mean() > 0.9
        assert np.array_equal(got[decided], ids[decided]), step
        assert not np.isin(got, [PAD_TOKEN_ID]).any()
        if top_k is not None:
            assert (logits.numpy()[np.arange(rows), got] >= thresholds).all()


def test_temperature_sampler_follows_softmax(cuda):
    """Frequencies over 65536 independent streams match softmax(logits / T)
    within five standard errors per column; PAD never appears."""
    from koemi_5hom_b200.runtime import SamplingPolicy, TokenSampler
    vocab, rows, temperature = 260, 65536, 0.8
    base = torch.zeros(vocab)
    base[:6] = torch.tensor([2.0, 1.0, 0.5, 0.0, -1.0, 3.0])
    base[6:] = -4.0
    base[PAD_TOKEN_ID] = 10.0
    sampler = TokenSampler(SamplingPolicy(temperature=temperature), cuda, stream_seed=7)
    ids = sampler(base.expand(rows, vocab).contiguous().to(cuda)).cpu().squeeze(1)
    counts = torch.bincount(ids, minlength=vocab).double()
    masked = base.clone()
    masked[PAD_TOKEN_ID] = float("-inf")
    p = torch.softmax(masked.double() / temperature, dim=0)
    assert counts[PAD_TOKEN_ID] == 0
    sigma = (rows * p * (1 - p)).sqrt()
    assert bool(((counts - rows * p).abs() <= 5 * sigma + 1).all())
