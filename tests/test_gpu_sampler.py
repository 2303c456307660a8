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
