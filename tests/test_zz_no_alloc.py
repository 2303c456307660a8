"""The allocation-free permutation entry point, called through the C ABI.

Some callers cannot allocate device memory: a host runtime that reaches the
library over FFI and only passes buffers it already owns, or code that must not
call cudaMalloc while other work is in flight. ``koemi_moe_permute_topk_static``
serves them with a fixed scratch array inside the library. This file checks
that it returns exactly what the workspace entry point returns, on two calls in
a row with different inputs (so nothing left in the shared scratch by the first
call leaks into the second), and that oversized requests are refused. It is
collected last so that a failure here never hides the other tests.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from koemi_5hom_b200 import _native

pytestmark = pytest.mark.gpu


def _permute(static: bool, context, assignments, valid, experts):
    lib = _native.library()
    tokens, top_k = assignments.shape
    width = context.shape[1]
    pairs = tokens * top_k
    device = context.device
    out = {
        "sorted_context": torch.empty(pairs, width, dtype=context.dtype, device=device),
        "sorted_rows": torch.empty(pairs, dtype=torch.int64, device=device),
        "sorted_experts": torch.empty(pairs, dtype=torch.int64, device=device),
        "segment_offsets": torch.empty(experts + 1, dtype=torch.int64, device=device),
        "pair_positions": torch.empty(pairs, dtype=torch.int64, device=device),
    }
    stream = torch.cuda.current_stream(device).cuda_stream
    common = (context.data_ptr(), assignments.data_ptr(), valid.data_ptr(), out["sorted_context"].data_ptr(),
              out["sorted_rows"].data_ptr(), out["sorted_experts"].data_ptr(), out["segment_offsets"].data_ptr(),
              out["pair_positions"].data_ptr(), tokens, width, top_k, experts, _native.dtype_code(context.dtype),
              _native.dtype_code(assignments.dtype))
    if static:
        status = lib.koemi_moe_permute_topk_static(*common, stream)
        _native.check("koemi_moe_permute_topk_static", status)
    else:
        size = lib.koemi_moe_permute_workspace(tokens, top_k, experts)
        workspace = torch.empty(max(size, 256), dtype=torch.uint8, device=device)
        status = lib.koemi_moe_permute_topk(*common, workspace.data_ptr(), workspace.numel(), stream)
        _native.check("koemi_moe_permute_topk", status)
    torch.cuda.synchronize(device)
    return out


@pytest.mark.parametrize("call", [0, 1])
def test_static_permute_matches_workspace_permute_on_consecutive_calls(call):
    device = torch.device("cuda", 0)
    results = []
    # the radix path (8000 pairs at 64 experts; 300 experts) and the one-CTA
    # path (2000 pairs at 16 experts), whose keys and counts live in the
    # scratch too
    shapes = ((4000, 64, 2, 96), (777, 300, 3, 40), (1000, 16, 2, 64))
    for seed, (tokens, experts, top_k, width) in enumerate(shapes):
        g = torch.Generator().manual_seed(100 * call + seed)
        assignments = torch.randint(-1, experts + 1, (tokens, top_k), generator=g).to(device)
        valid = (torch.rand(tokens, generator=g) > 0.1).to(device)
        context = torch.randn(tokens, width, generator=g).bfloat16().to(device)
        expected = _permute(False, context, assignments, valid, experts)
        got = _permute(True, context, assignments, valid, experts)
        for name in expected:
            assert torch.equal(got[name], expected[name]), (seed, name)  # bit-exact, like the permute tests
        results.append(got["segment_offsets"][-1].item())
    assert len(set(results)) == len(results)  # the calls really were different problems


def test_static_permute_refuses_oversized_requests():
    lib = _native.library()
    status = lib.koemi_moe_permute_topk_static(None, None, None, None, None, None, None, None, 200000, 64, 2, 64,
                                              _native.BF16, _native.I64, None)
    assert status == _native.KOEMI_ERR_UNSUPPORTED
    message = _native.last_error()
    need = lib.koemi_moe_permute_workspace(200000, 2, 64)
    assert f"needs {need} scratch bytes" in message and "65536 token-expert pairs always fit" in message


def test_static_permute_accepts_65536_pairs_at_any_expert_count():
    lib = _native.library()
    for experts in (1, 64, 255, 256, 2048, 1 << 20):
        assert lib.koemi_moe_permute_workspace(65536, 1, experts) <= 2 << 20
