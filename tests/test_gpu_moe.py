"""MoE front on the GPU: bit-exact routing / permutation, fp parity for the MLP and combines."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from koemi_5hom_b200.cuda_kernels import _ops
from koemi_5hom_b200.cuda_kernels.moe import (CudaMoeValidationError, combine_topk, grouped_expert_mlp_inference,
                                              permute_topk, route_topk_valid)
from oracle import ops

pytestmark = pytest.mark.gpu


def test_route_matches_reference_golden(golden_ops, cuda):
    g = golden_ops["route"]
    for key, expected in g["assignments"].items():
        experts, k = map(int, key.split("_"))
        if k > 1 and experts < 8:
            # the front rejects duplicates on valid tokens; compare the raw op
            got = _ops.route_topk(g["tokens"].to(cuda), g["previous"].to(cuda), g["valid"].to(cuda), experts, k)
            assert torch.equal(got.cpu().reshape(expected.shape), expected), key
            continue
        got = route_topk_valid(g["tokens"].to(cuda), g["previous"].to(cuda), g["valid"].to(cuda),
                               expert_count=experts, top_k=k)
        assert torch.equal(got.cpu(), expected), key
    for dtype in (torch.int32,):
        got = _ops.route_topk(g["tokens"].to(dtype).to(cuda), g["previous"].to(dtype).to(cuda), g["valid"].to(cuda), 64, 2)
        assert torch.equal(got.cpu().reshape(g["assignments"]["64_2"].shape), g["assignments"]["64_2"])


def test_route_known_answer(golden_ops, cuda):
    g = golden_ops["route_kat"]
    got = route_topk_valid(g["tokens"].to(cuda), g["previous"].to(cuda), (g["tokens"] != 256).to(cuda),
                           expert_count=4, top_k=1)
    assert got[..., 0].cpu().tolist() == [[1, 0, 0, -1]]


def test_route_front_rejects_duplicates(cuda):
    # with E=2, k=2 slot 1 can repeat slot 0 for some hashes
    tokens = torch.arange(200, device=cuda).reshape(1, 200)
    with pytest.raises(CudaMoeValidationError, match="duplicate"):
        for shift in range(50):
            route_topk_valid(tokens + shift, tokens, torch.ones_like(tokens, dtype=torch.bool), expert_count=3, top_k=3)


@pytest.mark.parametrize("key", ["4_2_50", "64_2_700", "5_3_41", "300_2_2000", "3000_2_4000"])
def test_permutation_is_bit_exact_with_stable_argsort(golden_ops, key, cuda):
    g = golden_ops["permute"][key]
    experts = int(key.split("_")[0])
    assignments, valid = g["assignments"], g["valid"]
    width = 24
    context = torch.randn(assignments.shape[0], width, generator=torch.Generator().manual_seed(1))
    sorted_context, rows, keys, offsets, positions = _ops.permute_topk(
        context.to(cuda), assignments.to(cuda), valid.to(cuda), experts, True)
    order = g["order"].numpy()
    top_k = assignments.shape[1]
    assert np.array_equal(rows.cpu().numpy(), order // top_k)
    assert np.array_equal(keys.cpu().numpy(), g["keys_sorted"].numpy())
    assert np.array_equal(np.diff(offsets.cpu().numpy()), g["counts"].numpy()[:experts])
    assert offsets[0].item() == 0
    inverse = np.empty_like(order)
    inverse[order] = np.arange(order.size)
    assert np.array_equal(positions.cpu().numpy(), inverse)
    n_valid = int(offsets[-1])
    assert torch.equal(sorted_context[:n_valid].cpu(), context[torch.from_numpy(order[:n_valid] // top_k)])
    assert bool((sorted_context[n_valid:] == 0).all())


@pytest.mark.parametrize("tokens,top_k,experts", [(2048, 2, 64), (2049, 2, 64), (1365, 3, 255), (1365, 3, 256),
                                                  (256, 2, 64), (1, 1, 1), (4096, 1, 7)])
def test_single_cta_and_radix_permutations_agree_with_oracle(tokens, top_k, experts, cuda):
    """Both sides of the one-CTA limit (4096 pairs, 255 experts), with dropped
    tokens, out-of-range ids and repeated slots in the assignments."""
    g = torch.Generator().manual_seed(tokens * 7 + experts)
    assignments = torch.randint(-1, experts + 2, (tokens, top_k), generator=g)
    if top_k > 1:
        assignments[::5, 1] = assignments[::5, 0]
    valid = torch.rand(tokens, generator=g) > 0.1
    order, rows_ref, keys_ref, offsets_ref, positions_ref = ops.permute_topk(assignments.numpy(), valid.numpy(),
                                                                            experts)
    context = torch.randn(tokens, 16, generator=g)
    for dtype in (torch.int64, torch.int32):
        sorted_context, rows, keys, offsets, positions = _ops.permute_topk(
            context.to(cuda), assignments.to(device=cuda, dtype=dtype), valid.to(cuda), experts, True)
        assert np.array_equal(rows.cpu().numpy(), rows_ref)
        assert np.array_equal(keys.cpu().numpy(), keys_ref)
        assert np.array_equal(offsets.cpu().numpy(), offsets_ref)
        assert np.array_equal(positions.cpu().numpy(), positions_ref)
        n_valid = int(offsets_ref[-1])
        assert torch.equal(sorted_context[:n_valid].cpu(), context[torch.from_numpy(rows_ref[:n_valid])])
        assert bool((sorted_context[n_valid:] == 0).all())


def test_permute_front_and_combine_preserve_stable_pairs(cuda):
    """tests/cuda/test_moe_cuda.py:60-82 of the reference, restated."""
    context = torch.arange(12, device=cuda, dtype=torch.float32).reshape(3, 4)
    assignments = torch.tensor([[1, 0], [0, 1], [1, 0]], device=cuda)
    valid = torch.tensor([True, True, False], device=cuda)
    sorted_context, sorted_rows, sorted_experts, offsets = permute_topk(context, assignments, valid, expert_count=2)
    valid_pairs = int(offsets[-1].item())
    assert sorted_context.shape[0] == 6 and valid_pairs == 4
    assert sorted_experts[:valid_pairs].tolist() == [0, 0, 1, 1]
    assert sorted_rows[:valid_pairs].tolist() == [0, 1, 0, 1]
    outputs = sorted_context + 10.0
    combined = combine_topk(outputs, sorted_rows, offsets, token_count=3, top_k=2)
    expected = torch.zeros_like(context)
    for pair in range(valid_pairs):
        expected[sorted_rows[pair]] += outputs[pair] / 2.0
    torch.testing.assert_close(combined, expected)


def _experts(e, h, d, dtype, seed, scale=0.2):
    g = torch.Generator().manual_seed(seed)
    t = lambda *s: (torch.randn(*s, generator=g) * scale).to(dtype)  # noqa: E731
    return t(e, h, d), t(e, h), t(e, h, d), t(e, h), t(e, d, h), t(e, d)


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 2e-4), (torch.bfloat16, 3e-2), (torch.float16, 5e-3)])
@pytest.mark.parametrize("e,h,d,tokens,k", [(2, 3, 4, 3, 1), (4, 512, 256, 300, 1), (8, 256, 128, 1000, 2),
                                            (16, 64, 96, 77, 2)])
def test_grouped_mlp_matches_oracle(dtype, tol, e, h, d, tokens, k, cuda):
    g = torch.Generator().manual_seed(e * 100 + h)
    context = torch.randn(tokens, d, generator=g).to(dtype)
    assignments = torch.stack([torch.randperm(e, generator=g)[:k] for _ in range(tokens)])
    valid = torch.rand(tokens, generator=g) > 0.1
    weights = _experts(e, h, d, dtype, seed=h)
    sc, rows, se, offsets, _ = _ops.permute_topk(context.to(cuda), assignments.to(cuda), valid.to(cuda), e, True)
    got = grouped_expert_mlp_inference(sc, se, offsets, *(w.to(cuda) for w in weights))
    expected = ops.grouped_mlp(sc.cpu(), se.cpu(), offsets.cpu(), *weights,
                               round_hidden_to=dtype if dtype != torch.float32 else None)
    scale = expected.abs().max().item() + 1e-6
    assert got.dtype == dtype
    torch.testing.assert_close(got.cpu().double() / scale, expected.to(dtype).double() / scale, rtol=tol, atol=tol)
    assert bool((got[int(offsets[-1]):] == 0).all())


def test_grouped_mlp_reference_contract(cuda):
    """tests/cuda/test_moe_cuda.py:84-113 of the reference, restated."""
    e, d, h, p = 2, 4, 3, 3
    sorted_context = torch.randn(p, d, device=cuda)
    sorted_experts = torch.tensor([0, 0, 1], device=cuda)
    offsets = torch.tensor([0, 2, 3], device=cuda)
    weights = [w.to(cuda) for w in _experts(e, h, d, torch.float32, seed=3, scale=1.0)]
    got = grouped_expert_mlp_inference(sorted_context, sorted_experts, offsets, *weights)
    rows = [ops.gated_ffn(sorted_context[i:i + 1].cpu(), *(w[x].cpu() for w in weights))[0]
            for i, x in enumerate([0, 0, 1])]
    torch.testing.assert_close(got.cpu().double(), torch.stack(rows), rtol=2e-4, atol=2e-4)


def test_combine_topk_matches_oracle_and_is_deterministic(cuda):
    g = torch.Generator().manual_seed(5)
    tokens, k, e, d = 500, 2, 16, 64
    assignments = torch.stack([torch.randperm(e, generator=g)[:k] for _ in range(tokens)])
    valid = torch.rand(tokens, generator=g) > 0.1
    context = torch.randn(tokens, d, generator=g)
    sc, rows, se, offsets, _ = _ops.permute_topk(context.to(cuda), assignments.to(cuda), valid.to(cuda), e, True)
    y = torch.randn(sc.shape, generator=g).to(cuda)
    first = combine_topk(y, rows, offsets, token_count=tokens, top_k=k)
    second = combine_topk(y, rows, offsets, token_count=tokens, top_k=k)
    assert torch.equal(first, second)
    torch.testing.assert_close(first.cpu().double(), ops.combine_topk(y.cpu(), rows.cpu(), offsets.cpu(), tokens, k),
                               rtol=1e-5, atol=1e-6)


def test_learned_topk_matches_reference_router(golden_ops, cuda):
    g = golden_ops["moe_learned"]
    flat = g["context"].reshape(-1, g["context"].shape[-1])
    valid = g["valid"].reshape(-1)
    logits = torch.where(valid.unsqueeze(-1), flat, torch.zeros_like(flat)) @ g["state"]["gate.weight"].T
    idx, weights, probs = _ops.learned_topk(logits.to(cuda), valid.to(cuda), 2, False)
    assert torch.equal(idx.cpu().reshape(g["assignments"].shape), g["assignments"])
    torch.testing.assert_close(weights.cpu().reshape(g["weights"].shape), g["weights"], rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(probs.sum(0).cpu(), g["probability_mass"], rtol=1e-5, atol=1e-5)


def test_combine_residual_rmsnorm_matches_reference_static_dispatch(golden_ops, cuda):
    g = golden_ops["moe_static"]
    s = g["state"]
    flat = g["context"].reshape(-1, 32)
    valid = g["valid"].reshape(-1)
    tokens_flat = g["ids"].reshape(-1)
    assignments = torch.from_numpy(ops.route_topk(tokens_flat.numpy(), g["prev"].reshape(-1).numpy(),
                                                  valid.numpy(), 6, 2))
    assert torch.equal(assignments.reshape(g["assignments"].shape), g["assignments"])
    stack = lambda name: torch.stack([s[f"experts.{i}.{name}"] for i in range(6)]).to(cuda)  # noqa: E731
    sc, rows, se, offsets, positions = _ops.permute_topk(flat.to(cuda), assignments.to(cuda), valid.to(cuda), 6, True)
    y = _ops.grouped_expert_mlp(sc, se, offsets, stack("gate_projection.weight"), stack("gate_projection.bias"),
                                stack("value_projection.weight"), stack("value_projection.bias"),
                                stack("output_projection.weight"), stack("output_projection.bias"))
    mixed = _ops.combine_residual_rmsnorm(flat.to(cuda), y, positions, offsets, None, valid.to(cuda),
                                          s["output_normalizer.weight"].to(cuda), 2, 1e-6)
    torch.testing.assert_close(mixed.cpu(), g["mixed"].reshape(-1, 32), rtol=2e-5, atol=2e-5)


def test_moe_baseline_config_routing_properties(cuda):
    """Config 4 routing at full size (131072 tokens, 64 experts, top-2): the
    hash route is bit-exact with the oracle and the permutation is a stable
    sort (checked through size-independent invariants)."""
    g = torch.Generator().manual_seed(4)
    tokens = torch.randint(0, 256, (131072,), generator=g)
    previous = torch.cat((torch.tensor([256]), tokens[:-1]))
    valid = torch.ones(131072, dtype=torch.bool)
    got = _ops.route_topk(tokens.to(cuda), previous.to(cuda), valid.to(cuda), 64, 2)
    assert np.array_equal(got.cpu().numpy(), ops.route_topk(tokens.numpy(), previous.numpy(), valid.numpy(), 64, 2))
    x = torch.randn(131072, 1024, generator=g).bfloat16().to(cuda)
    sc, rows, keys, offsets, positions = _ops.permute_topk(x, got, valid.to(cuda), 64, True)
    order, o_rows, o_keys, o_offsets, o_positions = ops.permute_topk(got.cpu().numpy(), valid.numpy(), 64)
    assert np.array_equal(rows.cpu().numpy(), o_rows)
    assert np.array_equal(offsets.cpu().numpy(), o_offsets)
    assert torch.equal(sc[:4096], x[rows[:4096]])


def _sampled_rows_check(sc, se, offsets, y, weights, rows, dtype, tol):
    """Oracle (fp64, hidden rounded to dtype) on a sample of sorted rows."""
    gw, gb, vw, vb, ow, ob = weights
    for i in rows:
        e = int(se[i])
        x = sc[i:i + 1].cpu().double()
        hidden = ops.silu(x @ gw[e].cpu().double().T + gb[e].cpu().double()) * (
            x @ vw[e].cpu().double().T + vb[e].cpu().double())
        hidden = hidden.to(dtype).double()
        expected = hidden @ ow[e].cpu().double().T + ob[e].cpu().double()
        got = y[i].cpu().double()
        scale = expected.abs().max().item() + 1e-6
        torch.testing.assert_close(got / scale, expected[0].to(dtype).double() / scale, rtol=tol, atol=tol)


@pytest.mark.parametrize("tokens,d,h,e,k", [(131072, 1024, 2048, 64, 2), (256, 2048, 4096, 64, 2),
                                             (32, 2048, 4096, 8, 2)])
def test_grouped_mlp_tensor_core_baseline_shapes(tokens, d, h, e, k, cuda):
    """Config 4 (131072 tokens, d=1024, d_ff=2048, 64 experts, top-2), the
    config-5 decode step (256 streams, d=2048, d_ff=4096) and one rank's share
    of it at 8 GPUs (32 streams, 8 experts: the narrow output tiles): sampled
    rows of every segment position class against the fp64 oracle."""
    g = torch.Generator(device=cuda).manual_seed(tokens)
    x = torch.randn(tokens, d, generator=g, device=cuda).bfloat16()
    scores = torch.rand(tokens, e, generator=g, device=cuda)
    assignments = scores.topk(k, dim=-1).indices
    valid = torch.ones(tokens, dtype=torch.bool, device=cuda)
    weights = tuple((torch.randn(*s, generator=g, device=cuda) * 0.02).bfloat16() for s in
                    ((e, h, d), (e, h), (e, h, d), (e, h), (e, d, h), (e, d)))
    sc, rows, se, offsets, _ = _ops.permute_topk(x, assignments, valid, e, True)
    y = _ops.grouped_expert_mlp(sc, se, offsets, *weights)
    torch.cuda.synchronize()
    off = offsets.cpu()
    sample = set()
    for expert in (0, 1, e // 2, e - 1):
        begin, end = int(off[expert]), int(off[expert + 1])
        for r in (begin, begin + 1, begin + 127, begin + 128, (begin + end) // 2, end - 1):
            if begin <= r < end:
                sample.add(r)
    _sampled_rows_check(sc, se, offsets, y, weights, sorted(sample), torch.bfloat16, 3e-2)
    assert bool(torch.isfinite(y).all())


@pytest.mark.parametrize("rows,n,k,stride,bias", [(256, 4096, 2048, 2048, True), (256, 2048, 8192, 8192, True),
                                                  (3000, 1000, 512, 512, False), (256, 16, 2048, 8192, True),
                                                  (7, 300, 64, 64, True), (32, 10242, 2048, 2048, True),
                                                  (200, 1030, 4096, 4096, True), (129, 2048, 8192, 8192, False),
                                                  (256, 6146, 2048, 2048, True), (8192, 4096, 2048, 2048, True),
                                                  (5000, 1000, 512, 512, True), (4100, 300, 64, 72, False),
                                                  (4608, 6146, 512, 512, True), (40, 4096, 2048, 2048, True),
                                                  (1, 8192, 1024, 1024, False), (64, 5000, 8192, 8200, True),
                                                  (17, 3600, 256, 264, True)])
def test_dense_projection_matches_fp64(rows, n, k, stride, bias, cuda):
    """tcgen05 projection (at most 64 rows: full-K column tiles with several
    TMEM accumulators; then cluster split-K, direct, or paired tiles in banded
    order from 4096 rows on, ragged last band included) against fp64 on the
    same bf16 operands."""
    g = torch.Generator(device=cuda).manual_seed(rows + n)
    wide = torch.randn(rows, stride, generator=g, device=cuda).bfloat16()
    a = wide[:, :k]
    w = (torch.randn(n, k, generator=g, device=cuda) * k ** -0.5).bfloat16()
    b = (torch.randn(n, generator=g, device=cuda) * 0.1).bfloat16() if bias else None
    out = _ops.dense_projection(a, w, b)
    expected = a.double() @ w.double().T + (b.double() if bias else 0.0)
    torch.testing.assert_close(out.double(), expected, rtol=1e-4, atol=1e-4)
    again = _ops.dense_projection(a, w, b)
    assert torch.equal(out, again)  # fixed-order split-K reduction
    # launched as for model parameters (weights requested before the wait on
    # the previous kernel): the same result
    assert torch.equal(_ops.dense_projection(a, w, b, True), out)


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_gather_rows_equals_permute_gather(out_dtype, cuda):
    g = torch.Generator().manual_seed(11)
    tokens, experts, width = 300, 16, 128
    context = torch.randn(tokens, width, generator=g).to(cuda)
    assignments = torch.randint(-1, experts + 1, (tokens, 2), generator=g).to(cuda)
    valid = (torch.rand(tokens, generator=g) > 0.1).to(cuda)
    sorted_ctx, rows, _, offsets, _ = _ops.permute_topk(context.to(out_dtype), assignments, valid, experts, True)
    got = _ops.gather_rows(context, rows, offsets, out_dtype)
    assert torch.equal(got, sorted_ctx)


@pytest.mark.parametrize("with_next", [True, False])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_combine_with_next_norm_equals_two_ops(with_next, out_dtype, cuda):
    from koemi_5hom_b200.cuda_kernels import _ops as ops_
    g = torch.Generator().manual_seed(12)
    tokens, experts, width, k = 256, 8, 2048, 2
    context = torch.randn(tokens, width, generator=g).to(cuda)
    assignments = torch.randint(0, experts, (tokens, k), generator=g).to(cuda)
    valid = (torch.rand(tokens, generator=g) > 0.1).to(cuda)
    _, rows, _, offsets, positions = ops_.permute_topk(context, assignments, valid, experts, False)
    expert_out = torch.randn(tokens * k, width, generator=g).bfloat16().to(cuda)
    norm = (1 + 0.1 * torch.randn(width, generator=g)).to(cuda)
    nxt = (1 + 0.1 * torch.randn(width, generator=g)).to(cuda) if with_next else None
    x = ops_.combine_residual_rmsnorm(context, expert_out, positions, offsets, None, valid, norm, k, 1e-6)
    expected = ops_.rms_norm(x, None, nxt, None, 1e-6, out_dtype) if with_next else x.to(out_dtype)
    got = ops_.combine_residual_rmsnorm_next(context, expert_out, positions, offsets, None, valid, norm, nxt, k, 1e-6,
                                             out_dtype)
    assert torch.equal(got, expected)




@pytest.mark.parametrize("groups,rows,n,k", [(4, 128, 256, 2048), (3, 100, 136, 64), (256, 128, 256, 2048),
                                             (2, 130, 2048, 256), (5, 7, 24, 8)])
def test_grouped_projection_matches_fp64(groups, rows, n, k, cuda):
    """Per-group products on tensor cores (the prefill's ring reads: queries x
    keys, weights x transposed values) against fp64 on the same bf16 operands;
    groups whose rows share a 128-row tile with the next group (rows < 128 or
    not a multiple of 128) keep their rows apart."""
    g = torch.Generator(device=cuda).manual_seed(groups * 1000 + rows + n)
    a = torch.randn(groups * rows, k, generator=g, device=cuda).bfloat16()
    b = (torch.randn(groups * n, k, generator=g, device=cuda) * k ** -0.5).bfloat16()
    out = _ops.grouped_projection(a, b, groups)
    expected = torch.bmm(a.double().view(groups, rows, k), b.double().view(groups, n, k).transpose(1, 2))
    torch.testing.assert_close(out.view(groups, rows, n).double(), expected, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("tokens,experts,top_k,width,hidden", [(256, 64, 2, 256, 512), (32, 8, 2, 128, 256),
                                                                 (77, 5, 3, 64, 128)])
def test_decode_norm_gather_and_mapped_mlp_equal_the_general_path(tokens, experts, top_k, width, hidden, cuda):
    """The decode step's expert path with one permutation per step: the
    fusion norm that also gathers each pair's row (koemi_moe_norm_gather) and
    the grouped MLP on a tile map computed once (koemi_moe_tile_prefix +
    koemi_moe_grouped_expert_mlp_mapped) equal the norm, the row gather and
    the grouped MLP bit for bit on every valid pair."""
    from koemi_5hom_b200 import _native
    g = torch.Generator().manual_seed(tokens + experts)
    fused = (torch.randn(tokens, width, generator=g) * 2.0).to(cuda)
    norm = (1.0 + 0.1 * torch.randn(width, generator=g)).to(cuda)
    assignments = torch.randint(-1, experts, (tokens, top_k), generator=g).to(cuda)
    valid = (torch.rand(tokens, generator=g) > 0.1).to(cuda)
    weights = tuple((torch.randn(*shape, generator=g) * 0.05).bfloat16().to(cuda) for shape in
                    ((experts, hidden, width), (experts, hidden), (experts, hidden, width), (experts, hidden),
                     (experts, width, hidden), (experts, width)))
    context = _ops.rms_norm(fused, None, norm, None, 1e-6, torch.float32)
    _, sorted_tokens, sorted_experts, offsets, positions = _ops.permute_topk(context, assignments, valid, experts,
                                                                              False)
    rows = _ops.gather_rows(context, sorted_tokens, offsets, torch.bfloat16)
    expected = _ops.grouped_expert_mlp(rows, sorted_experts, offsets, *weights)
    pairs = tokens * top_k
    stream = torch.cuda.current_stream(cuda).cuda_stream
    mine_context = torch.empty_like(context)
    mine_rows = torch.zeros(pairs, width, dtype=torch.bfloat16, device=cuda)
    _native.call("koemi_moe_norm_gather", fused.data_ptr(), norm.data_ptr(), 1e-6, mine_context.data_ptr(),
                 positions.data_ptr(), offsets.data_ptr(), experts, mine_rows.data_ptr(), _native.BF16, tokens, width,
                 top_k, stream)
    prefix = torch.empty(experts + 1, dtype=torch.int32, device=cuda)
    _native.call("koemi_moe_tile_prefix", offsets.data_ptr(), experts, prefix.data_ptr(), stream)
    out = torch.empty(pairs, width, dtype=torch.bfloat16, device=cuda)
    size = _native.library().koemi_moe_grouped_mlp_workspace(pairs, width, hidden, experts, _native.BF16)
    workspace = _native.workspace(size, cuda)
    _native.call("koemi_moe_grouped_expert_mlp_mapped", mine_rows.data_ptr(), prefix.data_ptr(), offsets.data_ptr(),
                 *(w.data_ptr() for w in weights), out.data_ptr(), pairs, width, hidden, experts, _native.BF16,
                 workspace.data_ptr(), workspace.numel(), stream)
    torch.cuda.synchronize()
    live = int(offsets[-1])
    assert torch.equal(mine_context, context)
    assert torch.equal(mine_rows[:live], rows[:live])
    assert torch.equal(out[:live], expected[:live])
