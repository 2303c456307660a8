"""The CPU oracle against the golden fixtures generated from the reference."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from herm_weights import HermShape, herm_parameters
from oracle import ops
from oracle.herm import HermConfig, HermOracle


def test_scan_matches_reference(golden_ops):
    g = golden_ops["scan"]
    torch.testing.assert_close(ops.affine_scan(g["a"], g["b"], g["h0"]).float(), g["h"], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(ops.affine_scan(g["a"], g["b"]).float(), g["h_zero"], rtol=1e-5, atol=1e-5)
    gb = golden_ops["scan_broadcast"]
    torch.testing.assert_close(ops.affine_scan(gb["a"], gb["b"]).float(), gb["h"], rtol=1e-5, atol=1e-5)


def test_rmsnorm_matches_reference(golden_ops):
    g = golden_ops["rmsnorm"]
    torch.testing.assert_close(ops.rms_norm(g["x"], g["w"]).float(), g["y"], rtol=1e-5, atol=1e-5)
    y, inv = ops.rmsnorm_silu(g["x"], g["w"])
    torch.testing.assert_close(y.float(), g["silu_y"], rtol=1e-5, atol=1e-5)
    assert inv.shape == (g["x"].shape[0],)


def test_content_hash_and_routing_bit_exact(golden_ops):
    g = golden_ops["route"]
    assert np.array_equal(ops.content_hash(g["tokens"].numpy(), g["previous"].numpy()).astype(np.int64),
                          g["hash"].numpy())
    for key, expected in g["assignments"].items():
        experts, k = map(int, key.split("_"))
        got = ops.route_topk(g["tokens"].numpy(), g["previous"].numpy(), g["valid"].numpy(), experts, k)
        assert np.array_equal(got, expected.numpy()), key


def test_routing_known_answer(golden_ops):
    g = golden_ops["route_kat"]
    got = ops.route_topk(g["tokens"].numpy(), g["previous"].numpy(), (g["tokens"] != 256).numpy(), 4, 1)
    assert got[..., 0].tolist() == [[1, 0, 0, -1]]  # tests/model/test_network.py:95-101
    assert g["hash"][0, :3].tolist() == [3804756533, 3473626764, 2599103304]


def test_pair_order_is_a_stable_argsort(golden_ops):
    for key, g in golden_ops["permute"].items():
        experts = int(key.split("_")[0])
        order, rows, keys, offsets, positions = ops.permute_topk(g["assignments"].numpy(), g["valid"].numpy(), experts)
        assert np.array_equal(order, g["order"].numpy()), key
        assert np.array_equal(keys, g["keys_sorted"].numpy()), key
        assert np.array_equal(np.diff(offsets), g["counts"].numpy()[:experts]), key
        assert np.array_equal(positions[order], np.arange(order.size))


def test_salient_tail_keeps_latest_admitted_in_order(golden_ops):
    for name, g in golden_ops["salient_tail"].items():
        k, v, valid = ops.salient_tail(g["carried_keys"], g["carried_values"], g["carried_valid"], g["keys"],
                                       g["values"], g["admission"], g["capacity"])
        assert k.shape == g["out_keys"].shape, name
        for (mk, mv), (rk, rv) in zip(ops.admitted_sequence(k, v, valid),
                                      ops.admitted_sequence(g["out_keys"], g["out_values"], g["out_valid"])):
            assert torch.equal(mk, rk) and torch.equal(mv, rv), name
        if name == "grow":  # short path is the plain concatenation
            assert torch.equal(valid, g["out_valid"])


def test_surprise_matches_reference(golden_ops):
    g = golden_ops["surprise"]
    keep = [i for i in range(g["head_weight"].shape[0]) if i != 256]
    target = torch.where(g["target"] > 256, g["target"] - 1, g["target"])
    got = ops.causal_surprise(g["prior"], g["head_weight"][keep], g["head_bias"][keep], target, g["valid"])
    torch.testing.assert_close(got.float(), g["surprise"], rtol=1e-5, atol=1e-6)


def test_learned_router_matches_reference(golden_ops):
    g = golden_ops["moe_learned"]
    flat = g["context"].reshape(-1, g["context"].shape[-1])
    valid = g["valid"].reshape(-1)
    logits = torch.where(valid.unsqueeze(-1), flat, torch.zeros_like(flat)) @ g["state"]["gate.weight"].T
    idx, weights, probs = ops.learned_topk(logits, valid, 2)
    assert torch.equal(idx.reshape(g["assignments"].shape), g["assignments"])
    torch.testing.assert_close(weights.float().reshape(g["weights"].shape), g["weights"], rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(probs.sum(0).float(), g["probability_mass"], rtol=1e-5, atol=1e-5)


def test_gated_ffn_matches_reference(golden_ops):
    g = golden_ops["moe_static"]
    s = g["state"]
    for i in range(g["ffn_in"].shape[0]):
        e = i % 6
        got = ops.gated_ffn(g["ffn_in"][i:i + 1], s[f"experts.{e}.gate_projection.weight"],
                            s[f"experts.{e}.gate_projection.bias"], s[f"experts.{e}.value_projection.weight"],
                            s[f"experts.{e}.value_projection.bias"], s[f"experts.{e}.output_projection.weight"],
                            s[f"experts.{e}.output_projection.bias"])
        torch.testing.assert_close(got[0].float(), g["ffn_out"][i], rtol=1e-5, atol=1e-5)


def _oracle_for(name: str):
    fx = load_golden(name)
    case = fx["case"]
    cfg = HermConfig.from_settings(case["settings"])
    shape = HermShape(cfg.vocabulary_size, cfg.embedding_size, cfg.memory_features, cfg.expert_count,
                      cfg.expert_routing, cfg.ablation)
    params = herm_parameters(shape, case["seed"], case["init"],
                             dtype=torch.bfloat16 if case.get("bf16") else torch.float32)
    return fx, HermOracle(cfg, {k: v.float() for k, v in params.items()}, torch.float32)


@pytest.mark.parametrize("name", ["c1", "c1_t065", "herm_learned", "c5_small"])
def test_herm_block_matches_reference_forward_and_decode(name):
    fx, oracle = _oracle_for(name)
    out = oracle.decode(fx["ids"], fx["case"]["decode"])
    prefill = out["prefill"]
    torch.testing.assert_close(prefill["logits"][:, fx["logit_positions"]], fx["logits"], rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(prefill["surprise"], fx["surprise"], rtol=1e-5, atol=1e-5)
    assert torch.equal(prefill["expert_indices"], fx["expert_indices"])
    assert torch.equal(prefill["active_expert_indices"], fx["active_expert_indices"])
    assert torch.equal(out["tokens"], fx["decode_tokens"])  # greedy decode is identical
    for field, expected in fx["state"].items():
        mine = prefill["state"][field]
        if field.startswith("salient"):
            continue
        assert mine.shape == expected.shape, field
        torch.testing.assert_close(mine.to(expected.dtype), expected, rtol=1e-4, atol=1e-5)
    for (mk, mv), (rk, rv) in zip(
            ops.admitted_sequence(prefill["state"]["salient_keys"], prefill["state"]["salient_values"],
                                  prefill["state"]["salient_valid"]),
            ops.admitted_sequence(fx["state"]["salient_keys"], fx["state"]["salient_values"],
                                  fx["state"]["salient_valid"])):
        assert mk.shape == rk.shape
        torch.testing.assert_close(mk, rk, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(mv, rv, rtol=1e-4, atol=1e-5)


def test_threshold_065_exercises_admission():
    fx = load_golden("c1_t065")
    assert int(fx["state"]["salient_valid"].sum()) > 0


def test_splitmix64_known_answers():
    """SplitMix64 from state 0: the first two outputs of the published
    generator (Steele, Lea and Flood, 2014)."""
    import numpy as np
    assert int(ops._splitmix64(np.uint64(0))) == 0xE220A8397B1DCDAF
    assert int(ops._splitmix64(np.uint64(0x9E3779B97F4A7C15))) == 0x6E789E6AA1B965F4


def test_gumbel_sampler_oracle_follows_softmax():
    """The counter-based Gumbel-max draws of the oracle (one per stream) have
    softmax(logits / T) frequencies, never PAD, never below a threshold."""
    import numpy as np
    rows, vocab, temperature = 40000, 300, 0.8
    base = np.full(vocab, -3.0)
    base[:4] = [1.0, 0.0, 2.0, -0.5]
    base[ops.PAD_TOKEN_ID] = 9.0
    ids, _ = ops.gumbel_sample(np.broadcast_to(base, (rows, vocab)), temperature, 99, 0, 0, ops.PAD_TOKEN_ID)
    counts = np.bincount(ids, minlength=vocab).astype(np.float64)
    masked = base.copy()
    masked[ops.PAD_TOKEN_ID] = -np.inf
    p = np.exp(masked / temperature - np.max(masked / temperature))
    p /= p.sum()
    assert counts[ops.PAD_TOKEN_ID] == 0
    assert (np.abs(counts - rows * p) <= 5 * np.sqrt(rows * p * (1 - p)) + 1).all()
    kept, _ = ops.gumbel_sample(np.broadcast_to(base, (64, vocab)), temperature, 99, 0, 1, ops.PAD_TOKEN_ID,
                                thresholds=np.full(64, 0.5))
    assert set(kept.tolist()) <= {0, 2}
