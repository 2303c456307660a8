"""Generate the golden fixtures under tests/golden/ from the reference itself.

Runs only where the Koemi-5HOM sources are available: ``KOEMI_REFERENCE_SRC``
must name the reference's ``src`` directory (the one holding ``koemi/``); the
fixtures it writes are committed, so nothing else ever imports the reference.

    KOEMI_REFERENCE_SRC=<reference checkout>/src PYTHONDONTWRITEBYTECODE=1 \
        python tests/golden/make_golden.py

Fixtures:
- ``ops.pt``: per-operator inputs and the reference's outputs (scan, norms,
  content hash + top-k routing, stable pair order, learned router, gated FFN,
  static dispatch, salient tail, surprise).
- ``herm_<case>.pt``: a full reference forward (``KoemiModel.forward``) over a
  prompt batch plus a ``BatchDecoder`` greedy decode, for seeded parameters
  from ``herm_weights.herm_parameters`` (only the seed is stored).
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from herm_weights import HermShape, herm_parameters  # noqa: E402

REFERENCE_SRC = os.environ.get("KOEMI_REFERENCE_SRC")
if not REFERENCE_SRC or not (Path(REFERENCE_SRC) / "koemi").is_dir():
    raise SystemExit("set KOEMI_REFERENCE_SRC to the reference's src directory (the one that holds koemi/)")
sys.path.insert(0, REFERENCE_SRC)

from koemi.configuration.settings import ModelSettings  # noqa: E402
from koemi.model.experts import DeterministicExpertMixture, content_dispatch_hash  # noqa: E402
from koemi.model.layers import GatedFeedForward, RootMeanSquareNorm  # noqa: E402
from koemi.model.memory import LocalKeyValueMemory  # noqa: E402
from koemi.model.network import KoemiModel  # noqa: E402
from koemi.model.router import LearnedExpertMixture  # noqa: E402
from koemi.model.scan import affine_scan  # noqa: E402
from koemi.runtime.fast_decode import BatchDecoder, SamplingPolicy, TokenSampler  # noqa: E402

PAD = 256


def ops_fixture() -> dict:
    g = torch.Generator().manual_seed(1234)
    out: dict = {}

    # affine scan (model/scan.py:17-30): odd sizes, with and without h0
    a = torch.rand(3, 37, 24, generator=g) * 0.98 + 0.01
    b = torch.randn(3, 37, 24, generator=g)
    h0 = torch.randn(3, 24, generator=g)
    out["scan"] = {"a": a, "b": b, "h0": h0, "h": affine_scan(a, b, h0), "h_zero": affine_scan(a, b)}
    a_bcast = torch.rand(2, 19, 1, generator=g)
    b2 = torch.randn(2, 19, 8, generator=g)
    out["scan_broadcast"] = {"a": a_bcast, "b": b2, "h": affine_scan(a_bcast, b2)}

    # RMSNorm (layers.py:8-16) and the fused RMSNorm+SiLU formula
    x = torch.randn(13, 96, generator=g) * 3.0
    norm = RootMeanSquareNorm(96)
    with torch.no_grad():
        norm.weight.copy_(1.0 + 0.1 * torch.randn(96, generator=g))
        rms = norm(x)
    out["rmsnorm"] = {"x": x, "w": norm.weight.detach().clone(), "y": rms, "silu_y": torch.nn.functional.silu(rms)}

    # content hash and top-k routing (experts.py:93-101, 346-352)
    tokens = torch.randint(0, 40000, (5, 33), generator=g)
    previous = torch.randint(0, 40000, (5, 33), generator=g)
    previous[:, 0] = PAD
    valid = torch.rand(5, 33, generator=g) > 0.15
    routes = {}
    for experts, k in ((4, 1), (6, 2), (6, 3), (64, 2), (128, 2), (7, 7)):
        mixture = DeterministicExpertMixture(8, experts, k)
        routes[f"{experts}_{k}"] = mixture.assign_top_k(tokens, previous, valid)
    out["route"] = {"tokens": tokens, "previous": previous, "valid": valid,
                    "hash": content_dispatch_hash(tokens, previous), "assignments": routes}
    # known answer of tests/model/test_network.py:95-101
    kat_tokens = torch.tensor([[65, 66, 67, PAD]])
    kat_previous = torch.tensor([[PAD, 65, 66, 67]])
    out["route_kat"] = {"tokens": kat_tokens, "previous": kat_previous,
                        "hash": content_dispatch_hash(kat_tokens, kat_previous),
                        "assignments": DeterministicExpertMixture(8, 4, 1).assign_top_k(
                            kat_tokens, kat_previous, kat_tokens != PAD)}

    # stable pair order with duplicate suppression (experts.py:245-257, 324-330)
    permutes = {}
    for experts, k, tokens_count in ((4, 2, 50), (64, 2, 700), (5, 3, 41), (300, 2, 2000), (3000, 2, 4000)):
        assignments = torch.randint(-1, experts + 1, (tokens_count, k), generator=g)
        valid_rows = torch.rand(tokens_count, generator=g) > 0.1
        mixture = DeterministicExpertMixture(8, experts, k)
        first = mixture._first_assignment_occurrence(assignments).reshape(-1)
        pair_experts = assignments.reshape(-1)
        pair_valid = pair_experts.ge(0) & pair_experts.lt(experts) & valid_rows.repeat_interleave(k) & first
        keys = torch.where(pair_valid, pair_experts, torch.full_like(pair_experts, experts))
        order = torch.argsort(keys, stable=True)
        counts = torch.bincount(keys, minlength=experts + 1)
        permutes[f"{experts}_{k}_{tokens_count}"] = {"assignments": assignments, "valid": valid_rows,
                                                     "order": order, "keys_sorted": keys[order], "counts": counts}
    out["permute"] = permutes

    # gated FFN (layers.py:19-29) and static dispatch (experts.py:172-206)
    torch.manual_seed(77)
    mixture = DeterministicExpertMixture(32, 6, 2).eval()
    with torch.no_grad():
        for p in mixture.parameters():
            p.copy_(torch.randn(p.shape, generator=g) * 0.2)
        context = torch.randn(3, 11, 32, generator=g)
        ids = torch.randint(0, 300, (3, 11), generator=g)
        prev = torch.randint(0, 300, (3, 11), generator=g)
        valid_m = torch.rand(3, 11, generator=g) > 0.2
        mixed, first_ids, assignments = mixture(context, ids, prev, valid_m)
        ffn_in = torch.randn(9, 32, generator=g)
        ffn_out = torch.stack([mixture.experts[i % 6](ffn_in[i]) for i in range(9)])
    out["moe_static"] = {"state": {k: v.clone() for k, v in mixture.state_dict().items()}, "context": context,
                         "ids": ids, "prev": prev, "valid": valid_m, "mixed": mixed, "assignments": assignments,
                         "ffn_in": ffn_in, "ffn_out": ffn_out}

    # learned router (router.py:43-97), k=2 of 8, raw (unrenormalised) weights
    learned = LearnedExpertMixture(32, 8, 2).eval()
    with torch.no_grad():
        for p in learned.parameters():
            p.copy_(torch.randn(p.shape, generator=g) * 0.2)
        context = torch.randn(4, 9, 32, generator=g)
        valid_l = torch.rand(4, 9, generator=g) > 0.2
        mixed_l, _, assign_l, stats = learned(context, ids[:, :9].repeat(2, 1)[:4], prev[:, :9].repeat(2, 1)[:4], valid_l)
        gate_probs = learned.gate(context.masked_fill(~valid_l.unsqueeze(-1), 0)).float().softmax(-1)
        weights_l, _ = gate_probs.topk(2, dim=-1)
    out["moe_learned"] = {"state": {k: v.clone() for k, v in learned.state_dict().items()}, "context": context,
                          "valid": valid_l, "mixed": mixed_l, "assignments": assign_l,
                          "weights": weights_l.masked_fill(~valid_l.unsqueeze(-1), 0),
                          "probability_mass": stats.probability_mass, "assignment_counts": stats.assignment_counts,
                          "valid_count": stats.valid_count}

    # salient tail (memory.py:431-455): only the admitted entries and their
    # order are defined; invalid slot placement follows topk tie order
    memory = LocalKeyValueMemory(16, 8)
    cases = {}
    for name, carried, length, capacity in (("grow", 0, 5, 8), ("compact", 8, 6, 8), ("long", 8, 40, 8)):
        ck = torch.randn(2, carried, 16, generator=g)
        cv = torch.randn(2, carried, 16, generator=g)
        cvalid = torch.rand(2, carried, generator=g) > 0.4
        keys = torch.randn(2, length, 16, generator=g)
        values = torch.randn(2, length, 16, generator=g)
        admission = torch.rand(2, length, generator=g) > 0.5
        ok, ov, ovalid = memory.salient_tail(ck, cv, cvalid, keys, values, admission, capacity)
        cases[name] = {"carried_keys": ck, "carried_values": cv, "carried_valid": cvalid, "keys": keys,
                       "values": values, "admission": admission, "capacity": capacity, "out_keys": ok,
                       "out_values": ov, "out_valid": ovalid}
    out["salient_tail"] = cases

    # causal surprise (network.py:677-698) through a small hybrid-vocab model
    settings = ModelSettings(vocabulary_size=300, embedding_size=32, expert_count=0)
    model = KoemiModel(settings).eval()
    with torch.no_grad():
        model.token_predictor.weight.copy_(torch.randn(300, 32, generator=g) * 0.3)
        model.token_predictor.bias.copy_(torch.randn(300, generator=g) * 0.3)
        prior = torch.randn(3, 10, 32, generator=g)
        target = torch.randint(0, 300, (3, 10), generator=g)
        target[target == PAD] = 5
        valid_s = torch.rand(3, 10, generator=g) > 0.2
        surprise = model.calculate_surprise(prior, target, valid_s)
    out["surprise"] = {"head_weight": model.token_predictor.weight.detach().clone(),
                       "head_bias": model.token_predictor.bias.detach().clone(), "prior": prior,
                       "target": target, "valid": valid_s, "surprise": surprise}
    return out


CASES = {
    # config 1 of BASELINE.json (reference defaults otherwise), threshold as given
    "c1": dict(settings=dict(vocabulary_size=257, embedding_size=256, memory_features=16, local_memory_size=32,
                             salience_memory_size=32, expert_count=4, expert_top_k=1, salience_threshold=0.75),
               batch=2, length=256, decode=64, seed=0, init="uniform", pad_rows=0),
    "c1_t065": dict(settings=dict(vocabulary_size=257, embedding_size=256, memory_features=16, local_memory_size=32,
                                  salience_memory_size=32, expert_count=4, expert_top_k=1, salience_threshold=0.65),
                    batch=2, length=256, decode=64, seed=0, init="uniform", pad_rows=0),
    # refine path, learned top-2 routing, hybrid vocabulary, padded prompts
    "herm_learned": dict(settings=dict(vocabulary_size=600, embedding_size=64, memory_features=8,
                                       local_memory_size=12, salience_memory_size=10, expert_count=6,
                                       expert_top_k=2, expert_routing="learned", ablation="herm",
                                       salience_threshold=0.5, scan_chunk=32),
                         batch=3, length=90, decode=24, seed=5, init="uniform", pad_rows=2),
    # hash top-2 over a hybrid vocabulary with bf16-rounded normal(0, 0.02)
    # weights, the structure of config 5 at a testable width
    "c5_small": dict(settings=dict(vocabulary_size=1024, embedding_size=128, memory_features=16,
                                   local_memory_size=48, salience_memory_size=40, expert_count=16,
                                   expert_top_k=2, salience_threshold=0.6, scan_chunk=64),
                     batch=3, length=150, decode=64, seed=11, init="normal", pad_rows=1, bf16=True),
    # config 5 at full width for one block: vocabulary 32768 (hybrid), d=2048,
    # 16 features, 128 + 128 slots, 64 experts top-2 (d_ff 4096), bf16-rounded
    # N(0, 0.02) weights, the bench's fixed threshold 0.64; two streams with a
    # short prompt (the reference's static dispatch gathers 100 MB of fp32
    # expert weights per token-expert pair). Rings are not stored (8 MB);
    # the admitted positions are, through the surprise values.
    "c5_width": dict(settings=dict(vocabulary_size=32768, embedding_size=2048, memory_features=16,
                                   local_memory_size=128, salience_memory_size=128, expert_count=64,
                                   expert_top_k=2, salience_threshold=0.64, scan_chunk=128),
                     batch=2, length=40, decode=64, seed=21, init="normal", pad_rows=0, bf16=True,
                     compact=True),
}


def herm_fixture(case: dict) -> dict:
    settings = ModelSettings(**case["settings"])
    shape = HermShape(vocabulary_size=settings.vocabulary_size, embedding_size=settings.embedding_size,
                      memory_features=settings.memory_features, expert_count=settings.expert_count,
                      expert_routing=settings.expert_routing, ablation=settings.ablation)
    params = herm_parameters(shape, case["seed"], case["init"],
                             dtype=torch.bfloat16 if case.get("bf16") else torch.float32)
    params = {k: v.float() for k, v in params.items()}
    model = KoemiModel(settings).eval()
    missing = model.load_state_dict(params, strict=True)
    assert not missing.missing_keys and not missing.unexpected_keys
    g = torch.Generator().manual_seed(case["seed"])
    vocab = settings.vocabulary_size
    ids = torch.randint(0, vocab - 1, (case["batch"], case["length"]), generator=g)
    ids = torch.where(ids >= PAD, ids + 1, ids)  # never PAD inside a prompt
    for row in range(case["pad_rows"]):  # left padding, as the batch prefill uses
        ids[row, : 7 * (row + 1)] = PAD
    with torch.no_grad():
        output = model(ids)
        decoder = BatchDecoder(model, cache_expert_weights=True)
        sampler = TokenSampler(SamplingPolicy(greedy=True), torch.device("cpu"))
        logits = decoder.prefill(ids)
        tokens, step_logits, top_values, top_ids = [], [], [], []
        for step in range(case["decode"]):
            nxt = sampler(logits)
            tokens.append(nxt)
            if step < 4:
                step_logits.append(logits.clone())
            # every step: the eight best content logits (PAD masked) and their ids
            scores = logits.clone()
            scores[:, PAD] = float("-inf")
            best = scores.topk(8, dim=-1)
            top_values.append(best.values)
            top_ids.append(best.indices)
            logits = decoder.step(nxt)
        final_state = decoder.state
    state = {name: getattr(output.state, name) for name in output.state.__dataclass_fields__ if name != "step_index"}
    decode_state = {name: getattr(final_state, name) for name in final_state.__dataclass_fields__
                    if name != "step_index"}
    if case.get("compact"):  # small state fields only; rings and bases summarised
        small = ("working_state", "memory_normalizer", "local_valid", "salient_valid", "last_token_ids")
        state = {name: value for name, value in state.items() if name in small}
        decode_state = {name: value for name, value in decode_state.items() if name in small}
    return {
        "case": {k: v for k, v in case.items()},
        "ids": ids,
        "logits": output.logits,
        "surprise": output.surprise_values,
        "expert_indices": output.expert_indices,
        "active_expert_indices": output.active_expert_indices,
        "valid_positions": output.valid_positions,
        "state": state,
        "decode_tokens": torch.cat(tokens, dim=1),
        "decode_logits": torch.stack(step_logits, dim=1),
        "decode_top_values": torch.stack(top_values, dim=1),
        "decode_top_ids": torch.stack(top_ids, dim=1),
        "decode_state": decode_state,
    }


def _compact(value):
    """Clone tensors so torch.save stores only their own elements, not the
    whole storage a view points into."""
    if isinstance(value, torch.Tensor):
        return value.detach().contiguous().clone()
    if isinstance(value, dict):
        return {k: _compact(v) for k, v in value.items()}
    return value


def main() -> None:
    """``make_golden.py [case ...]`` regenerates the named herm cases only
    (``ops`` names the per-operator fixture); no argument regenerates all."""
    wanted = set(sys.argv[1:]) or {"ops", *CASES}
    torch.manual_seed(0)
    if "ops" in wanted:
        torch.save(_compact(ops_fixture()), HERE / "ops.pt")
    for name, case in CASES.items():
        if name not in wanted:
            continue
        fixture = herm_fixture(case)
        # keep the fixture small: logits at every 8th position, the window
        # edges and the last position
        length = fixture["ids"].shape[1]
        keep = sorted(set(range(0, length, 8)) | {length - 1, 31, 32, 63, 64, 127, 128} & set(range(length)))
        fixture["logit_positions"] = torch.tensor(keep)
        fixture["logits"] = fixture["logits"][:, keep].clone()
        torch.save(_compact(fixture), HERE / f"herm_{name}.pt")
        print(name, {k: tuple(v.shape) for k, v in fixture.items() if isinstance(v, torch.Tensor)})


if __name__ == "__main__":
    main()
