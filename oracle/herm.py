"""CPU restatement of one HERM block (test infrastructure; see oracle/__init__.py).

Follows ``KoemiModel.forward_window`` (src/koemi/model/network.py:296-441)
window by window (``forward_parallel``, :174-197), but evaluates every memory
in its sequential form: the recurrent scan and both associative memories are
stepped one position at a time (the recurrence that the reference's closed
pairwise form in model/memory.py:97-144 sums), and the local/salient reads loop
over the slots each query may see (memory.py:332-429). Parameters are a dict
keyed by the reference's state-dict names (tests/golden/herm_weights.py).

``HermOracle.decode`` replays ``BatchDecoder`` (runtime/fast_decode.py:156-290)
with the greedy ``TokenSampler`` (:40-87).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from oracle import ops

PAD = ops.PAD_TOKEN_ID
STATE_FIELDS = (
    "working_state", "memory_basis", "memory_normalizer", "refine_basis", "refine_normalizer",
    "local_keys", "local_values", "local_valid", "salient_keys", "salient_values", "salient_valid",
    "last_token_ids",
)


@dataclass(frozen=True)
class HermConfig:
    """The ModelSettings fields the block reads (configuration/settings.py:15-32)."""

    vocabulary_size: int = 257
    embedding_size: int = 64
    memory_features: int = 16
    local_memory_size: int = 16
    salience_memory_size: int = 16
    salience_threshold: float = 0.75
    expert_count: int = 0
    expert_top_k: int = 1
    scan_chunk: int = 128
    refine_decay_rate: float = 0.0625
    ablation: str = "no_refine"
    expert_routing: str = "hash"

    @classmethod
    def from_settings(cls, settings: dict) -> "HermConfig":
        fields = cls.__dataclass_fields__
        return cls(**{k: v for k, v in settings.items() if k in fields})


class HermOracle:
    def __init__(self, config: HermConfig, params: dict[str, torch.Tensor], dtype: torch.dtype = torch.float32):
        self.config = config
        self.dtype = dtype
        self.p = {name: value.to(dtype) for name, value in params.items()}
        head_w, head_b = self.p["token_predictor.weight"], self.p["token_predictor.bias"]
        keep = [i for i in range(config.vocabulary_size) if i != PAD]
        self.content_w = head_w[keep]
        self.content_b = head_b[keep]

    # ------------------------------------------------------------ helpers
    def linear(self, name: str, x: torch.Tensor) -> torch.Tensor:
        y = x @ self.p[f"{name}.weight"].T
        bias = self.p.get(f"{name}.bias")
        return y if bias is None else y + bias

    def norm(self, name: str, x: torch.Tensor) -> torch.Tensor:
        return x * torch.rsqrt(x.pow(2).mean(dim=-1, keepdim=True) + 1e-6) * self.p[name]

    def initial_state(self, batch: int) -> dict[str, torch.Tensor]:
        c, d, m = self.config, self.config.embedding_size, self.config.memory_features
        zeros = lambda *shape: torch.zeros(*shape, dtype=self.dtype)  # noqa: E731
        return {
            "working_state": zeros(batch, d), "memory_basis": zeros(batch, d, m), "memory_normalizer": zeros(batch, m),
            "refine_basis": zeros(batch, d, m), "refine_normalizer": zeros(batch, m),
            "local_keys": zeros(batch, 0, d), "local_values": zeros(batch, 0, d),
            "local_valid": torch.zeros(batch, 0, dtype=torch.bool),
            "salient_keys": zeros(batch, 0, d), "salient_values": zeros(batch, 0, d),
            "salient_valid": torch.zeros(batch, 0, dtype=torch.bool),
            "last_token_ids": torch.full((batch,), PAD, dtype=torch.long),
        }

    # ------------------------------------------------------------ forward
    def forward(self, ids: torch.Tensor, state: dict | None = None) -> dict:
        state = state if state is not None else self.initial_state(ids.shape[0])
        pieces = []
        for start in range(0, ids.shape[1], self.config.scan_chunk):
            piece = self.window(ids[:, start:start + self.config.scan_chunk], state)
            pieces.append(piece)
            state = piece["state"]
        out = {k: torch.cat([p[k] for p in pieces], dim=1)
               for k in ("logits", "surprise", "expert_indices", "active_expert_indices", "valid_positions")}
        out["state"] = state
        return out

    def window(self, ids: torch.Tensor, state: dict, context: torch.Tensor | None = None,
               logits: bool = True) -> dict:
        """One window of the block. ``context`` (an extension for stacked
        blocks) replaces the embedding rows of ``ids`` as the block input;
        ``logits=False`` skips the head (blocks below the top of a stack)."""
        c = self.config
        batch, length = ids.shape
        width = c.embedding_size
        valid = ids != PAD
        v3 = valid.unsqueeze(-1)

        # embedding + input norm (network.py:703-707), bounded gates (memory.py:22-26)
        inputs = self.p["embedding.weight"][ids] if context is None else context
        u = self.norm("input_normalizer.weight", inputs)
        lo, hi = 2.0 ** -8, 1.0 - 2.0 ** -8
        a = lo + (hi - lo) * torch.sigmoid(self.linear("recurrent_state.retention_projection", u))
        b = (1.0 - a) * torch.tanh(self.linear("recurrent_state.candidate_projection", u))
        a = torch.where(v3, a, torch.ones_like(a))
        b = torch.where(v3, b, torch.zeros_like(b))
        h = torch.empty_like(b)
        carry = state["working_state"]
        for t in range(length):
            carry = a[:, t] * carry + b[:, t]
            h[:, t] = carry
        last_ids = self._last_valid(ids, valid, state["last_token_ids"])

        if c.ablation == "affine":  # network.py:443-480
            new_state = dict(state, working_state=h[:, -1], last_token_ids=last_ids)
            return {"logits": self.linear("token_predictor", h), "surprise": torch.zeros(batch, length, dtype=self.dtype),
                    "expert_indices": torch.full_like(ids, -1), "active_expert_indices": torch.full_like(ids, -1).unsqueeze(-1),
                    "valid_positions": valid, "state": new_state}

        prior = torch.cat((state["working_state"].unsqueeze(1), h[:, :-1]), dim=1)
        if c.ablation == "no_surprise":
            surprise = torch.zeros(batch, length, dtype=self.dtype)
        else:
            content_ids = torch.where(ids > PAD, ids - 1, ids) if c.vocabulary_size != PAD + 1 else ids
            surprise = ops.causal_surprise(prior, self.content_w, self.content_b, content_ids, valid,
                                           dtype=self.dtype)

        # local ring entries and sliding-window read (memory.py:297-383)
        keys = torch.where(v3, self.linear("local_memory.local_key_projection", h), torch.zeros_like(h))
        values = torch.where(v3, self.linear("local_memory.local_value_projection", h), torch.zeros_like(h))
        all_keys = torch.cat((state["local_keys"], keys), dim=1)
        all_values = torch.cat((state["local_values"], values), dim=1)
        all_valid = torch.cat((state["local_valid"], valid), dim=1)
        carried = state["local_keys"].shape[1]
        local_value = torch.zeros_like(h)
        novelty = torch.ones(batch, length, dtype=self.dtype)
        scale = 1.0 / math.sqrt(width)
        for t in range(length):
            own = carried + t
            first = max(0, own - c.local_memory_size)
            for row in range(batch):
                slots = [s for s in range(first, own) if all_valid[row, s]]
                if not slots:
                    continue
                k = all_keys[row, slots]
                q = h[row, t]
                weights = torch.softmax(k @ q * scale, dim=0)
                local_value[row, t] = weights @ all_values[row, slots]
                qn = q / q.norm().clamp_min(1e-12)
                kn = k / k.norm(dim=-1, keepdim=True).clamp_min(1e-12)
                novelty[row, t] = (1.0 - (kn @ qn).max()).clamp(0.0, 1.0)

        # associative memory (memory.py:82-144,244-255)
        key = self.linear("associative_memory.key_projection", h)
        features = torch.softmax(self.linear("associative_memory.feature_projection", key), dim=-1)
        query = self.linear("associative_memory.query_projection", h)
        query_features = torch.softmax(self.linear("associative_memory.feature_projection", query), dim=-1)
        mem_value = torch.tanh(self.linear("associative_memory.value_projection", h))
        dlo, dhi = 2.0 ** -12, 1.0 - 2.0 ** -12
        decay = dlo + (dhi - dlo) * torch.sigmoid(self.linear("associative_memory.decay_projection", h))
        write = torch.sigmoid(self.linear("associative_memory.write_projection", h)).squeeze(-1)
        fast_write = write * (0.25 + 0.75 * surprise.clamp(0.0, 1.0))
        fast_decay = torch.where(v3, decay, torch.ones_like(decay)).squeeze(-1)
        fast_write = torch.where(valid, fast_write, torch.zeros_like(fast_write))
        fast_read, basis, normalizer = self._scan_read(state["memory_basis"], state["memory_normalizer"],
                                                       fast_decay, mem_value, features, fast_write, query_features)

        # salient admission and read (network.py:349; memory.py:405-429)
        admission = valid & (surprise > c.salience_threshold)
        salient_value = torch.zeros_like(h)
        s_keys, s_values, s_valid = state["salient_keys"], state["salient_values"], state["salient_valid"]
        for row in range(batch):
            carried_slots = [s for s in range(s_keys.shape[1]) if s_valid[row, s]]
            for t in range(length):
                window_slots = [s for s in range(t) if admission[row, s]]
                k = torch.cat((s_keys[row, carried_slots], keys[row, window_slots]), dim=0)
                if k.shape[0] == 0:
                    continue
                vals = torch.cat((s_values[row, carried_slots], values[row, window_slots]), dim=0)
                salient_value[row, t] = torch.softmax(k @ h[row, t] * scale, dim=0) @ vals

        if c.ablation == "no_refine":
            memory_value = fast_read
            refine_basis, refine_normalizer = state["refine_basis"], state["refine_normalizer"]
        else:  # memory.py:257-268, network.py:366-386,709-721
            refine_decay = (1.0 - (1.0 - decay) * c.refine_decay_rate).clamp(max=1.0 - 2.0 ** -16)
            refine_decay = torch.where(v3, refine_decay, torch.ones_like(refine_decay)).squeeze(-1)
            refine_write = write * surprise.clamp(0.0, 1.0) * novelty.clamp(0.0, 1.0)
            refine_write = torch.where(valid, refine_write, torch.zeros_like(refine_write))
            error = (mem_value - fast_read).clamp(-2.0, 2.0)
            refine_read, refine_basis, refine_normalizer = self._scan_read(
                state["refine_basis"], state["refine_normalizer"], refine_decay, error, features, refine_write,
                query_features)
            gate = torch.sigmoid(self.linear("memory_refine_gate", torch.cat((h, fast_read, refine_read, local_value), -1)))
            memory_value = fast_read + gate * refine_read

        fused = self.norm("fusion_normalizer.weight",
                          self.linear("fusion_projection", torch.cat((h, memory_value, local_value, salient_value), -1)))
        previous = self._previous_ids(ids, valid, state["last_token_ids"])
        final, expert_indices, active = self._experts(fused, ids, previous, valid)
        head = self.linear("token_predictor", final) if logits else None

        local_keep = all_keys.shape[1] - min(all_keys.shape[1], c.local_memory_size)
        sk, sv, svalid = ops.salient_tail(s_keys, s_values, s_valid, keys, values, admission, c.salience_memory_size)
        new_state = {
            "working_state": h[:, -1], "memory_basis": basis, "memory_normalizer": normalizer,
            "refine_basis": refine_basis, "refine_normalizer": refine_normalizer,
            "local_keys": all_keys[:, local_keep:], "local_values": all_values[:, local_keep:],
            "local_valid": all_valid[:, local_keep:],
            "salient_keys": sk, "salient_values": sv, "salient_valid": svalid,
            "last_token_ids": last_ids,
        }
        return {"logits": head, "final": final, "surprise": surprise, "expert_indices": expert_indices,
                "active_expert_indices": active, "valid_positions": valid, "state": new_state}

    def _scan_read(self, basis, normalizer, decay, value, features, write, query_features):
        """Read at t from the memory before its own write, then write
        (B_t = d_t B_{t-1} + w_t v_t f_t^T); memory.py:91-95,248-251,279-287."""
        eps = 2.0 ** -8
        reads = torch.empty_like(value)
        for t in range(value.shape[1]):
            q = query_features[:, t]
            numerator = torch.einsum("bdm,bm->bd", basis, q)
            denominator = (normalizer * q).sum(-1, keepdim=True)
            regularized = denominator + eps
            reads[:, t] = (denominator / regularized) * numerator / regularized
            d = decay[:, t]
            w = write[:, t]
            basis = d[:, None, None] * basis + w[:, None, None] * value[:, t, :, None] * features[:, t, None, :]
            normalizer = d[:, None] * normalizer + w[:, None] * features[:, t]
        return reads, basis, normalizer

    def _experts(self, context, ids, previous, valid):
        c = self.config
        batch, length, width = context.shape
        if c.expert_count == 0:
            empty = torch.full_like(ids, -1)
            return context, empty, empty.unsqueeze(-1)
        flat = context.reshape(-1, width)
        flat_valid = valid.reshape(-1)
        if c.expert_routing == "learned":  # router.py:43-97
            gate_logits = (torch.where(flat_valid.unsqueeze(-1), flat, torch.zeros_like(flat))
                           @ self.p["experts.gate.weight"].T)
            assignments, weights, _ = ops.learned_topk(gate_logits.float(), flat_valid, c.expert_top_k)
            assignments, weights = assignments.to(torch.long), weights.to(self.dtype)
        else:  # experts.py:109-143,283-289
            assignments = torch.from_numpy(ops.route_topk(ids.reshape(-1).numpy(), previous.reshape(-1).numpy(),
                                                          flat_valid.numpy(), c.expert_count, c.expert_top_k))
            keys = ops.pair_keys(assignments.numpy(), flat_valid.numpy(), c.expert_count).reshape(-1, c.expert_top_k)
            weights = torch.where(torch.from_numpy(keys) < c.expert_count,
                                  torch.full(keys.shape, 1.0 / c.expert_top_k, dtype=self.dtype),
                                  torch.zeros(keys.shape, dtype=self.dtype))
        update = torch.zeros_like(flat)
        for slot in range(c.expert_top_k):
            experts = assignments[:, slot]
            for e in range(c.expert_count):
                rows = torch.nonzero((experts == e) & (weights[:, slot] != 0), as_tuple=False).squeeze(-1)
                if rows.numel() == 0:
                    continue
                prefix = f"experts.experts.{e}"
                y = ops.gated_ffn(flat[rows], self.p[f"{prefix}.gate_projection.weight"],
                                  self.p[f"{prefix}.gate_projection.bias"], self.p[f"{prefix}.value_projection.weight"],
                                  self.p[f"{prefix}.value_projection.bias"], self.p[f"{prefix}.output_projection.weight"],
                                  self.p[f"{prefix}.output_projection.bias"], dtype=self.dtype)
                update[rows] += y * weights[rows, slot].unsqueeze(-1)
        mixed = self.norm("experts.output_normalizer.weight", flat + update)
        mixed = torch.where(flat_valid.unsqueeze(-1), mixed, flat).reshape(batch, length, width)
        assignments = assignments.reshape(batch, length, c.expert_top_k)
        return mixed, assignments[..., 0], assignments

    @staticmethod
    def _previous_ids(ids, valid, carried):
        """Last valid id strictly before each position (network.py:742-749)."""
        out = torch.empty_like(ids)
        for row in range(ids.shape[0]):
            last = int(carried[row])
            for t in range(ids.shape[1]):
                out[row, t] = last
                if valid[row, t]:
                    last = int(ids[row, t])
        return out

    @staticmethod
    def _last_valid(ids, valid, carried):
        out = carried.clone()
        for row in range(ids.shape[0]):
            positions = torch.nonzero(valid[row], as_tuple=False)
            if positions.numel():
                out[row] = ids[row, int(positions[-1])]
        return out

    # ------------------------------------------------------------- decode
    def to_static(self, state: dict) -> dict:
        """Rings resized to capacity, zero/invalid slots leading (fast_decode.py:90-113,438-454)."""
        out = dict(state)
        for prefix, capacity in (("local", self.config.local_memory_size), ("salient", self.config.salience_memory_size)):
            k, v, valid = state[f"{prefix}_keys"], state[f"{prefix}_values"], state[f"{prefix}_valid"]
            n = k.shape[1]
            if n > capacity:
                k, v, valid = k[:, -capacity:], v[:, -capacity:], valid[:, -capacity:]
            elif n < capacity:
                pad = capacity - n
                k = torch.cat((k.new_zeros(k.shape[0], pad, k.shape[2]), k), dim=1)
                v = torch.cat((v.new_zeros(v.shape[0], pad, v.shape[2]), v), dim=1)
                valid = torch.cat((torch.zeros(valid.shape[0], pad, dtype=torch.bool), valid), dim=1)
            out[f"{prefix}_keys"], out[f"{prefix}_values"], out[f"{prefix}_valid"] = k, v, valid
        return out

    def greedy(self, logits: torch.Tensor) -> torch.Tensor:
        scores = logits.double().clone()
        scores[:, PAD] = float("-inf")
        return scores.argmax(dim=-1, keepdim=True)

    def decode(self, ids: torch.Tensor, steps: int) -> dict:
        prefill = self.forward(ids)
        state = self.to_static(prefill["state"])
        logits = prefill["logits"][:, -1]
        tokens, step_logits = [], []
        for _ in range(steps):
            step_logits.append(logits)
            nxt = self.greedy(logits)
            tokens.append(nxt)
            out = self.window(nxt, state)
            state, logits = out["state"], out["logits"][:, -1]
        return {"prefill": prefill, "tokens": torch.cat(tokens, dim=1), "logits": torch.stack(step_logits, dim=1),
                "state": state}
