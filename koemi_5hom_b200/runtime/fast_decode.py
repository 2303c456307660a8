"""Fixed-shape batched decode, mirroring ``koemi.runtime.fast_decode``.

``BatchDecoder`` keeps the reference's API (src/koemi/runtime/fast_decode.py:156-333):
``prefill(input_ids) -> [batch, vocab]`` logits of the last position,
``step(token_ids) -> [batch, vocab]``, ``extend``, ``adopt``, ``state``. The
state is held at ring capacity so every step has the same shapes; with
``capture_graph=True`` one step is captured into a CUDA graph on a side stream
after warm-up and replayed with static input/state buffers, so a decode step
is one graph launch with no host synchronisation.

Prefill asks the model for the last position's logits only
(``last_logits_only``), which is all ``prefill`` returns (:222).
``TokenSampler`` and ``SamplingPolicy`` follow :19-87 (greedy argmax or
softmax/temperature/top-k + multinomial, PAD always masked).
"""
from __future__ import annotations

from dataclasses import dataclass, replace

import torch
from torch import Tensor

from koemi_5hom_b200.cuda_kernels import _ops
from koemi_5hom_b200.model.decode import (RING_DTYPES, attach_head_pass, decode_step, from_koemi_state,
                                           supports_decode_path, to_koemi_state)
from koemi_5hom_b200.model.settings import PAD_TOKEN_ID
from koemi_5hom_b200.model.state import KOEMI_STATE_FIELDS, KoemiState, LayeredKoemiState

GRAPH_WARMUP_STEPS = 3


@dataclass(frozen=True)
class SamplingPolicy:
    temperature: float = 1.0
    top_k: int | None = None
    greedy: bool = False

    def __post_init__(self) -> None:
        if self.temperature <= 0.0:
            raise ValueError("temperature must be positive")
        if self.top_k is not None and (isinstance(self.top_k, bool) or not isinstance(self.top_k, int) or self.top_k < 1):
            raise ValueError("top_k must be a positive integer")


class TokenSampler:
    """Select decode tokens on the device (no host reads).

    Greedy runs the native argmax. Temperature sampling follows the reference
    (softmax + ``torch.multinomial`` with ``generator``) unless ``stream_seed``
    is given: then one native pass per row draws from the same distribution
    by counter-based Gumbel-max, seeded per stream (stream id
    ``stream_offset + row``) and per call (a device step counter advanced
    after every call, so the sampler can live inside a CUDA graph); a stream's
    tokens then do not depend on the batch it is decoded in."""

    def __init__(self, policy: SamplingPolicy, device: torch.device, generator: torch.Generator | None = None,
                 *, stream_seed: int | None = None, stream_offset: int = 0):
        self.policy = policy
        self.generator = generator
        self._padding = torch.tensor([PAD_TOKEN_ID], dtype=torch.long, device=device)
        self.stream_seed = stream_seed
        self.stream_offset = stream_offset
        self._step = torch.zeros(1, dtype=torch.int64, device=device) if stream_seed is not None else None

    def content_scores(self, logits: Tensor) -> Tensor:
        return logits.float().index_fill(-1, self._padding, float("-inf"))

    def __call__(self, logits: Tensor) -> Tensor:
        if logits.ndim != 2:
            raise ValueError("sampling requires logits with shape [batch, vocabulary]")
        if self.policy.greedy and logits.is_cuda and logits.dtype == torch.float32:
            # one native pass: PAD scored as -inf, torch.argmax tie and NaN order
            return _ops.greedy_tokens(logits, PAD_TOKEN_ID)
        if self.stream_seed is not None and not self.policy.greedy and logits.is_cuda and logits.dtype == torch.float32:
            thresholds = None
            if self.policy.top_k is not None:
                kept = min(self.policy.top_k, logits.shape[-1])
                thresholds = torch.topk(self.content_scores(logits), kept, dim=-1).values[:, -1].contiguous()
            tokens = _ops.temperature_tokens(logits, PAD_TOKEN_ID, float(self.policy.temperature), self.stream_seed,
                                             self.stream_offset, self._step, thresholds)
            self._step.add_(1)
            return tokens
        scores = self.content_scores(logits)
        if self.policy.greedy:
            return scores.argmax(dim=-1, keepdim=True)
        if self.policy.top_k is not None:
            kept = min(self.policy.top_k, scores.shape[-1])
            threshold = torch.topk(scores, kept, dim=-1).values[..., -1:]
            scores = scores.masked_fill(scores < threshold, float("-inf"))
        probabilities = torch.softmax(scores / self.policy.temperature, dim=-1)
        return torch.multinomial(probabilities, num_samples=1, generator=self.generator)


def _resize_ring(keys: Tensor, values: Tensor, valid: Tensor, capacity: int):
    length = keys.shape[1]
    if length == capacity:
        return keys, values, valid
    if length > capacity:
        return keys[:, -capacity:], values[:, -capacity:], valid[:, -capacity:]
    missing = capacity - length
    return (torch.cat((keys.new_zeros(keys.shape[0], missing, keys.shape[2]), keys), dim=1),
            torch.cat((values.new_zeros(values.shape[0], missing, values.shape[2]), values), dim=1),
            torch.cat((torch.zeros(valid.shape[0], missing, dtype=torch.bool, device=valid.device), valid), dim=1))


def to_static_state(state, local_memory_size: int, salience_memory_size: int):
    """Same state with both rings held at capacity (empty slots lead, zero,
    invalid), so reads are unchanged and shapes stay constant."""
    if isinstance(state, LayeredKoemiState):
        return LayeredKoemiState(tuple(to_static_state(layer, local_memory_size, salience_memory_size)
                                       for layer in state.layers), state.step_index)
    lk, lv, lvalid = _resize_ring(state.local_keys, state.local_values, state.local_valid, local_memory_size)
    sk, sv, svalid = _resize_ring(state.salient_keys, state.salient_values, state.salient_valid, salience_memory_size)
    return replace(state, local_keys=lk, local_values=lv, local_valid=lvalid, salient_keys=sk, salient_values=sv,
                   salient_valid=svalid)


def clone_state(state):
    if isinstance(state, LayeredKoemiState):
        return LayeredKoemiState(tuple(clone_state(layer) for layer in state.layers), state.step_index)
    return replace(state, **{f: getattr(state, f).clone() for f in KOEMI_STATE_FIELDS})


def _copy_state(destination, source) -> None:
    if isinstance(destination, LayeredKoemiState):
        for d, s in zip(destination.layers, source.layers):
            _copy_state(d, s)
        return
    for field in KOEMI_STATE_FIELDS:
        getattr(destination, field).copy_(getattr(source, field))


def _rows(state) -> int:
    return state.working_state.shape[0]


class BatchDecoder:
    """Fixed-shape recurrent decoding for a batch of sequences.

    When the model's configuration allows it (``supports_decode_path``) the
    state lives in a ``DecodeState`` and each step updates it in place with the
    fused decode kernels; otherwise each step runs the window path and the new
    state replaces the old. ``capture_graph`` records one step into a CUDA graph
    (after warm-up on a side stream) and replays it.
    """

    def __init__(self, model, *, capture_graph: bool = False, cache_expert_weights: bool = True,
                 in_place: bool = True, ring_dtype: torch.dtype = torch.float32):
        device = model.device
        if capture_graph and device.type != "cuda":
            raise RuntimeError("CUDA graph capture requires a model on a CUDA device")
        if capture_graph and getattr(model, "expert_shard", None) is not None and model.exchange == "nccl":
            raise RuntimeError("the NCCL expert exchange is not captured in CUDA graphs; use model.exchange = "
                               "'peer' or capture_graph=False")
        self.model = model
        self.device = device
        self._capture_graph = capture_graph
        self._in_place = in_place and device.type == "cuda" and supports_decode_path(model.settings)
        if ring_dtype not in RING_DTYPES:
            raise ValueError(f"ring_dtype must be one of {RING_DTYPES}")
        if ring_dtype != torch.float32 and not self._in_place:
            raise ValueError("a bf16 ring needs the in-place decode path")
        self._ring_dtype = ring_dtype
        self._graph: torch.cuda.CUDAGraph | None = None
        self._state = None       # window path: KoemiState / LayeredKoemiState
        self._dstate = None      # in-place path: DecodeState
        self._static_ids: Tensor | None = None
        self._static_logits: Tensor | None = None
        self._step_index = 0
        if cache_expert_weights:
            model.cache_inference_weights()

    @property
    def state(self):
        if self._state is None and self._dstate is None:
            raise RuntimeError("prefill must run before the state is available")
        state = to_koemi_state(self._dstate) if self._dstate is not None else self._state
        if isinstance(state, LayeredKoemiState):
            return state.with_step(self._step_index)
        return replace(state, step_index=self._step_index)

    def adopt(self, state, step_index: int | None = None) -> None:
        self._set_state(state)
        self._step_index = state.step_index if step_index is None else step_index

    def _set_state(self, state) -> None:
        s = self.model.settings
        static = to_static_state(state, s.local_memory_size, s.salience_memory_size)
        if self._in_place:
            self._dstate = from_koemi_state(static, s.local_memory_size, s.salience_memory_size, self._ring_dtype)
            attach_head_pass(self.model, self._dstate)
            self._state = None
        else:
            self._state = static
            self._dstate = None
        self._reset_graph()

    def prefill(self, input_ids: Tensor) -> Tensor:
        """Evaluate right-aligned (left-padded) prompts; return last logits."""
        self._validate_prompt(input_ids)
        trusted = not bool((input_ids == PAD_TOKEN_ID).any().item())
        output = self.model(input_ids, trusted_inputs=trusted, last_logits_only=True)
        self._set_state(output.state)
        self._step_index = input_ids.shape[1]
        return output.logits[:, -1]

    def step(self, token_ids: Tensor) -> Tensor:
        if self._state is None and self._dstate is None:
            raise RuntimeError("prefill must run before step")
        ids = self._normalize_step_input(token_ids)
        if self._capture_graph:
            return self._graph_step(ids)
        logits = self._eager_step(ids)
        self._step_index += 1
        return logits

    def _eager_step(self, ids: Tensor) -> Tensor:
        if self._dstate is not None:
            return decode_step(self.model, ids, self._dstate)
        output = self.model(ids, self._state, trusted_inputs=True)
        self._state = output.state
        return output.logits[:, -1]

    def extend(self, token_ids: Tensor) -> Tensor:
        if self._state is None and self._dstate is None:
            raise RuntimeError("prefill must run before extend")
        if not isinstance(token_ids, Tensor) or token_ids.ndim != 2 or token_ids.shape[1] == 0:
            raise ValueError("extend requires token ids with shape [batch, length]")
        output = self.model(token_ids, self.state, trusted_inputs=True)
        self._set_state(output.state)
        self._step_index += token_ids.shape[1]
        return output.logits

    def _graph_step(self, ids: Tensor) -> Tensor:
        if self._graph is None:
            self._static_ids = ids.clone()
            if self._dstate is None:
                self._state = clone_state(self._state)
            self._capture()
        self._static_ids.copy_(ids)
        self._graph.replay()
        self._step_index += 1
        return self._static_logits

    def _capture(self) -> None:
        """Warm up on a side stream, then record one step. The in-place path
        advances its state during warm-up, so it warms up on a copy."""
        stream = torch.cuda.Stream(device=self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            if self._dstate is not None:
                scratch = self._dstate.clone()
                for _ in range(GRAPH_WARMUP_STEPS):
                    decode_step(self.model, self._static_ids, scratch)
                del scratch
            else:
                for _ in range(GRAPH_WARMUP_STEPS):
                    self.model(self._static_ids, self._state, trusted_inputs=True)
        torch.cuda.current_stream(self.device).wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            if self._dstate is not None:
                self._static_logits = decode_step(self.model, self._static_ids, self._dstate)
            else:
                output = self.model(self._static_ids, self._state, trusted_inputs=True)
                self._static_logits = output.logits[:, -1]
                _copy_state(self._state, output.state)
        self._graph = graph

    def _reset_graph(self) -> None:
        self._graph = None
        self._static_ids = None
        self._static_logits = None

    def _rows(self) -> int:
        return self._dstate.last_token_ids.shape[0] if self._dstate is not None else _rows(self._state)

    def _normalize_step_input(self, token_ids: Tensor) -> Tensor:
        _enforce(_STEP_TYPE_RULE, token_ids, self)
        ids = token_ids.unsqueeze(-1) if token_ids.ndim == 1 else token_ids
        _enforce(_STEP_RULES, ids, self)
        return ids

    def _validate_prompt(self, input_ids: Tensor) -> None:
        _enforce(_PROMPT_RULES, input_ids, self)


# Input contracts of BatchDecoder (the reference's messages, in its order of
# checks, fast_decode.py:304-330): (broken(ids, decoder), exception, message).
_STEP_TYPE_RULE = ((lambda ids, dec: not isinstance(ids, Tensor), TypeError, "step token ids must be a torch.Tensor"),)
_STEP_RULES = (
    (lambda ids, dec: ids.ndim != 2 or ids.shape[1] != 1, ValueError, "step requires exactly one token id per row"),
    (lambda ids, dec: ids.shape[0] != dec._rows(), ValueError,
     "step token ids must carry one row per decoded sequence"),
    (lambda ids, dec: ids.dtype != torch.long, TypeError, "step token ids must use torch.long"),
    (lambda ids, dec: ids.device != dec.device, ValueError, "step token ids must live on the model device"),
)
_PROMPT_RULES = (
    (lambda ids, dec: not isinstance(ids, Tensor), TypeError, "prompt ids must be a torch.Tensor"),
    (lambda ids, dec: ids.ndim != 2 or 0 in ids.shape, ValueError, "prompt ids must have shape [batch, sequence]"),
    (lambda ids, dec: ids.dtype != torch.long, TypeError, "prompt ids must use torch.long"),
    (lambda ids, dec: ids.device != dec.device, ValueError, "prompt ids must live on the model device"),
    (lambda ids, dec: int(ids.min()) < 0 or int(ids.max()) >= dec.model.settings.vocabulary_size, ValueError,
     "prompt ids contain values outside the model vocabulary"),
)


def _enforce(rules, ids, decoder) -> None:
    for broken, error, message in rules:
        if broken(ids, decoder):
            raise error(message)


def generate_tokens(model, prompt_ids: Tensor, max_new_tokens: int, *, policy: SamplingPolicy | None = None,
                    generator: torch.Generator | None = None, capture_graph: bool = False) -> Tensor:
    """Prefill then decode ``max_new_tokens`` ids per row on the device
    (the loop of generate_batch, fast_decode.py:351-407, without text I/O)."""
    decoder = BatchDecoder(model, capture_graph=capture_graph)
    sampler = TokenSampler(policy or SamplingPolicy(greedy=True), model.device, generator)
    generated = torch.empty(prompt_ids.shape[0], max_new_tokens, dtype=torch.long, device=model.device)
    logits = decoder.prefill(prompt_ids)
    for index in range(max_new_tokens):
        token = sampler(logits)
        generated[:, index:index + 1].copy_(token)
        if index + 1 < max_new_tokens:
            logits = decoder.step(token)
    return generated


__all__ = ["BatchDecoder", "GRAPH_WARMUP_STEPS", "SamplingPolicy", "TokenSampler", "clone_state",
           "generate_tokens", "to_static_state"]
