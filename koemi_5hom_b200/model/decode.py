"""Decode-step path of the HERM stack: one token per stream, state in place.

``KoemiModel.forward`` follows the reference's window semantics and rebuilds
the rings every call (cat + slice). For decode, ``DecodeState`` keeps every
tensor of the state at a fixed address and updates it in place:

- local rings are circular, with one device-side head (the oldest slot) shared
  by all streams and blocks, since every stream writes one entry per step;
- salient rings are circular per stream (head + count of admitted entries);
- working state, associative bases and normalisers are overwritten in place.

A step is then: the hash route and its stable permutation once (the route
depends only on the ids); the surprise of every block at once -- block l
scores the token against the shared head from its working state before the
update, which is known for all blocks when the previous step ends. For 16-bit
models the previous step's head pass already folded the log-sum-exp of those
rows (the merged head pass: one tcgen05 read of the head per step gives this
step's logits and the next step's surprise partials), so only the target
logits remain; otherwise one tcgen05 head GEMM + online LSE over [blocks x
streams] rows reads the head once per step instead of once per block; per
block, rms_norm -> gate GEMM -> ``koemi_dense_decode_step`` -> one
local|assoc GEMM ->
``koemi_think_ring_decode_step`` -> ``koemi_assoc_decode_step`` (with the
feature projection of key and query fused in) -> fusion GEMM
(its input rows are written in place by the three kernels) -> rms_norm ->
row gather through the shared permutation -> grouped expert MLP -> combine,
which also writes the next block's normalised input; then the head pass (or
the logits GEMM). With fixed
addresses the whole step is one CUDA graph with no copy-back of the state.

``to_koemi_state`` restores the reference layout (rings oldest first, salient
entries packed at the end) whenever a caller asks for the state.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

from koemi_5hom_b200 import _native
from koemi_5hom_b200.cuda_kernels import _ops
from koemi_5hom_b200.model.settings import PAD_TOKEN_ID
from koemi_5hom_b200.model.state import KoemiState, LayeredKoemiState

MIN_RETENTION, MAX_RETENTION = 2.0 ** -8, 1.0 - 2.0 ** -8
NORM_EPSILON = 1e-6


def _assoc_step(call, ptr, block, st, assoc, surprise, valid, concat, batch, d, features, out_code, stream):
    """Associative read/update of one block (feature projection of key and
    query fused into the kernel), writing the memory columns of the fusion
    input in place."""
    call("koemi_assoc_decode_step", ptr(assoc), assoc.stride(0), None, ptr(block.feature_weight),
         ptr(block.feature_bias), _native.dtype_code(block.feature_weight.dtype), ptr(surprise), ptr(valid),
         ptr(st.memory_basis), ptr(st.memory_normalizer), ptr(concat[:, d:]), 4 * d, batch, d, features, out_code,
         stream)


@dataclass
class DecodeBlockState:
    working: Tensor
    memory_basis: Tensor
    memory_normalizer: Tensor
    refine_basis: Tensor
    refine_normalizer: Tensor
    local_keys: Tensor
    local_values: Tensor
    local_valid: Tensor
    salient_keys: Tensor
    salient_values: Tensor
    salient_valid: Tensor
    salient_head: Tensor   # int32 [B]
    salient_count: Tensor  # int32 [B]


@dataclass
class DecodeState:
    blocks: list[DecodeBlockState]
    local_head: Tensor      # int64 [1], slot of the oldest local entry (all streams, all blocks)
    last_token_ids: Tensor  # int64 [B]
    step_index: int
    layered: bool
    # merged head pass (16-bit models): rows [blocks * B + B, d] in the compute
    # dtype -- every block's working state (the next step's surprise priors)
    # then the final contexts -- and the log-sum-exp partials
    # [slices, blocks * B, 3] of the prior rows, written at the end of a step
    # and read at the start of the next one
    head_rows: Tensor | None = None
    head_partials: Tensor | None = None

    @property
    def ring_dtype(self) -> torch.dtype:
        return self.blocks[0].local_keys.dtype

    def clone(self) -> "DecodeState":
        """A deep copy at new addresses (same ring layout and dtype)."""
        blocks = [DecodeBlockState(**{f: getattr(b, f).clone() for f in DecodeBlockState.__dataclass_fields__})
                  for b in self.blocks]
        copy = lambda t: None if t is None else t.clone()  # noqa: E731
        return DecodeState(blocks, self.local_head.clone(), self.last_token_ids.clone(), self.step_index, self.layered,
                           copy(self.head_rows), copy(self.head_partials))


def supports_decode_path(settings) -> bool:
    """The in-place path covers the reference defaults and the config-5 stack
    (width a multiple of 8, so fp32 and bf16 ring rows pack in 16 bytes); the
    refine ablation ('herm') keeps the window path."""
    return settings.ablation in ("no_refine", "no_surprise") and settings.embedding_size % 8 == 0


RING_DTYPES = (torch.float32, torch.bfloat16)


def from_koemi_state(state, local_slots: int, salient_slots: int,
                     ring_dtype: torch.dtype = torch.float32) -> DecodeState:
    """Import a static (ring-at-capacity) state: local rings keep their
    oldest-first order (head 0); each salient ring is packed to its admitted
    entries, oldest first, at slots [0, count).

    ``ring_dtype`` is the storage type of the ring keys and values: fp32 (the
    reference's state type) or bf16, which halves the ring traffic of a decode
    step; the ring arithmetic is fp32 either way."""
    if ring_dtype not in RING_DTYPES:
        raise ValueError(f"ring_dtype must be one of {RING_DTYPES}")
    layers = state.layers if isinstance(state, LayeredKoemiState) else (state,)
    blocks = []
    for layer in layers:
        if layer.local_keys.shape[1] != local_slots or layer.salient_keys.shape[1] != salient_slots:
            raise ValueError("decode state needs rings at capacity; call to_static_state first")
        order = torch.argsort((~layer.salient_valid).to(torch.int8), dim=1, stable=True)
        gather = order.unsqueeze(-1).expand_as(layer.salient_keys)
        count = layer.salient_valid.sum(dim=1).to(torch.int32)
        blocks.append(DecodeBlockState(
            working=layer.working_state.float().contiguous().clone(),
            memory_basis=layer.memory_basis.float().contiguous().clone(),
            memory_normalizer=layer.memory_normalizer.float().contiguous().clone(),
            refine_basis=layer.refine_basis.float().contiguous().clone(),
            refine_normalizer=layer.refine_normalizer.float().contiguous().clone(),
            local_keys=layer.local_keys.to(ring_dtype).contiguous().clone(),
            local_values=layer.local_values.to(ring_dtype).contiguous().clone(),
            local_valid=layer.local_valid.contiguous().clone(),
            salient_keys=layer.salient_keys.to(ring_dtype).gather(1, gather).contiguous(),
            salient_values=layer.salient_values.to(ring_dtype).gather(1, gather).contiguous(),
            salient_valid=layer.salient_valid.gather(1, order).contiguous(),
            salient_head=torch.zeros_like(count),
            salient_count=count,
        ))
    device = layers[0].working_state.device
    return DecodeState(blocks=blocks, local_head=torch.zeros(1, dtype=torch.int64, device=device),
                       last_token_ids=layers[-1].last_token_ids.clone(), step_index=state.step_index,
                       layered=isinstance(state, LayeredKoemiState))


def to_koemi_state(dstate: DecodeState):
    """Export in the reference layout: local rings oldest first; salient rings
    with admitted entries oldest first, packed at the end behind empty slots."""
    layers = []
    for block in dstate.blocks:
        batch, local_slots, width = block.local_keys.shape
        salient_slots = block.salient_keys.shape[1]
        device = block.local_keys.device
        local_index = (dstate.local_head + torch.arange(local_slots, device=device)) % local_slots
        logical = torch.arange(salient_slots, device=device).unsqueeze(0)
        lead = salient_slots - block.salient_count.long().unsqueeze(1)
        physical = (block.salient_head.long().unsqueeze(1) + logical - lead) % salient_slots
        present = logical >= lead
        gather = physical.unsqueeze(-1).expand(batch, salient_slots, width)
        keep = present.unsqueeze(-1)
        layers.append(KoemiState(
            working_state=block.working.clone(),
            memory_basis=block.memory_basis.clone(),
            memory_normalizer=block.memory_normalizer.clone(),
            refine_basis=block.refine_basis.clone(),
            refine_normalizer=block.refine_normalizer.clone(),
            local_keys=block.local_keys.index_select(1, local_index).float(),
            local_values=block.local_values.index_select(1, local_index).float(),
            local_valid=block.local_valid.index_select(1, local_index),
            salient_keys=torch.where(keep, block.salient_keys.gather(1, gather).float(), 0.0),
            salient_values=torch.where(keep, block.salient_values.gather(1, gather).float(), 0.0),
            salient_valid=present & block.salient_valid.gather(1, physical),
            last_token_ids=dstate.last_token_ids.clone(),
            step_index=dstate.step_index,
        ))
    if dstate.layered:
        return LayeredKoemiState(tuple(layers), dstate.step_index)
    return layers[0]


def supports_head_pass(model) -> bool:
    """The merged head pass runs on the tcgen05 path: 16-bit weights, a
    surprise to score, and a width of whole 16-byte packets."""
    s = model.settings
    return (model.compute_dtype in (torch.bfloat16, torch.float16) and s.ablation != "no_surprise"
            and s.embedding_size % 8 == 0)


def attach_head_pass(model, dstate: DecodeState) -> None:
    """Give ``dstate`` the buffers of the merged head pass and fold the
    log-sum-exp partials of its current priors (every block's working state),
    which the next decode step reads. Call again whenever the working states
    were replaced (a new or adopted state); a no-op for models without the
    merged pass."""
    if not supports_head_pass(model):
        dstate.head_rows = dstate.head_partials = None
        return
    s = model.settings
    blocks, batch, d = len(dstate.blocks), dstate.last_token_ids.shape[0], s.embedding_size
    device = dstate.last_token_ids.device
    lib = _native.library()
    slices = lib.koemi_think_head_pass_slices(s.vocabulary_size)
    rows = torch.zeros((blocks + 1) * batch, d, dtype=model.compute_dtype, device=device)
    rows[:blocks * batch].view(blocks, batch, d).copy_(torch.stack([st.working for st in dstate.blocks]))
    partials = torch.empty(slices, blocks * batch, 3, dtype=torch.float32, device=device)
    _native.call("koemi_think_head_pass", _native.ptr(rows), blocks * batch, 0, d, _native.ptr(model.head_weight),
                 _native.ptr(model.head_bias), s.vocabulary_size, PAD_TOKEN_ID, _native.ptr(partials), None,
                 _native.dtype_code(model.compute_dtype), torch.cuda.current_stream(device).cuda_stream)
    dstate.head_rows, dstate.head_partials = rows, partials


def decode_step(model, token_ids: Tensor, dstate: DecodeState) -> Tensor:
    """Advance every stream by one token in place; return fp32 logits [B, V]."""
    s = model.settings
    cache = model._cache
    batch = token_ids.shape[0]
    d = s.embedding_size
    device = token_ids.device
    ids = token_ids.reshape(batch).contiguous()
    valid = ids != PAD_TOKEN_ID
    stream = torch.cuda.current_stream(device).cuda_stream
    call = _native.call
    ptr = _native.ptr
    prior_dtype = _native.dtype_code(model.compute_dtype)
    x = model.embedding_weight.index_select(0, ids).float()
    concat_dtype = model.compute_dtype
    out_code = _native.dtype_code(concat_dtype)
    ring_code = _native.dtype_code(dstate.ring_dtype)
    scoring = s.ablation != "no_surprise"
    merged = scoring and dstate.head_rows is not None
    if not scoring or merged:
        targets = None
    else:
        targets = torch.where(ids > PAD_TOKEN_ID, ids - 1, ids) if s.vocabulary_size != PAD_TOKEN_ID + 1 else ids
    # the hash route depends only on the ids, so one permutation serves every
    # block (each block gathers its own rows through it)
    shared_route = s.expert_count > 0 and s.expert_routing != "learned"
    if shared_route:
        assignments = _ops.route_topk(ids, dstate.last_token_ids, valid, s.expert_count, s.expert_top_k)
        _, sorted_tokens, sorted_experts, offsets, positions = _ops.permute_topk(
            x, assignments, valid, s.expert_count, False)
        weights = None
    # surprise of every block from its prior (the working state before this
    # step's update). With the merged head pass its log-sum-exp partials were
    # folded by the previous step's head read; only the target logits remain.
    # Otherwise one pass over the content head for the whole stack. Each
    # row's result is independent of the others.
    all_surprise = None
    count = len(model.blocks)
    if merged:
        all_surprise = torch.empty(count, batch, dtype=torch.float32, device=device)
        call("koemi_think_surprise_from_partials", ptr(dstate.head_rows), ptr(model.head_weight),
             ptr(model.head_bias), ptr(ids), ptr(valid), ptr(dstate.head_partials), dstate.head_partials.shape[0],
             count * batch, batch, d, s.vocabulary_size, PAD_TOKEN_ID, prior_dtype, ptr(all_surprise), stream)
    elif targets is not None:
        priors = torch.stack([st.working for st in dstate.blocks]).to(model.compute_dtype)
        all_surprise = _ops.causal_surprise_forward(
            priors.view(count * batch, d), cache["content_w"], cache["content_b"], targets.repeat(count),
            valid.repeat(count), torch.float32).view(count, batch)
    # the combine of block i also writes block i + 1's normalised input
    fused_combine = s.expert_count > 0 and d % 4 == 0 and d <= 2048 and s.expert_top_k <= 8
    exchange = (model.fused_return_exchange(batch * s.expert_top_k, d)
                if shared_route and fused_combine and model.expert_shard is not None else None)
    # one GPU with a shared route and 16-bit experts: the grouped GEMMs' tile
    # map is computed once per step (every block has the same segments) and
    # each block's fusion norm gathers its expert rows itself
    mapped = None
    if (shared_route and fused_combine and model.expert_shard is None and d % 8 == 0
            and model.compute_dtype in (torch.bfloat16, torch.float16)):
        pairs = sorted_tokens.shape[0]
        mapped = {"tile_prefix": torch.empty(s.expert_count + 1, dtype=torch.int32, device=device),
                  "workspace_bytes": _native.library().koemi_moe_grouped_mlp_workspace(
                      pairs, d, model.blocks[0].expert_gate_weight.shape[1], s.expert_count, prior_dtype)}
        call("koemi_moe_tile_prefix", ptr(offsets), s.expert_count, ptr(mapped["tile_prefix"]), stream)
    u = None
    for index, block in enumerate(model.blocks):
        bc = cache["blocks"][index]
        st = dstate.blocks[index]
        if u is None:
            u = _ops.rms_norm(x, None, bc["input_norm"], None, NORM_EPSILON, model.compute_dtype)
        pre = model._linear(u, block.gates_weight, block.gates_bias)
        # fusion input rows, written in place by the step kernels: h | memory | local | salient
        concat = torch.empty(batch, 4 * d, dtype=concat_dtype, device=device)
        # the new working state is also the next step's prior row of the head pass
        next_prior = ptr(dstate.head_rows[index * batch:(index + 1) * batch]) if merged else None
        call("koemi_dense_decode_step", ptr(pre), ptr(valid), ptr(st.working), None, ptr(concat), 4 * d,
             next_prior, batch, d, MIN_RETENTION, MAX_RETENTION, prior_dtype, stream)
        h = concat[:, :d]
        surprise = None if all_surprise is None else all_surprise[index]
        # local | assoc as one GEMM over h: fills the GPU better than two at
        # every decode batch (256 rows: 24.7 us against 13.2 + 16.1 us)
        local_assoc = model._linear(h, bc["local_assoc_weight"], bc["local_assoc_bias"])
        local, assoc = local_assoc[:, :2 * d], local_assoc[:, 2 * d:]
        scored = surprise if surprise is not None else torch.zeros(batch, device=device)
        # ring queries read the fp32 working state (the new h) directly
        call("koemi_think_ring_decode_step", ptr(st.working), d, ptr(local), local.stride(0), ptr(valid), ptr(scored),
             float(s.salience_threshold), ptr(st.local_keys), ptr(st.local_values), ptr(st.local_valid),
             ptr(dstate.local_head), ptr(st.salient_keys), ptr(st.salient_values), ptr(st.salient_valid),
             ptr(st.salient_head), ptr(st.salient_count), ptr(concat[:, 2 * d:]), ptr(concat[:, 3 * d:]), 4 * d,
             None, None, batch, d, st.local_keys.shape[1], st.salient_keys.shape[1], ring_code, out_code, stream)
        # (run beside the ring kernel on a side stream, a parallel graph
        # branch, it measured slower: at 32 streams the two cluster kernels
        # contend for SMs, ring 23.7 -> 36.7 us, step 4.24 -> 4.34 ms)
        _assoc_step(call, ptr, block, st, assoc, surprise, valid, concat, batch, d, s.memory_features,
                    out_code, stream)
        fused = model._linear(concat, block.fusion_weight, block.fusion_bias)
        if mapped is not None:
            # one GPU, one permutation per step: the fusion norm also writes each
            # pair's row at its sorted position
            context = torch.empty(batch, d, dtype=torch.float32, device=device)
            rows = torch.empty(pairs, d, dtype=model.compute_dtype, device=device)
            call("koemi_moe_norm_gather", ptr(fused), ptr(bc["fusion_norm"]), NORM_EPSILON, ptr(context),
                 ptr(positions), ptr(offsets), s.expert_count, ptr(rows), prior_dtype, batch, d, s.expert_top_k,
                 stream)
        elif exchange is not None:
            # expert parallel: the fusion norm dispatches each pair's row to its
            # owner; the owners' outputs come back into this rank's exchange
            # buffer, where the fused combine reads them
            context = exchange.dispatch_normed(fused, bc["fusion_norm"], NORM_EPSILON, positions, sorted_experts,
                                               offsets, s.expert_top_k)
        else:
            context = _ops.rms_norm(fused, None, bc["fusion_norm"], None, NORM_EPSILON, torch.float32)
        u = None
        if s.expert_count == 0:
            x = context
            continue
        if exchange is not None:
            exchange.serve_and_return(block.expert_weights())
        elif mapped is not None:
            expert_weights = block.expert_weights()
            expert_out = torch.empty(pairs, d, dtype=model.compute_dtype, device=device)
            workspace = _native.workspace(mapped["workspace_bytes"], device)
            call("koemi_moe_grouped_expert_mlp_mapped", ptr(rows), ptr(mapped["tile_prefix"]), ptr(offsets),
                 *(ptr(w) for w in expert_weights), ptr(expert_out), pairs, d, expert_weights[0].shape[1],
                 s.expert_count, prior_dtype, ptr(workspace), workspace.numel(), stream)
        elif shared_route:
            expert_out = model.expert_mlp_of_tokens(block, context, sorted_tokens, sorted_experts, offsets)
        else:
            gate_logits = model._linear(torch.where(valid.unsqueeze(-1), context, 0.0), block.router_weight, None)
            assignments, weights, _ = _ops.learned_topk(gate_logits, valid, s.expert_top_k, bool(s.router_renormalize))
            sorted_context, _, sorted_experts, offsets, positions = _ops.permute_topk(
                context.to(model.compute_dtype), assignments, valid, s.expert_count, True)
            expert_out = model.expert_mlp(block, sorted_context, sorted_experts, offsets, mode="padded")
        if fused_combine:
            last = index + 1 == len(model.blocks)
            next_norm = None if last else cache["blocks"][index + 1]["input_norm"]
            if exchange is not None:
                y = torch.empty(batch, d, dtype=model.compute_dtype, device=device)
                call("koemi_ep_combine_residual_rmsnorm_next", ptr(context), ptr(positions), ptr(offsets),
                     ptr(weights), ptr(valid), ptr(bc["expert_norm"]), ptr(next_norm), ptr(y),
                     _native.dtype_code(model.compute_dtype), batch, d, s.expert_top_k, s.expert_count,
                     NORM_EPSILON, _native.dtype_code(exchange.dtype), exchange.own, exchange.shard.world,
                     exchange.shard.local_count, exchange.capacity, stream)
            else:
                y = _ops.combine_residual_rmsnorm_next(context, expert_out, positions, offsets, weights, valid,
                                                       bc["expert_norm"], next_norm, s.expert_top_k, NORM_EPSILON,
                                                       model.compute_dtype)
            if last:
                x = y
            else:
                u = y
        else:
            x = _ops.combine_residual_rmsnorm(context, expert_out, positions, offsets, weights, valid,
                                              bc["expert_norm"], s.expert_top_k, NORM_EPSILON)
    if merged:
        # one read of the head: this step's logits and the next step's
        # surprise partials of every block's new working state
        dstate.head_rows[count * batch:].copy_(x)
        logits = torch.empty(batch, s.vocabulary_size, dtype=torch.float32, device=device)
        call("koemi_think_head_pass", ptr(dstate.head_rows), count * batch, batch, d, ptr(model.head_weight),
             ptr(model.head_bias), s.vocabulary_size, PAD_TOKEN_ID, ptr(dstate.head_partials), ptr(logits),
             prior_dtype, stream)
    else:
        logits = model._linear(x, model.head_weight, model.head_bias)
    dstate.last_token_ids.copy_(torch.where(valid, ids, dstate.last_token_ids))
    dstate.local_head.add_(1).remainder_(dstate.blocks[0].local_keys.shape[1])
    return logits
