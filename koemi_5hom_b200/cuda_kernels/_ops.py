"""``torch.library`` custom ops over the C-ABI of ``libkoemi_b200.so``.

Each op allocates its outputs and workspace from torch's caching allocator,
then launches the native kernels on the current stream through ctypes. The
ops are registered under the ``koemi_b200`` namespace with fake (meta)
implementations, so they can be captured in CUDA graphs and traced. There is
no CPU implementation: a CPU tensor reaching an op is a programming error,
reported by the fronts before dispatch.
"""
from __future__ import annotations

import torch
from torch import Tensor

from koemi_5hom_b200 import _native
from koemi_5hom_b200._native import call, dtype_code, ptr, stream_of

BF16_OR_F16 = (torch.bfloat16, torch.float16)


def _prepare(tensor: Tensor) -> int:
    _native.ensure_device(tensor.device)
    return stream_of(tensor)


def _dense(*tensors):
    """Row-major views of the inputs: the kernels take raw pointers, so a
    strided view (a window slice of the ids, a transposed weight) is copied."""
    return tuple(t if t is None or t.is_contiguous() else t.contiguous() for t in tensors)


# ---------------------------------------------------------------- dense front

@torch.library.custom_op("koemi_b200::affine_scan_forward", mutates_args=())
def affine_scan_forward(retention: Tensor, increment: Tensor, initial: Tensor, broadcast: bool) -> Tensor:
    retention, increment, initial = _dense(retention, increment, initial)
    stream = _prepare(increment)
    batch, length = increment.shape[0], increment.shape[1]
    features = increment.numel() // max(batch * length, 1) if batch * length else 0
    states = torch.empty_like(increment)
    code = dtype_code(increment.dtype)
    workspace_bytes = _native.library().koemi_dense_affine_scan_workspace(batch, length, features, code)
    workspace = torch.empty(workspace_bytes, dtype=torch.uint8, device=increment.device) if workspace_bytes else None
    call("koemi_dense_affine_scan_forward", ptr(retention), ptr(increment), ptr(initial), ptr(states),
         batch, length, features, int(broadcast), code, ptr(workspace), workspace_bytes, stream)
    return states


@affine_scan_forward.register_fake
def _(retention, increment, initial, broadcast):
    return torch.empty_like(increment)


@torch.library.custom_op("koemi_b200::affine_scan_backward", mutates_args=())
def affine_scan_backward(retention: Tensor, initial: Tensor, states: Tensor, grad_states: Tensor,
                         broadcast: bool) -> tuple[Tensor, Tensor, Tensor]:
    retention, initial, states, grad_states = _dense(retention, initial, states, grad_states)
    stream = _prepare(states)
    batch, length = states.shape[0], states.shape[1]
    features = states.numel() // max(batch * length, 1) if batch * length else 0
    grad_retention = torch.empty_like(states)
    grad_increment = torch.empty_like(states)
    grad_initial = torch.empty_like(initial)
    call("koemi_dense_affine_scan_backward", ptr(retention), ptr(initial), ptr(states), ptr(grad_states),
         ptr(grad_retention), ptr(grad_increment), ptr(grad_initial), batch, length, features,
         int(broadcast), dtype_code(states.dtype), stream)
    return grad_retention, grad_increment, grad_initial


@affine_scan_backward.register_fake
def _(retention, initial, states, grad_states, broadcast):
    return torch.empty_like(states), torch.empty_like(states), torch.empty_like(initial)


@torch.library.custom_op("koemi_b200::bounded_gates", mutates_args=())
def bounded_gates(projections: Tensor, valid: Tensor, minimum: float, maximum: float) -> tuple[Tensor, Tensor]:
    projections, valid = _dense(projections, valid)
    stream = _prepare(projections)
    rows, features = projections.shape[0], projections.shape[1] // 2
    retention = projections.new_empty(rows, features)
    increment = projections.new_empty(rows, features)
    call("koemi_dense_bounded_gates", ptr(projections), ptr(valid), ptr(retention), ptr(increment), rows,
         features, minimum, maximum, stream)
    return retention, increment


@bounded_gates.register_fake
def _(projections, valid, minimum, maximum):
    rows, features = projections.shape[0], projections.shape[1] // 2
    return projections.new_empty(rows, features), projections.new_empty(rows, features)


@torch.library.custom_op("koemi_b200::dense_projection", mutates_args=())
def dense_projection(a: Tensor, weight: Tensor, bias: Tensor | None, weights_ready: bool = False) -> Tensor:
    """fp32 [rows, n] = a [rows, k] @ weight[n, k]^T + bias on tensor cores
    (bf16/f16 operands); `a` may be a view with strided rows. With
    ``weights_ready`` (model parameters: nothing in flight on the stream
    writes weight or bias) the kernel starts loading weights while the
    previous kernel of the stream finishes."""
    weight, bias = _dense(weight, bias)
    if a.stride(-1) != 1:
        a = a.contiguous()
    stream = _prepare(weight)
    rows, k = a.shape
    n = weight.shape[0]
    out = torch.empty(rows, n, dtype=torch.float32, device=a.device)
    code = dtype_code(weight.dtype)
    size = _native.library().koemi_dense_projection_workspace(rows, n, k, code)
    scratch = _native.workspace(size, a.device)
    entry = "koemi_dense_projection_resident" if weights_ready else "koemi_dense_projection"
    call(entry, ptr(a), a.stride(0), ptr(weight), ptr(bias), ptr(out), n, rows, n, k, code,
         ptr(scratch), scratch.numel(), stream)
    return out


@dense_projection.register_fake
def _(a, weight, bias, weights_ready=False):
    return a.new_empty(a.shape[0], weight.shape[0], dtype=torch.float32)


@torch.library.custom_op("koemi_b200::grouped_projection", mutates_args=())
def grouped_projection(a: Tensor, b: Tensor, groups: int) -> Tensor:
    """fp32 [G * M, N] with out[g] = a[g] @ b[g]^T for G uniform groups:
    a [G * M, K], b [G * N, K] (bf16/f16, row-major) on tensor cores."""
    a, b = _dense(a, b)
    stream = _prepare(a)
    rows, k = a.shape
    n = b.shape[0] // groups
    out = torch.empty(rows, n, dtype=torch.float32, device=a.device)
    call("koemi_grouped_projection", ptr(a), ptr(b), ptr(out), groups, rows // groups, n, k, dtype_code(a.dtype),
         stream)
    return out


@grouped_projection.register_fake
def _(a, b, groups):
    return a.new_empty(a.shape[0], b.shape[0] // groups, dtype=torch.float32)


def _rows_view(t: Tensor) -> tuple[Tensor, int]:
    """A 2-D fp32 row block whose rows are contiguous, and its row stride."""
    if t.dim() != 2 or t.stride(1) != 1 or t.stride(0) % 2 or t.data_ptr() % (16 if t.stride(0) % 4 == 0 else 8):
        t = t.contiguous()
    return t, t.stride(0)


@torch.library.custom_op("koemi_b200::pack_rows", mutates_args=("out",))
def pack_rows(out: Tensor, sources: list[Tensor]) -> None:
    """out[:, o_p : o_p + w_p] = sources[p] converted to out's dtype, the fp32
    row blocks [rows, w_p] side by side (o_p = w_0 + ... + w_{p-1}); out is a
    2-D block [rows, >= sum w_p] with contiguous rows."""
    import ctypes
    stream = _prepare(out)
    views = [_rows_view(t) for t in sources]
    count = len(views)
    source_ptrs = (ctypes.c_void_p * count)(*[v.data_ptr() for v, _ in views])
    strides = (ctypes.c_int64 * count)(*[stride for _, stride in views])
    widths = (ctypes.c_int64 * count)(*[v.shape[1] for v, _ in views])
    call("koemi_window_pack_rows", ctypes.cast(source_ptrs, ctypes.c_void_p), ctypes.cast(strides, ctypes.c_void_p),
         ctypes.cast(widths, ctypes.c_void_p), count, out.shape[0], ptr(out), out.stride(0), dtype_code(out.dtype),
         stream)


@pack_rows.register_fake
def _(out, sources):
    return None


@torch.library.custom_op("koemi_b200::window_slot_operands", mutates_args=())
def window_slot_operands(carried_keys: Tensor, carried_values: Tensor, keys: Tensor, values: Tensor, padded: int,
                         dtype: torch.dtype) -> tuple[Tensor, Tensor]:
    """Stacked keys [B, padded, d] and transposed values [B, d, padded] in
    ``dtype`` of the slots [carried ; window] (fp32 [B, C, d] and [B, T, d]),
    zero past C + T: the B operands of a window ring read's two products."""
    def rows_of(t):
        return t if t.stride(2) == 1 and t.stride(1) == t.shape[2] and t.stride(0) % 4 == 0 else t.contiguous()
    carried_keys, carried_values = rows_of(carried_keys), rows_of(carried_values)
    keys, values = rows_of(keys), rows_of(values)
    if carried_keys.stride() != carried_values.stride():
        carried_keys, carried_values = carried_keys.contiguous(), carried_values.contiguous()
    if keys.stride() != values.stride():
        keys, values = keys.contiguous(), values.contiguous()
    stream = _prepare(keys)
    batch, length, width = keys.shape
    carried = carried_keys.shape[1]
    stacked = torch.empty(batch, padded, width, dtype=dtype, device=keys.device)
    transposed = torch.empty(batch, width, padded, dtype=dtype, device=keys.device)
    call("koemi_window_slot_operands", ptr(carried_keys), ptr(carried_values), carried_keys.stride(0), carried,
         ptr(keys), ptr(values), keys.stride(0), length, batch, width, padded, ptr(stacked), ptr(transposed),
         dtype_code(dtype), stream)
    return stacked, transposed


@window_slot_operands.register_fake
def _(carried_keys, carried_values, keys, values, padded, dtype):
    batch, _, width = keys.shape
    return (keys.new_empty(batch, padded, width, dtype=dtype), keys.new_empty(batch, width, padded, dtype=dtype))


# ----------------------------------------------------------------- core front

@torch.library.custom_op("koemi_b200::rmsnorm_silu_forward", mutates_args=())
def rmsnorm_silu_forward(x: Tensor, weight: Tensor, eps: float) -> tuple[Tensor, Tensor]:
    x, weight = _dense(x, weight)
    stream = _prepare(x)
    rows, hidden = x.shape
    y = torch.empty_like(x)
    inv_rms = torch.empty(rows, dtype=torch.float32, device=x.device)
    call("koemi_core_rmsnorm_silu_forward", ptr(x), ptr(weight), ptr(y), ptr(inv_rms), rows, hidden, eps,
         dtype_code(x.dtype), stream)
    return y, inv_rms


@rmsnorm_silu_forward.register_fake
def _(x, weight, eps):
    return torch.empty_like(x), x.new_empty(x.shape[0], dtype=torch.float32)


@torch.library.custom_op("koemi_b200::rmsnorm_silu_backward", mutates_args=())
def rmsnorm_silu_backward(grad_y: Tensor, x: Tensor, weight: Tensor, inv_rms: Tensor,
                          eps: float) -> tuple[Tensor, Tensor]:
    grad_y, x, weight, inv_rms = _dense(grad_y, x, weight, inv_rms)
    stream = _prepare(x)
    rows, hidden = x.shape
    grad_x = torch.empty_like(x)
    grad_weight = torch.empty(hidden, dtype=torch.float32, device=x.device)
    size = _native.library().koemi_core_rmsnorm_silu_backward_workspace(rows, hidden)
    scratch = _native.workspace(size, x.device)
    call("koemi_core_rmsnorm_silu_backward", ptr(grad_y), ptr(x), ptr(weight), ptr(inv_rms), ptr(grad_x),
         ptr(grad_weight), rows, hidden, ptr(scratch), scratch.numel(), dtype_code(x.dtype), stream)
    return grad_x, grad_weight


@rmsnorm_silu_backward.register_fake
def _(grad_y, x, weight, inv_rms, eps):
    return torch.empty_like(x), x.new_empty(x.shape[1], dtype=torch.float32)


@torch.library.custom_op("koemi_b200::gated_rmsnorm_silu", mutates_args=())
def gated_rmsnorm_silu(x: Tensor, gate: Tensor, weight: Tensor, eps: float) -> Tensor:
    x, gate, weight = _dense(x, gate, weight)
    stream = _prepare(x)
    rows, hidden = x.shape
    y = torch.empty_like(x)
    call("koemi_core_gated_rmsnorm_silu_forward", ptr(x), ptr(gate), ptr(weight), ptr(y), None, rows, hidden,
         eps, dtype_code(x.dtype), stream)
    return y


@gated_rmsnorm_silu.register_fake
def _(x, gate, weight, eps):
    return torch.empty_like(x)


@torch.library.custom_op("koemi_b200::rms_norm", mutates_args=())
def rms_norm(x: Tensor, residual: Tensor | None, weight: Tensor, keep: Tensor | None, eps: float,
             out_dtype: torch.dtype) -> Tensor:
    x, residual, weight, keep = _dense(x, residual, weight, keep)
    stream = _prepare(x)
    rows, hidden = x.shape
    y = torch.empty(rows, hidden, dtype=out_dtype, device=x.device)
    call("koemi_core_rmsnorm_forward", ptr(x), ptr(residual), ptr(weight), ptr(keep), ptr(y), rows, hidden,
         eps, dtype_code(x.dtype), dtype_code(out_dtype), stream)
    return y


@rms_norm.register_fake
def _(x, residual, weight, keep, eps, out_dtype):
    return x.new_empty(x.shape, dtype=out_dtype)


# ---------------------------------------------------------------- think front

@torch.library.custom_op("koemi_b200::causal_surprise_forward", mutates_args=())
def causal_surprise_forward(prior: Tensor, weight: Tensor, bias: Tensor, targets: Tensor, valid: Tensor,
                            out_dtype: torch.dtype) -> Tensor:
    prior, weight, bias, targets, valid = _dense(prior, weight, bias, targets, valid)
    stream = _prepare(prior)
    width = prior.shape[-1]
    rows = prior.numel() // width
    vocab = weight.shape[0]
    out = torch.empty(prior.shape[:-1], dtype=out_dtype, device=prior.device)
    size = _native.library().koemi_think_surprise_workspace(rows, width, vocab, dtype_code(prior.dtype))
    scratch = _native.workspace(size, prior.device)
    call("koemi_think_causal_surprise_forward", ptr(prior), ptr(weight), ptr(bias), ptr(targets), ptr(valid),
         ptr(out), None, rows, width, vocab, dtype_code(prior.dtype), dtype_code(out_dtype), ptr(scratch),
         scratch.numel(), stream)
    return out


@causal_surprise_forward.register_fake
def _(prior, weight, bias, targets, valid, out_dtype):
    return prior.new_empty(prior.shape[:-1], dtype=out_dtype)


@torch.library.custom_op("koemi_b200::causal_surprise_forward_nll", mutates_args=())
def causal_surprise_forward_nll(prior: Tensor, weight: Tensor, bias: Tensor, targets: Tensor, valid: Tensor,
                                out_dtype: torch.dtype) -> tuple[Tensor, Tensor]:
    """The surprise and the per-row fp32 NLL (kept for the backward)."""
    prior, weight, bias, targets, valid = _dense(prior, weight, bias, targets, valid)
    stream = _prepare(prior)
    width = prior.shape[-1]
    rows = prior.numel() // width
    vocab = weight.shape[0]
    out = torch.empty(prior.shape[:-1], dtype=out_dtype, device=prior.device)
    nll = torch.empty(prior.shape[:-1], dtype=torch.float32, device=prior.device)
    size = _native.library().koemi_think_surprise_workspace(rows, width, vocab, dtype_code(prior.dtype))
    scratch = _native.workspace(size, prior.device)
    call("koemi_think_causal_surprise_forward", ptr(prior), ptr(weight), ptr(bias), ptr(targets), ptr(valid),
         ptr(out), ptr(nll), rows, width, vocab, dtype_code(prior.dtype), dtype_code(out_dtype), ptr(scratch),
         scratch.numel(), stream)
    return out, nll


@causal_surprise_forward_nll.register_fake
def _(prior, weight, bias, targets, valid, out_dtype):
    return (prior.new_empty(prior.shape[:-1], dtype=out_dtype),
            prior.new_empty(prior.shape[:-1], dtype=torch.float32))


@torch.library.custom_op("koemi_b200::causal_surprise_dlogits", mutates_args=())
def causal_surprise_dlogits(prior: Tensor, weight: Tensor, bias: Tensor, targets: Tensor, valid: Tensor,
                            grad: Tensor, nll: Tensor) -> Tensor:
    """fp32 [rows, content_vocab] gradient of the loss with respect to the
    surprise logits (koemi_think_causal_surprise_backward)."""
    prior, weight, bias, targets, valid, grad, nll = _dense(prior, weight, bias, targets, valid, grad, nll)
    stream = _prepare(prior)
    width = prior.shape[-1]
    rows = prior.numel() // width
    vocab = weight.shape[0]
    dlogits = torch.empty(rows, vocab, dtype=torch.float32, device=prior.device)
    scratch = _native.workspace(_native.library().koemi_think_surprise_backward_workspace(rows), prior.device)
    call("koemi_think_causal_surprise_backward", ptr(prior), ptr(weight), ptr(bias), ptr(targets), ptr(valid),
         ptr(grad), ptr(nll), ptr(dlogits), rows, width, vocab, dtype_code(prior.dtype), ptr(scratch),
         scratch.numel(), stream)
    return dlogits


@causal_surprise_dlogits.register_fake
def _(prior, weight, bias, targets, valid, grad, nll):
    width = prior.shape[-1]
    return prior.new_empty(prior.numel() // width, weight.shape[0], dtype=torch.float32)


@torch.library.custom_op("koemi_b200::salient_admission", mutates_args=())
def salient_admission(carried_keys: Tensor, carried_values: Tensor, carried_valid: Tensor, keys: Tensor,
                      values: Tensor, surprise: Tensor, valid: Tensor, threshold: float,
                      capacity: int) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    carried_keys, carried_values, carried_valid, keys, values, surprise, valid = _dense(carried_keys, carried_values, carried_valid, keys, values, surprise, valid)
    stream = _prepare(keys)
    batch, length, width = keys.shape
    carried = carried_keys.shape[1]
    ring = min(carried + length, capacity)
    out_keys = keys.new_empty(batch, ring, width)
    out_values = keys.new_empty(batch, ring, width)
    out_valid = torch.empty(batch, ring, dtype=torch.bool, device=keys.device)
    admission = torch.empty(batch, length, dtype=torch.bool, device=keys.device)
    call("koemi_think_salient_admission", ptr(carried_keys), ptr(carried_values), ptr(carried_valid),
         ptr(keys), ptr(values), ptr(surprise), ptr(valid), threshold, ptr(out_keys), ptr(out_values),
         ptr(out_valid), ptr(admission), batch, carried, length, width, capacity, stream)
    return out_keys, out_values, out_valid, admission


@salient_admission.register_fake
def _(carried_keys, carried_values, carried_valid, keys, values, surprise, valid, threshold, capacity):
    batch, length, width = keys.shape
    ring = min(carried_keys.shape[1] + length, capacity)
    return (keys.new_empty(batch, ring, width), keys.new_empty(batch, ring, width),
            keys.new_empty(batch, ring, dtype=torch.bool), keys.new_empty(batch, length, dtype=torch.bool))


# ------------------------------------------------------------------ moe front

@torch.library.custom_op("koemi_b200::route_topk", mutates_args=())
def route_topk(token_ids: Tensor, previous_token_ids: Tensor, valid: Tensor, expert_count: int,
               top_k: int) -> Tensor:
    token_ids, previous_token_ids, valid = _dense(token_ids, previous_token_ids, valid)
    stream = _prepare(token_ids)
    count = token_ids.numel()
    out = torch.empty(count, top_k, dtype=torch.int64, device=token_ids.device)
    call("koemi_moe_route_topk", ptr(token_ids), ptr(previous_token_ids), ptr(valid), ptr(out), count,
         expert_count, top_k, dtype_code(token_ids.dtype), stream)
    return out


@route_topk.register_fake
def _(token_ids, previous_token_ids, valid, expert_count, top_k):
    return token_ids.new_empty(token_ids.numel(), top_k, dtype=torch.int64)


@torch.library.custom_op("koemi_b200::learned_topk", mutates_args=())
def learned_topk(gate_logits: Tensor, valid: Tensor, top_k: int, renormalize: bool) -> tuple[Tensor, Tensor, Tensor]:
    gate_logits, valid = _dense(gate_logits, valid)
    stream = _prepare(gate_logits)
    tokens, experts = gate_logits.shape
    assignments = torch.empty(tokens, top_k, dtype=torch.int64, device=gate_logits.device)
    weights = torch.empty(tokens, top_k, dtype=torch.float32, device=gate_logits.device)
    probabilities = torch.empty(tokens, experts, dtype=torch.float32, device=gate_logits.device)
    call("koemi_moe_learned_topk", ptr(gate_logits), ptr(valid), ptr(assignments), ptr(weights),
         ptr(probabilities), tokens, experts, top_k, int(renormalize), stream)
    return assignments, weights, probabilities


@learned_topk.register_fake
def _(gate_logits, valid, top_k, renormalize):
    tokens, experts = gate_logits.shape
    return (gate_logits.new_empty(tokens, top_k, dtype=torch.int64), gate_logits.new_empty(tokens, top_k),
            gate_logits.new_empty(tokens, experts))


@torch.library.custom_op("koemi_b200::permute_topk", mutates_args=())
def permute_topk(context: Tensor, assignments: Tensor, valid: Tensor, expert_count: int,
                 gather: bool) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    context, assignments, valid = _dense(context, assignments, valid)
    stream = _prepare(assignments)
    tokens, top_k = assignments.shape
    width = context.shape[-1]
    pairs = tokens * top_k
    device = assignments.device
    sorted_context = torch.empty(pairs if gather else 0, width, dtype=context.dtype, device=device)
    sorted_rows = torch.empty(pairs, dtype=torch.int64, device=device)
    sorted_experts = torch.empty(pairs, dtype=torch.int64, device=device)
    offsets = torch.empty(expert_count + 1, dtype=torch.int64, device=device)
    positions = torch.empty(pairs, dtype=torch.int64, device=device)
    size = _native.library().koemi_moe_permute_workspace(tokens, top_k, expert_count)
    scratch = _native.workspace(size, device)
    call("koemi_moe_permute_topk", ptr(context), ptr(assignments), ptr(valid),
         ptr(sorted_context) if gather else None, ptr(sorted_rows), ptr(sorted_experts), ptr(offsets),
         ptr(positions), tokens, width, top_k, expert_count, dtype_code(context.dtype),
         dtype_code(assignments.dtype), ptr(scratch), scratch.numel(), stream)
    return sorted_context, sorted_rows, sorted_experts, offsets, positions


@permute_topk.register_fake
def _(context, assignments, valid, expert_count, gather):
    tokens, top_k = assignments.shape
    pairs = tokens * top_k
    return (context.new_empty(pairs if gather else 0, context.shape[-1]),
            assignments.new_empty(pairs, dtype=torch.int64), assignments.new_empty(pairs, dtype=torch.int64),
            assignments.new_empty(expert_count + 1, dtype=torch.int64),
            assignments.new_empty(pairs, dtype=torch.int64))


@torch.library.custom_op("koemi_b200::grouped_expert_mlp", mutates_args=())
def grouped_expert_mlp(sorted_context: Tensor, sorted_experts: Tensor, segment_offsets: Tensor,
                       gate_weights: Tensor, gate_biases: Tensor, value_weights: Tensor, value_biases: Tensor,
                       output_weights: Tensor, output_biases: Tensor) -> Tensor:
    sorted_context, sorted_experts, segment_offsets, gate_weights, gate_biases, value_weights, value_biases, output_weights, output_biases = _dense(sorted_context, sorted_experts, segment_offsets, gate_weights, gate_biases, value_weights, value_biases, output_weights, output_biases)
    stream = _prepare(sorted_context)
    pairs, width = sorted_context.shape
    experts, hidden, _ = gate_weights.shape
    out = torch.empty_like(sorted_context)
    code = dtype_code(sorted_context.dtype)
    size = _native.library().koemi_moe_grouped_mlp_workspace(pairs, width, hidden, experts, code)
    scratch = _native.workspace(size, sorted_context.device)
    call("koemi_moe_grouped_expert_mlp", ptr(sorted_context), ptr(sorted_experts), ptr(segment_offsets),
         ptr(gate_weights), ptr(gate_biases), ptr(value_weights), ptr(value_biases), ptr(output_weights),
         ptr(output_biases), ptr(out), pairs, width, hidden, experts, code, ptr(scratch), scratch.numel(),
         stream)
    return out


@grouped_expert_mlp.register_fake
def _(sorted_context, sorted_experts, segment_offsets, gate_weights, gate_biases, value_weights, value_biases,
      output_weights, output_biases):
    return torch.empty_like(sorted_context)


@torch.library.custom_op("koemi_b200::combine_topk", mutates_args=())
def combine_topk(expert_outputs: Tensor, sorted_rows: Tensor, segment_offsets: Tensor, token_count: int,
                 top_k: int) -> Tensor:
    expert_outputs, sorted_rows, segment_offsets = _dense(expert_outputs, sorted_rows, segment_offsets)
    stream = _prepare(expert_outputs)
    pairs, width = expert_outputs.shape
    experts = segment_offsets.shape[0] - 1
    out = torch.empty(token_count, width, dtype=expert_outputs.dtype, device=expert_outputs.device)
    size = _native.library().koemi_moe_combine_workspace(token_count, pairs, top_k)
    scratch = _native.workspace(size, expert_outputs.device)
    call("koemi_moe_combine_topk", ptr(expert_outputs), ptr(sorted_rows), ptr(segment_offsets), ptr(out),
         pairs, width, token_count, top_k, experts, dtype_code(expert_outputs.dtype), ptr(scratch),
         scratch.numel(), stream)
    return out


@combine_topk.register_fake
def _(expert_outputs, sorted_rows, segment_offsets, token_count, top_k):
    return expert_outputs.new_empty(token_count, expert_outputs.shape[1])


@torch.library.custom_op("koemi_b200::combine_residual_rmsnorm", mutates_args=())
def combine_residual_rmsnorm(context: Tensor, expert_out: Tensor, pair_positions: Tensor,
                             segment_offsets: Tensor, weights: Tensor | None, valid: Tensor,
                             norm_weight: Tensor, top_k: int, eps: float) -> Tensor:
    context, expert_out, pair_positions, segment_offsets, weights, valid, norm_weight = _dense(context, expert_out, pair_positions, segment_offsets, weights, valid, norm_weight)
    stream = _prepare(context)
    tokens, width = context.shape
    experts = segment_offsets.shape[0] - 1
    out = torch.empty_like(context)
    call("koemi_moe_combine_residual_rmsnorm", ptr(context), ptr(expert_out), ptr(pair_positions),
         ptr(segment_offsets), ptr(weights), ptr(valid), ptr(norm_weight), ptr(out), tokens, width, top_k,
         experts, eps, dtype_code(expert_out.dtype), stream)
    return out


@combine_residual_rmsnorm.register_fake
def _(context, expert_out, pair_positions, segment_offsets, weights, valid, norm_weight, top_k, eps):
    return torch.empty_like(context)


# ------------------------------------------------------- expert parallelism

@torch.library.custom_op("koemi_b200::ep_pack", mutates_args=())
def ep_pack(sorted_rows: Tensor, sorted_experts: Tensor, segment_offsets: Tensor, ranks: int, local_experts: int,
            capacity: int) -> tuple[Tensor, Tensor]:
    """Dispatch slab [ranks * capacity, width] and owner-local expert ids
    (-1 = padding) of expert-major sorted rows; block g goes to rank g."""
    sorted_rows, sorted_experts, segment_offsets = _dense(sorted_rows, sorted_experts, segment_offsets)
    stream = _prepare(sorted_rows)
    pairs, width = sorted_rows.shape
    slab = torch.empty(ranks * capacity, width, dtype=sorted_rows.dtype, device=sorted_rows.device)
    slab_experts = torch.empty(ranks * capacity, dtype=torch.int32, device=sorted_rows.device)
    call("koemi_moe_ep_pack", ptr(sorted_rows), ptr(sorted_experts), ptr(segment_offsets), ptr(slab),
         ptr(slab_experts), pairs, width, ranks, local_experts, capacity, dtype_code(sorted_rows.dtype), stream)
    return slab, slab_experts


@ep_pack.register_fake
def _(sorted_rows, sorted_experts, segment_offsets, ranks, local_experts, capacity):
    return (sorted_rows.new_empty(ranks * capacity, sorted_rows.shape[1]),
            sorted_rows.new_empty(ranks * capacity, dtype=torch.int32))


@torch.library.custom_op("koemi_b200::ep_unpack", mutates_args=())
def ep_unpack(slab: Tensor, sorted_experts: Tensor, segment_offsets: Tensor, ranks: int, local_experts: int,
              capacity: int) -> Tensor:
    """Expert outputs back in the caller's sorted pair order (zero past the
    valid pairs) from the returned slab."""
    slab, sorted_experts, segment_offsets = _dense(slab, sorted_experts, segment_offsets)
    stream = _prepare(slab)
    pairs = sorted_experts.shape[0]
    width = slab.shape[1]
    out = torch.empty(pairs, width, dtype=slab.dtype, device=slab.device)
    call("koemi_moe_ep_unpack", ptr(slab), ptr(sorted_experts), ptr(segment_offsets), ptr(out), pairs, width,
         ranks, local_experts, capacity, dtype_code(slab.dtype), stream)
    return out


@ep_unpack.register_fake
def _(slab, sorted_experts, segment_offsets, ranks, local_experts, capacity):
    return slab.new_empty(sorted_experts.shape[0], slab.shape[1])


@torch.library.custom_op("koemi_b200::combine_residual_rmsnorm_next", mutates_args=())
def combine_residual_rmsnorm_next(context: Tensor, expert_out: Tensor, pair_positions: Tensor,
                                  segment_offsets: Tensor, weights: Tensor | None, valid: Tensor,
                                  norm_weight: Tensor, next_norm_weight: Tensor | None, top_k: int, eps: float,
                                  out_dtype: torch.dtype) -> Tensor:
    """``combine_residual_rmsnorm`` whose stored row is the next block's
    input RMSNorm(x) * next_norm_weight (or x itself without a next norm), in
    ``out_dtype``."""
    (context, expert_out, pair_positions, segment_offsets, weights, valid, norm_weight,
     next_norm_weight) = _dense(context, expert_out, pair_positions, segment_offsets, weights, valid, norm_weight,
                                next_norm_weight)
    stream = _prepare(context)
    tokens, width = context.shape
    experts = segment_offsets.shape[0] - 1
    out = torch.empty(tokens, width, dtype=out_dtype, device=context.device)
    call("koemi_moe_combine_residual_rmsnorm_next", ptr(context), ptr(expert_out), ptr(pair_positions),
         ptr(segment_offsets), ptr(weights), ptr(valid), ptr(norm_weight), ptr(next_norm_weight), ptr(out),
         dtype_code(out_dtype), tokens, width, top_k, experts, eps, dtype_code(expert_out.dtype), stream)
    return out


@combine_residual_rmsnorm_next.register_fake
def _(context, expert_out, pair_positions, segment_offsets, weights, valid, norm_weight, next_norm_weight, top_k, eps,
      out_dtype):
    return context.new_empty(context.shape, dtype=out_dtype)


@torch.library.custom_op("koemi_b200::gather_rows", mutates_args=())
def gather_rows(rows: Tensor, sorted_rows: Tensor, segment_offsets: Tensor, out_dtype: torch.dtype) -> Tensor:
    """Rows of an existing permutation (``sorted_rows`` from ``permute_topk``)
    in ``out_dtype``, zero past the valid pairs."""
    rows, sorted_rows, segment_offsets = _dense(rows, sorted_rows, segment_offsets)
    stream = _prepare(rows)
    pairs = sorted_rows.shape[0]
    width = rows.shape[1]
    out = torch.empty(pairs, width, dtype=out_dtype, device=rows.device)
    call("koemi_moe_gather_rows", ptr(rows), dtype_code(rows.dtype), ptr(sorted_rows), ptr(segment_offsets),
         segment_offsets.shape[0] - 1, ptr(out), dtype_code(out_dtype), pairs, width, stream)
    return out


@gather_rows.register_fake
def _(rows, sorted_rows, segment_offsets, out_dtype):
    return rows.new_empty(sorted_rows.shape[0], rows.shape[1], dtype=out_dtype)


# ------------------------------------------------------------------ sampling

@torch.library.custom_op("koemi_b200::greedy_tokens", mutates_args=())
def greedy_tokens(logits: Tensor, pad_id: int) -> Tensor:
    """[rows, vocab] fp32 logits -> int64 [rows, 1]: argmax with column
    pad_id masked (TokenSampler's greedy path, fast_decode.py:40-87)."""
    (logits,) = _dense(logits)
    stream = _prepare(logits)
    rows, vocab = logits.shape
    out = torch.empty(rows, 1, dtype=torch.int64, device=logits.device)
    call("koemi_sampler_greedy", ptr(logits), rows, vocab, vocab, pad_id, ptr(out), stream)
    return out


def temperature_tokens(logits: Tensor, pad_id: int, temperature: float, seed: int, stream_offset: int,
                       step: Tensor, thresholds: Tensor | None = None) -> Tensor:
    """[rows, vocab] fp32 logits -> int64 [rows, 1] drawn from
    softmax(logits / temperature) with column pad_id masked (and logits below
    ``thresholds[row]`` dropped), by the native counter-based Gumbel-max
    keyed by (seed, stream_offset + row, step[0], column)."""
    (logits,) = _dense(logits)
    stream = _prepare(logits)
    rows, vocab = logits.shape
    out = torch.empty(rows, 1, dtype=torch.int64, device=logits.device)
    call("koemi_sampler_temperature", ptr(logits), rows, vocab, vocab, pad_id, float(temperature),
         int(seed) & ((1 << 64) - 1), stream_offset, ptr(step), ptr(thresholds), ptr(out), stream)
    return out


@greedy_tokens.register_fake
def _(logits, pad_id):
    return logits.new_empty(logits.shape[0], 1, dtype=torch.int64)


# -------------------------------------------------------- associative memory

@torch.library.custom_op("koemi_b200::assoc_window_scan_read", mutates_args=())
def assoc_window_scan_read(basis: Tensor, normalizer: Tensor, decay: Tensor, value: Tensor, features: Tensor,
                           write: Tensor, query_features: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    """Window read and update of the rank-one associative memory (fp32):
    returns (read [B, T, d], new basis [B, d, m], new normaliser [B, m])."""
    decay, write, value, features, query_features = _dense(
        decay.float(), write.float(), value.float(), features.float(), query_features.float())
    stream = _prepare(value)
    batch, length, width = value.shape
    new_basis = basis.float().contiguous().clone()
    new_normalizer = normalizer.float().contiguous().clone()
    read = torch.empty_like(value)
    call("koemi_assoc_window_scan_read", ptr(decay), ptr(write), ptr(value), ptr(features), ptr(query_features),
         ptr(new_basis), ptr(new_normalizer), ptr(read), batch, length, width, features.shape[-1], stream)
    return read, new_basis, new_normalizer


@assoc_window_scan_read.register_fake
def _(basis, normalizer, decay, value, features, write, query_features):
    return torch.empty_like(value), torch.empty_like(basis), torch.empty_like(normalizer)
