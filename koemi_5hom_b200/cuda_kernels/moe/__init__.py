"""MoE front: route / permute / grouped expert MLP / combine, mirroring
``koemi.cuda_kernels.moe`` (src/koemi/cuda_kernels/moe/__init__.py:12-371).

Same function names, signatures, return layouts, limits (E <= 2^20,
k <= 256), inference-only rule, validation messages and exception types.
Differences that callers can observe only as improvements:

- every kernel runs on the *current* stream (the reference launches on the
  default stream);
- the permutation is a histogram/prefix-sum counting sort, bit-exact with a
  stable argsort, instead of a 64-bit CUB radix sort;
- bf16/f16 expert MLPs run on tcgen05 tensor cores;
- ``combine_topk`` sums each token's pairs in sorted order (deterministic)
  instead of float atomics;
- routing follows the torch runner's 64-bit slot arithmetic
  (experts.py:287-288) for every expert count.

The host-side checks that read device values (duplicates, ranges,
``segment_offsets[-1]``) are kept, as in the reference; the HERM block calls
the ``koemi_b200`` custom ops directly and never synchronises.
"""
from __future__ import annotations

from typing import Any

import torch
from torch import Tensor

from koemi_5hom_b200 import _native
from koemi_5hom_b200.cuda_kernels import _ops


class CudaMoeUnavailableError(RuntimeError):
    """Raised when the native MoE kernels cannot be loaded."""


class CudaMoeValidationError(ValueError):
    """Raised when a native MoE operation receives an unsafe contract."""


def load_native_extension() -> Any:
    """Open the native library on a CUDA host and return its handle."""
    if not torch.cuda.is_available():
        raise CudaMoeUnavailableError("Koemi MoE CUDA kernels require torch.cuda.is_available() == True")
    try:
        handle = _native.library()
    except _native.KoemiNativeUnavailableError as error:
        raise CudaMoeUnavailableError(f"Koemi MoE CUDA library failed to load: {error}") from error
    _native.ensure_device(torch.device("cuda", torch.cuda.current_device()))
    return handle


# Per-tensor rules, checked in order for every tensor a front receives: the
# first rule a tensor breaks raises (exception type, message with its name).
_TENSOR_RULES = (
    (lambda t: not isinstance(t, Tensor), TypeError, "{} must be a torch.Tensor"),
    (lambda t: not t.is_cuda, CudaMoeValidationError, "{} must be a CUDA tensor"),
    (lambda t: not t.is_contiguous(), CudaMoeValidationError, "{} must be contiguous"),
)
_FLOAT_DTYPES = (torch.float32, torch.float16, torch.bfloat16)
# Upper limits of the positive integer arguments (the kernels' index widths).
_COUNT_LIMITS = {"expert_count": 1 << 20, "top_k": 256, "token_count": 1 << 31}


def _check_tensors(tensors: dict[str, Tensor]) -> None:
    for name, tensor in tensors.items():
        for broken, error, message in _TENSOR_RULES:
            if broken(tensor):
                raise error(message.format(name))
    devices = sorted({str(tensor.device) for tensor in tensors.values()})
    if len(devices) > 1:
        raise CudaMoeValidationError(f"all MoE tensors must use one CUDA device, found {', '.join(devices)}")


def _check_float(tensor: Tensor, name: str) -> None:
    if tensor.dtype not in _FLOAT_DTYPES:
        raise CudaMoeValidationError(f"{name} must use float32, float16, or bfloat16; found {tensor.dtype}")


def _count(name: str, value: int) -> int:
    """``value`` if it is a positive int within ``_COUNT_LIMITS[name]``."""
    if type(value) is not int or value < 1:
        raise CudaMoeValidationError(f"{name} must be a positive integer")
    if value > _COUNT_LIMITS[name]:
        raise CudaMoeValidationError(f"{name} exceeds the CUDA MoE limit of {_COUNT_LIMITS[name]}")
    return value


def _inference_only(tensors: dict[str, Tensor]) -> None:
    tracked = [name for name in tensors if tensors[name].requires_grad]
    if tracked:
        raise RuntimeError("the native MoE path is inference-only; tensors require gradients: " + ", ".join(tracked))


def _reject_duplicates(assignments: Tensor, valid_mask: Tensor, message: str) -> None:
    """A valid token may not name one expert twice: after sorting its k
    slots, equal neighbours mark a repeat."""
    if assignments.shape[-1] < 2:
        return
    ordered = assignments.sort(dim=-1).values
    repeated = (ordered[..., 1:] == ordered[..., :-1]).any(dim=-1)
    if bool((repeated & valid_mask).any().item()):
        raise CudaMoeValidationError(message)


def route_topk_valid(token_ids: Tensor, previous_token_ids: Tensor, valid_mask: Tensor, *, expert_count: int,
                     top_k: int) -> Tensor:
    """Content-hash top-k routing; ``token_ids.shape + (top_k,)`` int64, -1 on
    invalid rows. Rejects duplicate experts on a valid token."""
    _check_tensors({"token_ids": token_ids, "previous_token_ids": previous_token_ids, "valid_mask": valid_mask})
    if token_ids.dtype not in (torch.int32, torch.int64):
        raise CudaMoeValidationError("token_ids must use int32 or int64")
    if previous_token_ids.dtype != token_ids.dtype:
        raise CudaMoeValidationError("token_ids and previous_token_ids must use one dtype")
    if valid_mask.dtype != torch.bool:
        raise CudaMoeValidationError("valid_mask must use boolean dtype")
    if token_ids.shape != previous_token_ids.shape or token_ids.shape != valid_mask.shape:
        raise CudaMoeValidationError("routing tensors must have equal shapes")
    expert_count = _count("expert_count", expert_count)
    top_k = _count("top_k", top_k)
    if top_k > expert_count:
        raise CudaMoeValidationError("top_k must not exceed expert_count")
    load_native_extension()
    assignments = _ops.route_topk(token_ids, previous_token_ids, valid_mask, expert_count, top_k)
    assignments = assignments.reshape(*token_ids.shape, top_k)
    _reject_duplicates(assignments, valid_mask, "MoE routing produced duplicate experts for a valid token")
    return assignments


def permute_topk(context: Tensor, assignments: Tensor, valid_mask: Tensor, *,
                 expert_count: int) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """Sort valid token-expert pairs into stable expert segments.

    Returns (sorted_context, sorted_rows, sorted_experts, segment_offsets);
    offsets are exclusive with ``expert_count + 1`` entries and invalid pairs
    follow every segment (expert id ``expert_count``).
    """
    _check_tensors({"context": context, "assignments": assignments, "valid_mask": valid_mask})
    _check_float(context, "context")
    if context.ndim < 2 or context.shape[-1] < 1:
        raise CudaMoeValidationError("context must have at least two dimensions and a non-empty width")
    if assignments.ndim != 2 or assignments.shape[0] != context.numel() // context.shape[-1]:
        raise CudaMoeValidationError("assignments must have shape [token_count, top_k]")
    if assignments.dtype not in (torch.int32, torch.int64):
        raise CudaMoeValidationError("assignments must use int32 or int64")
    if valid_mask.ndim != 1 or valid_mask.shape[0] != assignments.shape[0]:
        raise CudaMoeValidationError("valid_mask must have shape [token_count]")
    expert_count = _count("expert_count", expert_count)
    top_k = _count("top_k", int(assignments.shape[1]))
    if top_k > expert_count:
        raise CudaMoeValidationError("top_k must not exceed expert_count")
    out_of_range = ((assignments < 0) | (assignments >= expert_count)) & valid_mask.unsqueeze(-1)
    if bool(out_of_range.any().item()):
        raise CudaMoeValidationError("valid MoE assignments must be in [0, expert_count)")
    _reject_duplicates(assignments, valid_mask, "MoE permutation received duplicate experts for a valid token")
    load_native_extension()
    flat = context.reshape(-1, context.shape[-1])
    sorted_context, sorted_rows, sorted_experts, offsets, _ = _ops.permute_topk(
        flat, assignments, valid_mask, expert_count, True
    )
    return sorted_context, sorted_rows, sorted_experts, offsets


def grouped_expert_mlp_inference(sorted_context: Tensor, sorted_experts: Tensor, segment_offsets: Tensor,
                                 gate_weights: Tensor, gate_biases: Tensor, value_weights: Tensor,
                                 value_biases: Tensor, output_weights: Tensor, output_biases: Tensor) -> Tensor:
    """Grouped gated MLP of sorted pairs: weights ``[E, H, D]``, ``[E, H]``,
    ``[E, H, D]``, ``[E, H]``, ``[E, D, H]``, ``[E, D]``; rows past the valid
    count are zero. Inference only."""
    tensors = {
        "sorted_context": sorted_context,
        "sorted_experts": sorted_experts,
        "segment_offsets": segment_offsets,
        "gate_weights": gate_weights,
        "gate_biases": gate_biases,
        "value_weights": value_weights,
        "value_biases": value_biases,
        "output_weights": output_weights,
        "output_biases": output_biases,
    }
    _check_tensors(tensors)
    _check_float(sorted_context, "sorted_context")
    _inference_only(tensors)
    if sorted_context.ndim != 2:
        raise CudaMoeValidationError("sorted_context must have shape [pair_count, width]")
    if sorted_experts.ndim != 1 or sorted_experts.shape[0] != sorted_context.shape[0]:
        raise CudaMoeValidationError("sorted_experts must have shape [pair_count]")
    if sorted_experts.dtype != torch.int64:
        raise CudaMoeValidationError("sorted_experts must use int64")
    if segment_offsets.dtype != torch.int64 or segment_offsets.ndim != 1:
        raise CudaMoeValidationError("segment_offsets must be a one-dimensional int64 tensor")
    if gate_weights.ndim != 3 or value_weights.ndim != 3 or output_weights.ndim != 3:
        raise CudaMoeValidationError("expert weights must be three-dimensional")
    experts, hidden, width = gate_weights.shape
    shape_rules = (
        (width == sorted_context.shape[1], "gate weight input width does not match sorted_context"),
        (value_weights.shape == (experts, hidden, width), "value weights do not match gate weight shapes"),
        (output_weights.shape[0] == experts and output_weights.shape[1] == width,
         "output weights do not match expert and output widths"),
        (output_weights.shape[2] == hidden, "output weight hidden width does not match gate weights"),
        (gate_biases.shape == (experts, hidden), "gate biases do not match gate weights"),
        (value_biases.shape == (experts, hidden), "value biases do not match value weights"),
        (output_biases.shape == (experts, width), "output biases do not match output weights"),
        (segment_offsets.shape[0] == experts + 1, "segment_offsets must have expert_count + 1 entries"),
    )
    for passed, message in shape_rules:
        if not passed:
            raise CudaMoeValidationError(message)
    floats = [t for name, t in tensors.items() if name not in ("sorted_experts", "segment_offsets")]
    if any(t.dtype != sorted_context.dtype for t in floats):
        raise CudaMoeValidationError("all grouped MLP floating tensors must use one dtype")
    valid_pairs = int(segment_offsets[-1].item())
    if valid_pairs < 0 or valid_pairs > sorted_context.shape[0]:
        raise CudaMoeValidationError("segment_offsets final value is outside pair_count")
    if valid_pairs:
        chosen = sorted_experts[:valid_pairs]
        if bool((chosen < 0).any().item()) or bool((chosen >= experts).any().item()):
            raise CudaMoeValidationError("sorted expert ids are outside the expert catalog")
    load_native_extension()
    return _ops.grouped_expert_mlp(sorted_context, sorted_experts, segment_offsets, gate_weights, gate_biases,
                                   value_weights, value_biases, output_weights, output_biases)


def combine_topk(expert_outputs: Tensor, sorted_rows: Tensor, segment_offsets: Tensor, *, token_count: int,
                 top_k: int) -> Tensor:
    """Combine sorted expert outputs into token rows with weight ``1 / top_k``."""
    tensors = {"expert_outputs": expert_outputs, "sorted_rows": sorted_rows, "segment_offsets": segment_offsets}
    _check_tensors(tensors)
    _check_float(expert_outputs, "expert_outputs")
    _inference_only(tensors)
    if expert_outputs.ndim != 2:
        raise CudaMoeValidationError("expert_outputs must have shape [pair_count, width]")
    if sorted_rows.dtype != torch.int64 or sorted_rows.ndim != 1:
        raise CudaMoeValidationError("sorted_rows must be a one-dimensional int64 tensor")
    if sorted_rows.shape[0] != expert_outputs.shape[0]:
        raise CudaMoeValidationError("sorted_rows must match expert_outputs pair_count")
    if segment_offsets.dtype != torch.int64 or segment_offsets.ndim != 1:
        raise CudaMoeValidationError("segment_offsets must be a one-dimensional int64 tensor")
    token_count = _count("token_count", token_count)
    top_k = _count("top_k", top_k)
    valid_pairs = int(segment_offsets[-1].item())
    if valid_pairs < 0 or valid_pairs > expert_outputs.shape[0]:
        raise CudaMoeValidationError("segment_offsets final value is outside pair_count")
    if valid_pairs:
        rows = sorted_rows[:valid_pairs]
        if bool((rows < 0).any().item()) or bool((rows >= token_count).any().item()):
            raise CudaMoeValidationError("sorted rows are outside token_count")
    load_native_extension()
    return _ops.combine_topk(expert_outputs, sorted_rows, segment_offsets, token_count, top_k)


__all__ = [
    "CudaMoeUnavailableError",
    "CudaMoeValidationError",
    "combine_topk",
    "grouped_expert_mlp_inference",
    "load_native_extension",
    "permute_topk",
    "route_topk_valid",
]
