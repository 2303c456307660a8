"""Think front: causal surprise, mirroring ``koemi.cuda_kernels.think``.

``causal_surprise`` keeps the reference signature, output dtype, limits and
validation contract (src/koemi/cuda_kernels/think/surprise.py:91-251). The
forward is ``koemi_think_causal_surprise_forward``: the head contraction and
the log-sum-exp/NLL reduction run fused, so the ``[rows, content_vocab]``
logits are never written to memory. The backward is
``koemi_think_causal_surprise_backward``: the logits recomputed tile by tile
(tcgen05 for 16-bit inputs) and turned into dlogits in the same kernel; the
three contractions with dlogits are fp32 library GEMMs, as in the reference.
``salient_admission`` exposes the admission + ring compaction kernel the HERM
block uses after the surprise.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from time import perf_counter

import torch
from torch import Tensor

from koemi_5hom_b200 import _native
from koemi_5hom_b200.cuda_kernels import _ops

__all__ = [
    "CudaThinkBenchmark",
    "CudaThinkUnavailableError",
    "CudaThinkValidationError",
    "benchmark_causal_surprise",
    "causal_surprise",
    "salient_admission",
]

_SUPPORTED_DTYPES: tuple[torch.dtype, ...] = (torch.float16, torch.bfloat16, torch.float32)


class CudaThinkUnavailableError(RuntimeError):
    """Raised when the native think kernel cannot run without CUDA."""


class CudaThinkValidationError(ValueError):
    """Raised when the causal-surprise tensors violate the native kernel contract."""


@dataclass(frozen=True)
class CudaThinkBenchmark:
    """Synchronized native-kernel timing for one causal-surprise shape."""

    elapsed_seconds: float
    latency_milliseconds: float
    positions_per_second: float
    position_count: int
    warmup_iterations: int
    measured_iterations: int


def causal_surprise(prior_states: Tensor, content_weight: Tensor, content_bias: Tensor, target_ids: Tensor,
                    valid_mask: Tensor, *, validate_targets: bool = True) -> Tensor:
    """Normalised causal surprise ``1 - exp(-NLL / ln C)`` per position.

    Shapes: ``[batch, sequence, width]``, ``[content_vocab, width]``,
    ``[content_vocab]``, ``[batch, sequence]`` (int64) and ``[batch, sequence]``
    (bool). ``prior_states[:, t]`` is the state before position ``t``; invalid
    positions return zero and get no gradient. ``validate_targets=False``
    skips the host-side range check for already checked ids.
    """
    _validate_inputs(prior_states, content_weight, content_bias, target_ids, valid_mask, validate_targets)
    if prior_states.shape[1] == 0:
        return prior_states.sum(dim=-1)[:, :0]
    _load(prior_states.device)
    return _CausalSurpriseFunction.apply(prior_states, content_weight, content_bias, target_ids, valid_mask)


def benchmark_causal_surprise(prior_states: Tensor, content_weight: Tensor, content_bias: Tensor,
                              target_ids: Tensor, valid_mask: Tensor, *, warmup_iterations: int = 10,
                              measured_iterations: int = 50, validate_targets: bool = True) -> CudaThinkBenchmark:
    """Measure synchronized native forward latency and positions per second."""
    if isinstance(warmup_iterations, bool) or not isinstance(warmup_iterations, int) or warmup_iterations < 0:
        raise CudaThinkValidationError("warmup_iterations must be a non-negative integer")
    if isinstance(measured_iterations, bool) or not isinstance(measured_iterations, int) or measured_iterations <= 0:
        raise CudaThinkValidationError("measured_iterations must be a positive integer")
    _validate_inputs(prior_states, content_weight, content_bias, target_ids, valid_mask, validate_targets)
    arguments = (prior_states, content_weight, content_bias, target_ids, valid_mask)
    with torch.no_grad():
        for _ in range(warmup_iterations):
            causal_surprise(*arguments, validate_targets=False)
        torch.cuda.synchronize(prior_states.device)
        started = perf_counter()
        for _ in range(measured_iterations):
            causal_surprise(*arguments, validate_targets=False)
        torch.cuda.synchronize(prior_states.device)
        elapsed = perf_counter() - started
    positions = prior_states.shape[0] * prior_states.shape[1]
    mean = elapsed / measured_iterations
    return CudaThinkBenchmark(
        elapsed_seconds=elapsed,
        latency_milliseconds=mean * 1000.0,
        positions_per_second=positions / mean if mean > 0.0 else math.inf,
        position_count=positions,
        warmup_iterations=warmup_iterations,
        measured_iterations=measured_iterations,
    )


def salient_admission(carried_keys: Tensor, carried_values: Tensor, carried_valid: Tensor, keys: Tensor,
                      values: Tensor, surprise: Tensor, valid_mask: Tensor, threshold: float,
                      capacity: int) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """Admit ``valid & (surprise > threshold)`` and keep the latest ``capacity``
    admitted entries of ``[carried ; window]`` (network.py:349,
    memory.py:431-455). Returns (keys, values, valid, admission)."""
    for name, value in (("keys", keys), ("values", values), ("carried_keys", carried_keys)):
        if value.dtype != torch.float32 or value.device.type != "cuda":
            raise CudaThinkValidationError(f"{name} must be a float32 CUDA tensor")
    return _ops.salient_admission(
        carried_keys.contiguous(), carried_values.contiguous(), carried_valid.contiguous(), keys.contiguous(),
        values.contiguous(), surprise.float().contiguous(), valid_mask.contiguous(), float(threshold), int(capacity)
    )


def _load(device: torch.device) -> None:
    try:
        _native.library()
        _native.ensure_device(device)
    except _native.KoemiNativeUnavailableError as error:
        raise CudaThinkUnavailableError(str(error)) from error


class _CausalSurpriseFunction(torch.autograd.Function):
    @staticmethod
    def forward(context, prior_states, content_weight, content_bias, target_ids, valid_mask):
        inputs = tuple(t.contiguous() for t in (prior_states, content_weight, content_bias, target_ids, valid_mask))
        surprise, nll = _ops.causal_surprise_forward_nll(*inputs, prior_states.dtype)
        context.save_for_backward(*inputs, nll)
        return surprise

    @staticmethod
    def backward(context, gradient):
        """The native kernel forms dlogits = dL/dNLL (softmax - onehot) from
        recomputed logits (never stored); the three contractions run in fp32
        as the reference's (think/surprise_kernel.cu:248-251)."""
        prior, weight, bias, targets, valid, nll = context.saved_tensors
        width = prior.shape[-1]
        dlogits = _ops.causal_surprise_dlogits(prior, weight, bias, targets, valid,
                                               gradient.to(prior.dtype).contiguous(), nll)
        rows = prior.reshape(-1, width).float()
        grad_prior = (dlogits @ weight.float()).reshape(prior.shape)
        grad_weight = dlogits.T @ rows
        grad_bias = dlogits.sum(dim=0)
        return grad_prior.to(prior.dtype), grad_weight.to(weight.dtype), grad_bias.to(bias.dtype), None, None


def _validate_inputs(prior_states, content_weight, content_bias, target_ids, valid_mask, validate_targets) -> int:
    """Reference contract (think/surprise.py:190-251), same order and messages."""
    named = {
        "prior_states": prior_states,
        "content_weight": content_weight,
        "content_bias": content_bias,
        "target_ids": target_ids,
        "valid_mask": valid_mask,
    }
    for name, value in named.items():
        if not isinstance(value, Tensor):
            raise CudaThinkValidationError(f"{name} must be a torch.Tensor")
    structural = (
        (prior_states.ndim == 3, "prior_states must have shape [batch, sequence, width]"),
        (content_weight.ndim == 2, "content_weight must have shape [content_vocab, width]"),
        (content_bias.ndim == 1, "content_bias must have shape [content_vocab]"),
    )
    for passed, message in structural:
        if not passed:
            raise CudaThinkValidationError(message)
    sequence_shape = prior_states.shape[:2]
    batch, _, width = prior_states.shape
    vocab = content_weight.shape[0]
    contract = (
        (target_ids.shape == sequence_shape and valid_mask.shape == sequence_shape,
         "target_ids and valid_mask must match [batch, sequence]"),
        (content_weight.shape[1] == width and content_bias.shape[0] == vocab,
         "content head dimensions must match prior_states width"),
        (batch >= 1 and vocab >= 2 and width >= 1, "batch, content_vocab and width must be positive"),
        (width <= 4096, "width must be at most 4096 for the shared-memory backward kernel"),
        (prior_states.dtype in _SUPPORTED_DTYPES, "prior_states dtype must be float16, bfloat16 or float32"),
        (content_weight.dtype == prior_states.dtype and content_bias.dtype == prior_states.dtype,
         "prior_states, content_weight and content_bias must share a dtype"),
        (target_ids.dtype == torch.long, "target_ids must use torch.int64"),
        (valid_mask.dtype == torch.bool, "valid_mask must use torch.bool"),
        (isinstance(validate_targets, bool), "validate_targets must be a boolean"),
    )
    for passed, message in contract:
        if not passed:
            raise CudaThinkValidationError(message)
    if not torch.cuda.is_available():
        raise CudaThinkUnavailableError("native think CUDA kernel is unavailable: torch.cuda.is_available() is False")
    off_device = [str(t.device) for t in named.values() if t.device.type != "cuda"]
    if off_device:
        raise CudaThinkValidationError(f"all think tensors must be on CUDA; found {', '.join(off_device)}")
    devices = {t.device for t in named.values()}
    if len(devices) != 1:
        raise CudaThinkValidationError(
            f"all think tensors must use one CUDA device; found {', '.join(sorted(map(str, devices)))}"
        )
    if validate_targets and target_ids.numel() > 0:
        low, high = int(target_ids.amin().item()), int(target_ids.amax().item())
        if low < 0 or high >= vocab:
            raise CudaThinkValidationError(f"target_ids must be in [0, {vocab}); found [{low}, {high}]")
    return vocab
