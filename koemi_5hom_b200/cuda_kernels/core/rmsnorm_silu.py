"""Core front: fused RMSNorm + SiLU, mirroring ``koemi.cuda_kernels.core``.

Same names, signatures, dtype set, validation messages and error types as
src/koemi/cuda_kernels/core/rmsnorm_silu.py:31-100. The forward and backward
run ``koemi_core_rmsnorm_silu_forward`` / ``_backward`` (single-pass row
kernels on the current stream). ``gated_rmsnorm_silu`` and ``rms_norm`` are
the two other norm forms the HERM block and the config-3 workload use.
"""
from __future__ import annotations

import math
from typing import Any

import torch
from torch import Tensor

from koemi_5hom_b200.cuda_kernels import _ops
from koemi_5hom_b200.cuda_kernels.loader import CudaExtensionValidationError, load_cuda_extension

__all__ = ["fused_rmsnorm_silu", "gated_rmsnorm_silu", "load_core_extension", "rms_norm"]

_SUPPORTED_DTYPES = frozenset({torch.float16, torch.bfloat16, torch.float32})


def load_core_extension(*, device: torch.device | str | int | None = None, verbose: bool = False) -> Any:
    """Open the native library (the core kernels live in libkoemi_b200.so)."""
    return load_cuda_extension(device=device, verbose=verbose)


def fused_rmsnorm_silu(input_tensor: Tensor, weight: Tensor, eps: float = 1e-6) -> Tensor:
    """Apply RMSNorm and SiLU in one CUDA forward with an autograd backward."""
    _validate_inputs(input_tensor, weight, eps)
    load_core_extension(device=input_tensor.device)
    return _FusedRMSNormSiLU.apply(input_tensor, weight, float(eps))


def gated_rmsnorm_silu(input_tensor: Tensor, gate: Tensor, weight: Tensor, eps: float = 1e-6) -> Tensor:
    """Return ``silu(gate) * rmsnorm(input_tensor) * weight`` (forward only)."""
    _validate_inputs(input_tensor, weight, eps)
    if not isinstance(gate, Tensor) or gate.shape != input_tensor.shape or gate.dtype != input_tensor.dtype:
        raise CudaExtensionValidationError("gate must match input_tensor in shape and dtype")
    if gate.device != input_tensor.device or not gate.is_contiguous():
        raise CudaExtensionValidationError("gate must be a contiguous tensor on the input device")
    load_core_extension(device=input_tensor.device)
    return _ops.gated_rmsnorm_silu(input_tensor, gate, weight, float(eps))


def rms_norm(values: Tensor, weight: Tensor, eps: float = 1e-6, *, residual: Tensor | None = None,
             keep: Tensor | None = None, out_dtype: torch.dtype | None = None) -> Tensor:
    """RMSNorm of ``values (+ residual)`` times ``weight``; rows where ``keep`` is
    false return ``values`` unchanged (RootMeanSquareNorm, model/layers.py:8-16,
    with the residual/select of model/experts.py:204-205)."""
    shape = values.shape
    flat = values.reshape(-1, shape[-1])
    flat_residual = residual.reshape(-1, shape[-1]) if residual is not None else None
    flat_keep = keep.reshape(-1) if keep is not None else None
    if flat_residual is not None and flat_residual.dtype != flat.dtype:
        raise CudaExtensionValidationError("residual must match values' dtype")
    if weight.dtype != flat.dtype:
        weight = weight.to(flat.dtype)
    if flat.device.type != "cuda":
        raise CudaExtensionValidationError(f"values must be on CUDA, got {flat.device}")
    out = _ops.rms_norm(flat.contiguous(), None if flat_residual is None else flat_residual.contiguous(),
                        weight.contiguous(), flat_keep, float(eps), out_dtype or values.dtype)
    return out.reshape(shape)


class _FusedRMSNormSiLU(torch.autograd.Function):
    @staticmethod
    def forward(context: Any, input_tensor: Tensor, weight: Tensor, eps: float) -> Tensor:
        output, inverse_rms = _ops.rmsnorm_silu_forward(input_tensor, weight, eps)
        context.save_for_backward(input_tensor, weight, inverse_rms)
        context.eps = eps
        return output

    @staticmethod
    def backward(context: Any, gradient_output: Tensor) -> tuple[Tensor | None, Tensor | None, None]:
        input_tensor, weight, inverse_rms = context.saved_tensors
        gradient_input, gradient_weight = _ops.rmsnorm_silu_backward(
            gradient_output.contiguous(), input_tensor, weight, inverse_rms, context.eps
        )
        return gradient_input, gradient_weight.to(weight.dtype), None


def _validate_inputs(input_tensor: Tensor, weight: Tensor, eps: float) -> None:
    """Enforce the reference contract (core/rmsnorm_silu.py:74-100): same
    checks, order, messages and exception types, so callers see no change."""
    for name, value in (("input_tensor", input_tensor), ("weight", weight)):
        if not isinstance(value, Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
    hidden = input_tensor.shape[1] if input_tensor.ndim == 2 else None
    eps_ok = (not isinstance(eps, bool) and isinstance(eps, (float, int))
              and math.isfinite(float(eps)) and float(eps) > 0.0)
    checks = (
        (input_tensor.ndim == 2, "input_tensor must have shape [rows, hidden]"),
        (hidden != 0, "input_tensor hidden dimension must be positive"),
        (weight.ndim == 1 and weight.shape[0] == hidden,
         lambda: f"weight must have shape {(hidden,)}, got {tuple(weight.shape)}"),
        (input_tensor.dtype in _SUPPORTED_DTYPES and weight.dtype in _SUPPORTED_DTYPES,
         "input_tensor and weight must use float16, bfloat16 or float32"),
        (input_tensor.dtype == weight.dtype, "input_tensor and weight must have the same dtype"),
        (input_tensor.device == weight.device, "input_tensor and weight must use the same device"),
        (input_tensor.device.type == "cuda", lambda: f"input_tensor must be on CUDA, got {input_tensor.device}"),
        (input_tensor.is_contiguous() and weight.is_contiguous(),
         "input_tensor and weight must be contiguous"),
        (eps_ok, "eps must be a finite positive number"),
    )
    for passed, message in checks:
        if not passed:
            raise CudaExtensionValidationError(message() if callable(message) else message)
