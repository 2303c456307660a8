"""Dense front: native affine scan, mirroring ``koemi.cuda_kernels.dense``.

``dense_affine_scan(retention, increment, initial=None)`` keeps the reference
signature, broadcasting rule, dtype set {f16, bf16, f32, f64}, validation
order/messages and exception types (src/koemi/cuda_kernels/dense/affine_scan.py:33-255).
The forward is ``koemi_dense_affine_scan_forward`` with a workspace from the
caching allocator: segments of the sequence scanned by separate CTAs from
TMA-staged tiles, carries passed by decoupled look-back, fp32 state (f64 input
takes the workspace-free kernel, one CTA walking each lane group in fp64). The backward is
``koemi_dense_affine_scan_backward`` (reverse-time adjoint). There is no CPU
fallback.
"""
from __future__ import annotations

import torch
from torch import Tensor

from koemi_5hom_b200 import _native
from koemi_5hom_b200.cuda_kernels import _ops

__all__ = [
    "DenseCudaBuildError",
    "DenseCudaUnavailableError",
    "DenseCudaValidationError",
    "dense_affine_scan",
    "native_cuda_available",
]

_SUPPORTED_CUDA_DTYPES: tuple[torch.dtype, ...] = (torch.float16, torch.bfloat16, torch.float32, torch.float64)


class DenseCudaUnavailableError(RuntimeError):
    """Raised when the native dense kernel cannot run in the current process."""


class DenseCudaBuildError(DenseCudaUnavailableError):
    """Raised when the native library is missing or cannot be loaded."""


class DenseCudaValidationError(ValueError):
    """Raised when tensors violate the native dense affine-scan contract."""


def native_cuda_available() -> bool:
    """Return whether CUDA tensors and the built kernel library are available."""
    return bool(torch.cuda.is_available() and _native.LIBRARY_PATH.is_file())


def dense_affine_scan(retention: Tensor, increment: Tensor, initial: Tensor | None = None) -> Tensor:
    """Run the native affine scan h_t = retention_t * h_{t-1} + increment_t.

    ``retention`` and ``increment`` are ``[batch, sequence, ...]``; retention
    may broadcast over the state dimensions. ``initial`` is ``[batch, ...]``
    (zeros when omitted). Every tensor shares one CUDA device and dtype.
    Differentiable to first order.
    """
    _validate_inputs(retention, increment, initial)
    if not native_cuda_available():
        raise DenseCudaUnavailableError("native dense CUDA scan requires torch CUDA support, a CUDA device, and the built kernel library")
    _load_library(increment.device)
    start = initial if initial is not None else increment.new_zeros((increment.shape[0],) + tuple(increment.shape[2:]))
    return _DenseAffineScanFunction.apply(retention, increment.contiguous(), start.contiguous())


def _load_library(device: torch.device) -> None:
    try:
        _native.library()
        _native.ensure_device(device)
    except _native.KoemiNativeUnavailableError as error:
        raise DenseCudaBuildError(f"failed to load the native dense CUDA library: {error}") from error


class _DenseAffineScanFunction(torch.autograd.Function):
    @staticmethod
    def forward(context, retention: Tensor, increment: Tensor, initial: Tensor) -> Tensor:
        coefficients, broadcast = _coefficients(retention, increment)
        states = _ops.affine_scan_forward(coefficients, increment, initial, broadcast)
        context.save_for_backward(coefficients, initial, states)
        context.broadcast = broadcast
        context.retention_shape = retention.shape
        return states

    @staticmethod
    def backward(context, gradient_states: Tensor):
        coefficients, initial, states = context.saved_tensors
        grad_retention, grad_increment, grad_initial = _ops.affine_scan_backward(
            coefficients, initial, states, gradient_states.contiguous(), context.broadcast
        )
        return _sum_to(grad_retention, context.retention_shape), grad_increment, grad_initial


def _coefficients(retention: Tensor, increment: Tensor) -> tuple[Tensor, bool]:
    """Full-shape retention, or one coefficient per (batch, position)."""
    if retention.shape == increment.shape:
        return retention.contiguous(), False
    if all(size == 1 for size in retention.shape[2:]):
        return retention.reshape(retention.shape[0], retention.shape[1]).contiguous(), True
    return retention.expand_as(increment).contiguous(), False


def _sum_to(gradient: Tensor, shape: torch.Size) -> Tensor:
    """Reduce a full [batch, sequence, ...] gradient to the retention shape."""
    if gradient.shape == shape:
        return gradient
    reduced = gradient
    while reduced.ndim > len(shape):
        reduced = reduced.sum(dim=-1)
    keep = [d for d in range(2, reduced.ndim) if shape[d] == 1 and reduced.shape[d] != 1]
    if keep:
        reduced = reduced.sum(dim=keep, keepdim=True)
    if reduced.shape != shape:
        raise DenseCudaValidationError(
            f"native gradient shape {tuple(reduced.shape)} does not match {tuple(shape)}"
        )
    return reduced


def _validate_inputs(retention: Tensor, increment: Tensor, initial: Tensor | None) -> None:
    """Reference contract (dense/affine_scan.py:146-219), same order and messages."""
    named = [("retention", retention), ("increment", increment)]
    if initial is not None:
        named.append(("initial", initial))
    for name, value in named:
        if not isinstance(value, Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
    tensors = [value for _, value in named]

    def fail(message: str) -> None:
        raise DenseCudaValidationError(message)

    if retention.ndim < 2 or increment.ndim < 2:
        fail("retention and increment must have at least two dimensions")
    if retention.ndim != increment.ndim:
        fail("retention and increment must have the same rank")
    if retention.shape[:2] != increment.shape[:2]:
        fail("retention and increment must have the same batch and sequence dimensions")
    try:
        broadcast_ok = torch.broadcast_shapes(retention.shape, increment.shape) == increment.shape
    except RuntimeError:
        broadcast_ok = False
    if not broadcast_ok:
        fail("retention must broadcast to increment's shape")
    dtypes = {value.dtype for value in tensors}
    unsupported = sorted(str(dtype) for dtype in dtypes if dtype not in _SUPPORTED_CUDA_DTYPES)
    if unsupported:
        fail(f"unsupported CUDA dtype(s): {', '.join(unsupported)}")
    if len(dtypes) != 1:
        fail("retention, increment and initial must have the same dtype")
    if initial is not None:
        expected = (increment.shape[0],) + tuple(increment.shape[2:])
        if initial.shape != expected:
            fail(f"initial must have shape {expected}, got {tuple(initial.shape)}")
    if not torch.cuda.is_available():
        raise DenseCudaUnavailableError("native dense CUDA scan is unavailable: torch.cuda.is_available() is False")
    off_device = [str(value.device) for value in tensors if value.device.type != "cuda"]
    if off_device:
        fail(f"all dense scan tensors must be on CUDA; found {', '.join(off_device)}")
    devices = {value.device for value in tensors}
    if len(devices) != 1:
        fail(f"all dense scan tensors must use one CUDA device; found {', '.join(sorted(map(str, devices)))}")
