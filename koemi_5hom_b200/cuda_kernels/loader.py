"""Native-library status and ABI contract, mirroring ``koemi.cuda_kernels.loader``.

The reference JIT-compiles one extension per front with
``torch.utils.cpp_extension.load`` (src/koemi/cuda_kernels/loader.py:170-221)
and checks ``KOEMI_CUDA_ABI_VERSION`` on it. Here every front lives in one
prebuilt sm_100a library, ``libkoemi_b200.so``; "loading an extension" means
opening that library, checking its ABI version and initialising the device.
No compiler runs at first call.
"""
from __future__ import annotations

import shutil
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch

from koemi_5hom_b200 import _native

__all__ = [
    "CUDA_EXTENSION_ABI_VERSION",
    "CudaExtensionLoadError",
    "CudaExtensionUnavailableError",
    "CudaExtensionValidationError",
    "CudaToolchainStatus",
    "cuda_extension_available",
    "detect_cuda_toolchain",
    "load_cuda_extension",
]

CUDA_EXTENSION_ABI_VERSION = _native.ABI_VERSION


class CudaExtensionUnavailableError(RuntimeError):
    """Raised when the local CUDA runtime cannot run the native library."""


class CudaExtensionValidationError(ValueError):
    """Raised when a call violates a native operator contract."""


class CudaExtensionLoadError(RuntimeError):
    """Raised when the native library is missing or reports a wrong ABI."""


@dataclass(frozen=True)
class CudaToolchainStatus:
    """Snapshot of the CUDA runtime and the prebuilt native library."""

    runtime_available: bool
    torch_cuda_version: str | None
    library_path: Path
    library_present: bool
    nvcc_path: Path | None
    reason: str

    @property
    def ready(self) -> bool:
        return self.runtime_available and self.library_present


def detect_cuda_toolchain() -> CudaToolchainStatus:
    """Inspect the CUDA runtime and whether ``libkoemi_b200.so`` is built."""
    runtime = bool(torch.cuda.is_available())
    path = _native.LIBRARY_PATH
    nvcc = shutil.which("nvcc")
    missing = []
    if not runtime:
        missing.append("torch.cuda.is_available() is False")
    if not path.is_file():
        missing.append(f"{path.name} is not built")
    return CudaToolchainStatus(
        runtime_available=runtime,
        torch_cuda_version=torch.version.cuda,
        library_path=path,
        library_present=path.is_file(),
        nvcc_path=Path(nvcc) if nvcc else None,
        reason="; ".join(missing) if missing else "ready",
    )


def cuda_extension_available() -> bool:
    return detect_cuda_toolchain().ready


def load_cuda_extension(*, device: torch.device | str | int | None = None, verbose: bool = False) -> Any:
    """Open the native library for ``device`` and return the ctypes handle.

    Raises :class:`CudaExtensionUnavailableError` without a CUDA runtime and
    :class:`CudaExtensionLoadError` when the library is missing or stale.
    """
    if not torch.cuda.is_available():
        raise CudaExtensionUnavailableError(
            "native CUDA kernels are unavailable: torch.cuda.is_available() is False"
        )
    try:
        handle = _native.library()
    except _native.KoemiNativeUnavailableError as error:
        raise CudaExtensionLoadError(str(error)) from error
    resolved = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if resolved.type == "cuda":
        _native.ensure_device(resolved)
    if verbose:
        print(f"koemi_b200: loaded {_native.LIBRARY_PATH} (ABI {CUDA_EXTENSION_ABI_VERSION})")
    return handle
