"""ctypes binding of ``lib/libkoemi_b200.so`` (declared in ``include/koemi_b200.h``).

Every entry point is bound with explicit argument types. Loading the library
needs no GPU: the status and ABI functions can be called on any host, which is
what the CPU tests use. Compute calls must go to CUDA tensors; this module
never falls back to a host implementation.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIBRARY_PATH = Path(__file__).resolve().parent / "lib" / "libkoemi_b200.so"
ABI_VERSION = 1

KOEMI_OK = 0
KOEMI_ERR_INVALID = -1
KOEMI_ERR_CUDA = -2
KOEMI_ERR_UNSUPPORTED = -3
KOEMI_ERR_TIMEOUT = -4
KOEMI_ERR_WORKSPACE = -5

F32, F16, BF16, F64, I32, I64, BOOL = range(7)

DTYPE_CODES = {
    torch.float32: F32,
    torch.float16: F16,
    torch.bfloat16: BF16,
    torch.float64: F64,
    torch.int32: I32,
    torch.int64: I64,
    torch.bool: BOOL,
}

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/koemi_b200.h.
SIGNATURES: dict[str, tuple[object, tuple[object, ...]]] = {
    "koemi_abi_version": (_int, ()),
    "koemi_last_error": (_sz, (ctypes.c_char_p, _sz)),
    "koemi_device_status": (_int, (_int, ctypes.POINTER(_int))),
    "koemi_device_init": (_int, (_int,)),
    "koemi_sampler_greedy": (_int, (_p, _i64, _i64, _i64, _i64, _p, _p)),
    "koemi_sampler_temperature": (_int, (_p, _i64, _i64, _i64, _i64, _f, ctypes.c_uint64, _i64, _p, _p, _p, _p)),
    "koemi_assoc_window_scan_read": (_int, (_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _p)),
    "koemi_dense_affine_scan_workspace": (_sz, (_i64, _i64, _i64, _int)),
    "koemi_dense_affine_scan_forward": (_int, (_p, _p, _p, _p, _i64, _i64, _i64, _int, _int, _p, _sz, _p)),
    "koemi_dense_affine_scan_backward": (
        _int, (_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _int, _p)),
    "koemi_dense_bounded_gates": (_int, (_p, _p, _p, _p, _i64, _i64, _f, _f, _p)),
    "koemi_dense_decode_step": (_int, (_p, _p, _p, _p, _p, _i64, _p, _i64, _i64, _f, _f, _int, _p)),
    "koemi_think_surprise_backward_workspace": (_sz, (_i64,)),
    "koemi_think_causal_surprise_backward": (
        _int, (_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p, _sz, _p)),
    "koemi_think_head_pass_slices": (_i64, (_i64,)),
    "koemi_think_head_pass": (_int, (_p, _i64, _i64, _i64, _p, _p, _i64, _i64, _p, _p, _int, _p)),
    "koemi_think_surprise_from_partials": (
        _int, (_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _int, _p, _p)),
    "koemi_think_ring_decode_step": (
        _int, (_p, _i64, _p, _i64, _p, _p, _f, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _p, _p, _i64,
               _i64, _i64, _i64, _int, _int, _p)),
    "koemi_assoc_decode_step": (_int, (_p, _i64, _p, _p, _p, _int, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _int,
                                       _p)),
    "koemi_dense_projection_workspace": (_sz, (_i64, _i64, _i64, _int)),
    "koemi_dense_projection": (_int, (_p, _i64, _p, _p, _p, _i64, _i64, _i64, _i64, _int, _p, _sz, _p)),
    "koemi_dense_projection_resident": (_int, (_p, _i64, _p, _p, _p, _i64, _i64, _i64, _i64, _int, _p, _sz, _p)),
    "koemi_grouped_projection": (_int, (_p, _p, _p, _i64, _i64, _i64, _i64, _int, _p)),
    "koemi_window_pack_rows": (_int, (_p, _p, _p, _int, _i64, _p, _i64, _int, _p)),
    "koemi_window_slot_operands": (_int, (_p, _p, _i64, _i64, _p, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _int, _p)),
    "koemi_core_rmsnorm_silu_forward": (_int, (_p, _p, _p, _p, _i64, _i64, _f, _int, _p)),
    "koemi_core_rmsnorm_silu_backward_workspace": (_sz, (_i64, _i64)),
    "koemi_core_rmsnorm_silu_backward": (
        _int, (_p, _p, _p, _p, _p, _p, _i64, _i64, _p, _sz, _int, _p)),
    "koemi_core_gated_rmsnorm_silu_forward": (_int, (_p, _p, _p, _p, _p, _i64, _i64, _f, _int, _p)),
    "koemi_core_rmsnorm_forward": (_int, (_p, _p, _p, _p, _p, _i64, _i64, _f, _int, _int, _p)),
    "koemi_think_surprise_workspace": (_sz, (_i64, _i64, _i64, _int)),
    "koemi_think_causal_surprise_forward": (
        _int, (_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _int, _p, _sz, _p)),
    "koemi_think_salient_admission": (
        _int, (_p, _p, _p, _p, _p, _p, _p, _f, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p)),
    "koemi_moe_route_topk": (_int, (_p, _p, _p, _p, _i64, _i64, _i64, _int, _p)),
    "koemi_moe_learned_topk": (_int, (_p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p)),
    "koemi_moe_permute_workspace": (_sz, (_i64, _i64, _i64)),
    "koemi_moe_permute_topk": (
        _int, (_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _int, _int, _p, _sz, _p)),
    "koemi_moe_permute_topk_static": (
        _int, (_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _int, _int, _p)),
    "koemi_moe_grouped_mlp_workspace": (_sz, (_i64, _i64, _i64, _i64, _int)),
    "koemi_moe_grouped_expert_mlp": (
        _int, (_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _int, _p, _sz, _p)),
    "koemi_moe_combine_workspace": (_sz, (_i64, _i64, _i64)),
    "koemi_moe_combine_topk": (
        _int, (_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _int, _p, _sz, _p)),
    "koemi_moe_ep_pack": (_int, (_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _int, _p)),
    "koemi_moe_ep_unpack": (_int, (_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _int, _p)),
    "koemi_moe_combine_residual_rmsnorm_next": (
        _int, (_p, _p, _p, _p, _p, _p, _p, _p, _p, _int, _i64, _i64, _i64, _i64, _f, _int, _p)),
    "koemi_moe_tile_prefix": (_int, (_p, _i64, _p, _p)),
    "koemi_moe_grouped_expert_mlp_mapped": (_int, (_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _int,
                                                   _p, _sz, _p)),
    "koemi_moe_norm_gather": (_int, (_p, _p, _f, _p, _p, _p, _i64, _p, _int, _i64, _i64, _i64, _p)),
    "koemi_moe_gather_rows": (_int, (_p, _int, _p, _p, _i64, _p, _int, _i64, _i64, _p)),
    "koemi_peer_exchange_bytes": (_sz, (_i64, _i64, _i64, _int)),
    "koemi_peer_exchange_offsets": (_int, (_i64, _i64, _i64, _int, _p, _p)),
    "koemi_peer_buffer_alloc": (_int, (_sz, _p, _p)),
    "koemi_peer_buffer_open": (_int, (_p, _p)),
    "koemi_peer_buffer_close": (_int, (_p,)),
    "koemi_peer_buffer_free": (_int, (_p,)),
    "koemi_ep_dispatch": (_int, (_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _int, _p)),
    "koemi_ep_dispatch_gather": (
        _int, (_p, _int, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _int, _p)),
    "koemi_ep_norm_dispatch": (_int, (_p, _p, _f, _p, _p, _p, _p, _i64, _i64, _p, _p, _i64, _i64, _i64, _i64, _i64,
                                      _int, _p)),
    "koemi_ep_owner_sort": (_int, (_p, _p, _i64, _i64, _i64, _i64, _i64, _int, _p, _p, _p, _p, _p, _p, _p)),
    "koemi_ep_expert_mlp_return": (_int, (_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _int, _p,
                                          _sz, _p, _p, _i64, _i64, _i64, _p)),
    "koemi_ep_combine_residual_rmsnorm_next": (_int, (_p, _p, _p, _p, _p, _p, _p, _p, _int, _i64, _i64, _i64, _i64,
                                                      _f, _int, _p, _i64, _i64, _i64, _p)),
    "koemi_ep_wait_dispatch": (_int, (_p, _i64, _p)),
    "koemi_ep_return": (_int, (_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _int, _p)),
    "koemi_ep_collect": (_int, (_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _int, _p)),
    "koemi_moe_combine_residual_rmsnorm": (
        _int, (_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _f, _int, _p)),
}


class KoemiNativeUnavailableError(RuntimeError):
    """Raised when libkoemi_b200.so is missing, stale or cannot be loaded."""


class KoemiNativeError(RuntimeError):
    """Raised when a native entry point returns a nonzero status."""

    def __init__(self, function: str, status: int, message: str) -> None:
        super().__init__(f"{function} failed with status {status}: {message}")
        self.function = function
        self.status = status


_LOCK = threading.RLock()
_LIBRARY: ctypes.CDLL | None = None
_INITIALISED_DEVICES: set[int] = set()


def library() -> ctypes.CDLL:
    """Load (once) and return the kernel library with bound signatures."""
    global _LIBRARY
    if _LIBRARY is not None:
        return _LIBRARY
    with _LOCK:
        if _LIBRARY is not None:
            return _LIBRARY
        override = os.environ.get("KOEMI_B200_LIBRARY")
        path = Path(override) if override else LIBRARY_PATH
        if not path.is_file():
            raise KoemiNativeUnavailableError(
                f"{path} is missing; build it with `python -m koemi_5hom_b200.build`"
            )
        try:
            handle = ctypes.CDLL(str(path))
        except OSError as error:
            raise KoemiNativeUnavailableError(f"cannot load {path}: {error}") from error
        for name, (restype, argtypes) in SIGNATURES.items():
            try:
                function = getattr(handle, name)
            except AttributeError as error:
                raise KoemiNativeUnavailableError(f"{path} does not export {name}") from error
            function.restype = restype
            function.argtypes = list(argtypes)
        version = handle.koemi_abi_version()
        if version != ABI_VERSION:
            raise KoemiNativeUnavailableError(
                f"{path} reports ABI version {version}, expected {ABI_VERSION}"
            )
        _LIBRARY = handle
    return _LIBRARY


def last_error() -> str:
    lib = library()
    size = lib.koemi_last_error(None, 0)
    buffer = ctypes.create_string_buffer(size + 1)
    lib.koemi_last_error(buffer, size + 1)
    return buffer.value.decode("utf-8", errors="replace")


def check(function: str, status: int) -> None:
    if status != KOEMI_OK:
        raise KoemiNativeError(function, status, last_error())


def call(function: str, *arguments) -> None:
    """Call a status-returning entry point and raise on a nonzero status."""
    check(function, getattr(library(), function)(*arguments))


def ensure_device(device: torch.device) -> None:
    """Initialise the per-device state once, outside any graph capture."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    if index in _INITIALISED_DEVICES:
        return
    handle = library()  # takes _LOCK itself on the first load
    with _LOCK:
        if index not in _INITIALISED_DEVICES:
            check("koemi_device_init", handle.koemi_device_init(index))
            _INITIALISED_DEVICES.add(index)


def device_status(device: torch.device) -> int:
    index = device.index if device.index is not None else torch.cuda.current_device()
    value = ctypes.c_int(0)
    check("koemi_device_status", library().koemi_device_status(index, ctypes.byref(value)))
    return value.value


def raise_for_device_status(device: torch.device) -> None:
    """Read (and clear) the device status word; raise if a bounded
    device-side wait gave up since the last read. Synchronises the device."""
    status = device_status(device)
    if status != KOEMI_OK:
        raise KoemiNativeError("device status", status,
                               "a bounded device-side wait gave up (a peer or producer never signalled)")


def stream_of(tensor: torch.Tensor) -> int:
    """Raw handle of the current stream of ``tensor``'s device."""
    return torch.cuda.current_stream(tensor.device).cuda_stream


def ptr(tensor: torch.Tensor | None) -> int | None:
    return None if tensor is None else tensor.data_ptr()


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return DTYPE_CODES[dtype]
    except KeyError as error:
        raise ValueError(f"dtype {dtype} has no native code") from error


def workspace(size: int, device: torch.device) -> torch.Tensor:
    """Caller-owned scratch from torch's caching allocator (at least 256 bytes)."""
    return torch.empty(max(int(size), 256), dtype=torch.uint8, device=device)


def exported_symbols() -> list[str]:
    return list(SIGNATURES)
