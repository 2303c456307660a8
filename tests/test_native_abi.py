"""libkoemi_b200.so loads on any host and exports every symbol of include/koemi_b200.h."""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from koemi_5hom_b200 import _native

HEADER = Path(__file__).resolve().parent.parent / "include" / "koemi_b200.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"KOEMI_API\s+\w+\s+(koemi_\w+)\s*\(", text)))


def test_header_and_binding_table_agree():
    assert declared_symbols() == sorted(_native.SIGNATURES)


def test_library_loads_and_reports_abi():
    lib = _native.library()
    assert lib.koemi_abi_version() == _native.ABI_VERSION == 1


def test_library_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", str(_native.LIBRARY_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (koemi_\w+)", out))
    missing = set(declared_symbols()) - exported
    assert not missing, missing
    # nothing but the C ABI leaks out of the library
    assert all(name.startswith("koemi_") for name in exported)


def test_invalid_arguments_fail_before_touching_the_device():
    lib = _native.library()
    status = lib.koemi_moe_route_topk(None, None, None, None, 4, 0, 1, _native.I64, None)
    assert status == _native.KOEMI_ERR_INVALID
    assert "expert_count" in _native.last_error()
    status = lib.koemi_core_rmsnorm_silu_forward(None, None, None, None, 4, 8, -1.0, _native.F32, None)
    assert status == _native.KOEMI_ERR_INVALID
    assert "eps" in _native.last_error()
    status = lib.koemi_dense_affine_scan_forward(None, None, None, None, 1, 4, 8, 0, 99, None, 0, None)
    assert status == _native.KOEMI_ERR_INVALID
    with pytest.raises(_native.KoemiNativeError, match="status -1"):
        _native.call("koemi_moe_learned_topk", None, None, None, None, None, 3, 4, 9, 0, None)


def test_empty_work_is_a_no_op():
    lib = _native.library()
    assert lib.koemi_dense_affine_scan_forward(None, None, None, None, 0, 5, 8, 0, _native.F32, None, 0, None) == 0
    assert lib.koemi_moe_route_topk(None, None, None, None, 0, 4, 2, _native.I64, None) == 0


def test_workspace_queries_are_host_only():
    lib = _native.library()
    assert lib.koemi_moe_permute_workspace(131072, 2, 64) >= 4 * 131072 * 2 * 4
    assert lib.koemi_think_surprise_workspace(256, 2048, 32767, _native.BF16) > 0
    assert lib.koemi_moe_grouped_mlp_workspace(512, 2048, 4096, 64, _native.BF16) > 0


def test_scan_workspace_query():
    lib = _native.library()
    # bf16: tiles of 128 positions x 64 features, 768 B of records each after a 256 B head
    assert lib.koemi_dense_affine_scan_workspace(8, 4096, 1024, _native.BF16) == 256 + 8 * 16 * 32 * 768
    # fp32 tiles are 64 positions long
    assert lib.koemi_dense_affine_scan_workspace(8, 4096, 1024, _native.F32) == 256 + 8 * 16 * 64 * 768
    # decode steps (length <= 8) and fp64 take the workspace-free kernels
    assert lib.koemi_dense_affine_scan_workspace(256, 1, 2048, _native.BF16) == 0
    assert lib.koemi_dense_affine_scan_workspace(8, 4096, 1024, _native.F64) == 0


def test_sampler_and_window_memory_reject_bad_arguments_on_the_host():
    lib = _native.library()
    assert lib.koemi_sampler_greedy(None, 4, 0, 0, 256, None, None) == _native.KOEMI_ERR_INVALID
    assert lib.koemi_sampler_greedy(None, 0, 10, 10, 256, None, None) == _native.KOEMI_OK  # no rows
    status = lib.koemi_assoc_window_scan_read(None, None, None, None, None, None, None, None, 2, 5, 64, 12, None)
    assert status == _native.KOEMI_ERR_UNSUPPORTED  # the model pads 12 features to 16 before calling
    assert "4, 8, 16 or 32 memory features" in _native.last_error()


def test_last_error_is_truncated_safely():
    lib = _native.library()
    lib.koemi_moe_route_topk(None, None, None, None, 4, 0, 1, _native.I64, None)
    buffer = ctypes.create_string_buffer(8)
    full = lib.koemi_last_error(buffer, 8)
    assert full > 7 and len(buffer.value) == 7


def test_device_init_path_loads_library_without_deadlock(monkeypatch):
    """ensure_device() as the first call into the library (the model's path)
    must not self-deadlock on the loader lock."""
    import threading

    monkeypatch.setattr(_native, "_LIBRARY", None)
    monkeypatch.setattr(_native, "_INITIALISED_DEVICES", set())
    calls = []

    class FakeDevice:
        index = 0

    def run():
        try:
            _native.ensure_device(FakeDevice())
        except _native.KoemiNativeError as error:  # no GPU here: init reports a CUDA error
            calls.append(error)
        else:
            calls.append(None)

    worker = threading.Thread(target=run, daemon=True)
    worker.start()
    worker.join(timeout=30)
    assert not worker.is_alive(), "ensure_device deadlocked"
    assert calls


def test_window_operand_builders_reject_bad_arguments_on_the_host():
    lib = _native.library()
    assert lib.koemi_window_pack_rows(None, None, None, 0, 4, None, 8, _native.BF16, None) == _native.KOEMI_ERR_INVALID
    assert "1 to 8 parts" in _native.last_error()
    status = lib.koemi_window_slot_operands(None, None, 0, 3, None, None, 0, 4, 2, 64, 12, None, None, _native.BF16,
                                            None)
    assert status == _native.KOEMI_ERR_INVALID
    assert "multiple of 8" in _native.last_error()
