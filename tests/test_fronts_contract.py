"""Front contracts on a host without CUDA: typed errors, never a CPU fallback.

Mirrors the reference's contract tests (tests/cuda/test_core_cuda.py:21-52,
test_dense_cuda.py:36-65, test_moe_cuda.py:23-42, test_think_cuda.py:35-69).
"""
from __future__ import annotations

import pytest
import torch

from koemi_5hom_b200.cuda_kernels import core, dense, moe, think
from koemi_5hom_b200.cuda_kernels.loader import CudaExtensionValidationError, detect_cuda_toolchain

cpu_only = pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-CUDA contract")


def test_core_rejects_cpu_and_bad_shapes():
    with pytest.raises(CudaExtensionValidationError, match="must be on CUDA"):
        core.fused_rmsnorm_silu(torch.ones(2, 4), torch.ones(4))
    with pytest.raises(CudaExtensionValidationError, match=r"weight must have shape \(4,\)"):
        core.fused_rmsnorm_silu(torch.ones(2, 4), torch.ones(5))
    with pytest.raises(CudaExtensionValidationError, match="float16, bfloat16 or float32"):
        core.fused_rmsnorm_silu(torch.ones(2, 4, dtype=torch.float64), torch.ones(4, dtype=torch.float64))
    with pytest.raises(CudaExtensionValidationError, match="same dtype"):
        core.fused_rmsnorm_silu(torch.ones(2, 4), torch.ones(4, dtype=torch.float16))
    with pytest.raises(CudaExtensionValidationError, match="must be on CUDA"):  # device is checked before eps
        core.fused_rmsnorm_silu(torch.ones(2, 4), torch.ones(4), eps=0.0)
    with pytest.raises(TypeError):
        core.fused_rmsnorm_silu([1.0], torch.ones(4))


def test_dense_validation_messages():
    a = torch.rand(2, 3, 4)
    with pytest.raises(dense.DenseCudaValidationError, match="at least two dimensions"):
        dense.dense_affine_scan(torch.rand(3), torch.rand(3))
    with pytest.raises(dense.DenseCudaValidationError, match="same rank"):
        dense.dense_affine_scan(torch.rand(2, 3), a)
    with pytest.raises(dense.DenseCudaValidationError, match="broadcast"):
        dense.dense_affine_scan(torch.rand(2, 3, 2), a)
    with pytest.raises(dense.DenseCudaValidationError, match="unsupported CUDA dtype"):
        dense.dense_affine_scan(a.int(), a.int())
    with pytest.raises(dense.DenseCudaValidationError, match="initial must have shape"):
        dense.dense_affine_scan(a, a, torch.rand(2, 5))


@cpu_only
def test_dense_reports_unavailable_without_cuda():
    a = torch.rand(2, 3, 4)
    with pytest.raises(dense.DenseCudaUnavailableError, match="torch.cuda.is_available"):
        dense.dense_affine_scan(a, a)
    assert not dense.native_cuda_available()


def test_think_validation_messages():
    prior = torch.rand(2, 3, 8)
    w, b = torch.rand(10, 8), torch.rand(10)
    t = torch.zeros(2, 3, dtype=torch.long)
    v = torch.ones(2, 3, dtype=torch.bool)
    with pytest.raises(think.CudaThinkValidationError, match=r"\[batch, sequence, width\]"):
        think.causal_surprise(prior[0], w, b, t, v)
    with pytest.raises(think.CudaThinkValidationError, match="torch.int64"):
        think.causal_surprise(prior, w, b, t.int(), v)
    with pytest.raises(think.CudaThinkValidationError, match="at most 4096"):
        think.causal_surprise(torch.rand(1, 1, 4097), torch.rand(2, 4097), torch.rand(2), t[:1, :1], v[:1, :1])
    with pytest.raises(think.CudaThinkValidationError, match="share a dtype"):
        think.causal_surprise(prior, w.half(), b, t, v)


@cpu_only
def test_think_reports_unavailable_without_cuda():
    with pytest.raises(think.CudaThinkUnavailableError, match="torch.cuda.is_available"):
        think.causal_surprise(torch.rand(2, 3, 8), torch.rand(10, 8), torch.rand(10),
                              torch.zeros(2, 3, dtype=torch.long), torch.ones(2, 3, dtype=torch.bool))


def test_moe_rejects_cpu_without_fallback():
    ids = torch.tensor([[1, 2]])
    with pytest.raises(moe.CudaMoeValidationError, match="must be a CUDA tensor"):
        moe.route_topk_valid(ids, ids, torch.ones_like(ids, dtype=torch.bool), expert_count=4, top_k=2)
    with pytest.raises(moe.CudaMoeValidationError, match="must be a CUDA tensor"):
        moe.permute_topk(torch.ones(2, 4), torch.tensor([[0, 1], [1, 0]]), torch.ones(2, dtype=torch.bool),
                         expert_count=2)


@cpu_only
def test_moe_load_reports_unavailable_without_cuda():
    with pytest.raises(moe.CudaMoeUnavailableError, match="torch.cuda.is_available"):
        moe.load_native_extension()


def test_toolchain_status_reports_library():
    status = detect_cuda_toolchain()
    assert status.library_present
    assert status.library_path.name == "libkoemi_b200.so"
