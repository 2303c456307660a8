from koemi_5hom_b200.cuda_kernels.dense.affine_scan import (
    DenseCudaBuildError,
    DenseCudaUnavailableError,
    DenseCudaValidationError,
    dense_affine_scan,
    native_cuda_available,
)

__all__ = [
    "DenseCudaBuildError",
    "DenseCudaUnavailableError",
    "DenseCudaValidationError",
    "dense_affine_scan",
    "native_cuda_available",
]
