from koemi_5hom_b200.cuda_kernels.core.rmsnorm_silu import (
    fused_rmsnorm_silu,
    gated_rmsnorm_silu,
    load_core_extension,
    rms_norm,
)

__all__ = ["fused_rmsnorm_silu", "gated_rmsnorm_silu", "load_core_extension", "rms_norm"]
