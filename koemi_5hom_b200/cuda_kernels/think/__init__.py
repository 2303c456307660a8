from koemi_5hom_b200.cuda_kernels.think.surprise import (
    CudaThinkBenchmark,
    CudaThinkUnavailableError,
    CudaThinkValidationError,
    benchmark_causal_surprise,
    causal_surprise,
    salient_admission,
)

__all__ = [
    "CudaThinkBenchmark",
    "CudaThinkUnavailableError",
    "CudaThinkValidationError",
    "benchmark_causal_surprise",
    "causal_surprise",
    "salient_admission",
]
