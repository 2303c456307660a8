// tcgen05 tensor-core paths (grouped expert MLP, surprise head). Until the
// tensor-core kernels are enabled these entry points decline the work and the
// callers run their fp32 FMA kernels.
#include "common.cuh"

namespace koemi {

int grouped_mlp_umma(const void *, const int64_t *, const void *, const void *, const void *, const void *,
                     const void *, const void *, void *, int64_t, int64_t, int64_t, int64_t, int, void *,
                     size_t, cudaStream_t, bool *handled) {
    *handled = false;
    return KOEMI_OK;
}

size_t grouped_mlp_umma_workspace(int64_t, int64_t, int64_t, int64_t, int) { return 0; }

int surprise_umma_forward(const void *, const void *, const void *, const int64_t *, int64_t, int64_t, int64_t,
                          int, float *, int64_t, cudaStream_t, bool *handled) {
    *handled = false;
    return KOEMI_OK;
}

int64_t surprise_umma_slices(int64_t, int64_t, int64_t, int) { return 0; }

}  // namespace koemi
