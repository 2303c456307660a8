// Library-wide host plumbing: ABI version, thread-local error messages, the
// per-device status word used by bounded waits, SM counts and the TMA
// descriptor encoder resolved through the runtime's driver entry point.
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"

namespace koemi {
namespace {

thread_local std::string g_last_error;

constexpr int kMaxDevices = 64;
std::mutex g_device_mutex;
int *g_status_words[kMaxDevices] = {};
int g_sm_counts[kMaxDevices] = {};

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode_tiled = nullptr;
std::once_flag g_encode_once;

}  // namespace

int fail(int code, const char *format, ...) {
    char buffer[1024];
    va_list args;
    va_start(args, format);
    std::vsnprintf(buffer, sizeof(buffer), format, args);
    va_end(args);
    g_last_error.assign(buffer);
    return code;
}

void clear_error() { g_last_error.clear(); }

int *device_status_word() {
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lock(g_device_mutex);
    if (g_status_words[device] == nullptr) {
        int *word = nullptr;
        if (cudaMalloc(&word, sizeof(int)) != cudaSuccess) return nullptr;
        if (cudaMemset(word, 0, sizeof(int)) != cudaSuccess) return nullptr;
        g_status_words[device] = word;
    }
    return g_status_words[device];
}

int sm_count() {
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) return 148;
    if (g_sm_counts[device] == 0) {
        int count = 0;
        cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device);
        g_sm_counts[device] = count > 0 ? count : 148;
    }
    return g_sm_counts[device];
}

int encode_tensor_map(CUtensorMap *map, CUtensorMapDataType type, uint32_t rank, const void *base,
                      const uint64_t *dims, const uint64_t *strides_bytes, const uint32_t *box,
                      CUtensorMapSwizzle swizzle) {
    std::call_once(g_encode_once, [] {
        void *entry = nullptr;
        cudaDriverEntryPointQueryResult query;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &entry, cudaEnableDefault, &query) ==
                cudaSuccess &&
            query == cudaDriverEntryPointSuccess) {
            g_encode_tiled = reinterpret_cast<EncodeTiledFn>(entry);
        }
    });
    if (g_encode_tiled == nullptr) {
        return fail(KOEMI_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
    }
    cuuint32_t element_strides[5] = {1, 1, 1, 1, 1};
    CUresult result = g_encode_tiled(map, type, rank, const_cast<void *>(base),
                                     reinterpret_cast<const cuuint64_t *>(dims),
                                     reinterpret_cast<const cuuint64_t *>(strides_bytes),
                                     reinterpret_cast<const cuuint32_t *>(box), element_strides,
                                     CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (result != CUDA_SUCCESS) {
        return fail(KOEMI_ERR_CUDA, "cuTensorMapEncodeTiled failed with CUresult %d", int(result));
    }
    return KOEMI_OK;
}

}  // namespace koemi

extern "C" int koemi_abi_version(void) { return KOEMI_ABI_VERSION; }

extern "C" size_t koemi_last_error(char *buffer, size_t capacity) {
    const std::string &message = koemi::g_last_error;
    if (buffer != nullptr && capacity > 0) {
        size_t n = message.size() < capacity - 1 ? message.size() : capacity - 1;
        std::memcpy(buffer, message.data(), n);
        buffer[n] = '\0';
    }
    return message.size();
}

extern "C" int koemi_device_init(int device) {
    int previous = 0;
    KOEMI_CUDA_TRY(cudaGetDevice(&previous));
    KOEMI_CUDA_TRY(cudaSetDevice(device));
    int *word = koemi::device_status_word();
    koemi::sm_count();
    cudaSetDevice(previous);
    if (word == nullptr) return koemi::fail(KOEMI_ERR_CUDA, "allocating the status word failed");
    return KOEMI_OK;
}

extern "C" int koemi_device_status(int device, int *status_out) {
    if (status_out == nullptr) return koemi::fail(KOEMI_ERR_INVALID, "status_out is NULL");
    int previous = 0;
    KOEMI_CUDA_TRY(cudaGetDevice(&previous));
    KOEMI_CUDA_TRY(cudaSetDevice(device));
    int *word = koemi::device_status_word();
    int value = 0;
    if (word != nullptr) {
        cudaError_t e = cudaMemcpy(&value, word, sizeof(int), cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = cudaMemset(word, 0, sizeof(int));
        cudaSetDevice(previous);
        if (e != cudaSuccess) {
            return koemi::fail(KOEMI_ERR_CUDA, "reading the device status failed: %s",
                               cudaGetErrorString(e));
        }
    } else {
        cudaSetDevice(previous);
    }
    *status_out = value;
    return KOEMI_OK;
}
