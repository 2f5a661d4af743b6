// C-ABI plumbing: thread-local error messages, launch checks, version.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace popkv {

static thread_local char g_message[512] = "";

int fail(int code, const char* fmt, ...) {
    va_list args;
    va_start(args, fmt);
    vsnprintf(g_message, sizeof g_message, fmt, args);
    va_end(args);
    return code;
}

int check_launch(const char* what) {
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess)
        return fail(POPKV_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
    return POPKV_OK;
}

bool valid_dtype(int dtype) {
    return dtype == POPKV_DTYPE_F32 || dtype == POPKV_DTYPE_F16 || dtype == POPKV_DTYPE_BF16;
}

size_t dtype_size(int dtype) { return dtype == POPKV_DTYPE_F32 ? 4 : 2; }

int allow_dynamic_smem_impl(const void* kernel, int bytes) {
    // (kernel, device mask) pairs already configured; a handful of kernels use this.
    constexpr int kSlots = 64;
    static std::mutex mutex;
    static const void* kernels[kSlots] = {};
    static unsigned long long masks[kSlots] = {};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return fail(POPKV_ERR_CUDA, "cudaGetDevice failed");
    const unsigned long long bit = 1ull << (device & 63);
    std::lock_guard<std::mutex> lock(mutex);
    int slot = -1;
    for (int i = 0; i < kSlots; ++i) {
        if (kernels[i] == kernel) {
            slot = i;
            break;
        }
        if (kernels[i] == nullptr) {
            kernels[i] = kernel;
            slot = i;
            break;
        }
    }
    if (slot >= 0 && (masks[slot] & bit)) return POPKV_OK;
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (err != cudaSuccess)
        return fail(POPKV_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(err));
    // Prefer the largest shared-memory carveout so that several CTAs fit per SM.
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                               cudaSharedmemCarveoutMaxShared);
    if (err != cudaSuccess)
        return fail(POPKV_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(err));
    if (slot >= 0) masks[slot] |= bit;  // beyond kSlots kernels: set every call
    return POPKV_OK;
}

float score_scale_for(int64_t head_dim) {
    volatile float root = std::sqrt(static_cast<float>(head_dim));
    return 1.0f / root;
}

}  // namespace popkv

extern "C" const char* popkv_last_error(void) { return popkv::g_message; }

extern "C" int popkv_abi_version(void) { return POPKV_ABI_VERSION; }
