// C-ABI plumbing: thread-local error messages, launch checks, version.
#include <cmath>
#include <cstdarg>
#include <cstdio>

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

float score_scale_for(int64_t head_dim) {
    volatile float root = std::sqrt(static_cast<float>(head_dim));
    return 1.0f / root;
}

}  // namespace popkv

extern "C" const char* popkv_last_error(void) { return popkv::g_message; }

extern "C" int popkv_abi_version(void) { return POPKV_ABI_VERSION; }
