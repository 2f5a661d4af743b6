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
    // Dynamic shared-memory limit already set, per (kernel, device); a handful
    // of kernels use this.  A larger request raises the limit again.
    constexpr int kSlots = 64, kDevices = 64;
    static std::mutex mutex;
    static const void* kernels[kSlots] = {};
    static int configured[kSlots][kDevices] = {};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return fail(POPKV_ERR_CUDA, "cudaGetDevice failed");
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
    const bool known = slot >= 0 && device >= 0 && device < kDevices;
    if (known && configured[slot][device] >= bytes) return POPKV_OK;
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (err != cudaSuccess)
        return fail(POPKV_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(err));
    // Prefer the largest shared-memory carveout so that several CTAs fit per SM.
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                               cudaSharedmemCarveoutMaxShared);
    if (err != cudaSuccess)
        return fail(POPKV_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(err));
    if (known) configured[slot][device] = bytes;  // otherwise: set on every call
    return POPKV_OK;
}

float score_scale_for(int64_t head_dim) {
    volatile float root = std::sqrt(static_cast<float>(head_dim));
    return 1.0f / root;
}

}  // namespace popkv

extern "C" const char* popkv_last_error(void) { return popkv::g_message; }

extern "C" int popkv_abi_version(void) { return POPKV_ABI_VERSION; }

namespace popkv {
namespace {

// Copies `n16` 16-byte units from host-mapped (or device) memory to the device.
__global__ void __launch_bounds__(256) stage_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                                    int64_t n16) {
    pdl_wait();
    pdl_launch_dependents();
    for (int64_t i = blockIdx.x * 256ll + threadIdx.x; i < n16; i += gridDim.x * 256ll) dst[i] = src[i];
}

}  // namespace
}  // namespace popkv

extern "C" int popkv_stage(const void* src, void* dst, int64_t bytes, void* stream) {
    using namespace popkv;
    if (bytes < 0 || (bytes % 16) != 0)
        return fail(POPKV_ERR_INVALID, "popkv_stage: bytes must be a non-negative multiple of 16");
    if (bytes == 0) return POPKV_OK;
    if (!src || !dst || !aligned(src, 16) || !aligned(dst, 16))
        return fail(POPKV_ERR_INVALID, "popkv_stage: buffers must be non-null and 16-byte aligned");
    const int64_t n16 = bytes / 16;
    const unsigned blocks = static_cast<unsigned>(n16 > 256 * 64 ? 64 : (n16 + 255) / 256);
    const cudaError_t err = launch_pdl(stage_kernel, dim3(blocks), dim3(256), 0, static_cast<cudaStream_t>(stream), 1,
                                       static_cast<const uint4*>(src), static_cast<uint4*>(dst), n16);
    if (err != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_stage: %s", cudaGetErrorString(err));
    return check_launch("popkv_stage");
}
