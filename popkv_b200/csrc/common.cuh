// Shared helpers of the PopKV B200 kernels: element loads, exact conversions,
// error reporting for the C ABI.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "popkv_b200.h"

namespace popkv {

// ---------------------------------------------------------------------------
// Host-side error state (thread-local message, see popkv_last_error()).
// ---------------------------------------------------------------------------
int fail(int code, const char* fmt, ...);
int check_launch(const char* what);
bool valid_dtype(int dtype);
size_t dtype_size(int dtype);

// Raise a kernel's dynamic shared-memory limit once per (kernel, device)
// (needed above 48 KB).  Kernels are told apart by address: instantiations of
// one template share a function type.
int allow_dynamic_smem_impl(const void* kernel, int bytes);

template <typename Kernel>
int allow_dynamic_smem(Kernel kernel, int bytes) {
    return allow_dynamic_smem_impl(reinterpret_cast<const void*>(kernel), bytes);
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch (PDL) between the kernels of a decode step.
// A kernel launched with launch_pdl may start while the previous kernel on the
// stream is finishing; it calls pdl_wait() before its first global memory
// access, which returns once the previous grid has completed and its writes
// are visible.  pdl_launch_dependents() lets the next kernel start early.
// Both are no-ops for a plain launch.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// cudaLaunchKernelEx with programmatic stream serialization (and a 1-D
// cluster when cluster_x > 1).
template <typename... ExpTypes, typename... ActTypes>
cudaError_t launch_pdl(void (*kernel)(ExpTypes...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, unsigned cluster_x, ActTypes&&... args) {
    cudaLaunchConfig_t config = {};
    config.gridDim = grid;
    config.blockDim = block;
    config.dynamicSmemBytes = smem;
    config.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    int n = 1;
    if (cluster_x > 1) {
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = cluster_x;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        n = 2;
    }
    config.attrs = attr;
    config.numAttrs = n;
    return cudaLaunchKernelEx(&config, kernel, static_cast<ActTypes&&>(args)...);
}

inline bool aligned(const void* p, size_t bytes) {
    return (reinterpret_cast<uintptr_t>(p) % bytes) == 0;
}

// ---------------------------------------------------------------------------
// Element access.  Loads widen to fp32 exactly (bf16/fp16 -> fp32 is exact).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float to_float(float v) { return v; }
__device__ __forceinline__ float to_float(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ float load_float(const T* p) { return to_float(*p); }

__device__ __forceinline__ float bf16_lo(uint32_t pair) { return __uint_as_float(pair << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t pair) { return __uint_as_float(pair & 0xFFFF0000u); }

__device__ __forceinline__ float half_bits_to_float(uint16_t bits) {
    return __half2float(__ushort_as_half(bits));
}

// Exact conversion of a small integer (|c| < 2^22) to float on the FP32 pipe:
// 0x4B400000 is 1.5 * 2^23, whose ulp is 1, so (1.5*2^23 + c) - 1.5*2^23 == c.
__device__ __forceinline__ float small_int_to_float(int c) {
    return __fsub_rn(__int_as_float(0x4B400000 + c), 12582912.0f);
}

// fp32 -> fp16 round-to-nearest-even, returned as the 16-bit pattern.
__device__ __forceinline__ uint16_t float_to_half_bits(float v) {
    return __half_as_ushort(__float2half_rn(v));
}

// Order-preserving 16-bit key of an fp16 score: a larger score has a larger key;
// -0 and +0 share a key; NaN takes the largest key.
__device__ __forceinline__ uint32_t order_key16(uint16_t h) {
    if ((h & 0x7FFFu) == 0) h = 0;
    if ((h & 0x7C00u) == 0x7C00u && (h & 0x3FFu)) return 0xFFFFu;
    return (h & 0x8000u) ? (~static_cast<uint32_t>(h) & 0xFFFFu) : (static_cast<uint32_t>(h) | 0x8000u);
}

// Bucket means shared by every encoder (reference csrc/popkv_ext.cu:128-135):
// an empty low bucket copies the high mean, an empty high bucket copies the
// low mean, both empty give 0.  Divisions are correctly rounded.
__device__ __forceinline__ void bucket_means(float low_sum, int low_count, float high_sum,
                                             int high_count, float& low, float& delta) {
    float high;
    if (low_count == 0) {
        low = high_count ? __fdiv_rn(high_sum, (float)high_count) : 0.0f;
        high = low;
    } else {
        low = __fdiv_rn(low_sum, (float)low_count);
        high = high_count ? __fdiv_rn(high_sum, (float)high_count) : low;
    }
    delta = __fsub_rn(high, low);
}

// Score scale fp32(1 / fp32(sqrt(head_dim))), computed on the host with IEEE
// single-precision sqrt and divide: 0x3DB504F3 for head_dim 128.
float score_scale_for(int64_t head_dim);

}  // namespace popkv
