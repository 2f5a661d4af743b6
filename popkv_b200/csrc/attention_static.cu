// popkv_attn_partial_merge_static: popkv_attn_partial_merge with its scratch
// (split partial states and the per-row completion counters) in a file-scope
// device array instead of caller buffers, so the call allocates nothing.
//
// Setup, once per device, on the first call made with that device current:
// cudaGetSymbolAddress of the array (checked) and a clear of the counter
// region, followed by a device synchronize.  Later calls only read the cached
// address.  The kernels leave the counters zero after every call, so nothing
// has to be cleared again.  All calls on one device share the one array.
#include <mutex>

#include "common.cuh"

namespace {

// Per-row completion counters: one int32 per (batch, query head) row.
constexpr int64_t kStaticCounterRows = 65536;
// Split partial states: rows * splits * (head_dim + 2) fp32 values.
constexpr int64_t kStaticPartialFloats = int64_t(1) << 20;  // 4 MiB
constexpr size_t kStaticCounterBytes = static_cast<size_t>(kStaticCounterRows) * sizeof(int32_t);
constexpr size_t kStaticScratchBytes =
    kStaticCounterBytes + static_cast<size_t>(kStaticPartialFloats) * sizeof(float);
constexpr int kMaxDevices = 64;

std::mutex g_setup_mutex;
unsigned char* g_scratch_ptr[kMaxDevices] = {};

}  // namespace

// Counters at offset 0, partials at kStaticCounterBytes (a multiple of 256).
static __device__ __align__(256) unsigned char g_attn_static_scratch[kStaticScratchBytes];

namespace {

// Address of this device's scratch, set up on first use.  Returns null and
// records the error on failure.
unsigned char* scratch_for_current_device(int* status) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        *status = popkv::fail(POPKV_ERR_CUDA, "popkv_attn_partial_merge_static: cudaGetDevice: %s",
                              cudaGetErrorString(e));
        return nullptr;
    }
    if (dev < 0 || dev >= kMaxDevices) {
        *status = popkv::fail(POPKV_ERR_UNSUPPORTED,
                              "popkv_attn_partial_merge_static: device %d beyond %d", dev, kMaxDevices);
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (g_scratch_ptr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attn_static_scratch);
        if (e != cudaSuccess || p == nullptr) {
            *status = popkv::fail(POPKV_ERR_CUDA,
                                  "popkv_attn_partial_merge_static: cudaGetSymbolAddress: %s",
                                  cudaGetErrorString(e));
            return nullptr;
        }
        e = cudaMemset(p, 0, kStaticCounterBytes);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess) {
            *status = popkv::fail(POPKV_ERR_CUDA,
                                  "popkv_attn_partial_merge_static: clearing counters: %s",
                                  cudaGetErrorString(e));
            return nullptr;
        }
        g_scratch_ptr[dev] = static_cast<unsigned char*>(p);
    }
    return g_scratch_ptr[dev];
}

}  // namespace

extern "C" int popkv_attn_partial_merge_static(
    const void* queries, int queries_dtype, int64_t batch, int64_t q_heads, int64_t head_dim,
    const void* prefix_keys, const void* prefix_values, int kv_dtype, int64_t kv_heads,
    int64_t prefix_tokens, int64_t k_batch_stride, int64_t k_head_stride, int64_t k_token_stride,
    int64_t v_batch_stride, int64_t v_head_stride, int64_t v_token_stride,
    const void* current_keys, const void* current_values, const int64_t* indices, int64_t selected,
    const uint8_t* valid, const int64_t* head_to_kv, int64_t split_tokens, void* out, int out_dtype,
    void* stream) {
    using namespace popkv;
    // Size checks first: they need no device and run before any CUDA call.
    if (batch < 0 || q_heads <= 0 || head_dim <= 0 || selected <= 0 || split_tokens <= 0)
        return fail(POPKV_ERR_INVALID, "popkv_attn_partial_merge_static: invalid sizes");
    const int64_t rows = batch * q_heads;
    const int64_t splits = (selected + split_tokens - 1) / split_tokens;
    if (rows > kStaticCounterRows)
        return fail(POPKV_ERR_CAPACITY,
                    "popkv_attn_partial_merge_static: %lld rows exceed the static scratch (%lld)",
                    static_cast<long long>(rows), static_cast<long long>(kStaticCounterRows));
    if (head_dim > 256 || splits > kStaticPartialFloats ||
        rows * splits > kStaticPartialFloats / (head_dim + 2))
        return fail(POPKV_ERR_CAPACITY,
                    "popkv_attn_partial_merge_static: rows*splits*(head_dim+2) = %lld fp32 exceeds the "
                    "static scratch (%lld)",
                    static_cast<long long>(rows * splits * (head_dim + 2)),
                    static_cast<long long>(kStaticPartialFloats));
    if (batch == 0) return POPKV_OK;
    int status = POPKV_OK;
    unsigned char* base = scratch_for_current_device(&status);
    if (base == nullptr) return status;
    int32_t* counters = reinterpret_cast<int32_t*>(base);
    float* partials = reinterpret_cast<float*>(base + kStaticCounterBytes);
    return popkv_attn_partial_merge(queries, queries_dtype, batch, q_heads, head_dim, prefix_keys,
                                    prefix_values, kv_dtype, kv_heads, prefix_tokens, k_batch_stride,
                                    k_head_stride, k_token_stride, v_batch_stride, v_head_stride,
                                    v_token_stride, current_keys, current_values, indices, selected,
                                    valid, head_to_kv, split_tokens, partials, counters, out,
                                    out_dtype, stream);
}
