// Per-token glue of the Llama decode loop around the retrieval path:
// residual add + RMSNorm, rotary embedding + KV-cache append at a
// device-resident position, and the SwiGLU gate.  Each follows the bf16
// rounding points of the reference model's eager ops so that a graph-replayed
// decode step tracks the reference decode (popkv.py:988-1115) closely:
//   * RMSNorm (transformers LlamaRMSNorm, reached from popkv.py:1011 and
//     :1109): x in fp32, x * rsqrt(mean(x^2) + eps) rounded to bf16, then
//     weight * that rounded to bf16;
//   * residual adds (popkv.py:1104, decode_runtime.py:39): bf16 + bf16 -> bf16;
//   * rotary embedding (_apply_rope, popkv.py:745-749) with bf16 cos/sin:
//     q * cos and rotate_half(q) * sin each rounded to bf16, their sum rounded;
//   * SwiGLU (LlamaMLP): silu(gate) rounded to bf16, times up rounded to bf16.
#include "common.cuh"

namespace popkv {
namespace {

constexpr int kNormThreads = 512;

__device__ __forceinline__ float bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// One CTA per row.  With `delta`, hidden <- bf16(hidden + delta) first (written
// back), then out = RMSNorm(hidden).  dim % 8 == 0, dim <= 16384.
__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(
    const __nv_bfloat16* __restrict__ delta, __nv_bfloat16* __restrict__ hidden,
    const __nv_bfloat16* __restrict__ weight, __nv_bfloat16* __restrict__ out, int dim, float eps) {
    extern __shared__ float row[];  // [dim]
    __shared__ float red[kNormThreads / 32];
    pdl_wait();
    const int64_t r = blockIdx.x;
    const int tid = threadIdx.x;
    __nv_bfloat16* h = hidden + r * dim;
    float ss = 0.0f;
    for (int i = tid * 8; i < dim; i += kNormThreads * 8) {
        uint4 hv = *reinterpret_cast<const uint4*>(h + i);
        __nv_bfloat16* he = reinterpret_cast<__nv_bfloat16*>(&hv);
        if (delta) {
            const uint4 dv = *reinterpret_cast<const uint4*>(delta + r * dim + i);
            const __nv_bfloat16* de = reinterpret_cast<const __nv_bfloat16*>(&dv);
#pragma unroll
            for (int j = 0; j < 8; ++j)
                he[j] = __float2bfloat16_rn(__bfloat162float(he[j]) + __bfloat162float(de[j]));
            *reinterpret_cast<uint4*>(h + i) = hv;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float x = __bfloat162float(he[j]);
            row[i + j] = x;
            ss = __fmaf_rn(x, x, ss);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float total = 0.0f;
#pragma unroll
    for (int w = 0; w < kNormThreads / 32; ++w) total += red[w];
    const float inv = rsqrtf(total / static_cast<float>(dim) + eps);
    pdl_launch_dependents();
    for (int i = tid * 8; i < dim; i += kNormThreads * 8) {
        const uint4 wv = *reinterpret_cast<const uint4*>(weight + i);
        const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
        uint4 ov;
        __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
        for (int j = 0; j < 8; ++j)
            oe[j] = __float2bfloat16_rn(__bfloat162float(we[j]) * bf(row[i + j] * inv));
        *reinterpret_cast<uint4*>(out + r * dim + i) = ov;
    }
}

// Grid (batch, q_heads + kv_heads): CTA (b, h) rotates query head h (h <
// q_heads) or key head h - q_heads, and the key CTAs also copy the value head;
// 64 threads, one per rotation pair (d, d + 64).  qkv rows are
// [q_heads | kv_heads | kv_heads] x 128.  Keys and values go to the current
// buffers and to the caches at row *position.
__global__ void __launch_bounds__(64) rope_append_kernel(
    const __nv_bfloat16* __restrict__ qkv, int q_heads, int kv_heads,
    const __nv_bfloat16* __restrict__ cos_tab, const __nv_bfloat16* __restrict__ sin_tab,
    const int64_t* __restrict__ position, int64_t max_position, __nv_bfloat16* __restrict__ q_out,
    __nv_bfloat16* __restrict__ k_cur, __nv_bfloat16* __restrict__ v_cur,
    __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache, int64_t kbs,
    int64_t khs, int64_t kts, int64_t vbs, int64_t vhs, int64_t vts) {
    pdl_wait();
    const int64_t b = blockIdx.x;
    const int h = blockIdx.y;
    const int d = threadIdx.x;
    int64_t pos = *position;
    pos = pos < 0 ? 0 : (pos > max_position ? max_position : pos);
    const int heads = q_heads + 2 * kv_heads;
    const __nv_bfloat16* src = qkv + (b * heads + h) * 128;
    const float c = __bfloat162float(cos_tab[pos * 64 + d]);
    const float s = __bfloat162float(sin_tab[pos * 64 + d]);
    const float x0 = __bfloat162float(src[d]), x1 = __bfloat162float(src[d + 64]);
    // rotate_half(x) = (-x[64:], x[:64]); cos/sin repeat over the two halves.
    const __nv_bfloat16 y0 = __float2bfloat16_rn(bf(x0 * c) + bf(-x1 * s));
    const __nv_bfloat16 y1 = __float2bfloat16_rn(bf(x1 * c) + bf(x0 * s));
    pdl_launch_dependents();
    if (h < q_heads) {
        __nv_bfloat16* q = q_out + (b * q_heads + h) * 128;
        q[d] = y0;
        q[d + 64] = y1;
        return;
    }
    const int kh = h - q_heads;
    __nv_bfloat16* kc = k_cur + (b * kv_heads + kh) * 128;
    __nv_bfloat16* kr = k_cache + b * kbs + kh * khs + pos * kts;
    kc[d] = y0;
    kc[d + 64] = y1;
    kr[d] = y0;
    kr[d + 64] = y1;
    const __nv_bfloat16* vs = qkv + (b * heads + q_heads + kv_heads + kh) * 128;
    __nv_bfloat16* vc = v_cur + (b * kv_heads + kh) * 128;
    __nv_bfloat16* vr = v_cache + b * vbs + kh * vhs + pos * vts;
    vc[d] = vs[d];
    vc[d + 64] = vs[d + 64];
    vr[d] = vs[d];
    vr[d + 64] = vs[d + 64];
}

// act[r, i] = bf16(bf16(silu(gate[r, i])) * up[r, i]), gate_up rows = [gate | up].
__global__ void __launch_bounds__(256) silu_mul_kernel(const __nv_bfloat16* __restrict__ gate_up,
                                                       int64_t rows, int64_t inter,
                                                       __nv_bfloat16* __restrict__ act) {
    pdl_wait();
    const int64_t n8 = rows * inter / 8;
    for (int64_t v = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; v < n8;
         v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t e = v * 8, r = e / inter, i = e % inter;
        const uint4 gv = *reinterpret_cast<const uint4*>(gate_up + r * 2 * inter + i);
        const uint4 uv = *reinterpret_cast<const uint4*>(gate_up + r * 2 * inter + inter + i);
        const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(&gv);
        const __nv_bfloat16* u = reinterpret_cast<const __nv_bfloat16*>(&uv);
        uint4 ov;
        __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float x = __bfloat162float(g[j]);
            const float sx = bf(x / (1.0f + expf(-x)));
            o[j] = __float2bfloat16_rn(sx * __bfloat162float(u[j]));
        }
        *reinterpret_cast<uint4*>(act + e) = ov;
    }
    pdl_launch_dependents();
}

}  // namespace
}  // namespace popkv

extern "C" int popkv_rms_norm(const void* delta, void* hidden, const void* weight, int64_t rows,
                              int64_t dim, float eps, void* out, void* stream) {
    using namespace popkv;
    if (rows < 0 || dim <= 0 || dim % 8 || dim > 16384)
        return fail(POPKV_ERR_INVALID, "popkv_rms_norm: dim must be a positive multiple of 8, at most 16384");
    if (rows == 0) return POPKV_OK;
    if (rows > 0x7FFFFFFFll) return fail(POPKV_ERR_UNSUPPORTED, "popkv_rms_norm: too many rows");
    if (!hidden || !weight || !out) return fail(POPKV_ERR_INVALID, "popkv_rms_norm: null pointer");
    if (!aligned(hidden, 16) || !aligned(weight, 16) || !aligned(out, 16) || (delta && !aligned(delta, 16)))
        return fail(POPKV_ERR_INVALID, "popkv_rms_norm: buffers must be 16-byte aligned");
    const size_t smem = sizeof(float) * static_cast<size_t>(dim);
    const int st = allow_dynamic_smem(rms_norm_kernel, static_cast<int>(smem));
    if (st != POPKV_OK) return st;
    const cudaError_t err = launch_pdl(
        rms_norm_kernel, dim3(static_cast<unsigned>(rows)), dim3(kNormThreads), smem,
        static_cast<cudaStream_t>(stream), 1, static_cast<const __nv_bfloat16*>(delta),
        static_cast<__nv_bfloat16*>(hidden), static_cast<const __nv_bfloat16*>(weight),
        static_cast<__nv_bfloat16*>(out), static_cast<int>(dim), eps);
    if (err != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_rms_norm: %s", cudaGetErrorString(err));
    return check_launch("popkv_rms_norm");
}

extern "C" int popkv_rope_append(const void* qkv, int64_t batch, int64_t q_heads, int64_t kv_heads,
                                 int64_t head_dim, const void* cos_table, const void* sin_table,
                                 const int64_t* position_dev, int64_t max_position, void* q_out,
                                 void* k_cur, void* v_cur, void* k_cache, void* v_cache,
                                 int64_t k_batch_stride, int64_t k_head_stride, int64_t k_token_stride,
                                 int64_t v_batch_stride, int64_t v_head_stride, int64_t v_token_stride,
                                 void* stream) {
    using namespace popkv;
    if (head_dim != 128) return fail(POPKV_ERR_UNSUPPORTED, "popkv_rope_append: head_dim must be 128");
    if (batch < 0 || q_heads <= 0 || kv_heads <= 0 || max_position < 0)
        return fail(POPKV_ERR_INVALID, "popkv_rope_append: invalid shape");
    if (batch > 65535 || q_heads + kv_heads > 65535)
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_rope_append: too many rows");
    if (batch == 0) return POPKV_OK;
    if (!qkv || !cos_table || !sin_table || !position_dev || !q_out || !k_cur || !v_cur || !k_cache || !v_cache)
        return fail(POPKV_ERR_INVALID, "popkv_rope_append: null pointer");
    const cudaError_t err = launch_pdl(
        rope_append_kernel, dim3(static_cast<unsigned>(batch), static_cast<unsigned>(q_heads + kv_heads)),
        dim3(64), 0, static_cast<cudaStream_t>(stream), 1, static_cast<const __nv_bfloat16*>(qkv),
        static_cast<int>(q_heads), static_cast<int>(kv_heads), static_cast<const __nv_bfloat16*>(cos_table),
        static_cast<const __nv_bfloat16*>(sin_table), position_dev, max_position,
        static_cast<__nv_bfloat16*>(q_out), static_cast<__nv_bfloat16*>(k_cur),
        static_cast<__nv_bfloat16*>(v_cur), static_cast<__nv_bfloat16*>(k_cache),
        static_cast<__nv_bfloat16*>(v_cache), k_batch_stride, k_head_stride, k_token_stride,
        v_batch_stride, v_head_stride, v_token_stride);
    if (err != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_rope_append: %s", cudaGetErrorString(err));
    return check_launch("popkv_rope_append");
}

extern "C" int popkv_silu_mul(const void* gate_up, int64_t rows, int64_t inter, void* act, void* stream) {
    using namespace popkv;
    if (rows < 0 || inter <= 0 || inter % 8) return fail(POPKV_ERR_INVALID, "popkv_silu_mul: inter must be a positive multiple of 8");
    if (rows == 0) return POPKV_OK;
    if (!gate_up || !act) return fail(POPKV_ERR_INVALID, "popkv_silu_mul: null pointer");
    if (!aligned(gate_up, 16) || !aligned(act, 16))
        return fail(POPKV_ERR_INVALID, "popkv_silu_mul: buffers must be 16-byte aligned");
    const int64_t n8 = rows * inter / 8;
    const int64_t blocks = (n8 + 255) / 256;
    const cudaError_t err = launch_pdl(silu_mul_kernel,
                                       dim3(static_cast<unsigned>(blocks < 1184 ? blocks : 1184)), dim3(256),
                                       0, static_cast<cudaStream_t>(stream), 1,
                                       static_cast<const __nv_bfloat16*>(gate_up), rows, inter,
                                       static_cast<__nv_bfloat16*>(act));
    if (err != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_silu_mul: %s", cudaGetErrorString(err));
    return check_launch("popkv_silu_mul");
}
