// Key bit-plane prepack and per-token append (PopKV subsystem 1).
//
// Reference: csrc/popkv_ext.cu:381-500 (fused G16/G64 encoders),
// :79-143 (G32 encoder), :284-374 (generic head dim), launched from
// :1014-1206 and reached through popkv_cuda.pack_keys / pack_keys_into
// (popkv_cuda.py:53-87).
//
// One CTA encodes one token group of one KV head:
//   staging (when the group's rows fit and are 16-byte aligned): every thread
//            issues its 16-byte loads of the group's rows at once, into shared
//            memory, so the two phases below read shared memory instead of
//            walking the rows with dependent global loads;
//   phase 1: per-dimension min/max over the group's tokens (split across row
//            slices, combined in shared memory), stored as the magnitude
//            thresholds 0.5*max and 0.5*min;
//   phase 2: one warp per token row, lane l owning dim 32*w + l of word w:
//            two ballots give the sign and magnitude words, and the bucket sums
//            of each representative group are reduced by a butterfly whose lane-0
//            result equals the reference's shuffle-down tree
//            (s[i] += s[i + o], o = 16, 8, 4, 2, 1; width 16 for G16).
// Counts come from popcounts of the ballots, so only the two sums need shuffles.
#include <cstdint>
#include <type_traits>

#include "common.cuh"

namespace popkv {
namespace {

constexpr int kPackThreads = 256;

__device__ __forceinline__ float butterfly16(float x) {
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) x = __fadd_rn(x, __shfl_xor_sync(0xFFFFFFFFu, x, o));
    return x;
}

__device__ __forceinline__ float butterfly32(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x = __fadd_rn(x, __shfl_xor_sync(0xFFFFFFFFu, x, o));
    return x;
}

template <typename T, int G, int W, bool STAGED>
__global__ void __launch_bounds__(kPackThreads) pack_kernel(
    const T* __restrict__ keys, int64_t head_stride, int64_t token_stride, int64_t tokens,
    int head_dim, int64_t token_group, int32_t* __restrict__ k_sign, int32_t* __restrict__ k_mag,
    uint16_t* __restrict__ k_low, uint16_t* __restrict__ k_delta, int64_t capacity,
    int64_t token_offset) {
    extern __shared__ __align__(16) float smem[];
    float* thr_hi = smem;                      // [head_dim]  0.5 * max
    float* thr_lo = smem + head_dim;           // [head_dim]  0.5 * min
    float* part = smem + 2 * head_dim;         // [slices][2][head_dim] partial extrema

    const int64_t kvh = blockIdx.y;
    const int64_t t0 = static_cast<int64_t>(blockIdx.x) * token_group;
    const int64_t t1 = min(t0 + token_group, tokens);
    const T* head = keys + kvh * head_stride;
    const int tid = threadIdx.x;
    const int slices0 = max(1, kPackThreads / head_dim);
    // Staged rows [t1 - t0][head_dim] after the extrema scratch, 16-byte aligned.
    T* tile = reinterpret_cast<T*>(smem + ((2 + 2 * slices0) * head_dim + 3) / 4 * 4);
    if constexpr (STAGED) {
        const int chunks = head_dim * static_cast<int>(sizeof(T)) / 16;  // per row
        const int total = static_cast<int>(t1 - t0) * chunks;
#pragma unroll 4
        for (int i = tid; i < total; i += kPackThreads) {
            const int r = i / chunks, c = i % chunks;
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(head + (t0 + r) * token_stride) + c);
            reinterpret_cast<uint4*>(tile + static_cast<int64_t>(r) * head_dim)[c] = v;
        }
        __syncthreads();
    }
    auto row_ptr = [&](int64_t t) -> const T* {
        if constexpr (STAGED) return tile + (t - t0) * head_dim;
        else return head + t * token_stride;
    };

    // Phase 1: extrema.  `slices` row slices of head_dim threads each
    // (head_dim <= 256 == kPackThreads, so every dim has a thread).
    const int slices = max(1, kPackThreads / head_dim);
    if (tid < slices * head_dim) {
        const int d = tid % head_dim, s = tid / head_dim;
        float mn = INFINITY, mx = -INFINITY;
#pragma unroll 4
        for (int64_t t = t0 + s; t < t1; t += slices) {
            float v = load_float(row_ptr(t) + d);
            mn = fminf(mn, v);
            mx = fmaxf(mx, v);
        }
        part[(s * 2 + 0) * head_dim + d] = mn;
        part[(s * 2 + 1) * head_dim + d] = mx;
    }
    __syncthreads();
    for (int d = tid; d < head_dim; d += kPackThreads) {
        float mn = part[d], mx = part[head_dim + d];
        for (int s = 1; s < slices; ++s) {
            mn = fminf(mn, part[(s * 2 + 0) * head_dim + d]);
            mx = fmaxf(mx, part[(s * 2 + 1) * head_dim + d]);
        }
        thr_lo[d] = __fmul_rn(mn, 0.5f);
        thr_hi[d] = __fmul_rn(mx, 0.5f);
    }
    __syncthreads();

    // Phase 2: one warp per token row.
    const int lane = tid & 31, warp = tid >> 5;
    constexpr int kWarps = kPackThreads / 32;
    const int reps = (head_dim + G - 1) / G;
    for (int64_t t = t0 + warp; t < t1; t += kWarps) {
        const T* row = row_ptr(t);
        const int64_t out_row = kvh * capacity + token_offset + t;
        float a_low[W], a_high[W];
        uint32_t sw[W], mw[W], vw[W];
#pragma unroll
        for (int w = 0; w < W; ++w) {
            const int d = w * 32 + lane;
            const bool valid = d < head_dim;
            const float v = valid ? load_float(row + d) : 0.0f;
            const bool sign = valid && v >= 0.0f;
            const bool mag = valid && (sign ? (v > thr_hi[d]) : (v < thr_lo[d]));
            sw[w] = __ballot_sync(0xFFFFFFFFu, sign);
            mw[w] = __ballot_sync(0xFFFFFFFFu, mag);
            vw[w] = __ballot_sync(0xFFFFFFFFu, valid);
            const float a = fabsf(v);
            a_low[w] = (valid && !mag) ? a : 0.0f;
            a_high[w] = mag ? a : 0.0f;
        }
        if (lane == 0) {
            if constexpr (W == 4) {
                reinterpret_cast<uint4*>(k_sign)[out_row] = make_uint4(sw[0], sw[1], sw[2], sw[3]);
                reinterpret_cast<uint4*>(k_mag)[out_row] = make_uint4(mw[0], mw[1], mw[2], mw[3]);
            } else {
#pragma unroll
                for (int w = 0; w < W; ++w) {
                    k_sign[out_row * W + w] = static_cast<int32_t>(sw[w]);
                    k_mag[out_row * W + w] = static_cast<int32_t>(mw[w]);
                }
            }
        }
        if constexpr (G == 16) {
#pragma unroll
            for (int w = 0; w < W; ++w) {
                const float lo = butterfly16(a_low[w]);
                const float hi = butterfly16(a_high[w]);
                const int half = lane >> 4;
                const int rep = 2 * w + half;
                if ((lane & 15) == 0 && rep < reps) {
                    const uint32_t m = half ? 0xFFFF0000u : 0x0000FFFFu;
                    const int low_count = __popc(vw[w] & ~mw[w] & m);
                    const int high_count = __popc(mw[w] & m);
                    float low, delta;
                    bucket_means(lo, low_count, hi, high_count, low, delta);
                    k_low[out_row * reps + rep] = float_to_half_bits(low);
                    k_delta[out_row * reps + rep] = float_to_half_bits(delta);
                }
            }
        } else if constexpr (G == 32) {
#pragma unroll
            for (int w = 0; w < W; ++w) {
                const float lo = butterfly32(a_low[w]);
                const float hi = butterfly32(a_high[w]);
                if (lane == 0 && w < reps) {
                    const int low_count = __popc(vw[w] & ~mw[w]);
                    const int high_count = __popc(mw[w]);
                    float low, delta;
                    bucket_means(lo, low_count, hi, high_count, low, delta);
                    k_low[out_row * reps + w] = float_to_half_bits(low);
                    k_delta[out_row * reps + w] = float_to_half_bits(delta);
                }
            }
        } else {
#pragma unroll
            for (int r = 0; r < (W + 1) / 2; ++r) {
                const bool has_second = 2 * r + 1 < W;
                const float x_lo = has_second ? __fadd_rn(a_low[2 * r], a_low[2 * r + 1]) : a_low[2 * r];
                const float x_hi = has_second ? __fadd_rn(a_high[2 * r], a_high[2 * r + 1]) : a_high[2 * r];
                const float lo = butterfly32(x_lo);
                const float hi = butterfly32(x_hi);
                if (lane == 0 && r < reps) {
                    const uint32_t m1 = has_second ? mw[2 * r + 1] : 0u;
                    const uint32_t v1 = has_second ? vw[2 * r + 1] : 0u;
                    const int low_count = __popc(vw[2 * r] & ~mw[2 * r]) + __popc(v1 & ~m1);
                    const int high_count = __popc(mw[2 * r]) + __popc(m1);
                    float low, delta;
                    bucket_means(lo, low_count, hi, high_count, low, delta);
                    k_low[out_row * reps + r] = float_to_half_bits(low);
                    k_delta[out_row * reps + r] = float_to_half_bits(delta);
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// head_dim 128, staged rows: one thread per token row in phase 2.
//
// The warp-per-row phase above spends ~300 warp instructions per row on
// ballots and shuffle trees, only 32 values per instruction.  Here each
// thread encodes a whole row from shared memory (rows padded by 16 bytes so a
// warp's 16-byte loads of 32 different rows spread over the banks), builds the
// sign/magnitude words with shifts, and reproduces the reference's lane-0
// shuffle-down tree (s[i] += s[i + o], o = 16 .. 1, width 16 for G16) with
// in-register pairwise adds, so the sums are the same bit for bit.
// ---------------------------------------------------------------------------
template <int N>
__device__ __forceinline__ float tree_sum(float* a) {  // lane-0 result of a width-N shuffle-down tree
#pragma unroll
    for (int o = N / 2; o > 0; o >>= 1)
#pragma unroll
        for (int i = 0; i < o; ++i) a[i] = __fadd_rn(a[i], a[i + o]);
    return a[0];
}

template <typename T>
__device__ __forceinline__ void load32(const unsigned char* p, float* v) {  // 32 consecutive elements
    if constexpr (sizeof(T) == 4) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint4 u = *reinterpret_cast<const uint4*>(p + 16 * j);
            v[4 * j] = __uint_as_float(u.x); v[4 * j + 1] = __uint_as_float(u.y);
            v[4 * j + 2] = __uint_as_float(u.z); v[4 * j + 3] = __uint_as_float(u.w);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint4 u = *reinterpret_cast<const uint4*>(p + 16 * j);
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                if constexpr (std::is_same<T, __nv_bfloat16>::value) {
                    v[8 * j + 2 * e] = bf16_lo(w[e]);
                    v[8 * j + 2 * e + 1] = bf16_hi(w[e]);
                } else {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
                    v[8 * j + 2 * e] = f.x;
                    v[8 * j + 2 * e + 1] = f.y;
                }
            }
        }
    }
}

constexpr int kRowThreads = 128;  // one thread per token row of a group of up to 128

// With `new_keys` set (append): the group is rows [t0, tokens) of `keys` where
// the last row, index tokens - 1, is taken from new_keys [KVH, 128] instead and
// written to `keys`, and new_values to `values` at that row (the KV append of
// the decoded token, fused with its re-encode).
template <typename T, int G>
__global__ void __launch_bounds__(kRowThreads) pack_rows_kernel(
    const T* __restrict__ keys, int64_t head_stride, int64_t token_stride, int64_t tokens,
    int64_t token_group, int32_t* __restrict__ k_sign, int32_t* __restrict__ k_mag,
    uint16_t* __restrict__ k_low, uint16_t* __restrict__ k_delta, int64_t capacity,
    int64_t token_offset, const T* __restrict__ new_keys = nullptr, const T* __restrict__ new_values = nullptr,
    T* __restrict__ values = nullptr, int64_t v_head_stride = 0, int64_t v_token_stride = 0,
    const int64_t* __restrict__ dyn_position = nullptr) {
    constexpr int D = 128, R = D / G, kSlices = kRowThreads / D;
    constexpr int kRowBytes = D * static_cast<int>(sizeof(T)) + 16;
    constexpr int kChunks = D * static_cast<int>(sizeof(T)) / 16;
    extern __shared__ __align__(16) float smem[];
    float* thr_hi = smem;                // [D]
    float* thr_lo = smem + D;            // [D]
    float* part = smem + 2 * D;          // [kSlices][2][D]
    unsigned char* tile = reinterpret_cast<unsigned char*>(smem + (2 + 2 * kSlices) * D);

    if (dyn_position) {
        // Append at a device-resident position (one CTA column, the graph-replayed
        // decode loop, launched with programmatic dependent launch): `tokens`
        // bounds the position; the open group runs from the last group boundary
        // to it.
        pdl_wait();
        pdl_launch_dependents();
        int64_t pos = *dyn_position;
        pos = pos < 0 ? 0 : (pos < tokens ? pos : tokens - 1);
        const int64_t sealed = pos - pos % token_group;
        keys += sealed * token_stride;
        if (values) values += sealed * v_token_stride;
        token_offset = sealed;
        tokens = pos - sealed + 1;
    }
    const int64_t kvh = blockIdx.y;
    const int64_t t0 = static_cast<int64_t>(blockIdx.x) * token_group;
    const int64_t t1 = min(t0 + token_group, tokens);
    const int rows = static_cast<int>(t1 - t0);
    const T* head = keys + kvh * head_stride;
    const int tid = threadIdx.x;

    const int cached_rows = new_keys ? rows - 1 : rows;
    for (int i = tid; i < cached_rows * kChunks; i += kRowThreads) {
        const int r = i / kChunks, c = i % kChunks;
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(head + (t0 + r) * token_stride) + c);
        *reinterpret_cast<uint4*>(tile + r * kRowBytes + c * 16) = v;
    }
    if (new_keys && tid < 2 * kChunks) {  // the appended token: stage its key, store its key and value
        const int c = tid % kChunks;
        const int64_t t = t1 - 1;
        if (tid < kChunks) {
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(new_keys + kvh * D) + c);
            *reinterpret_cast<uint4*>(tile + (rows - 1) * kRowBytes + c * 16) = v;
            reinterpret_cast<uint4*>(const_cast<T*>(head) + t * token_stride)[c] = v;
        } else {
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(new_values + kvh * D) + c);
            reinterpret_cast<uint4*>(values + kvh * v_head_stride + t * v_token_stride)[c] = v;
        }
    }
    __syncthreads();

    // Phase 1: extrema per dim.
    {
        const int d = tid % D, sl = tid / D;
        float mn = INFINITY, mx = -INFINITY;
        for (int r = sl; r < rows; r += kSlices) {
            const float v = load_float(reinterpret_cast<const T*>(tile + r * kRowBytes) + d);
            mn = fminf(mn, v);
            mx = fmaxf(mx, v);
        }
        part[(sl * 2 + 0) * D + d] = mn;
        part[(sl * 2 + 1) * D + d] = mx;
    }
    __syncthreads();
    if (tid < D) {
        float mn = part[tid], mx = part[D + tid];
#pragma unroll
        for (int sl = 1; sl < kSlices; ++sl) {
            mn = fminf(mn, part[(sl * 2 + 0) * D + tid]);
            mx = fmaxf(mx, part[(sl * 2 + 1) * D + tid]);
        }
        thr_lo[tid] = __fmul_rn(mn, 0.5f);
        thr_hi[tid] = __fmul_rn(mx, 0.5f);
    }
    __syncthreads();

    // Phase 2: one thread per row.
    for (int r = tid; r < rows; r += kRowThreads) {
        const unsigned char* rowp = tile + r * kRowBytes;
        const int64_t out_row = kvh * capacity + token_offset + t0 + r;
        uint32_t sw[4], mw[4];
        float lows[R], deltas[R];
        float pend_lo[32], pend_hi[32];  // G64: the first word of a pair, summed per lane with the second
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            float v[32];
            load32<T>(rowp + w * 32 * static_cast<int>(sizeof(T)), v);
            uint32_t sb = 0, mb = 0;
            float lo[32], hi[32];
#pragma unroll
            for (int l = 0; l < 32; ++l) {
                const int d = w * 32 + l;
                const bool sign = v[l] >= 0.0f;
                const bool mag = sign ? (v[l] > thr_hi[d]) : (v[l] < thr_lo[d]);
                sb |= static_cast<uint32_t>(sign) << l;
                mb |= static_cast<uint32_t>(mag) << l;
                const float a = fabsf(v[l]);
                lo[l] = mag ? 0.0f : a;
                hi[l] = mag ? a : 0.0f;
            }
            sw[w] = sb;
            mw[w] = mb;
            if constexpr (G == 16) {
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const uint32_t m = half ? 0xFFFF0000u : 0x0000FFFFu;
                    const float ls = tree_sum<16>(lo + 16 * half);
                    const float hs = tree_sum<16>(hi + 16 * half);
                    float low, delta;
                    bucket_means(ls, __popc(~mb & m), hs, __popc(mb & m), low, delta);
                    lows[2 * w + half] = low;
                    deltas[2 * w + half] = delta;
                }
            } else if constexpr (G == 32) {
                const float ls = tree_sum<32>(lo), hs = tree_sum<32>(hi);
                float low, delta;
                bucket_means(ls, __popc(~mb), hs, __popc(mb), low, delta);
                lows[w] = low;
                deltas[w] = delta;
            } else {
                if ((w & 1) == 0) {
#pragma unroll
                    for (int l = 0; l < 32; ++l) {
                        pend_lo[l] = lo[l];
                        pend_hi[l] = hi[l];
                    }
                } else {
#pragma unroll
                    for (int l = 0; l < 32; ++l) {
                        pend_lo[l] = __fadd_rn(pend_lo[l], lo[l]);
                        pend_hi[l] = __fadd_rn(pend_hi[l], hi[l]);
                    }
                    const float ls = tree_sum<32>(pend_lo), hs = tree_sum<32>(pend_hi);
                    float low, delta;
                    bucket_means(ls, __popc(~mw[w - 1]) + __popc(~mb), hs, __popc(mw[w - 1]) + __popc(mb),
                                 low, delta);
                    lows[w / 2] = low;
                    deltas[w / 2] = delta;
                }
            }
        }
        reinterpret_cast<uint4*>(k_sign)[out_row] = make_uint4(sw[0], sw[1], sw[2], sw[3]);
        reinterpret_cast<uint4*>(k_mag)[out_row] = make_uint4(mw[0], mw[1], mw[2], mw[3]);
        uint32_t lw[R / 2], dw[R / 2];
#pragma unroll
        for (int j = 0; j < R / 2; ++j) {
            lw[j] = static_cast<uint32_t>(float_to_half_bits(lows[2 * j])) |
                    (static_cast<uint32_t>(float_to_half_bits(lows[2 * j + 1])) << 16);
            dw[j] = static_cast<uint32_t>(float_to_half_bits(deltas[2 * j])) |
                    (static_cast<uint32_t>(float_to_half_bits(deltas[2 * j + 1])) << 16);
        }
        if constexpr (R == 8) {
            reinterpret_cast<uint4*>(k_low)[out_row] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            reinterpret_cast<uint4*>(k_delta)[out_row] = make_uint4(dw[0], dw[1], dw[2], dw[3]);
        } else if constexpr (R == 4) {
            reinterpret_cast<uint2*>(k_low)[out_row] = make_uint2(lw[0], lw[1]);
            reinterpret_cast<uint2*>(k_delta)[out_row] = make_uint2(dw[0], dw[1]);
        } else {
            reinterpret_cast<uint32_t*>(k_low)[out_row] = lw[0];
            reinterpret_cast<uint32_t*>(k_delta)[out_row] = dw[0];
        }
    }
}

template <typename T, int G>
int launch_pack_g(const void* keys, int64_t kv_heads, int64_t tokens, int64_t head_dim,
                  int64_t hs, int64_t ts, int32_t* k_sign, int32_t* k_mag, uint16_t* k_low,
                  uint16_t* k_delta, int64_t capacity, int64_t token_offset, int64_t tg,
                  cudaStream_t stream) {
    const int64_t groups = (tokens + tg - 1) / tg;
    const int words = static_cast<int>((head_dim + 31) / 32);
    const int slices = head_dim >= kPackThreads ? 1 : kPackThreads / static_cast<int>(head_dim);
    const size_t scratch = sizeof(float) * ((static_cast<size_t>(head_dim) * (2 + 2 * slices) + 3) / 4 * 4);
    const int64_t group_rows = tg < tokens ? tg : tokens;
    const size_t tile = sizeof(T) * static_cast<size_t>(group_rows) * static_cast<size_t>(head_dim);
    const bool staged = (head_dim * static_cast<int64_t>(sizeof(T))) % 16 == 0 &&
                        (ts * static_cast<int64_t>(sizeof(T))) % 16 == 0 &&
                        (hs * static_cast<int64_t>(sizeof(T))) % 16 == 0 && aligned(keys, 16) &&
                        tile <= 96 * 1024;
    const size_t smem = scratch + (staged ? tile : 0);
    dim3 grid(static_cast<unsigned>(groups), static_cast<unsigned>(kv_heads));
    const T* k = static_cast<const T*>(keys);
    if (staged && head_dim == 128) {  // thread-per-row encoder
        const size_t rows_smem = sizeof(float) * 128 * (2 + 2 * (kRowThreads / 128)) +
                                 static_cast<size_t>(group_rows) * (128 * sizeof(T) + 16);
        if (rows_smem <= 96 * 1024) {
            const int st = allow_dynamic_smem(pack_rows_kernel<T, G>, static_cast<int>(rows_smem));
            if (st != POPKV_OK) return st;
            pack_rows_kernel<T, G><<<grid, kRowThreads, rows_smem, stream>>>(
                k, hs, ts, tokens, tg, k_sign, k_mag, k_low, k_delta, capacity, token_offset);
            return check_launch("popkv_pack");
        }
    }
#define POPKV_PACK_CASE(NW)                                                                          \
    case NW:                                                                                         \
        if (staged) {                                                                                \
            const int st = allow_dynamic_smem(pack_kernel<T, G, NW, true>, static_cast<int>(smem));  \
            if (st != POPKV_OK) return st;                                                           \
            pack_kernel<T, G, NW, true><<<grid, kPackThreads, smem, stream>>>(                       \
                k, hs, ts, tokens, static_cast<int>(head_dim), tg, k_sign, k_mag, k_low, k_delta,    \
                capacity, token_offset);                                                             \
        } else {                                                                                     \
            pack_kernel<T, G, NW, false><<<grid, kPackThreads, smem, stream>>>(                      \
                k, hs, ts, tokens, static_cast<int>(head_dim), tg, k_sign, k_mag, k_low, k_delta,    \
                capacity, token_offset);                                                             \
        }                                                                                            \
        break;
    switch (words) {
        POPKV_PACK_CASE(1)
        POPKV_PACK_CASE(2)
        POPKV_PACK_CASE(3)
        POPKV_PACK_CASE(4)
        POPKV_PACK_CASE(5)
        POPKV_PACK_CASE(6)
        POPKV_PACK_CASE(7)
        POPKV_PACK_CASE(8)
        default:
            return fail(POPKV_ERR_UNSUPPORTED, "popkv_pack: head_dim %lld exceeds 256",
                        static_cast<long long>(head_dim));
    }
#undef POPKV_PACK_CASE
    return check_launch("popkv_pack");
}

template <typename T>
int launch_pack(const void* keys, int64_t kv_heads, int64_t tokens, int64_t head_dim, int64_t hs,
                int64_t ts, int32_t* k_sign, int32_t* k_mag, uint16_t* k_low, uint16_t* k_delta,
                int64_t capacity, int64_t token_offset, int64_t tg, int64_t g,
                cudaStream_t stream) {
    if (g == 16)
        return launch_pack_g<T, 16>(keys, kv_heads, tokens, head_dim, hs, ts, k_sign, k_mag,
                                    k_low, k_delta, capacity, token_offset, tg, stream);
    if (g == 32)
        return launch_pack_g<T, 32>(keys, kv_heads, tokens, head_dim, hs, ts, k_sign, k_mag,
                                    k_low, k_delta, capacity, token_offset, tg, stream);
    return launch_pack_g<T, 64>(keys, kv_heads, tokens, head_dim, hs, ts, k_sign, k_mag, k_low,
                                k_delta, capacity, token_offset, tg, stream);
}

}  // namespace
}  // namespace popkv

extern "C" int popkv_pack(const void* keys, int keys_dtype, int64_t kv_heads, int64_t tokens,
                          int64_t head_dim, int64_t key_head_stride, int64_t key_token_stride,
                          int32_t* k_sign, int32_t* k_mag, uint16_t* k_low, uint16_t* k_delta,
                          int64_t capacity, int64_t token_offset, int64_t token_group_size,
                          int64_t dim_group_size, void* stream) {
    using namespace popkv;
    if (!valid_dtype(keys_dtype)) return fail(POPKV_ERR_INVALID, "popkv_pack: keys must be fp32/fp16/bf16");
    if (kv_heads < 0 || tokens < 0 || head_dim <= 0)
        return fail(POPKV_ERR_INVALID, "keys must be [KVH, T, D] with a non-empty head dim");
    if (token_group_size < 1 || token_group_size > 4096)
        return fail(POPKV_ERR_INVALID, "token_group_size must be between 1 and 4096");
    if (dim_group_size != 16 && dim_group_size != 32 && dim_group_size != 64)
        return fail(POPKV_ERR_INVALID, "dim_group_size must be 16, 32, or 64");
    if (token_offset < 0 || token_offset + tokens > capacity)
        return fail(POPKV_ERR_CAPACITY, "Pop-KV cache capacity exceeded");
    if (kv_heads == 0 || tokens == 0) return POPKV_OK;
    if (!keys || !k_sign || !k_mag || !k_low || !k_delta)
        return fail(POPKV_ERR_INVALID, "popkv_pack: null pointer");
    if ((head_dim + 31) / 32 == 4 && (!aligned(k_sign, 16) || !aligned(k_mag, 16)))
        return fail(POPKV_ERR_INVALID, "popkv_pack: bit-planes must be 16-byte aligned");
    if ((tokens + token_group_size - 1) / token_group_size > 0x7FFFFFFF || kv_heads > 65535)
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_pack: grid too large");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (keys_dtype) {
        case POPKV_DTYPE_F32:
            return launch_pack<float>(keys, kv_heads, tokens, head_dim, key_head_stride,
                                      key_token_stride, k_sign, k_mag, k_low, k_delta, capacity,
                                      token_offset, token_group_size, dim_group_size, s);
        case POPKV_DTYPE_F16:
            return launch_pack<__half>(keys, kv_heads, tokens, head_dim, key_head_stride,
                                       key_token_stride, k_sign, k_mag, k_low, k_delta, capacity,
                                       token_offset, token_group_size, dim_group_size, s);
        default:
            return launch_pack<__nv_bfloat16>(keys, kv_heads, tokens, head_dim, key_head_stride,
                                              key_token_stride, k_sign, k_mag, k_low, k_delta,
                                              capacity, token_offset, token_group_size,
                                              dim_group_size, s);
    }
}

extern "C" int popkv_append_kv(const void* new_keys, const void* new_values, int dtype, int64_t kv_heads,
                               int64_t head_dim, void* cache_keys, void* cache_values, int64_t k_head_stride,
                               int64_t k_token_stride, int64_t v_head_stride, int64_t v_token_stride,
                               int64_t position, int32_t* k_sign, int32_t* k_mag, uint16_t* k_low,
                               uint16_t* k_delta, int64_t capacity, int64_t sealed, int64_t token_group_size,
                               int64_t dim_group_size, void* stream) {
    using namespace popkv;
    if (!valid_dtype(dtype)) return fail(POPKV_ERR_INVALID, "popkv_append_kv: keys must be fp32/fp16/bf16");
    if (head_dim != 128) return fail(POPKV_ERR_UNSUPPORTED, "popkv_append_kv: head_dim must be 128");
    if (kv_heads <= 0 || kv_heads > 65535) return fail(POPKV_ERR_INVALID, "popkv_append_kv: invalid KV head count");
    if (dim_group_size != 16 && dim_group_size != 32 && dim_group_size != 64)
        return fail(POPKV_ERR_INVALID, "dim_group_size must be 16, 32, or 64");
    if (token_group_size < 1 || token_group_size > 128)
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_append_kv: token_group_size must be at most 128");
    if (sealed < 0 || sealed % token_group_size || position < sealed || position - sealed >= token_group_size)
        return fail(POPKV_ERR_INVALID, "popkv_append_kv: position must lie in the open group after `sealed`");
    if (position >= capacity) return fail(POPKV_ERR_CAPACITY, "Pop-KV cache capacity exceeded");
    if (!new_keys || !new_values || !cache_keys || !cache_values || !k_sign || !k_mag || !k_low || !k_delta)
        return fail(POPKV_ERR_INVALID, "popkv_append_kv: null pointer");
    const int64_t es = static_cast<int64_t>(dtype_size(dtype));
    if (!aligned(new_keys, 16) || !aligned(new_values, 16) || !aligned(cache_keys, 16) ||
        !aligned(cache_values, 16) || (k_head_stride * es) % 16 || (k_token_stride * es) % 16 ||
        (v_head_stride * es) % 16 || (v_token_stride * es) % 16 || !aligned(k_sign, 16) || !aligned(k_mag, 16))
        return fail(POPKV_ERR_INVALID, "popkv_append_kv: buffers and strides must be 16-byte aligned");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t rows = position - sealed + 1;
    const dim3 grid(1, static_cast<unsigned>(kv_heads));
    auto run = [&](auto tag, auto gtag) -> int {
        using T = decltype(tag);
        constexpr int G = decltype(gtag)::value;
        const size_t smem = sizeof(float) * 128 * (2 + 2 * (kRowThreads / 128)) +
                            static_cast<size_t>(rows) * (128 * sizeof(T) + 16);
        const int st = allow_dynamic_smem(pack_rows_kernel<T, G>, static_cast<int>(smem));
        if (st != POPKV_OK) return st;
        // One group of `rows` rows starting at row `sealed` of the caches.
        pack_rows_kernel<T, G><<<grid, kRowThreads, smem, s>>>(
            static_cast<const T*>(cache_keys) + sealed * k_token_stride, k_head_stride, k_token_stride, rows,
            rows, k_sign, k_mag, k_low, k_delta, capacity, sealed, static_cast<const T*>(new_keys),
            static_cast<const T*>(new_values), static_cast<T*>(cache_values) + sealed * v_token_stride,
            v_head_stride, v_token_stride);
        return check_launch("popkv_append_kv");
    };
    auto by_g = [&](auto tag) -> int {
        if (dim_group_size == 16) return run(tag, std::integral_constant<int, 16>{});
        if (dim_group_size == 32) return run(tag, std::integral_constant<int, 32>{});
        return run(tag, std::integral_constant<int, 64>{});
    };
    if (dtype == POPKV_DTYPE_F32) return by_g(float{});
    if (dtype == POPKV_DTYPE_F16) return by_g(__half{});
    return by_g(__nv_bfloat16{});
}

extern "C" int popkv_append_kv_dyn(const void* new_keys, const void* new_values, int dtype,
                                   int64_t kv_heads, int64_t head_dim, void* cache_keys,
                                   void* cache_values, int64_t k_head_stride, int64_t k_token_stride,
                                   int64_t v_head_stride, int64_t v_token_stride,
                                   const int64_t* position_dev, int64_t max_tokens, int32_t* k_sign,
                                   int32_t* k_mag, uint16_t* k_low, uint16_t* k_delta,
                                   int64_t capacity, int64_t token_group_size,
                                   int64_t dim_group_size, void* stream) {
    using namespace popkv;
    if (!valid_dtype(dtype)) return fail(POPKV_ERR_INVALID, "popkv_append_kv_dyn: keys must be fp32/fp16/bf16");
    if (head_dim != 128) return fail(POPKV_ERR_UNSUPPORTED, "popkv_append_kv_dyn: head_dim must be 128");
    if (kv_heads <= 0 || kv_heads > 65535) return fail(POPKV_ERR_INVALID, "popkv_append_kv_dyn: invalid KV head count");
    if (dim_group_size != 16 && dim_group_size != 32 && dim_group_size != 64)
        return fail(POPKV_ERR_INVALID, "dim_group_size must be 16, 32, or 64");
    if (token_group_size < 1 || token_group_size > 128)
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_append_kv_dyn: token_group_size must be at most 128");
    if (max_tokens <= 0 || max_tokens > capacity)
        return fail(POPKV_ERR_CAPACITY, "popkv_append_kv_dyn: max_tokens must be in [1, capacity]");
    if ((new_keys == nullptr) != (new_values == nullptr))
        return fail(POPKV_ERR_INVALID, "popkv_append_kv_dyn: new keys and values go together");
    if (!cache_keys || !cache_values || !k_sign || !k_mag || !k_low || !k_delta || !position_dev)
        return fail(POPKV_ERR_INVALID, "popkv_append_kv_dyn: null pointer");
    const int64_t es = static_cast<int64_t>(dtype_size(dtype));
    if ((new_keys && (!aligned(new_keys, 16) || !aligned(new_values, 16))) || !aligned(cache_keys, 16) ||
        !aligned(cache_values, 16) || (k_head_stride * es) % 16 || (k_token_stride * es) % 16 ||
        (v_head_stride * es) % 16 || (v_token_stride * es) % 16 || !aligned(k_sign, 16) || !aligned(k_mag, 16))
        return fail(POPKV_ERR_INVALID, "popkv_append_kv_dyn: buffers and strides must be 16-byte aligned");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const dim3 grid(1, static_cast<unsigned>(kv_heads));
    auto run = [&](auto tag, auto gtag) -> int {
        using T = decltype(tag);
        constexpr int G = decltype(gtag)::value;
        const size_t smem = sizeof(float) * 128 * (2 + 2 * (kRowThreads / 128)) +
                            static_cast<size_t>(token_group_size) * (128 * sizeof(T) + 16);
        const int st = allow_dynamic_smem(pack_rows_kernel<T, G>, static_cast<int>(smem));
        if (st != POPKV_OK) return st;
        const cudaError_t err = launch_pdl(
            pack_rows_kernel<T, G>, grid, dim3(kRowThreads), smem, s, 1, static_cast<const T*>(cache_keys),
            k_head_stride, k_token_stride, max_tokens, static_cast<int64_t>(token_group_size), k_sign, k_mag,
            k_low, k_delta, capacity, static_cast<int64_t>(0), static_cast<const T*>(new_keys),
            static_cast<const T*>(new_values), static_cast<T*>(cache_values), v_head_stride, v_token_stride,
            position_dev);
        if (err != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_append_kv_dyn: %s", cudaGetErrorString(err));
        return check_launch("popkv_append_kv_dyn");
    };
    auto by_g = [&](auto tag) -> int {
        if (dim_group_size == 16) return run(tag, std::integral_constant<int, 16>{});
        if (dim_group_size == 32) return run(tag, std::integral_constant<int, 32>{});
        return run(tag, std::integral_constant<int, 64>{});
    };
    if (dtype == POPKV_DTYPE_F32) return by_g(float{});
    if (dtype == POPKV_DTYPE_F16) return by_g(__half{});
    return by_g(__nv_bfloat16{});
}
