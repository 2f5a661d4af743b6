// Split-token sparse attention over the selected cache rows (PopKV subsystem 4).
//
// Reference: sparse_kernels.py:237-294 (_indexed_attention_split_kernel) and
// :297-318 (_indexed_attention_merge_kernel), launched from
// indexed_attention_split_partial / _merge (sparse_kernels.py:321-387).
//
// Partial kernel, head_dim 128: one CTA per (batch*query head, split).  The
// split's slots are processed in chunks of 256: the slot -> cache-row map is
// staged in shared memory, then thread t (segment c = t % 16 of 8 dims, row
// group g = t / 16) issues 16-byte loads of its 16 K rows and 16 V rows up front
// (256 rows x 512 B per chunk in flight), reduces q.k across the 16 threads of
// a row with shuffles, and folds the chunk into a running (max, sum, acc)
// online-softmax state.  Arithmetic is fp32; the state is written as
// [max, sum, acc[D]] per (row, split) exactly like the reference's partials.
// A generic warp-per-split kernel covers other head dims.
//
// Slot semantics follow the reference: index == prefix_tokens selects the
// current token's key/value, any other index reads prefix row
// clamp(index, 0, prefix_tokens - 1); a masked slot contributes nothing.  A
// split without a live slot keeps max = -inf, sum = 0, acc = 0 (the reference
// produces NaN when a split's first 16-slot tile is fully masked).
#include <cstdint>
#include <type_traits>

#include "common.cuh"

// Phase timestamps for profiling builds (-DPOPKV_ATTN_TIMING): thread 0 of each
// CTA of the pipelined kernel records %globaltimer at its phase boundaries.
#ifdef POPKV_ATTN_TIMING
__device__ unsigned long long g_attn_phase_ns[4096][8];
#define POPKV_ATTN_PHASE(i)                                                              \
    do {                                                                                 \
        const unsigned cta_ = blockIdx.y * gridDim.x + blockIdx.x;                       \
        if (threadIdx.x == 0 && cta_ < 4096) {                                           \
            unsigned long long t_;                                                       \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                      \
            g_attn_phase_ns[cta_][i] = t_;                                               \
        }                                                                                \
    } while (0)
extern "C" __attribute__((visibility("default"))) int popkv_attn_phase_ns(unsigned long long* host, int ctas) {
    return static_cast<int>(cudaMemcpyFromSymbol(host, g_attn_phase_ns, sizeof(unsigned long long) * 8 * ctas));
}
#else
#define POPKV_ATTN_PHASE(i) \
    do {                    \
    } while (0)
#endif

namespace popkv {
namespace {

constexpr int kAttnThreads = 256;
constexpr int kChunk = 256;
constexpr int kSegThreads = 16;                            // threads per row (8 dims each)
constexpr int kRowGroups = kAttnThreads / kSegThreads;     // 16
constexpr int kRowsPerThread = kChunk / kRowGroups;        // 16
constexpr int kSlotMasked = -2;
constexpr int kSlotCurrent = -1;

struct Raw8 {
    uint4 a, b;  // b used only for fp32 elements
};

template <typename T>
__device__ __forceinline__ Raw8 load_raw8(const T* p) {
    Raw8 r;
    r.a = __ldg(reinterpret_cast<const uint4*>(p));
    if constexpr (sizeof(T) == 4) r.b = __ldg(reinterpret_cast<const uint4*>(p) + 1);
    else r.b = make_uint4(0, 0, 0, 0);
    return r;
}

template <typename T>
__device__ __forceinline__ void unpack8(const Raw8& r, float* f) {
    if constexpr (sizeof(T) == 4) {
        f[0] = __uint_as_float(r.a.x); f[1] = __uint_as_float(r.a.y);
        f[2] = __uint_as_float(r.a.z); f[3] = __uint_as_float(r.a.w);
        f[4] = __uint_as_float(r.b.x); f[5] = __uint_as_float(r.b.y);
        f[6] = __uint_as_float(r.b.z); f[7] = __uint_as_float(r.b.w);
    } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        const uint32_t w[4] = {r.a.x, r.a.y, r.a.z, r.a.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            f[2 * j] = bf16_lo(w[j]);
            f[2 * j + 1] = bf16_hi(w[j]);
        }
    } else {
        const uint32_t w[4] = {r.a.x, r.a.y, r.a.z, r.a.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
            f[2 * j] = v.x;
            f[2 * j + 1] = v.y;
        }
    }
}

template <typename QT, typename KT>
__global__ void __launch_bounds__(kAttnThreads, 1) attn_partial128_kernel(
    const QT* __restrict__ queries, const KT* __restrict__ prefix_k, const KT* __restrict__ prefix_v,
    const KT* __restrict__ cur_k, const KT* __restrict__ cur_v, const int64_t* __restrict__ indices,
    const uint8_t* __restrict__ valid, const int64_t* __restrict__ head_to_kv,
    float* __restrict__ partials, int q_heads, int kv_heads, int64_t prefix_tokens,
    int64_t kbs, int64_t khs, int64_t kts, int64_t vbs, int64_t vhs, int64_t vts,
    int64_t selected, int64_t split_tokens, int splits, float scale) {
    __shared__ int s_row[kChunk];
    __shared__ float s_red[kAttnThreads / 32];
    __shared__ float s_acc[kAttnThreads / 32][kSegThreads][8];
    __shared__ float s_sum[kAttnThreads / 32];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int c = tid & (kSegThreads - 1), g = tid / kSegThreads;
    const int64_t row = blockIdx.y;
    const int64_t b = row / q_heads;
    const int qh = static_cast<int>(row % q_heads);
    const int64_t kvh = head_to_kv[qh];
    const int split = blockIdx.x;
    const int64_t slot0 = static_cast<int64_t>(split) * split_tokens;
    const int64_t slot_end = min(slot0 + split_tokens, selected);

    float q8[8];
    {
        const QT* qp = queries + row * 128 + 8 * c;
#pragma unroll
        for (int j = 0; j < 8; ++j) q8[j] = load_float(qp + j);
    }
    const KT* kbase = prefix_k + b * kbs + kvh * khs + 8 * c;
    const KT* vbase = prefix_v + b * vbs + kvh * vhs + 8 * c;
    const KT* ckp = cur_k + (b * kv_heads + kvh) * 128 + 8 * c;
    const KT* cvp = cur_v + (b * kv_heads + kvh) * 128 + 8 * c;
    const int64_t* idx_row = indices + row * selected;
    const uint8_t* valid_row = valid ? valid + row * selected : nullptr;

    float run_max = -INFINITY, run_sum = 0.0f;
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.0f;

    for (int64_t chunk0 = slot0; chunk0 < slot_end; chunk0 += kChunk) {
        {
            const int64_t slot = chunk0 + tid;
            int r = kSlotMasked;
            if (slot < slot_end && (!valid_row || valid_row[slot])) {
                const int64_t idx = idx_row[slot];
                r = idx == prefix_tokens ? kSlotCurrent
                                         : static_cast<int>(idx < 0 ? 0 : (idx > prefix_tokens - 1 ? prefix_tokens - 1 : idx));
            }
            s_row[tid] = r;
        }
        __syncthreads();

        // 16-bit K/V: issue the K and V loads of all 16 rows before any math
        // (16 x 2 x 16 B in flight per thread).  fp32 K/V would need twice the
        // registers, so its V loads follow the logits.
        constexpr bool kEarlyV = sizeof(KT) == 2;
        Raw8 kraw[kRowsPerThread], vraw[kRowsPerThread];
        int rid[kRowsPerThread];
#pragma unroll
        for (int i = 0; i < kRowsPerThread; ++i) {
            rid[i] = s_row[g + kRowGroups * i];
            if (rid[i] >= 0) {
                kraw[i] = load_raw8(kbase + static_cast<int64_t>(rid[i]) * kts);
                if constexpr (kEarlyV) vraw[i] = load_raw8(vbase + static_cast<int64_t>(rid[i]) * vts);
            } else if (rid[i] == kSlotCurrent) {
                kraw[i] = load_raw8(ckp);
                if constexpr (kEarlyV) vraw[i] = load_raw8(cvp);
            } else {
                kraw[i].a = kraw[i].b = make_uint4(0, 0, 0, 0);
                if constexpr (kEarlyV) vraw[i].a = vraw[i].b = make_uint4(0, 0, 0, 0);
            }
        }

        float logit[kRowsPerThread];
        float chunk_max = -INFINITY;
#pragma unroll
        for (int i = 0; i < kRowsPerThread; ++i) {
            float kf[8];
            unpack8<KT>(kraw[i], kf);
            float dot = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j) dot = __fmaf_rn(kf[j], q8[j], dot);
#pragma unroll
            for (int o = kSegThreads / 2; o > 0; o >>= 1) dot += __shfl_xor_sync(0xFFFFFFFFu, dot, o);
            logit[i] = rid[i] == kSlotMasked ? -INFINITY : dot * scale;
            chunk_max = fmaxf(chunk_max, logit[i]);
        }
        if constexpr (!kEarlyV) {
#pragma unroll
            for (int i = 0; i < kRowsPerThread; ++i) {
                if (rid[i] >= 0) vraw[i] = load_raw8(vbase + static_cast<int64_t>(rid[i]) * vts);
                else if (rid[i] == kSlotCurrent) vraw[i] = load_raw8(cvp);
                else vraw[i].a = vraw[i].b = make_uint4(0, 0, 0, 0);
            }
        }
        chunk_max = fmaxf(chunk_max, __shfl_xor_sync(0xFFFFFFFFu, chunk_max, 16));
        if (lane == 0) s_red[warp] = chunk_max;
        __syncthreads();
        chunk_max = s_red[0];
#pragma unroll
        for (int w = 1; w < kAttnThreads / 32; ++w) chunk_max = fmaxf(chunk_max, s_red[w]);

        const float new_max = fmaxf(run_max, chunk_max);
        if (new_max != -INFINITY) {
            const float alpha = run_max == -INFINITY ? 0.0f : expf(run_max - new_max);
            run_sum *= alpha;
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] *= alpha;
#pragma unroll
            for (int i = 0; i < kRowsPerThread; ++i) {
                const float p = rid[i] == kSlotMasked ? 0.0f : expf(logit[i] - new_max);
                run_sum += p;
                float vf[8];
                unpack8<KT>(vraw[i], vf);
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[j] = __fmaf_rn(p, vf[j], acc[j]);
            }
            run_max = new_max;
        }
        __syncthreads();  // s_row / s_red reuse
    }

    // Combine the 16 row groups: lanes g and g^1 share a warp, then 8 warps via smem.
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] += __shfl_xor_sync(0xFFFFFFFFu, acc[j], 16);
    float sum = run_sum + __shfl_xor_sync(0xFFFFFFFFu, run_sum, 16);
    if (lane < kSegThreads) {
#pragma unroll
        for (int j = 0; j < 8; ++j) s_acc[warp][lane][j] = acc[j];
    }
    if (lane == 0) s_sum[warp] = sum;
    __syncthreads();
    float* out = partials + (row * splits + split) * (128 + 2);
    if (tid < 128) {
        const int seg = tid / 8, j = tid % 8;
        float a = 0.0f;
#pragma unroll
        for (int w = 0; w < kAttnThreads / 32; ++w) a += s_acc[w][seg][j];
        out[2 + tid] = a;
    }
    if (tid == 0) {
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < kAttnThreads / 32; ++w) s += s_sum[w];
        out[0] = run_max;
        out[1] = s;
    }
}

// ---------------------------------------------------------------------------
// Pairs of dims (2j, 2j+1) of one 16-byte unit as float2, for packed fp32 math.
template <typename KT>
__device__ __forceinline__ void unpack_unit2(const uint4& u, float2* f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        if constexpr (std::is_same<KT, __nv_bfloat16>::value) f[j] = make_float2(bf16_lo(w[j]), bf16_hi(w[j]));
        else f[j] = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
    }
}

// Pipelined partial kernel (head_dim 128, 16-bit K/V).
//
// Thread t owns row group r = t / 8 and 16-byte units c and c + 8 of the
// head dim (dims 8c..8c+7 and 64+8c..64+8c+7).  The split is walked in
// sub-chunks of 32 slots; for each, thread t copies exactly the K and V units
// it will later read (cp.async, 16 B, L2-only) into a kPipeStages-deep ring of
// shared-memory stages, so the copy -> compute hand-off is a per-thread
// cp.async.wait_group with no block barrier.  The 8 threads of a row reduce
// q.k with shuffles; each row group keeps its own online-softmax state and the
// 32 states are combined once at the end.  Eight threads read one 256-byte row
// per phase, which touches all 32 banks once: no conflicts.
// ---------------------------------------------------------------------------
constexpr int kPipeRowGroups = 32;  // 8 threads per row -> 32 row groups per CTA
constexpr int kPipeRowsPerGroup = 1; // rows per row group per sub-chunk
constexpr int kPipeRows = kPipeRowGroups * kPipeRowsPerGroup;  // 32 slots per sub-chunk
constexpr int kPipeStages = 3;       // ring depth (2 sub-chunks in flight while computing)
constexpr int kPipeMaxSub = 8;       // sub-chunks per split (splits <= 256 slots)
constexpr int kRowBytes = 256;       // 128 x 16-bit
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kMaxFusedSplits = 64;
constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

template <typename KT>
__device__ __forceinline__ void unpack_unit(const uint4& u, float* f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        if constexpr (std::is_same<KT, __nv_bfloat16>::value) {
            f[2 * j] = bf16_lo(w[j]);
            f[2 * j + 1] = bf16_hi(w[j]);
        } else {
            const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
            f[2 * j] = v.x;
            f[2 * j + 1] = v.y;
        }
    }
}

// Pipelined partial kernel (head_dim 128, 16-bit K/V).
//
// Thread t owns row group r = t / 8 and 16-byte units c and c + 8 (dims
// 8c..8c+7 and 64+8c..64+8c+7) of each row it handles.  The split is walked
// in sub-chunks of 32 slots, one row per row group; thread t cp.async-copies
// exactly the K and V units it will read into a kPipeStages-deep ring, so the
// hand-off is a per-thread cp.async.wait_group with no block barrier.  Logits
// are kept in the base-2 domain (scale * log2 e folded in) so each softmax
// weight is one exp2; the running sum/accumulator are rescaled only when the
// running maximum grows.  The partial's max is written back in natural units.
template <typename OT>
__device__ __forceinline__ void store_out(OT* p, float v) {
    if constexpr (std::is_same<OT, float>::value) *p = v;
    else if constexpr (std::is_same<OT, __half>::value) *p = __float2half_rn(v);
    else *p = __float2bfloat16_rn(v);
}

// When OT is not void the kernel also merges: the last CTA to finish a row
// (counted with counters[row], which it resets to 0) combines the row's split
// states, read back through L2, into out[row].
template <typename QT, typename KT, typename OT>
__global__ void __launch_bounds__(kAttnThreads, 4) attn_partial_pipe_kernel(
    const QT* __restrict__ queries, const KT* __restrict__ prefix_k, const KT* __restrict__ prefix_v,
    const KT* __restrict__ cur_k, const KT* __restrict__ cur_v, const int64_t* __restrict__ indices,
    const uint8_t* __restrict__ valid, const int64_t* __restrict__ head_to_kv,
    float* __restrict__ partials, int q_heads, int kv_heads, int64_t prefix_tokens,
    int64_t kbs, int64_t khs, int64_t kts, int64_t vbs, int64_t vhs, int64_t vts,
    int64_t selected, int64_t split_tokens, int splits, float scale, int* __restrict__ counters,
    OT* __restrict__ merged, int64_t index_stride, const int64_t* __restrict__ dyn_tokens) {
    extern __shared__ __align__(16) unsigned char ring[];  // [stage][K|V][32 rows][256 B]
    POPKV_ATTN_PHASE(0);
    pdl_wait();
    pdl_launch_dependents();
    if (dyn_tokens) {
        // Device-resident prefix length: `prefix_tokens` and `selected` are the
        // upper bounds the grid was sized for.  Without indices every prefix
        // token is a slot (dense attention), plus the current one.
        const int64_t t = *dyn_tokens;
        prefix_tokens = t < 0 ? 0 : (t < prefix_tokens ? t : prefix_tokens);
        selected = indices ? min(selected - 1, prefix_tokens) + 1 : prefix_tokens + 1;
    }
    __shared__ float s_m[kAttnThreads / 32], s_s[kAttnThreads / 32];
    __shared__ float s_acc[kAttnThreads / 32][8][16];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int r = tid >> 3, c = tid & 7;
    const int64_t row = blockIdx.y;
    const int64_t b = row / q_heads;
    const int qh = static_cast<int>(row % q_heads);
    const int64_t kvh = head_to_kv[qh];
    const int split = blockIdx.x;
    const int64_t slot0 = static_cast<int64_t>(split) * split_tokens;
    const int64_t slot_end = min(slot0 + split_tokens, selected);
    const int nsub = slot_end > slot0 ? static_cast<int>((slot_end - slot0 + kPipeRows - 1) / kPipeRows) : 0;

    const unsigned char* kb = reinterpret_cast<const unsigned char*>(prefix_k + b * kbs + kvh * khs) + c * 16;
    const unsigned char* vb = reinterpret_cast<const unsigned char*>(prefix_v + b * vbs + kvh * vhs) + c * 16;
    const unsigned char* ckb = reinterpret_cast<const unsigned char*>(cur_k + (b * kv_heads + kvh) * 128) + c * 16;
    const unsigned char* cvb = reinterpret_cast<const unsigned char*>(cur_v + (b * kv_heads + kvh) * 128) + c * 16;
    const int64_t kstride = kts * 2, vstride = vts * 2;

    // Slot -> cache row map of the split, loaded with one coalesced pass and
    // staged in shared memory; thread t then copies slot i*32 + r for each i.
    __shared__ int s_rid[kPipeRows * kPipeMaxSub];
    for (int j = tid; j < kPipeRows * kPipeMaxSub; j += kAttnThreads) {
        const int64_t slot = slot0 + j;
        int id = kSlotMasked;
        if (slot < slot_end && (!valid || valid[row * index_stride + slot])) {
            const int64_t idx = indices ? __ldg(indices + row * index_stride + slot) : slot;
            id = idx == prefix_tokens ? kSlotCurrent
                                      : static_cast<int>(idx < 0 ? 0 : (idx > prefix_tokens - 1 ? prefix_tokens - 1 : idx));
        }
        s_rid[j] = id;
    }
    __syncthreads();
    int rid[kPipeMaxSub][kPipeRowsPerGroup];
#pragma unroll
    for (int i = 0; i < kPipeMaxSub; ++i)
#pragma unroll
        for (int h = 0; h < kPipeRowsPerGroup; ++h) rid[i][h] = s_rid[i * kPipeRows + h * kPipeRowGroups + r];

    auto stage_k = [&](int st, int h) {
        return ring + ((st * 2 + 0) * kPipeRows + h * kPipeRowGroups + r) * kRowBytes + c * 16;
    };
    auto stage_v = [&](int st, int h) {
        return ring + ((st * 2 + 1) * kPipeRows + h * kPipeRowGroups + r) * kRowBytes + c * 16;
    };
    auto issue = [&](int i) {
        if (i < nsub) {
            const int st = i % kPipeStages;
#pragma unroll
            for (int h = 0; h < kPipeRowsPerGroup; ++h) {
                const int id = rid[i][h];
                if (id != kSlotMasked) {
                    const unsigned char* ks = id == kSlotCurrent ? ckb : kb + static_cast<int64_t>(id) * kstride;
                    const unsigned char* vs = id == kSlotCurrent ? cvb : vb + static_cast<int64_t>(id) * vstride;
                    cp_async16(stage_k(st, h), ks);
                    cp_async16(stage_k(st, h) + 128, ks + 128);
                    cp_async16(stage_v(st, h), vs);
                    cp_async16(stage_v(st, h) + 128, vs + 128);
                }
            }
        }
        cp_async_commit();
    };

    POPKV_ATTN_PHASE(1);
#pragma unroll
    for (int i = 0; i < kPipeStages - 1; ++i) issue(i);
    POPKV_ATTN_PHASE(2);

    float q[16];
    {
        const QT* qp = queries + row * 128;
        const float qscale = scale * kLog2e;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            q[j] = load_float(qp + 8 * c + j) * qscale;
            q[8 + j] = load_float(qp + 64 + 8 * c + j) * qscale;
        }
    }

    float m = -INFINITY, ssum = 0.0f;  // m in log2 units
    // Dims (2j, 2j+1) of this thread's 16 as pairs: the products and the
    // accumulator updates run as packed fp32 operations (each element rounded
    // as a single fma would round it).
    float2 q2[8], acc2[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        q2[j] = make_float2(q[2 * j], q[2 * j + 1]);
        acc2[j] = make_float2(0.0f, 0.0f);
    }

#pragma unroll
    for (int i = 0; i < kPipeMaxSub; ++i) {
        if (i >= nsub) break;
        issue(i + kPipeStages - 1);
        cp_async_wait<kPipeStages - 1>();
        const int st = i % kPipeStages;
#pragma unroll
        for (int h = 0; h < kPipeRowsPerGroup; ++h) {
            const int id = rid[i][h];  // uniform across the 8 lanes of the row group
            float2 kf[8];
            if (id != kSlotMasked) {
                unpack_unit2<KT>(*reinterpret_cast<const uint4*>(stage_k(st, h)), kf);
                unpack_unit2<KT>(*reinterpret_cast<const uint4*>(stage_k(st, h) + 128), kf + 4);
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) kf[j] = make_float2(0.0f, 0.0f);
            }
            float2 d2 = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int j = 0; j < 8; ++j) d2 = __ffma2_rn(kf[j], q2[j], d2);
            float dot = d2.x + d2.y;
            dot += __shfl_xor_sync(0xFFFFFFFFu, dot, 4);
            dot += __shfl_xor_sync(0xFFFFFFFFu, dot, 2);
            dot += __shfl_xor_sync(0xFFFFFFFFu, dot, 1);
            if (id != kSlotMasked) {
                float2 vf[8];
                unpack_unit2<KT>(*reinterpret_cast<const uint4*>(stage_v(st, h)), vf);
                unpack_unit2<KT>(*reinterpret_cast<const uint4*>(stage_v(st, h) + 128), vf + 4);
                if (dot > m) {  // new maximum: rescale what has been accumulated
                    const float alpha = exp2f(m - dot);  // 0 when m == -inf
                    ssum = __fmaf_rn(ssum, alpha, 1.0f);
                    const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc2[j] = __ffma2_rn(acc2[j], a2, vf[j]);
                    m = dot;
                } else {
                    const float p = exp2f(dot - m);
                    ssum += p;
                    const float2 p2 = make_float2(p, p);
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc2[j] = __ffma2_rn(p2, vf[j], acc2[j]);
                }
            }
        }
    }
    cp_async_wait<0>();
    float acc[16];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        acc[2 * j] = acc2[j].x;
        acc[2 * j + 1] = acc2[j].y;
    }
    POPKV_ATTN_PHASE(3);

    // Combine the 4 row groups of this warp (lanes with equal c), then the 8 warps.
#pragma unroll
    for (int o = 8; o <= 16; o <<= 1) {
        const float m2 = __shfl_xor_sync(0xFFFFFFFFu, m, o);
        const float s2 = __shfl_xor_sync(0xFFFFFFFFu, ssum, o);
        const float M = fmaxf(m, m2);
        const float f1 = m == -INFINITY ? 0.0f : exp2f(m - M);
        const float f2 = m2 == -INFINITY ? 0.0f : exp2f(m2 - M);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const float a2 = __shfl_xor_sync(0xFFFFFFFFu, acc[j], o);
            acc[j] = acc[j] * f1 + a2 * f2;
        }
        ssum = ssum * f1 + s2 * f2;
        m = M;
    }
    if (lane < 8) {
#pragma unroll
        for (int j = 0; j < 16; ++j) s_acc[warp][lane][j] = acc[j];
        if (lane == 0) {
            s_m[warp] = m;
            s_s[warp] = ssum;
        }
    }
    __syncthreads();
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnThreads / 32; ++w) M = fmaxf(M, s_m[w]);
    float* out = partials + (row * splits + split) * (128 + 2);
    if (tid < 128) {
        const int d = tid;
        const int cc = (d & 63) >> 3, j = (d & 7) + (d >= 64 ? 8 : 0);
        float a = 0.0f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kAttnThreads / 32; ++w)
                if (s_m[w] != -INFINITY) a = __fmaf_rn(s_acc[w][cc][j], exp2f(s_m[w] - M), a);
        }
        out[2 + d] = a;
    }
    if (tid == 0) {
        float total = 0.0f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kAttnThreads / 32; ++w)
                if (s_m[w] != -INFINITY) total = __fmaf_rn(s_s[w], exp2f(s_m[w] - M), total);
        }
        out[0] = M == -INFINITY ? -INFINITY : M * kLn2;
        out[1] = total;
    }
    POPKV_ATTN_PHASE(4);
    if constexpr (!std::is_same<OT, void>::value) {
        __shared__ int s_last;
        __shared__ float s_w[kMaxFusedSplits];
        __shared__ float s_den;
        __threadfence();
        __syncthreads();
        if (tid == 0) s_last = atomicAdd(counters + row, 1) == splits - 1;
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        const float* pr = partials + row * splits * (128 + 2);
        __shared__ float s_ps[kMaxFusedSplits];
        if (tid < splits) {  // one thread per split: all loads in flight at once
            s_w[tid] = __ldcg(pr + tid * 130);
            s_ps[tid] = __ldcg(pr + tid * 130 + 1);
        }
        __syncthreads();
        if (tid == 0) {
            float gm = -INFINITY;
            for (int sp = 0; sp < splits; ++sp) gm = fmaxf(gm, s_w[sp]);
            float den = 0.0f;
            for (int sp = 0; sp < splits; ++sp) {
                const float w = expf(s_w[sp] - gm);
                s_w[sp] = w;
                den = __fmaf_rn(s_ps[sp], w, den);
            }
            s_den = den;
            counters[row] = 0;
        }
        __syncthreads();
        if (tid < 128) {
            float num = 0.0f;
#pragma unroll 8
            for (int sp = 0; sp < splits; ++sp) num = __fmaf_rn(__ldcg(pr + sp * 130 + 2 + tid), s_w[sp], num);
            store_out(merged + row * 128 + tid, num / s_den);
        }
    }
}

// Generic head dims: one warp per (row, split), serial over slots.
template <typename QT, typename KT>
__global__ void attn_partial_generic_kernel(
    const QT* __restrict__ queries, const KT* __restrict__ prefix_k, const KT* __restrict__ prefix_v,
    const KT* __restrict__ cur_k, const KT* __restrict__ cur_v, const int64_t* __restrict__ indices,
    const uint8_t* __restrict__ valid, const int64_t* __restrict__ head_to_kv,
    float* __restrict__ partials, int q_heads, int kv_heads, int head_dim, int64_t prefix_tokens,
    int64_t kbs, int64_t khs, int64_t kts, int64_t vbs, int64_t vhs, int64_t vts,
    int64_t selected, int64_t split_tokens, int splits, float scale) {
    constexpr int kMaxPerLane = 8;  // head_dim <= 256
    const int lane = threadIdx.x & 31;
    const int64_t row = blockIdx.y;
    const int64_t b = row / q_heads;
    const int qh = static_cast<int>(row % q_heads);
    const int64_t kvh = head_to_kv[qh];
    const int split = blockIdx.x;
    const int64_t slot0 = static_cast<int64_t>(split) * split_tokens;
    const int64_t slot_end = min(slot0 + split_tokens, selected);
    float q[kMaxPerLane], acc[kMaxPerLane];
#pragma unroll
    for (int j = 0; j < kMaxPerLane; ++j) {
        const int d = lane + 32 * j;
        q[j] = d < head_dim ? load_float(queries + row * head_dim + d) : 0.0f;
        acc[j] = 0.0f;
    }
    float run_max = -INFINITY, run_sum = 0.0f;
    for (int64_t slot = slot0; slot < slot_end; ++slot) {
        if (valid && !valid[row * selected + slot]) continue;
        const int64_t idx = indices[row * selected + slot];
        const KT *kp, *vp;
        if (idx == prefix_tokens) {
            kp = cur_k + (b * kv_heads + kvh) * head_dim;
            vp = cur_v + (b * kv_heads + kvh) * head_dim;
        } else {
            const int64_t r = (idx < 0 ? int64_t(0) : (idx > prefix_tokens - 1 ? prefix_tokens - 1 : idx));
            kp = prefix_k + b * kbs + kvh * khs + r * kts;
            vp = prefix_v + b * vbs + kvh * vhs + r * vts;
        }
        float dot = 0.0f;
#pragma unroll
        for (int j = 0; j < kMaxPerLane; ++j) {
            const int d = lane + 32 * j;
            if (d < head_dim) dot = __fmaf_rn(load_float(kp + d), q[j], dot);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xFFFFFFFFu, dot, o);
        const float logit = dot * scale;
        const float new_max = fmaxf(run_max, logit);
        const float alpha = run_max == -INFINITY ? 0.0f : expf(run_max - new_max);
        const float p = expf(logit - new_max);
        run_sum = run_sum * alpha + p;
#pragma unroll
        for (int j = 0; j < kMaxPerLane; ++j) {
            const int d = lane + 32 * j;
            const float v = d < head_dim ? load_float(vp + d) : 0.0f;
            acc[j] = __fmaf_rn(p, v, acc[j] * alpha);
        }
        run_max = new_max;
    }
    float* out = partials + (row * splits + split) * (head_dim + 2);
#pragma unroll
    for (int j = 0; j < kMaxPerLane; ++j) {
        const int d = lane + 32 * j;
        if (d < head_dim) out[2 + d] = acc[j];
    }
    if (lane == 0) {
        out[0] = run_max;
        out[1] = run_sum;
    }
}

// Merge: one CTA per row; the split maxima/sums are staged in shared memory and
// turned into weights once, then thread d reduces output dim d over the splits.
constexpr int kMergeMaxSplits = 1024;

template <typename OT>
__global__ void attn_merge_kernel(const float* __restrict__ partials, int64_t splits, int head_dim,
                                  OT* __restrict__ out) {
    __shared__ float s_w[kMergeMaxSplits];
    __shared__ float s_red[32];
    __shared__ float s_den;
    pdl_wait();
    pdl_launch_dependents();
    const int64_t row = blockIdx.x;
    const int64_t state = head_dim + 2;
    const float* p = partials + row * splits * state;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
    // Up to 16 splits: each thread loads its dim of every split's accumulator up
    // front, so those loads overlap the max/sum pass instead of following it.
    constexpr int kPre = 16;
    const bool pre = splits <= kPre && head_dim <= static_cast<int>(blockDim.x);
    float acc_pre[kPre];
    if (pre && tid < head_dim) {
#pragma unroll
        for (int sp = 0; sp < kPre; ++sp) acc_pre[sp] = sp < splits ? p[sp * state + 2 + tid] : 0.0f;
    }
    float gm = -INFINITY;
    for (int64_t sp = tid; sp < splits; sp += blockDim.x) gm = fmaxf(gm, p[sp * state]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) gm = fmaxf(gm, __shfl_xor_sync(0xFFFFFFFFu, gm, o));
    if (lane == 0) s_red[warp] = gm;
    __syncthreads();
    gm = s_red[0];
    for (int w = 1; w < nwarps; ++w) gm = fmaxf(gm, s_red[w]);
    __syncthreads();
    float den = 0.0f;
    for (int64_t sp = tid; sp < splits; sp += blockDim.x) {
        const float w = expf(p[sp * state] - gm);
        s_w[sp] = w;
        den = __fmaf_rn(p[sp * state + 1], w, den);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xFFFFFFFFu, den, o);
    if (lane == 0) s_red[warp] = den;
    __syncthreads();
    if (tid == 0) {
        float d = 0.0f;
        for (int w = 0; w < nwarps; ++w) d += s_red[w];
        s_den = d;
    }
    __syncthreads();
    den = s_den;
    for (int d = tid; d < head_dim; d += blockDim.x) {
        float num = 0.0f;
        if (pre) {
#pragma unroll
            for (int sp = 0; sp < kPre; ++sp)
                if (sp < splits) num = __fmaf_rn(acc_pre[sp], s_w[sp], num);
        } else {
#pragma unroll 4
            for (int64_t sp = 0; sp < splits; ++sp) num = __fmaf_rn(p[sp * state + 2 + d], s_w[sp], num);
        }
        const float v = num / den;
        if constexpr (std::is_same<OT, float>::value) out[row * head_dim + d] = v;
        else if constexpr (std::is_same<OT, __half>::value) out[row * head_dim + d] = __float2half_rn(v);
        else out[row * head_dim + d] = __float2bfloat16_rn(v);
    }
}

template <typename QT, typename KT>
int launch_partial(const void* queries, int64_t batch, int64_t q_heads, int64_t head_dim,
                   const void* pk, const void* pv, int64_t kv_heads, int64_t prefix_tokens,
                   int64_t kbs, int64_t khs, int64_t kts, int64_t vbs, int64_t vhs, int64_t vts,
                   const void* ck, const void* cv, const int64_t* indices, int64_t selected,
                   const uint8_t* valid, const int64_t* head_to_kv, int64_t split_tokens,
                   float* partials, cudaStream_t stream) {
    const int64_t splits = (selected + split_tokens - 1) / split_tokens;
    dim3 grid(static_cast<unsigned>(splits), static_cast<unsigned>(batch * q_heads));
    const float scale = score_scale_for(head_dim);
    const size_t es = sizeof(KT);
    const bool vec_ok = head_dim == 128 && aligned(pk, 16) && aligned(pv, 16) && aligned(ck, 16) &&
                        aligned(cv, 16) && (kbs * es) % 16 == 0 && (khs * es) % 16 == 0 &&
                        (kts * es) % 16 == 0 && (vbs * es) % 16 == 0 && (vhs * es) % 16 == 0 &&
                        (vts * es) % 16 == 0;
    if (vec_ok && sizeof(KT) == 2 && split_tokens <= kPipeRows * kPipeMaxSub) {
        constexpr size_t ring_bytes = static_cast<size_t>(kPipeStages) * 2 * kPipeRows * kRowBytes;
        const int st = allow_dynamic_smem(attn_partial_pipe_kernel<QT, KT, void>, static_cast<int>(ring_bytes));
        if (st != POPKV_OK) return st;
        const cudaError_t err = launch_pdl(
            attn_partial_pipe_kernel<QT, KT, void>, grid, dim3(kAttnThreads), ring_bytes, stream, 1,
            static_cast<const QT*>(queries), static_cast<const KT*>(pk), static_cast<const KT*>(pv),
            static_cast<const KT*>(ck), static_cast<const KT*>(cv), indices, valid, head_to_kv,
            partials, static_cast<int>(q_heads), static_cast<int>(kv_heads), prefix_tokens, kbs,
            khs, kts, vbs, vhs, vts, selected, split_tokens, static_cast<int>(splits), scale,
            static_cast<int*>(nullptr), static_cast<void*>(nullptr), selected,
            static_cast<const int64_t*>(nullptr));
        if (err != cudaSuccess)
            return fail(POPKV_ERR_CUDA, "popkv_attn_partial: %s", cudaGetErrorString(err));
    } else if (vec_ok) {
        attn_partial128_kernel<QT, KT><<<grid, kAttnThreads, 0, stream>>>(
            static_cast<const QT*>(queries), static_cast<const KT*>(pk), static_cast<const KT*>(pv),
            static_cast<const KT*>(ck), static_cast<const KT*>(cv), indices, valid, head_to_kv,
            partials, static_cast<int>(q_heads), static_cast<int>(kv_heads), prefix_tokens, kbs,
            khs, kts, vbs, vhs, vts, selected, split_tokens, static_cast<int>(splits), scale);
    } else {
        attn_partial_generic_kernel<QT, KT><<<grid, 32, 0, stream>>>(
            static_cast<const QT*>(queries), static_cast<const KT*>(pk), static_cast<const KT*>(pv),
            static_cast<const KT*>(ck), static_cast<const KT*>(cv), indices, valid, head_to_kv,
            partials, static_cast<int>(q_heads), static_cast<int>(kv_heads),
            static_cast<int>(head_dim), prefix_tokens, kbs, khs, kts, vbs, vhs, vts, selected,
            split_tokens, static_cast<int>(splits), scale);
    }
    return check_launch("popkv_attn_partial");
}

// Partials + merge in one launch when the pipelined kernel applies; otherwise
// the two-launch path.  Returns POPKV_ERR_UNSUPPORTED (without launching) when
// the single-launch form does not apply, so the caller can fall back.
template <typename QT, typename KT, typename OT>
int launch_partial_merged(const void* queries, int64_t batch, int64_t q_heads, int64_t head_dim,
                          const void* pk, const void* pv, int64_t kv_heads, int64_t prefix_tokens,
                          int64_t kbs, int64_t khs, int64_t kts, int64_t vbs, int64_t vhs,
                          int64_t vts, const void* ck, const void* cv, const int64_t* indices,
                          int64_t selected, const uint8_t* valid, const int64_t* head_to_kv,
                          int64_t split_tokens, float* partials, int* counters, void* out,
                          cudaStream_t stream) {
    const int64_t splits = (selected + split_tokens - 1) / split_tokens;
    const size_t es = sizeof(KT);
    const bool ok = sizeof(KT) == 2 && head_dim == 128 && split_tokens <= kPipeRows * kPipeMaxSub &&
                    splits <= kMaxFusedSplits && aligned(pk, 16) && aligned(pv, 16) &&
                    aligned(ck, 16) && aligned(cv, 16) && (kbs * es) % 16 == 0 &&
                    (khs * es) % 16 == 0 && (kts * es) % 16 == 0 && (vbs * es) % 16 == 0 &&
                    (vhs * es) % 16 == 0 && (vts * es) % 16 == 0;
    if (!ok) return POPKV_ERR_UNSUPPORTED;
    if constexpr (sizeof(KT) == 2) {
        dim3 grid(static_cast<unsigned>(splits), static_cast<unsigned>(batch * q_heads));
        constexpr size_t ring_bytes = static_cast<size_t>(kPipeStages) * 2 * kPipeRows * kRowBytes;
        const int st = allow_dynamic_smem(attn_partial_pipe_kernel<QT, KT, OT>, static_cast<int>(ring_bytes));
        if (st != POPKV_OK) return st;
        attn_partial_pipe_kernel<QT, KT, OT><<<grid, kAttnThreads, ring_bytes, stream>>>(
            static_cast<const QT*>(queries), static_cast<const KT*>(pk), static_cast<const KT*>(pv),
            static_cast<const KT*>(ck), static_cast<const KT*>(cv), indices, valid, head_to_kv,
            partials, static_cast<int>(q_heads), static_cast<int>(kv_heads), prefix_tokens, kbs,
            khs, kts, vbs, vhs, vts, selected, split_tokens, static_cast<int>(splits),
            score_scale_for(head_dim), counters, static_cast<OT*>(out), selected,
            static_cast<const int64_t*>(nullptr));
        return check_launch("popkv_attn_partial_merge");
    }
    return POPKV_ERR_UNSUPPORTED;
}

template <typename QT>
int dispatch_kv(int kv_dtype, const void* queries, int64_t batch, int64_t q_heads, int64_t head_dim,
                const void* pk, const void* pv, int64_t kv_heads, int64_t prefix_tokens, int64_t kbs,
                int64_t khs, int64_t kts, int64_t vbs, int64_t vhs, int64_t vts, const void* ck,
                const void* cv, const int64_t* indices, int64_t selected, const uint8_t* valid,
                const int64_t* head_to_kv, int64_t split_tokens, float* partials,
                cudaStream_t stream) {
    if (kv_dtype == POPKV_DTYPE_F32)
        return launch_partial<QT, float>(queries, batch, q_heads, head_dim, pk, pv, kv_heads,
                                         prefix_tokens, kbs, khs, kts, vbs, vhs, vts, ck, cv,
                                         indices, selected, valid, head_to_kv, split_tokens,
                                         partials, stream);
    if (kv_dtype == POPKV_DTYPE_F16)
        return launch_partial<QT, __half>(queries, batch, q_heads, head_dim, pk, pv, kv_heads,
                                          prefix_tokens, kbs, khs, kts, vbs, vhs, vts, ck, cv,
                                          indices, selected, valid, head_to_kv, split_tokens,
                                          partials, stream);
    return launch_partial<QT, __nv_bfloat16>(queries, batch, q_heads, head_dim, pk, pv, kv_heads,
                                             prefix_tokens, kbs, khs, kts, vbs, vhs, vts, ck, cv,
                                             indices, selected, valid, head_to_kv, split_tokens,
                                             partials, stream);
}

}  // namespace
}  // namespace popkv

extern "C" int popkv_attn_partial(const void* queries, int queries_dtype, int64_t batch,
                                  int64_t q_heads, int64_t head_dim, const void* prefix_keys,
                                  const void* prefix_values, int kv_dtype, int64_t kv_heads,
                                  int64_t prefix_tokens, int64_t k_batch_stride,
                                  int64_t k_head_stride, int64_t k_token_stride,
                                  int64_t v_batch_stride, int64_t v_head_stride,
                                  int64_t v_token_stride, const void* current_keys,
                                  const void* current_values, const int64_t* indices,
                                  int64_t selected, const uint8_t* valid,
                                  const int64_t* head_to_kv, int64_t split_tokens, float* partials,
                                  void* stream) {
    using namespace popkv;
    if (!valid_dtype(queries_dtype) || !valid_dtype(kv_dtype))
        return fail(POPKV_ERR_INVALID, "popkv_attn_partial: tensors must be fp32/fp16/bf16");
    if (batch < 0 || q_heads <= 0 || kv_heads <= 0 || head_dim <= 0)
        return fail(POPKV_ERR_INVALID, "invalid indexed-attention tensor ranks or K/V shapes");
    if (prefix_tokens <= 0 || selected <= 0)
        return fail(POPKV_ERR_INVALID, "indexed attention requires non-empty prefix and selection");
    if (split_tokens <= 0 || split_tokens % 16)
        return fail(POPKV_ERR_INVALID, "split_tokens must be a positive multiple of 16");
    if (head_dim > 256)
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_attn_partial: head_dim %lld exceeds 256",
                    static_cast<long long>(head_dim));
    const int64_t splits = (selected + split_tokens - 1) / split_tokens;
    if (splits > 0x7FFFFFFFll || batch * q_heads > 65535 || prefix_tokens >= 0x7FFFFFFFll)
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_attn_partial: grid too large");
    if (batch == 0) return POPKV_OK;
    if (!queries || !prefix_keys || !prefix_values || !current_keys || !current_values ||
        !indices || !head_to_kv || !partials)
        return fail(POPKV_ERR_INVALID, "popkv_attn_partial: null pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (queries_dtype == POPKV_DTYPE_F32)
        return dispatch_kv<float>(kv_dtype, queries, batch, q_heads, head_dim, prefix_keys,
                                  prefix_values, kv_heads, prefix_tokens, k_batch_stride,
                                  k_head_stride, k_token_stride, v_batch_stride, v_head_stride,
                                  v_token_stride, current_keys, current_values, indices, selected,
                                  valid, head_to_kv, split_tokens, partials, s);
    if (queries_dtype == POPKV_DTYPE_F16)
        return dispatch_kv<__half>(kv_dtype, queries, batch, q_heads, head_dim, prefix_keys,
                                   prefix_values, kv_heads, prefix_tokens, k_batch_stride,
                                   k_head_stride, k_token_stride, v_batch_stride, v_head_stride,
                                   v_token_stride, current_keys, current_values, indices, selected,
                                   valid, head_to_kv, split_tokens, partials, s);
    return dispatch_kv<__nv_bfloat16>(kv_dtype, queries, batch, q_heads, head_dim, prefix_keys,
                                      prefix_values, kv_heads, prefix_tokens, k_batch_stride,
                                      k_head_stride, k_token_stride, v_batch_stride, v_head_stride,
                                      v_token_stride, current_keys, current_values, indices,
                                      selected, valid, head_to_kv, split_tokens, partials, s);
}

extern "C" int popkv_attn_merge(const float* partials, int64_t rows, int64_t splits,
                                int64_t head_dim, void* out, int out_dtype, void* stream) {
    using namespace popkv;
    if (!valid_dtype(out_dtype))
        return fail(POPKV_ERR_INVALID, "popkv_attn_merge: output must be fp32/fp16/bf16");
    if (rows < 0 || splits <= 0 || head_dim <= 0)
        return fail(POPKV_ERR_INVALID, "partial/output shape mismatch");
    if (rows == 0) return POPKV_OK;
    if (!partials || !out) return fail(POPKV_ERR_INVALID, "popkv_attn_merge: null pointer");
    if (rows > 0x7FFFFFFFll) return fail(POPKV_ERR_UNSUPPORTED, "popkv_attn_merge: too many rows");
    if (splits > kMergeMaxSplits)
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_attn_merge: more than %d splits", kMergeMaxSplits);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const unsigned threads = head_dim >= 128 ? 128 : 32 * static_cast<unsigned>((head_dim + 31) / 32);
    const int d = static_cast<int>(head_dim);
    const dim3 grid(static_cast<unsigned>(rows)), block(threads);
    cudaError_t err;
    if (out_dtype == POPKV_DTYPE_F32)
        err = launch_pdl(attn_merge_kernel<float>, grid, block, 0, s, 1, partials, splits, d,
                         static_cast<float*>(out));
    else if (out_dtype == POPKV_DTYPE_F16)
        err = launch_pdl(attn_merge_kernel<__half>, grid, block, 0, s, 1, partials, splits, d,
                         static_cast<__half*>(out));
    else
        err = launch_pdl(attn_merge_kernel<__nv_bfloat16>, grid, block, 0, s, 1, partials, splits, d,
                         static_cast<__nv_bfloat16*>(out));
    if (err != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_attn_merge: %s", cudaGetErrorString(err));
    return check_launch("popkv_attn_merge");
}

extern "C" int popkv_attn_partial_merge(
    const void* queries, int queries_dtype, int64_t batch, int64_t q_heads, int64_t head_dim,
    const void* prefix_keys, const void* prefix_values, int kv_dtype, int64_t kv_heads,
    int64_t prefix_tokens, int64_t k_batch_stride, int64_t k_head_stride, int64_t k_token_stride,
    int64_t v_batch_stride, int64_t v_head_stride, int64_t v_token_stride,
    const void* current_keys, const void* current_values, const int64_t* indices, int64_t selected,
    const uint8_t* valid, const int64_t* head_to_kv, int64_t split_tokens, float* partials,
    int32_t* counters, void* out, int out_dtype, void* stream) {
    using namespace popkv;
    if (!valid_dtype(out_dtype))
        return fail(POPKV_ERR_INVALID, "popkv_attn_partial_merge: output must be fp32/fp16/bf16");
    if (!counters || !out) return fail(POPKV_ERR_INVALID, "popkv_attn_partial_merge: null pointer");
    if (queries_dtype == POPKV_DTYPE_BF16 && kv_dtype == POPKV_DTYPE_BF16 && batch > 0 &&
        q_heads > 0 && q_heads * batch <= 65535 && prefix_tokens > 0 && prefix_tokens < 0x7FFFFFFFll &&
        selected > 0 && split_tokens > 0 && split_tokens % 16 == 0 && queries && prefix_keys &&
        prefix_values && current_keys && current_values && indices && head_to_kv && partials) {
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        int st = POPKV_ERR_UNSUPPORTED;
        if (out_dtype == POPKV_DTYPE_BF16)
            st = launch_partial_merged<__nv_bfloat16, __nv_bfloat16, __nv_bfloat16>(
                queries, batch, q_heads, head_dim, prefix_keys, prefix_values, kv_heads, prefix_tokens,
                k_batch_stride, k_head_stride, k_token_stride, v_batch_stride, v_head_stride,
                v_token_stride, current_keys, current_values, indices, selected, valid, head_to_kv,
                split_tokens, partials, counters, out, s);
        else if (out_dtype == POPKV_DTYPE_F32)
            st = launch_partial_merged<__nv_bfloat16, __nv_bfloat16, float>(
                queries, batch, q_heads, head_dim, prefix_keys, prefix_values, kv_heads, prefix_tokens,
                k_batch_stride, k_head_stride, k_token_stride, v_batch_stride, v_head_stride,
                v_token_stride, current_keys, current_values, indices, selected, valid, head_to_kv,
                split_tokens, partials, counters, out, s);
        if (st != POPKV_ERR_UNSUPPORTED) return st;
    }
    // General case: two launches.
    int st = popkv_attn_partial(queries, queries_dtype, batch, q_heads, head_dim, prefix_keys,
                                prefix_values, kv_dtype, kv_heads, prefix_tokens, k_batch_stride,
                                k_head_stride, k_token_stride, v_batch_stride, v_head_stride,
                                v_token_stride, current_keys, current_values, indices, selected,
                                valid, head_to_kv, split_tokens, partials, stream);
    if (st != POPKV_OK) return st;
    return popkv_attn_merge(partials, batch * q_heads, (selected + split_tokens - 1) / split_tokens,
                            head_dim, out, out_dtype, stream);
}

namespace popkv {
namespace {

template <typename QT, typename KT>
int launch_partial_dyn(const void* queries, int64_t batch, int64_t q_heads, const void* pk,
                       const void* pv, int64_t kv_heads, int64_t max_tokens, int64_t kbs, int64_t khs,
                       int64_t kts, int64_t vbs, int64_t vhs, int64_t vts, const void* ck,
                       const void* cv, const int64_t* tokens_dev, const int64_t* indices,
                       int64_t index_stride, int64_t max_selected, const int64_t* head_to_kv,
                       int64_t split_tokens, int64_t splits, float* partials, cudaStream_t stream) {
    constexpr size_t ring_bytes = static_cast<size_t>(kPipeStages) * 2 * kPipeRows * kRowBytes;
    const int st = allow_dynamic_smem(attn_partial_pipe_kernel<QT, KT, void>, static_cast<int>(ring_bytes));
    if (st != POPKV_OK) return st;
    const dim3 grid(static_cast<unsigned>(splits), static_cast<unsigned>(batch * q_heads));
    const cudaError_t err = launch_pdl(
        attn_partial_pipe_kernel<QT, KT, void>, grid, dim3(kAttnThreads), ring_bytes, stream, 1,
        static_cast<const QT*>(queries), static_cast<const KT*>(pk), static_cast<const KT*>(pv),
        static_cast<const KT*>(ck), static_cast<const KT*>(cv), indices,
        static_cast<const uint8_t*>(nullptr), head_to_kv, partials, static_cast<int>(q_heads),
        static_cast<int>(kv_heads), max_tokens, kbs, khs, kts, vbs, vhs, vts, max_selected,
        split_tokens, static_cast<int>(splits), score_scale_for(128), static_cast<int*>(nullptr),
        static_cast<void*>(nullptr), index_stride, tokens_dev);
    if (err != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_attn_dyn: %s", cudaGetErrorString(err));
    return check_launch("popkv_attn_dyn");
}

}  // namespace
}  // namespace popkv

extern "C" int popkv_attn_dyn(const void* queries, int queries_dtype, int64_t batch, int64_t q_heads,
                              const void* prefix_keys, const void* prefix_values, int kv_dtype,
                              int64_t kv_heads, int64_t max_tokens, int64_t k_batch_stride,
                              int64_t k_head_stride, int64_t k_token_stride, int64_t v_batch_stride,
                              int64_t v_head_stride, int64_t v_token_stride, const void* current_keys,
                              const void* current_values, const int64_t* tokens_dev,
                              const int64_t* indices, int64_t index_stride, int64_t k_max,
                              const int64_t* head_to_kv, int64_t split_tokens, float* partials,
                              void* out, int out_dtype, void* stream) {
    using namespace popkv;
    if (queries_dtype != POPKV_DTYPE_BF16 && queries_dtype != POPKV_DTYPE_F16)
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_attn_dyn: queries must be fp16/bf16");
    if (kv_dtype != queries_dtype)
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_attn_dyn: keys/values must have the query dtype");
    if (!valid_dtype(out_dtype)) return fail(POPKV_ERR_INVALID, "popkv_attn_dyn: output must be fp32/fp16/bf16");
    if (batch < 0 || q_heads <= 0 || kv_heads <= 0 || max_tokens < 0 || split_tokens <= 0)
        return fail(POPKV_ERR_INVALID, "popkv_attn_dyn: invalid shape");
    if (split_tokens > kPipeRows * kPipeMaxSub)
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_attn_dyn: split_tokens above %d", kPipeRows * kPipeMaxSub);
    if (indices && (k_max < 0 || index_stride < k_max + 1))
        return fail(POPKV_ERR_INVALID, "popkv_attn_dyn: index rows must hold k_max + 1 slots");
    const int64_t max_selected = indices ? (k_max < max_tokens ? k_max : max_tokens) + 1 : max_tokens + 1;
    const int64_t splits = (max_selected + split_tokens - 1) / split_tokens;
    if (splits > kMergeMaxSplits)
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_attn_dyn: more than %d splits", kMergeMaxSplits);
    if (batch * q_heads > 65535) return fail(POPKV_ERR_UNSUPPORTED, "popkv_attn_dyn: batch * q_heads above 65535");
    if (batch == 0) return POPKV_OK;
    if (!queries || !prefix_keys || !prefix_values || !current_keys || !current_values || !tokens_dev ||
        !head_to_kv || !partials)
        return fail(POPKV_ERR_INVALID, "popkv_attn_dyn: null pointer");
    const int64_t es = 2;
    if (!aligned(prefix_keys, 16) || !aligned(prefix_values, 16) || !aligned(current_keys, 16) ||
        !aligned(current_values, 16) || (k_batch_stride * es) % 16 || (k_head_stride * es) % 16 ||
        (k_token_stride * es) % 16 || (v_batch_stride * es) % 16 || (v_head_stride * es) % 16 ||
        (v_token_stride * es) % 16)
        return fail(POPKV_ERR_INVALID, "popkv_attn_dyn: K/V buffers and strides must be 16-byte aligned");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int st =
        queries_dtype == POPKV_DTYPE_BF16
            ? launch_partial_dyn<__nv_bfloat16, __nv_bfloat16>(
                  queries, batch, q_heads, prefix_keys, prefix_values, kv_heads, max_tokens,
                  k_batch_stride, k_head_stride, k_token_stride, v_batch_stride, v_head_stride,
                  v_token_stride, current_keys, current_values, tokens_dev, indices, index_stride,
                  max_selected, head_to_kv, split_tokens, splits, partials, s)
            : launch_partial_dyn<__half, __half>(
                  queries, batch, q_heads, prefix_keys, prefix_values, kv_heads, max_tokens,
                  k_batch_stride, k_head_stride, k_token_stride, v_batch_stride, v_head_stride,
                  v_token_stride, current_keys, current_values, tokens_dev, indices, index_stride,
                  max_selected, head_to_kv, split_tokens, splits, partials, s);
    if (st != POPKV_OK || !out) return st;
    return popkv_attn_merge(partials, batch * q_heads, splits, 128, out, out_dtype, stream);
}
