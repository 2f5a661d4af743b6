// Query encoding and popcount scoring (PopKV subsystem 2).
//
// Reference: query encoding csrc/popkv_ext.cu:911-957 (G16/G64) and :235-281
// (G32); scoring csrc/popkv_ext.cu:757-876 (GQA tiled, head_dim 128, fp16 out)
// with the four-count reconstruction of :502-515, and :145-230 / :517-675
// (other head dims, fp32 out).  Entry points replace ext.query_encode_out,
// ext.score_encoded, ext.score and ext.score_dim (popkv_cuda.py:157-204).
//
// Score of query row q against key token t, per representative group r (in order):
//   match = ~(qs ^ ks) restricted to r's bits
//   c_sign = 2 popc(match) - |r|, c_q = 2 popc(match & qm) - popc(qm),
//   c_k = 2 popc(match & km) - popc(km), c_qk = 2 popc(match & qm & km) - popc(qm & km)
//   total += fma(ql*kl, c_sign, fma(dq*kl, c_q, fma(ql*dk, c_k, (dq*dk)*c_qk)))
// then fp16(total * scale).  Every fp32 operation is written with an explicit
// rounding intrinsic so the result is bit-identical to the CPU oracle.
//
// head_dim 128 kernel: one CTA per (batch, GQA group, token tile); each thread
// owns kTokensPerThread tokens of the tile, loads their planes with 128-bit
// coalesced loads, and scores them against every query head of the group; the
// group's encoded query state sits in shared memory (broadcast reads).  The
// count-to-float conversion uses the FP32 pipe (small_int_to_float) instead of
// the slower integer-conversion unit, leaving the popcount unit as the only
// narrow pipe.
#include <atomic>
#include <cstdint>

#include "common.cuh"
#include "score_tc8.cuh"
#include "score_impl.cuh"
#include "score_mma.cuh"

namespace popkv {
namespace {

constexpr int kEncodeWarps = 4;

template <typename T, int W>
__global__ void __launch_bounds__(kEncodeWarps * 32) query_encode_kernel(
    const T* __restrict__ queries, int64_t rows, int head_dim, int G, int32_t* __restrict__ q_sign,
    int32_t* __restrict__ q_mag, float* __restrict__ q_low, float* __restrict__ q_delta) {
    __shared__ float scratch[kEncodeWarps][2 * 32 * W];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * kEncodeWarps + warp;
    if (row >= rows) return;
    const int reps = (head_dim + G - 1) / G;
    encode_query_row<T, W>(queries + row * head_dim, head_dim, G, lane, scratch[warp],
                           reinterpret_cast<uint32_t*>(q_sign + row * W),
                           reinterpret_cast<uint32_t*>(q_mag + row * W), q_low + row * reps,
                           q_delta + row * reps);
}

// ---------------------------------------------------------------------------
// head_dim 128 scorer.
// ---------------------------------------------------------------------------

constexpr int kScoreThreads = 256;
constexpr int kTokensPerThread = 1;
constexpr int kScoreTile = kScoreThreads * kTokensPerThread;
constexpr int kMaxGroupHeads = 16;

// With HIST the kernel also counts every score's top 11 key bits
// (order_key16 >> 5) per query row into hist [rows][2048] (global, must hold
// zeros on entry): per-CTA shared-memory histograms flushed with one global
// atomic per non-empty bin.  That is the first radix pass of the top-k.
constexpr int kHistBins11 = 2048;
constexpr int kMaxHistHeads = 4;

template <int G, typename QT, bool RAW, bool HIST = false>
__global__ void __launch_bounds__(kScoreThreads, 4) score128_kernel(
    const QT* __restrict__ queries, const int32_t* __restrict__ q_sign,
    const int32_t* __restrict__ q_mag, const float* __restrict__ q_low,
    const float* __restrict__ q_delta, const int32_t* __restrict__ k_sign,
    const int32_t* __restrict__ k_mag, const uint16_t* __restrict__ k_low,
    const uint16_t* __restrict__ k_delta, const int64_t* __restrict__ head_to_kv,
    uint16_t* __restrict__ scores, int q_heads, int group_heads, int64_t capacity,
    int64_t tokens, float scale, uint32_t* __restrict__ hist, int64_t score_stride,
    const int64_t* __restrict__ dyn_tokens) {
    constexpr int R = 128 / G;
    extern __shared__ uint32_t hist_s[];  // [group_heads][2048] when HIST
    __shared__ QueryState<G> states[kMaxGroupHeads];
    __shared__ float scratch[kScoreThreads / 32][2 * 32 * 4];

    pdl_wait();
    if (dyn_tokens) {
        // Device-resident token count (the graph-replayed decode loop); the grid
        // and `tokens` cover its upper bound.
        const int64_t t = *dyn_tokens;
        tokens = t < 0 ? 0 : (t < tokens ? t : tokens);
        if (static_cast<int64_t>(blockIdx.x) * kScoreTile >= tokens) return;
    }
    const int groups = q_heads / group_heads;
    const int64_t b = blockIdx.y / groups;
    const int grp = blockIdx.y % groups;
    const int qh0 = grp * group_heads;
    const int64_t row0 = b * q_heads + qh0;
    const int64_t kvh = head_to_kv[qh0];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

    if constexpr (RAW) {
        for (int h = warp; h < group_heads; h += kScoreThreads / 32) {
            encode_query_row<QT, 4>(queries + (row0 + h) * 128, 128, G, lane, scratch[warp],
                                    states[h].qs, states[h].qm, states[h].ql, states[h].dq);
        }
    } else {
        for (int i = threadIdx.x; i < group_heads * (8 + 2 * R); i += kScoreThreads) {
            const int h = i / (8 + 2 * R), j = i % (8 + 2 * R);
            const int64_t row = row0 + h;
            if (j < 4) states[h].qs[j] = static_cast<uint32_t>(q_sign[row * 4 + j]);
            else if (j < 8) states[h].qm[j - 4] = static_cast<uint32_t>(q_mag[row * 4 + j - 4]);
            else if (j < 8 + R) states[h].ql[j - 8] = q_low[row * R + j - 8];
            else states[h].dq[j - 8 - R] = q_delta[row * R + j - 8 - R];
        }
    }
    if constexpr (HIST) {
        for (int i = threadIdx.x; i < group_heads * kHistBins11; i += kScoreThreads) hist_s[i] = 0;
    }
    __syncthreads();
    if (threadIdx.x < group_heads) finish_state<G>(states[threadIdx.x]);
    __syncthreads();

    const int64_t tile0 = static_cast<int64_t>(blockIdx.x) * kScoreTile;
    const uint4* sign4 = reinterpret_cast<const uint4*>(k_sign) + kvh * capacity;
    const uint4* mag4 = reinterpret_cast<const uint4*>(k_mag) + kvh * capacity;
    const uint16_t* lowp = k_low + kvh * capacity * R;
    const uint16_t* deltap = k_delta + kvh * capacity * R;

    TokenPlanes<G> tp[kTokensPerThread];
    bool live[kTokensPerThread];
#pragma unroll
    for (int i = 0; i < kTokensPerThread; ++i) {
        const int64_t t = tile0 + threadIdx.x + i * kScoreThreads;
        live[i] = t < tokens;
        load_token<G>(sign4, mag4, lowp, deltap, live[i] ? t : 0, tp[i]);
    }

    for (int h = 0; h < group_heads; ++h) {
        const QueryState<G>& st = states[h];
        uint16_t* out = scores + (row0 + h) * score_stride;
#pragma unroll
        for (int i = 0; i < kTokensPerThread; ++i) {
            const float total = score_token<G>(st, tp[i]);
            if (live[i]) {
                const int64_t t = tile0 + threadIdx.x + i * kScoreThreads;
                const uint16_t bits = float_to_half_bits(__fmul_rn(total, scale));
                out[t] = bits;
                if constexpr (HIST) atomicAdd(&hist_s[h * kHistBins11 + (order_key16(bits) >> 5)], 1u);
            }
        }
    }
    pdl_launch_dependents();
    if constexpr (HIST) {
        __syncthreads();
        for (int i = threadIdx.x; i < group_heads * kHistBins11; i += kScoreThreads) {
            const uint32_t c = hist_s[i];
            if (c) atomicAdd(hist + (row0 + i / kHistBins11) * kHistBins11 + (i % kHistBins11), c);
        }
    }
}

// ---------------------------------------------------------------------------
// Generic head-dim scorer (fp32 out): one CTA per (query row, token tile).
// ---------------------------------------------------------------------------

constexpr int kGenericThreads = 256;

template <typename QT, int W>
__global__ void __launch_bounds__(kGenericThreads) score_generic_kernel(
    const QT* __restrict__ queries, const int32_t* __restrict__ k_sign,
    const int32_t* __restrict__ k_mag, const uint16_t* __restrict__ k_low,
    const uint16_t* __restrict__ k_delta, const int64_t* __restrict__ head_to_kv,
    float* __restrict__ scores, int q_heads, int head_dim, int G, int64_t capacity,
    int64_t tokens, float scale) {
    __shared__ uint32_t s_qs[W], s_qm[W];
    __shared__ float s_ql[W * 2], s_dq[W * 2];
    __shared__ float scratch[2 * 32 * W];
    const int64_t row = blockIdx.y;
    const int qh = static_cast<int>(row % q_heads);
    const int64_t kvh = head_to_kv[qh];
    const int reps = (head_dim + G - 1) / G;
    if (threadIdx.x < 32)
        encode_query_row<QT, W>(queries + row * head_dim, head_dim, G, threadIdx.x, scratch, s_qs,
                                s_qm, s_ql, s_dq);
    __syncthreads();
    const int64_t t = static_cast<int64_t>(blockIdx.x) * kGenericThreads + threadIdx.x;
    if (t >= tokens) return;
    const int64_t key_row = kvh * capacity + t;
    float total = 0.0f;
    for (int r = 0; r < reps; ++r) {
        const int start = r * G, end = min(start + G, head_dim);
        int c_sign = 0, c_q = 0, c_k = 0, c_qk = 0;
        for (int w = start / 32; w <= (end - 1) / 32; ++w) {
            const int ws = w * 32;
            const int bgn = max(start, ws) - ws, fin = min(end, ws + 32) - ws;
            const int width = fin - bgn;
            const uint32_t m = width == 32 ? 0xFFFFFFFFu : (((1u << width) - 1u) << bgn);
            const uint32_t qm = s_qm[w] & m;
            const uint32_t km = static_cast<uint32_t>(k_mag[key_row * W + w]) & m;
            const uint32_t match = ~(s_qs[w] ^ static_cast<uint32_t>(k_sign[key_row * W + w])) & m;
            const uint32_t both = qm & km;
            c_sign += 2 * __popc(match) - __popc(m);
            c_q += 2 * __popc(match & qm) - __popc(qm);
            c_k += 2 * __popc(match & km) - __popc(km);
            c_qk += 2 * __popc(match & both) - __popc(both);
        }
        const float ql = s_ql[r], dq = s_dq[r];
        const float kl = half_bits_to_float(k_low[key_row * reps + r]);
        const float dk = half_bits_to_float(k_delta[key_row * reps + r]);
        const float t1 = __fmul_rn(ql, kl), t2 = __fmul_rn(dq, kl), t3 = __fmul_rn(ql, dk);
        const float t4 = __fmul_rn(__fmul_rn(dq, dk), static_cast<float>(c_qk));
        total = __fadd_rn(total, __fmaf_rn(t1, static_cast<float>(c_sign),
                                           __fmaf_rn(t2, static_cast<float>(c_q),
                                                     __fmaf_rn(t3, static_cast<float>(c_k), t4))));
    }
    scores[row * tokens + t] = __fmul_rn(total, scale);
}

// ---------------------------------------------------------------------------
// Launchers.
// ---------------------------------------------------------------------------

// Scorer choice for head_dim 128 (popkv_score_dispatch): 0 picks the faster
// kernel for the shape, 1 always the popcount kernel, 2 the fp8 tensor-core
// kernel wherever it applies.  All three give the same bits.
std::atomic<int> g_score_dispatch{0};

inline bool use_tc8(int G, int64_t capacity, int group_heads, int64_t rows, int64_t tokens) {
    const int mode = g_score_dispatch.load(std::memory_order_relaxed);
    if (mode == 1 || !score_tc8_eligible(G, capacity, group_heads)) return false;
    return mode == 2 || score_tc8_pays(G, rows, tokens);
}

template <int G, typename QT, bool RAW>
int launch_score128_hist(const void* queries, int64_t batch, int64_t q_heads, const int32_t* k_sign,
                         const int32_t* k_mag, const uint16_t* k_low, const uint16_t* k_delta,
                         int64_t kv_heads, int64_t capacity, const int64_t* head_to_kv,
                         int64_t tokens, uint16_t* scores, uint32_t* hist, cudaStream_t stream) {
    const int group_heads = static_cast<int>(q_heads / kv_heads);
    if (use_tc8(G, capacity, group_heads, batch * kv_heads, tokens)) {
        return launch_score128_tc8<G, QT, RAW, true>(
            static_cast<const QT*>(queries), nullptr, nullptr, nullptr, nullptr, batch, q_heads, k_sign, k_mag,
            k_low, k_delta, kv_heads, capacity, head_to_kv, tokens, scores, stream, tokens, nullptr, hist);
    }
    const int64_t tiles = (tokens + kScoreTile - 1) / kScoreTile;
    dim3 grid(static_cast<unsigned>(tiles), static_cast<unsigned>(batch * kv_heads));
    const size_t smem = sizeof(uint32_t) * kHistBins11 * group_heads;
    const cudaError_t err = launch_pdl(
        score128_kernel<G, QT, RAW, true>, grid, dim3(kScoreThreads), smem, stream, 1,
        static_cast<const QT*>(queries), static_cast<const int32_t*>(nullptr),
        static_cast<const int32_t*>(nullptr), static_cast<const float*>(nullptr),
        static_cast<const float*>(nullptr), k_sign, k_mag, k_low, k_delta, head_to_kv, scores,
        static_cast<int>(q_heads), group_heads, capacity, tokens, score_scale_for(128), hist, tokens,
        static_cast<const int64_t*>(nullptr));
    if (err != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_score_hist: %s", cudaGetErrorString(err));
    return check_launch("popkv_score_hist");
}

template <int G, typename QT, bool RAW>
int launch_score128(const void* queries, const int32_t* q_sign, const int32_t* q_mag,
                    const float* q_low, const float* q_delta, int64_t batch, int64_t q_heads,
                    const int32_t* k_sign, const int32_t* k_mag, const uint16_t* k_low,
                    const uint16_t* k_delta, int64_t kv_heads, int64_t capacity,
                    const int64_t* head_to_kv, int64_t tokens, uint16_t* scores,
                    cudaStream_t stream, int64_t score_stride = -1,
                    const int64_t* dyn_tokens = nullptr, bool popcount_only = false) {
    const int group_heads = static_cast<int>(q_heads / kv_heads);
    if (!popcount_only && use_tc8(G, capacity, group_heads, batch * kv_heads, tokens)) {
        return launch_score128_tc8<G, QT, RAW>(
            static_cast<const QT*>(queries), q_sign, q_mag, q_low, q_delta, batch, q_heads, k_sign, k_mag,
            k_low, k_delta, kv_heads, capacity, head_to_kv, tokens, scores, stream,
            score_stride < 0 ? tokens : score_stride, dyn_tokens);
    }
    const int64_t tiles = (tokens + kScoreTile - 1) / kScoreTile;
    dim3 grid(static_cast<unsigned>(tiles), static_cast<unsigned>(batch * kv_heads));
    const cudaError_t err = launch_pdl(
        score128_kernel<G, QT, RAW, false>, grid, dim3(kScoreThreads), 0, stream, 1,
        static_cast<const QT*>(queries), q_sign, q_mag, q_low, q_delta, k_sign, k_mag, k_low,
        k_delta, head_to_kv, scores, static_cast<int>(q_heads), group_heads, capacity, tokens,
        score_scale_for(128), static_cast<uint32_t*>(nullptr), score_stride < 0 ? tokens : score_stride,
        dyn_tokens);
    if (err != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_score: %s", cudaGetErrorString(err));
    return check_launch("popkv_score");
}

template <typename QT, bool RAW>
int dispatch_score128(int64_t g, const void* queries, const int32_t* q_sign, const int32_t* q_mag,
                      const float* q_low, const float* q_delta, int64_t batch, int64_t q_heads,
                      const int32_t* k_sign, const int32_t* k_mag, const uint16_t* k_low,
                      const uint16_t* k_delta, int64_t kv_heads, int64_t capacity,
                      const int64_t* head_to_kv, int64_t tokens, uint16_t* scores,
                      cudaStream_t stream, bool popcount_only = false) {
    if (g == 16)
        return launch_score128<16, QT, RAW>(queries, q_sign, q_mag, q_low, q_delta, batch, q_heads,
                                            k_sign, k_mag, k_low, k_delta, kv_heads, capacity,
                                            head_to_kv, tokens, scores, stream, -1, nullptr,
                                            popcount_only);
    if (g == 32)
        return launch_score128<32, QT, RAW>(queries, q_sign, q_mag, q_low, q_delta, batch, q_heads,
                                            k_sign, k_mag, k_low, k_delta, kv_heads, capacity,
                                            head_to_kv, tokens, scores, stream, -1, nullptr,
                                            popcount_only);
    return launch_score128<64, QT, RAW>(queries, q_sign, q_mag, q_low, q_delta, batch, q_heads,
                                        k_sign, k_mag, k_low, k_delta, kv_heads, capacity,
                                        head_to_kv, tokens, scores, stream, -1, nullptr, popcount_only);
}

}  // namespace

int score_sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!cached[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

int read_score_tc8_timeouts(uint32_t* count) {
    const cudaError_t e = cudaMemcpyFromSymbol(count, g_score_tc8_timeouts, sizeof(uint32_t));
    return e == cudaSuccess ? POPKV_OK : fail(POPKV_ERR_CUDA, "score timeouts: %s", cudaGetErrorString(e));
}

int check_score_common(int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t capacity,
                       int64_t tokens, int64_t g, const void* head_to_kv) {
    if (g != 16 && g != 32 && g != 64)
        return fail(POPKV_ERR_INVALID, "dim_group_size must be 16, 32, or 64");
    if (batch < 0 || q_heads <= 0 || kv_heads <= 0)
        return fail(POPKV_ERR_INVALID, "invalid batch or head counts");
    if (tokens <= 0 || tokens > capacity) return fail(POPKV_ERR_INVALID, "invalid score token count");
    if (q_heads % kv_heads != 0)
        return fail(POPKV_ERR_INVALID, "GQA query heads must be divisible by KV heads");
    if (!head_to_kv) return fail(POPKV_ERR_INVALID, "head mapping is null");
    if (batch * kv_heads > 65535 || batch * q_heads > 65535)
        return fail(POPKV_ERR_UNSUPPORTED, "batch * heads exceeds 65535");
    return POPKV_OK;
}

}  // namespace popkv

extern "C" int popkv_query_encode(const void* queries, int queries_dtype, int64_t rows,
                                  int64_t head_dim, int64_t dim_group_size, int32_t* q_sign,
                                  int32_t* q_mag, float* q_low, float* q_delta, void* stream) {
    using namespace popkv;
    if (!valid_dtype(queries_dtype))
        return fail(POPKV_ERR_INVALID, "queries must be fp32/fp16/bf16");
    if (dim_group_size != 16 && dim_group_size != 32 && dim_group_size != 64)
        return fail(POPKV_ERR_INVALID, "dim_group_size must be 16, 32, or 64");
    if (rows < 0 || head_dim <= 0)
        return fail(POPKV_ERR_INVALID, "queries must be [batch, query heads, non-empty head dim]");
    if (head_dim > 256)
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_query_encode: head_dim %lld exceeds 256",
                    static_cast<long long>(head_dim));
    if (rows == 0) return POPKV_OK;
    if (!queries || !q_sign || !q_mag || !q_low || !q_delta)
        return fail(POPKV_ERR_INVALID, "popkv_query_encode: null pointer");
    const int words = static_cast<int>((head_dim + 31) / 32);
    const unsigned blocks = static_cast<unsigned>((rows + kEncodeWarps - 1) / kEncodeWarps);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int g = static_cast<int>(dim_group_size), d = static_cast<int>(head_dim);
#define POPKV_ENC(T, NW)                                                                            \
    query_encode_kernel<T, NW><<<blocks, kEncodeWarps * 32, 0, s>>>(static_cast<const T*>(queries), \
                                                                    rows, d, g, q_sign, q_mag,      \
                                                                    q_low, q_delta)
#define POPKV_ENC_T(T)                          \
    switch (words) {                            \
        case 1: POPKV_ENC(T, 1); break;         \
        case 2: POPKV_ENC(T, 2); break;         \
        case 3: POPKV_ENC(T, 3); break;         \
        case 4: POPKV_ENC(T, 4); break;         \
        case 5: POPKV_ENC(T, 5); break;         \
        case 6: POPKV_ENC(T, 6); break;         \
        case 7: POPKV_ENC(T, 7); break;         \
        default: POPKV_ENC(T, 8); break;        \
    }
    if (queries_dtype == POPKV_DTYPE_F32) { POPKV_ENC_T(float) }
    else if (queries_dtype == POPKV_DTYPE_F16) { POPKV_ENC_T(__half) }
    else { POPKV_ENC_T(__nv_bfloat16) }
#undef POPKV_ENC_T
#undef POPKV_ENC
    return check_launch("popkv_query_encode");
}

extern "C" int popkv_score_encoded(const int32_t* q_sign, const int32_t* q_mag, const float* q_low,
                                   const float* q_delta, int64_t batch, int64_t q_heads,
                                   const int32_t* k_sign, const int32_t* k_mag,
                                   const uint16_t* k_low, const uint16_t* k_delta, int64_t kv_heads,
                                   int64_t capacity, const int64_t* head_to_kv, int64_t tokens,
                                   int64_t dim_group_size, uint16_t* scores, void* stream) {
    using namespace popkv;
    int st = check_score_common(batch, q_heads, kv_heads, capacity, tokens, dim_group_size, head_to_kv);
    if (st != POPKV_OK) return st;
    if (q_heads / kv_heads > kMaxGroupHeads)
        return fail(POPKV_ERR_UNSUPPORTED, "more than %d query heads per KV head", kMaxGroupHeads);
    if (batch == 0) return POPKV_OK;
    if (!q_sign || !q_mag || !q_low || !q_delta || !k_sign || !k_mag || !k_low || !k_delta || !scores)
        return fail(POPKV_ERR_INVALID, "popkv_score_encoded: null pointer");
    if (!aligned(k_sign, 16) || !aligned(k_mag, 16) || !aligned(k_low, 16) || !aligned(k_delta, 16))
        return fail(POPKV_ERR_INVALID, "packed planes must be 16-byte aligned");
    return dispatch_score128<float, false>(dim_group_size, nullptr, q_sign, q_mag, q_low, q_delta,
                                           batch, q_heads, k_sign, k_mag, k_low, k_delta, kv_heads,
                                           capacity, head_to_kv, tokens, scores,
                                           static_cast<cudaStream_t>(stream));
}

namespace popkv {
static int score_entry(const void* queries, int queries_dtype, int64_t batch, int64_t q_heads,
                       int64_t head_dim, const int32_t* k_sign, const int32_t* k_mag,
                       const uint16_t* k_low, const uint16_t* k_delta, int64_t kv_heads,
                       int64_t capacity, const int64_t* head_to_kv, int64_t tokens,
                       int64_t dim_group_size, void* scores, int scores_dtype, void* stream,
                       bool popcount_only) {
    if (!valid_dtype(queries_dtype)) return fail(POPKV_ERR_INVALID, "queries must be fp32/fp16/bf16");
    int st = check_score_common(batch, q_heads, kv_heads, capacity, tokens, dim_group_size, head_to_kv);
    if (st != POPKV_OK) return st;
    if (head_dim <= 0) return fail(POPKV_ERR_INVALID, "queries must have a non-empty head dim");
    if (head_dim > 256)
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_score: head_dim %lld exceeds 256",
                    static_cast<long long>(head_dim));
    if (batch == 0) return POPKV_OK;
    if (!queries || !k_sign || !k_mag || !k_low || !k_delta || !scores)
        return fail(POPKV_ERR_INVALID, "popkv_score: null pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (head_dim == 128) {
        if (scores_dtype != POPKV_DTYPE_F16)
            return fail(POPKV_ERR_INVALID, "head_dim 128 scores are fp16");
        if (q_heads / kv_heads > kMaxGroupHeads)
            return fail(POPKV_ERR_UNSUPPORTED, "more than %d query heads per KV head", kMaxGroupHeads);
        if (!aligned(k_sign, 16) || !aligned(k_mag, 16) || !aligned(k_low, 16) || !aligned(k_delta, 16))
            return fail(POPKV_ERR_INVALID, "packed planes must be 16-byte aligned");
        uint16_t* out = static_cast<uint16_t*>(scores);
        if (queries_dtype == POPKV_DTYPE_F32)
            return dispatch_score128<float, true>(dim_group_size, queries, nullptr, nullptr, nullptr,
                                                  nullptr, batch, q_heads, k_sign, k_mag, k_low,
                                                  k_delta, kv_heads, capacity, head_to_kv, tokens,
                                                  out, s, popcount_only);
        if (queries_dtype == POPKV_DTYPE_F16)
            return dispatch_score128<__half, true>(dim_group_size, queries, nullptr, nullptr, nullptr,
                                                   nullptr, batch, q_heads, k_sign, k_mag, k_low,
                                                   k_delta, kv_heads, capacity, head_to_kv, tokens,
                                                   out, s, popcount_only);
        return dispatch_score128<__nv_bfloat16, true>(dim_group_size, queries, nullptr, nullptr,
                                                      nullptr, nullptr, batch, q_heads, k_sign,
                                                      k_mag, k_low, k_delta, kv_heads, capacity,
                                                      head_to_kv, tokens, out, s, popcount_only);
    }
    if (scores_dtype != POPKV_DTYPE_F32)
        return fail(POPKV_ERR_INVALID, "scores for head_dim != 128 are fp32");
    const int words = static_cast<int>((head_dim + 31) / 32);
    dim3 grid(static_cast<unsigned>((tokens + kGenericThreads - 1) / kGenericThreads),
              static_cast<unsigned>(batch * q_heads));
    float* out = static_cast<float*>(scores);
    const float scale = score_scale_for(head_dim);
    const int d = static_cast<int>(head_dim), g = static_cast<int>(dim_group_size);
    const int qh = static_cast<int>(q_heads);
#define POPKV_GEN(T, NW)                                                                          \
    score_generic_kernel<T, NW><<<grid, kGenericThreads, 0, s>>>(                                 \
        static_cast<const T*>(queries), k_sign, k_mag, k_low, k_delta, head_to_kv, out, qh, d, g, \
        capacity, tokens, scale)
#define POPKV_GEN_T(T)                   \
    switch (words) {                     \
        case 1: POPKV_GEN(T, 1); break;  \
        case 2: POPKV_GEN(T, 2); break;  \
        case 3: POPKV_GEN(T, 3); break;  \
        case 4: POPKV_GEN(T, 4); break;  \
        case 5: POPKV_GEN(T, 5); break;  \
        case 6: POPKV_GEN(T, 6); break;  \
        case 7: POPKV_GEN(T, 7); break;  \
        default: POPKV_GEN(T, 8); break; \
    }
    if (queries_dtype == POPKV_DTYPE_F32) { POPKV_GEN_T(float) }
    else if (queries_dtype == POPKV_DTYPE_F16) { POPKV_GEN_T(__half) }
    else { POPKV_GEN_T(__nv_bfloat16) }
#undef POPKV_GEN_T
#undef POPKV_GEN
    return check_launch("popkv_score");
}
}  // namespace popkv

extern "C" int popkv_score(const void* queries, int queries_dtype, int64_t batch, int64_t q_heads,
                           int64_t head_dim, const int32_t* k_sign, const int32_t* k_mag,
                           const uint16_t* k_low, const uint16_t* k_delta, int64_t kv_heads,
                           int64_t capacity, const int64_t* head_to_kv, int64_t tokens,
                           int64_t dim_group_size, void* scores, int scores_dtype, void* stream) {
    return popkv::score_entry(queries, queries_dtype, batch, q_heads, head_dim, k_sign, k_mag, k_low,
                              k_delta, kv_heads, capacity, head_to_kv, tokens, dim_group_size, scores,
                              scores_dtype, stream, false);
}

extern "C" int popkv_score_popcount(const void* queries, int queries_dtype, int64_t batch, int64_t q_heads,
                                    int64_t head_dim, const int32_t* k_sign, const int32_t* k_mag,
                                    const uint16_t* k_low, const uint16_t* k_delta, int64_t kv_heads,
                                    int64_t capacity, const int64_t* head_to_kv, int64_t tokens,
                                    int64_t dim_group_size, void* scores, int scores_dtype, void* stream) {
    return popkv::score_entry(queries, queries_dtype, batch, q_heads, head_dim, k_sign, k_mag, k_low,
                              k_delta, kv_heads, capacity, head_to_kv, tokens, dim_group_size, scores,
                              scores_dtype, stream, true);
}

extern "C" int popkv_score_dispatch(int mode) {
    using namespace popkv;
    if (mode < 0 || mode > 2)
        return fail(POPKV_ERR_INVALID, "popkv_score_dispatch: mode must be 0 (auto), 1 (popcount) or 2 (fp8)");
    g_score_dispatch.store(mode, std::memory_order_relaxed);
    return POPKV_OK;
}

extern "C" int popkv_score_hist(const void* queries, int queries_dtype, int64_t batch, int64_t q_heads,
                                const int32_t* k_sign, const int32_t* k_mag, const uint16_t* k_low,
                                const uint16_t* k_delta, int64_t kv_heads, int64_t capacity,
                                const int64_t* head_to_kv, int64_t tokens, int64_t dim_group_size,
                                uint16_t* scores, uint32_t* hist, void* stream) {
    using namespace popkv;
    if (!valid_dtype(queries_dtype)) return fail(POPKV_ERR_INVALID, "queries must be fp32/fp16/bf16");
    int st = check_score_common(batch, q_heads, kv_heads, capacity, tokens, dim_group_size, head_to_kv);
    if (st != POPKV_OK) return st;
    if (q_heads / kv_heads > kMaxHistHeads)
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_score_hist: more than %d query heads per KV head",
                    kMaxHistHeads);
    if (batch == 0) return POPKV_OK;
    if (!queries || !k_sign || !k_mag || !k_low || !k_delta || !scores || !hist)
        return fail(POPKV_ERR_INVALID, "popkv_score_hist: null pointer");
    if (!aligned(k_sign, 16) || !aligned(k_mag, 16) || !aligned(k_low, 16) || !aligned(k_delta, 16))
        return fail(POPKV_ERR_INVALID, "packed planes must be 16-byte aligned");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
#define POPKV_SH(G_, T_)                                                                             \
    return launch_score128_hist<G_, T_, true>(queries, batch, q_heads, k_sign, k_mag, k_low, k_delta, \
                                               kv_heads, capacity, head_to_kv, tokens, scores, hist, s)
#define POPKV_SH_T(T_)                         \
    if (dim_group_size == 16) { POPKV_SH(16, T_); } \
    if (dim_group_size == 32) { POPKV_SH(32, T_); } \
    POPKV_SH(64, T_);
    if (queries_dtype == POPKV_DTYPE_F32) { POPKV_SH_T(float) }
    if (queries_dtype == POPKV_DTYPE_F16) { POPKV_SH_T(__half) }
    POPKV_SH_T(__nv_bfloat16)
#undef POPKV_SH_T
#undef POPKV_SH
}

extern "C" int popkv_score_dyn(const void* queries, int queries_dtype, int64_t batch, int64_t q_heads,
                               const int32_t* k_sign, const int32_t* k_mag, const uint16_t* k_low,
                               const uint16_t* k_delta, int64_t kv_heads, int64_t capacity,
                               const int64_t* head_to_kv, const int64_t* tokens_dev,
                               int64_t max_tokens, int64_t dim_group_size, uint16_t* scores,
                               int64_t score_stride, void* stream) {
    using namespace popkv;
    if (!valid_dtype(queries_dtype)) return fail(POPKV_ERR_INVALID, "queries must be fp32/fp16/bf16");
    int st = check_score_common(batch, q_heads, kv_heads, capacity, max_tokens, dim_group_size, head_to_kv);
    if (st != POPKV_OK) return st;
    if (q_heads / kv_heads > kMaxGroupHeads)
        return fail(POPKV_ERR_UNSUPPORTED, "more than %d query heads per KV head", kMaxGroupHeads);
    if (score_stride < max_tokens) return fail(POPKV_ERR_INVALID, "popkv_score_dyn: score_stride < max_tokens");
    if (batch == 0) return POPKV_OK;
    if (!queries || !k_sign || !k_mag || !k_low || !k_delta || !scores || !tokens_dev)
        return fail(POPKV_ERR_INVALID, "popkv_score_dyn: null pointer");
    if (!aligned(k_sign, 16) || !aligned(k_mag, 16) || !aligned(k_low, 16) || !aligned(k_delta, 16))
        return fail(POPKV_ERR_INVALID, "packed planes must be 16-byte aligned");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    auto by_g = [&](auto tag) -> int {
        using QT = decltype(tag);
        const QT* q = static_cast<const QT*>(queries);
#define POPKV_SD(G_)                                                                                  \
    return launch_score128<G_, QT, true>(q, nullptr, nullptr, nullptr, nullptr, batch, q_heads, k_sign, \
                                         k_mag, k_low, k_delta, kv_heads, capacity, head_to_kv,         \
                                         max_tokens, scores, s, score_stride, tokens_dev)
        if (dim_group_size == 16) POPKV_SD(16);
        if (dim_group_size == 32) POPKV_SD(32);
        POPKV_SD(64);
#undef POPKV_SD
    };
    if (queries_dtype == POPKV_DTYPE_F32) return by_g(float{});
    if (queries_dtype == POPKV_DTYPE_F16) return by_g(__half{});
    return by_g(__nv_bfloat16{});
}
