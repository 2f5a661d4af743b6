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
#include <cstdint>

#include "common.cuh"

namespace popkv {
namespace {

constexpr int kEncodeWarps = 4;

// ---------------------------------------------------------------------------
// Query encoding: whole-head thresholds, sequential representative sums.
// ---------------------------------------------------------------------------

// Encodes one query row with one warp.  `scratch` holds 2 * 32 * W floats.
template <typename T, int W>
__device__ void encode_query_row(const T* __restrict__ q, int head_dim, int G, int lane,
                                 float* scratch, uint32_t* sign_out, uint32_t* mag_out,
                                 float* low_out, float* delta_out) {
    float v[W];
    float mn = INFINITY, mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < W; ++w) {
        const int d = w * 32 + lane;
        v[w] = d < head_dim ? load_float(q + d) : 0.0f;
        if (d < head_dim) {
            mn = fminf(mn, v[w]);
            mx = fmaxf(mx, v[w]);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xFFFFFFFFu, mn, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    }
    const float neg = __fmul_rn(mn, 0.5f), pos = __fmul_rn(mx, 0.5f);
    float* lows = scratch;
    float* highs = scratch + 32 * W;
    uint32_t sw[W], mw[W], vw[W];
#pragma unroll
    for (int w = 0; w < W; ++w) {
        const int d = w * 32 + lane;
        const bool valid = d < head_dim;
        const bool sign = valid && v[w] >= 0.0f;
        const bool mag = valid && (sign ? (v[w] > pos) : (v[w] < neg));
        sw[w] = __ballot_sync(0xFFFFFFFFu, sign);
        mw[w] = __ballot_sync(0xFFFFFFFFu, mag);
        vw[w] = __ballot_sync(0xFFFFFFFFu, valid);
        const float a = fabsf(v[w]);
        lows[d] = (valid && !mag) ? a : 0.0f;
        highs[d] = mag ? a : 0.0f;
        if (lane == w) {
            sign_out[w] = sw[w];
            mag_out[w] = mw[w];
        }
    }
    __syncwarp();
    const int reps = (head_dim + G - 1) / G;
    if (lane < reps) {
        const int start = lane * G;
        const int end = min(start + G, head_dim);
        float low_sum = 0.0f, high_sum = 0.0f;
        for (int d = start; d < end; ++d) {  // sequential, as popkv_ext.cu:942-947
            low_sum = __fadd_rn(low_sum, lows[d]);
            high_sum = __fadd_rn(high_sum, highs[d]);
        }
        int low_count = 0, high_count = 0;
#pragma unroll
        for (int w = 0; w < W; ++w) {
            const int ws = w * 32;
            const int b = max(start, ws) - ws, e = min(end, ws + 32) - ws;
            if (e > b) {
                const uint32_t m = (e - b == 32) ? 0xFFFFFFFFu : (((1u << (e - b)) - 1u) << b);
                low_count += __popc(vw[w] & ~mw[w] & m);
                high_count += __popc(mw[w] & m);
            }
        }
        float low, delta;
        bucket_means(low_sum, low_count, high_sum, high_count, low, delta);
        low_out[lane] = low;
        delta_out[lane] = delta;
    }
    __syncwarp();
}

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
constexpr int kTokensPerThread = 2;
constexpr int kScoreTile = kScoreThreads * kTokensPerThread;
constexpr int kMaxGroupHeads = 16;

// Per query head, per representative group r: the query words it reads and the
// constants that depend on the query only.
template <int G>
struct QueryState {
    static constexpr int R = 128 / G;
    uint32_t qs[4];
    uint32_t qm[4];   // magnitude words (masked per rep inside the loop for G16)
    int pq[R];        // popc(qm restricted to r)
    float ql[R];
    float dq[R];
};

template <int G>
__device__ __forceinline__ void finish_state(QueryState<G>& st) {
    constexpr int R = QueryState<G>::R;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        if constexpr (G == 16) st.pq[r] = __popc(st.qm[r >> 1] & ((r & 1) ? 0xFFFF0000u : 0x0000FFFFu));
        else if constexpr (G == 32) st.pq[r] = __popc(st.qm[r]);
        else st.pq[r] = __popc(st.qm[2 * r]) + __popc(st.qm[2 * r + 1]);
    }
}

template <int G, typename QT, bool RAW>
__global__ void __launch_bounds__(kScoreThreads) score128_kernel(
    const QT* __restrict__ queries, const int32_t* __restrict__ q_sign,
    const int32_t* __restrict__ q_mag, const float* __restrict__ q_low,
    const float* __restrict__ q_delta, const int32_t* __restrict__ k_sign,
    const int32_t* __restrict__ k_mag, const uint16_t* __restrict__ k_low,
    const uint16_t* __restrict__ k_delta, const int64_t* __restrict__ head_to_kv,
    uint16_t* __restrict__ scores, int q_heads, int group_heads, int64_t capacity,
    int64_t tokens, float scale) {
    constexpr int R = 128 / G;
    __shared__ QueryState<G> states[kMaxGroupHeads];
    __shared__ float scratch[kScoreThreads / 32][2 * 32 * 4];

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
    __syncthreads();
    if (threadIdx.x < group_heads) finish_state<G>(states[threadIdx.x]);
    __syncthreads();

    const int64_t tile0 = static_cast<int64_t>(blockIdx.x) * kScoreTile;
    const uint4* sign4 = reinterpret_cast<const uint4*>(k_sign) + kvh * capacity;
    const uint4* mag4 = reinterpret_cast<const uint4*>(k_mag) + kvh * capacity;
    const uint16_t* lowp = k_low + kvh * capacity * R;
    const uint16_t* deltap = k_delta + kvh * capacity * R;

    // Token-side data of this thread's tokens.
    uint32_t ks[kTokensPerThread][4], km[kTokensPerThread][4];
    float kl[kTokensPerThread][R], dk[kTokensPerThread][R];
    int pk[kTokensPerThread][R];
    bool live[kTokensPerThread];
#pragma unroll
    for (int i = 0; i < kTokensPerThread; ++i) {
        const int64_t t = tile0 + threadIdx.x + i * kScoreThreads;
        live[i] = t < tokens;
        const int64_t tt = live[i] ? t : 0;
        const uint4 s4 = sign4[tt], m4 = mag4[tt];
        ks[i][0] = s4.x; ks[i][1] = s4.y; ks[i][2] = s4.z; ks[i][3] = s4.w;
        km[i][0] = m4.x; km[i][1] = m4.y; km[i][2] = m4.z; km[i][3] = m4.w;
        if constexpr (R == 8) {
            const uint4 l4 = reinterpret_cast<const uint4*>(lowp)[tt];
            const uint4 d4 = reinterpret_cast<const uint4*>(deltap)[tt];
            const uint32_t lw[4] = {l4.x, l4.y, l4.z, l4.w}, dw[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                kl[i][2 * j] = half_bits_to_float(static_cast<uint16_t>(lw[j] & 0xFFFFu));
                kl[i][2 * j + 1] = half_bits_to_float(static_cast<uint16_t>(lw[j] >> 16));
                dk[i][2 * j] = half_bits_to_float(static_cast<uint16_t>(dw[j] & 0xFFFFu));
                dk[i][2 * j + 1] = half_bits_to_float(static_cast<uint16_t>(dw[j] >> 16));
            }
        } else if constexpr (R == 4) {
            const uint2 l2 = reinterpret_cast<const uint2*>(lowp)[tt];
            const uint2 d2 = reinterpret_cast<const uint2*>(deltap)[tt];
            const uint32_t lw[2] = {l2.x, l2.y}, dw[2] = {d2.x, d2.y};
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                kl[i][2 * j] = half_bits_to_float(static_cast<uint16_t>(lw[j] & 0xFFFFu));
                kl[i][2 * j + 1] = half_bits_to_float(static_cast<uint16_t>(lw[j] >> 16));
                dk[i][2 * j] = half_bits_to_float(static_cast<uint16_t>(dw[j] & 0xFFFFu));
                dk[i][2 * j + 1] = half_bits_to_float(static_cast<uint16_t>(dw[j] >> 16));
            }
        } else {
            const uint32_t lw = reinterpret_cast<const uint32_t*>(lowp)[tt];
            const uint32_t dw = reinterpret_cast<const uint32_t*>(deltap)[tt];
            kl[i][0] = half_bits_to_float(static_cast<uint16_t>(lw & 0xFFFFu));
            kl[i][1] = half_bits_to_float(static_cast<uint16_t>(lw >> 16));
            dk[i][0] = half_bits_to_float(static_cast<uint16_t>(dw & 0xFFFFu));
            dk[i][1] = half_bits_to_float(static_cast<uint16_t>(dw >> 16));
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            if constexpr (G == 16) pk[i][r] = __popc(km[i][r >> 1] & ((r & 1) ? 0xFFFF0000u : 0x0000FFFFu));
            else if constexpr (G == 32) pk[i][r] = __popc(km[i][r]);
            else pk[i][r] = __popc(km[i][2 * r]) + __popc(km[i][2 * r + 1]);
        }
    }

    for (int h = 0; h < group_heads; ++h) {
        const QueryState<G>& st = states[h];
        uint16_t* out = scores + (row0 + h) * tokens;
#pragma unroll
        for (int i = 0; i < kTokensPerThread; ++i) {
            float total = 0.0f;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                int c_sign, c_q, c_k, c_qk;
                if constexpr (G == 64) {
                    int p1 = 0, p2 = 0, p3 = 0, p4 = 0, p5 = 0;
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        const int w = 2 * r + half;
                        const uint32_t match = ~(st.qs[w] ^ ks[i][w]);
                        const uint32_t both = st.qm[w] & km[i][w];
                        p1 += __popc(match);
                        p2 += __popc(match & st.qm[w]);
                        p3 += __popc(match & km[i][w]);
                        p4 += __popc(match & both);
                        p5 += __popc(both);
                    }
                    c_sign = 2 * p1 - 64;
                    c_q = 2 * p2 - st.pq[r];
                    c_k = 2 * p3 - pk[i][r];
                    c_qk = 2 * p4 - p5;
                } else {
                    const int w = (G == 16) ? (r >> 1) : r;
                    const uint32_t m = (G == 16) ? ((r & 1) ? 0xFFFF0000u : 0x0000FFFFu) : 0xFFFFFFFFu;
                    const uint32_t match = ~(st.qs[w] ^ ks[i][w]) & m;
                    const uint32_t qm = st.qm[w] & m;
                    const uint32_t kmr = km[i][w] & m;
                    const uint32_t both = qm & kmr;
                    c_sign = 2 * __popc(match) - G;
                    c_q = 2 * __popc(match & qm) - st.pq[r];
                    c_k = 2 * __popc(match & kmr) - pk[i][r];
                    c_qk = 2 * __popc(match & both) - __popc(both);
                }
                const float ql = st.ql[r], dq = st.dq[r];
                const float t1 = __fmul_rn(ql, kl[i][r]);
                const float t2 = __fmul_rn(dq, kl[i][r]);
                const float t3 = __fmul_rn(ql, dk[i][r]);
                const float t4 = __fmul_rn(__fmul_rn(dq, dk[i][r]), small_int_to_float(c_qk));
                const float chain = __fmaf_rn(t1, small_int_to_float(c_sign),
                                              __fmaf_rn(t2, small_int_to_float(c_q),
                                                        __fmaf_rn(t3, small_int_to_float(c_k), t4)));
                total = __fadd_rn(total, chain);
            }
            if (live[i]) {
                const int64_t t = tile0 + threadIdx.x + i * kScoreThreads;
                out[t] = float_to_half_bits(__fmul_rn(total, scale));
            }
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

template <int G, typename QT, bool RAW>
int launch_score128(const void* queries, const int32_t* q_sign, const int32_t* q_mag,
                    const float* q_low, const float* q_delta, int64_t batch, int64_t q_heads,
                    const int32_t* k_sign, const int32_t* k_mag, const uint16_t* k_low,
                    const uint16_t* k_delta, int64_t kv_heads, int64_t capacity,
                    const int64_t* head_to_kv, int64_t tokens, uint16_t* scores,
                    cudaStream_t stream) {
    const int group_heads = static_cast<int>(q_heads / kv_heads);
    const int64_t tiles = (tokens + kScoreTile - 1) / kScoreTile;
    dim3 grid(static_cast<unsigned>(tiles), static_cast<unsigned>(batch * kv_heads));
    score128_kernel<G, QT, RAW><<<grid, kScoreThreads, 0, stream>>>(
        static_cast<const QT*>(queries), q_sign, q_mag, q_low, q_delta, k_sign, k_mag, k_low,
        k_delta, head_to_kv, scores, static_cast<int>(q_heads), group_heads, capacity, tokens,
        score_scale_for(128));
    return check_launch("popkv_score");
}

template <typename QT, bool RAW>
int dispatch_score128(int64_t g, const void* queries, const int32_t* q_sign, const int32_t* q_mag,
                      const float* q_low, const float* q_delta, int64_t batch, int64_t q_heads,
                      const int32_t* k_sign, const int32_t* k_mag, const uint16_t* k_low,
                      const uint16_t* k_delta, int64_t kv_heads, int64_t capacity,
                      const int64_t* head_to_kv, int64_t tokens, uint16_t* scores,
                      cudaStream_t stream) {
    if (g == 16)
        return launch_score128<16, QT, RAW>(queries, q_sign, q_mag, q_low, q_delta, batch, q_heads,
                                            k_sign, k_mag, k_low, k_delta, kv_heads, capacity,
                                            head_to_kv, tokens, scores, stream);
    if (g == 32)
        return launch_score128<32, QT, RAW>(queries, q_sign, q_mag, q_low, q_delta, batch, q_heads,
                                            k_sign, k_mag, k_low, k_delta, kv_heads, capacity,
                                            head_to_kv, tokens, scores, stream);
    return launch_score128<64, QT, RAW>(queries, q_sign, q_mag, q_low, q_delta, batch, q_heads,
                                        k_sign, k_mag, k_low, k_delta, kv_heads, capacity,
                                        head_to_kv, tokens, scores, stream);
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

}  // namespace
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

extern "C" int popkv_score(const void* queries, int queries_dtype, int64_t batch, int64_t q_heads,
                           int64_t head_dim, const int32_t* k_sign, const int32_t* k_mag,
                           const uint16_t* k_low, const uint16_t* k_delta, int64_t kv_heads,
                           int64_t capacity, const int64_t* head_to_kv, int64_t tokens,
                           int64_t dim_group_size, void* scores, int scores_dtype, void* stream) {
    using namespace popkv;
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
                                                  out, s);
        if (queries_dtype == POPKV_DTYPE_F16)
            return dispatch_score128<__half, true>(dim_group_size, queries, nullptr, nullptr, nullptr,
                                                   nullptr, batch, q_heads, k_sign, k_mag, k_low,
                                                   k_delta, kv_heads, capacity, head_to_kv, tokens,
                                                   out, s);
        return dispatch_score128<__nv_bfloat16, true>(dim_group_size, queries, nullptr, nullptr,
                                                      nullptr, nullptr, batch, q_heads, k_sign,
                                                      k_mag, k_low, k_delta, kv_heads, capacity,
                                                      head_to_kv, tokens, out, s);
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
