// Device building blocks of the popcount scorer, shared by the standalone
// score kernels (score.cu) and the fused retrieval kernel (retrieve.cu).
//
// Reference arithmetic: csrc/popkv_ext.cu:502-515 (four-count reconstruction),
// :757-876 (GQA-tiled head_dim-128 scorer), :911-957 (query encoding).
#pragma once

#include <cstdint>

#include "common.cuh"

namespace popkv {

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


// One key token's planes and representatives, widened for scoring.
template <int G>
struct TokenPlanes {
    static constexpr int R = 128 / G;
    uint32_t ks[4], km[4];
    float kl[R], dk[R];
    int pk[R];  // popc(km restricted to r)
};

template <int G>
__device__ __forceinline__ void load_token(const uint4* __restrict__ sign4, const uint4* __restrict__ mag4,
                                           const uint16_t* __restrict__ lowp,
                                           const uint16_t* __restrict__ deltap, int64_t t,
                                           TokenPlanes<G>& tp) {
    constexpr int R = 128 / G;
    const uint4 s4 = sign4[t], m4 = mag4[t];
    tp.ks[0] = s4.x; tp.ks[1] = s4.y; tp.ks[2] = s4.z; tp.ks[3] = s4.w;
    tp.km[0] = m4.x; tp.km[1] = m4.y; tp.km[2] = m4.z; tp.km[3] = m4.w;
    if constexpr (R == 8) {
        const uint4 l4 = reinterpret_cast<const uint4*>(lowp)[t];
        const uint4 d4 = reinterpret_cast<const uint4*>(deltap)[t];
        const uint32_t lw[4] = {l4.x, l4.y, l4.z, l4.w}, dw[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            tp.kl[2 * j] = half_bits_to_float(static_cast<uint16_t>(lw[j] & 0xFFFFu));
            tp.kl[2 * j + 1] = half_bits_to_float(static_cast<uint16_t>(lw[j] >> 16));
            tp.dk[2 * j] = half_bits_to_float(static_cast<uint16_t>(dw[j] & 0xFFFFu));
            tp.dk[2 * j + 1] = half_bits_to_float(static_cast<uint16_t>(dw[j] >> 16));
        }
    } else if constexpr (R == 4) {
        const uint2 l2 = reinterpret_cast<const uint2*>(lowp)[t];
        const uint2 d2 = reinterpret_cast<const uint2*>(deltap)[t];
        const uint32_t lw[2] = {l2.x, l2.y}, dw[2] = {d2.x, d2.y};
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            tp.kl[2 * j] = half_bits_to_float(static_cast<uint16_t>(lw[j] & 0xFFFFu));
            tp.kl[2 * j + 1] = half_bits_to_float(static_cast<uint16_t>(lw[j] >> 16));
            tp.dk[2 * j] = half_bits_to_float(static_cast<uint16_t>(dw[j] & 0xFFFFu));
            tp.dk[2 * j + 1] = half_bits_to_float(static_cast<uint16_t>(dw[j] >> 16));
        }
    } else {
        const uint32_t lw = reinterpret_cast<const uint32_t*>(lowp)[t];
        const uint32_t dw = reinterpret_cast<const uint32_t*>(deltap)[t];
        tp.kl[0] = half_bits_to_float(static_cast<uint16_t>(lw & 0xFFFFu));
        tp.kl[1] = half_bits_to_float(static_cast<uint16_t>(lw >> 16));
        tp.dk[0] = half_bits_to_float(static_cast<uint16_t>(dw & 0xFFFFu));
        tp.dk[1] = half_bits_to_float(static_cast<uint16_t>(dw >> 16));
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
        if constexpr (G == 16) tp.pk[r] = __popc(tp.km[r >> 1] & ((r & 1) ? 0xFFFF0000u : 0x0000FFFFu));
        else if constexpr (G == 32) tp.pk[r] = __popc(tp.km[r]);
        else tp.pk[r] = __popc(tp.km[2 * r]) + __popc(tp.km[2 * r + 1]);
    }
}

// Popcounts of the two 16-bit halves of x, in bytes 0 and 2 of the result,
// computed on the integer pipe.
__device__ __forceinline__ uint32_t swar_half_counts(uint32_t x) {
    uint32_t v = x - ((x >> 1) & 0x55555555u);
    v = (v & 0x33333333u) + ((v >> 2) & 0x33333333u);
    v = (v + (v >> 4)) & 0x0F0F0F0Fu;
    return v + (v >> 8);
}

// Unscaled score of one (query head, key token) pair: the sum over
// representative groups of fma(ql*kl, c_sign, fma(dq*kl, c_q, fma(ql*dk, c_k,
// (dq*dk)*c_qk))), every operation rounded as written.
template <int G>
__device__ __forceinline__ float score_token(const QueryState<G>& st, const TokenPlanes<G>& tp) {
    constexpr int R = 128 / G;
    float total = 0.0f;
    // G16: the two groups of each 32-bit word share one SWAR popcount of the
    // sign agreements (on the integer pipe, not the popcount pipe).
    uint32_t agree[4] = {0u, 0u, 0u, 0u};
    if constexpr (G == 16) {
#pragma unroll
        for (int w = 0; w < 4; ++w) agree[w] = swar_half_counts(~(st.qs[w] ^ tp.ks[w]));
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
        int c_sign, c_q, c_k, c_qk;
        if constexpr (G == 64) {
            int p1 = 0, p2 = 0, p3 = 0, p4 = 0, p5 = 0;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int w = 2 * r + half;
                const uint32_t match = ~(st.qs[w] ^ tp.ks[w]);
                const uint32_t both = st.qm[w] & tp.km[w];
                p1 += __popc(match);
                p2 += __popc(match & st.qm[w]);
                p3 += __popc(match & tp.km[w]);
                p4 += __popc(match & both);
                p5 += __popc(both);
            }
            c_sign = 2 * p1 - 64;
            c_q = 2 * p2 - st.pq[r];
            c_k = 2 * p3 - tp.pk[r];
            c_qk = 2 * p4 - p5;
        } else {
            const int w = (G == 16) ? (r >> 1) : r;
            const uint32_t m = (G == 16) ? ((r & 1) ? 0xFFFF0000u : 0x0000FFFFu) : 0xFFFFFFFFu;
            const uint32_t match = ~(st.qs[w] ^ tp.ks[w]) & m;
            const uint32_t qm = st.qm[w] & m;
            const uint32_t kmr = tp.km[w] & m;
            const uint32_t both = qm & kmr;
            if constexpr (G == 16) {
                const uint32_t v = agree[w];
                c_sign = 2 * static_cast<int>((r & 1) ? ((v >> 16) & 0xFFu) : (v & 0xFFu)) - G;
            } else {
                c_sign = 2 * __popc(match) - G;
            }
            c_q = 2 * __popc(match & qm) - st.pq[r];
            c_k = 2 * __popc(match & kmr) - tp.pk[r];
            c_qk = 2 * __popc(match & both) - __popc(both);
        }
        const float ql = st.ql[r], dq = st.dq[r];
        const float t1 = __fmul_rn(ql, tp.kl[r]);
        const float t2 = __fmul_rn(dq, tp.kl[r]);
        const float t3 = __fmul_rn(ql, tp.dk[r]);
        const float t4 = __fmul_rn(__fmul_rn(dq, tp.dk[r]), small_int_to_float(c_qk));
        const float chain = __fmaf_rn(t1, small_int_to_float(c_sign),
                                      __fmaf_rn(t2, small_int_to_float(c_q),
                                                __fmaf_rn(t3, small_int_to_float(c_k), t4)));
        total = __fadd_rn(total, chain);
    }
    return total;
}

}  // namespace popkv
