// head_dim-128 popcount scorer on the 5th-generation tensor cores: the four
// counts of every (key token, query head, representative group) come out of
// tcgen05.mma kind::f8f6f4 as exact fp32 values in tensor memory.
//
// Reference arithmetic: csrc/popkv_ext.cu:502-515 (four-count reconstruction)
// and :757-876 (GQA-tiled head_dim-128 scorer, fp16 out).  The scores are bit
// for bit those of score128_kernel (score.cu) and of the CPU oracle.
//
// The counts as dot products.  With s = +1 for a set sign bit and -1 otherwise,
// and r a representative group's dims,
//   c_sign = 2 popc(match & r)        - |r|        = sum_r s_q s_k
//   c_q    = 2 popc(match & qm & r)   - popc(qm&r)  = sum_r (qm s_q) s_k
//   c_k    = 2 popc(match & km & r)   - popc(km&r)  = sum_r s_q (km s_k)
//   c_qk   = 2 popc(match & both & r) - popc(both)  = sum_r (qm s_q)(km s_k)
// i.e. products of the query vectors {s_q, qm s_q} with the key vectors
// {s_k, km s_k}, all in {-1, 0, +1}.  In e4m3 those are exact (0x38 = +1,
// 0xB8 = -1, 0x00 = 0) and so is a sum of 128 of them in fp32.
//
// Per tile of 128 key tokens and per key plane p (0: s_k, 1: km s_k):
//   A (128 x 128 fp8, tensor memory): row = token, the plane's 128 dims
//   B (128 x N fp8, shared memory, K-major): column (head, qt, group r) =
//     (qt ? qm s_q : s_q) of the head restricted to group r, N = 8 R
//   D_p (128 x N fp32, tensor memory) = A_p B, four K-blocks of 32 accumulated
// so D_0 holds c_sign (qt 0) and c_q (qt 1), D_1 holds c_k and c_qk, for every
// head and group of the token, in its own tensor-memory lane.  Two threads own
// a token (warps w and w+4 share TMEM lane quarter w): thread group P expands
// words 2P, 2P+1 of both planes into A and runs the fp32 chain of heads 2P,
// 2P+1 -- the reference's fma(ql*kl, c_sign, fma(dq*kl, c_q, fma(ql*dk, c_k,
// (dq*dk)*c_qk))) -- on groups (r, r+1) at once as packed f32x2 ops, summing
// the groups in order.
//
// Key bits become fp8 bytes with a shift, one prmt in sign-replicate mode (bit
// 7 of each byte -> 0x00/0xFF) and one logic op.  The k order inside a word is
// a permutation both operands share: A column 8w + s of a row holds, in byte e,
// dim 32w + 8e + 7 - s (s = 0..7).
//
// Pipeline per CTA: lane 0 of the last warp streams plane tiles (sign,
// magnitude, low, delta; 128 tokens) into a 4-stage shared-memory ring with
// cp.async.bulk copies on mbarriers.  A is double-buffered in tensor memory, so
// tile i+1 is expanded while thread 0's MMAs of tile i run; D is read back with
// tcgen05.ld.  Tensor memory: A0 [0, 64), A1 [64, 128), D [128, 128 + 16 R)
// columns of a 256-column allocation, so two CTAs share an SM.  Every wait is
// bounded; a wait that gives up is counted in g_score_tc8_timeouts and the
// kernel carries on to its end.
#pragma once

#include <cstdint>

#include "common.cuh"
#include "mbarrier.cuh"
#include "score_impl.cuh"

namespace popkv {
namespace tc8 {

constexpr int kWarps = 8;            // two threads per token: warps w and w+4 share TMEM lane quarter w
constexpr int kThreads = kWarps * 32;
constexpr int kTile = 128;          // tokens per tile (MMA M)
constexpr int kStages = 4;          // plane ring depth
constexpr int kMaxHeads = 4;        // query heads per KV head
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColA0 = 0, kColA1 = 64, kColD = 128;  // A buffers (two planes x 32 columns), D

template <int G>
struct Layout {
    static constexpr int R = 128 / G;
    static constexpr int N = 8 * R;                           // MMA N: 4 heads x 2 x R
    static constexpr int kStageBytes = kTile * (32 + 4 * R);  // sign, mag, low, delta
    static constexpr int kBBlockBytes = N * 32;               // one K-block of B
    static constexpr int kRingBytes = kStages * kStageBytes;
    static constexpr int kUsedBytes = kRingBytes + 4 * kBBlockBytes;  // ring + B (offset 1024-aligned)
    // Optional first-pass top-k histograms: 2048 bins per query head.
    static constexpr int kHistOffset = kUsedBytes;
    static constexpr int kHistBytes = kMaxHeads * 2048 * 4;
    // Padded so that at most two CTAs share an SM: a third CTA's 256-column
    // tensor-memory allocation would wait for one of them to finish.
    static constexpr int kSmemBytes = 80 * 1024;
    static_assert(kRingBytes % 1024 == 0, "B must start 1024-aligned");
    static_assert(kHistOffset % 16 == 0 && kHistOffset + kHistBytes <= kSmemBytes, "histograms fit the padding");
};

// Sign-replicated bytes: byte e of the result is 0xFF if bit 8e+7 of x is set, else 0.
__device__ __forceinline__ uint32_t byte_masks(uint32_t x) {
    uint32_t r;
    asm("prmt.b32 %0, %1, 0, 0xBA98;" : "=r"(r) : "r"(x));
    return r;
}

// e4m3 +-1 bytes from sign bits (bit 8e+7 of `x` set -> +1): 0xB8 (-1) with
// bit 7 cleared where the mask is set gives 0x38 (+1).
__device__ __forceinline__ uint32_t pm_one(uint32_t x) {
    uint32_t r;
    asm("lop3.b32 %0, %1, 0x80808080, 0xB8B8B8B8, 0x6a;" : "=r"(r) : "r"(byte_masks(x)));
    return r;
}

// fp16 half `which` (0: low, 1: high) of a 32-bit word, widened exactly.
__device__ __forceinline__ float half_of(uint32_t w, int which) {
    float f;
    if (which) asm("{.reg .b16 l, h; mov.b32 {l, h}, %1; cvt.f32.f16 %0, h;}" : "=f"(f) : "r"(w));
    else asm("{.reg .b16 l, h; mov.b32 {l, h}, %1; cvt.f32.f16 %0, l;}" : "=f"(f) : "r"(w));
    return f;
}

// The reference's score term of groups (r, r+1) at once; c* = {group r, group r+1}.
__device__ __forceinline__ float2 chain_pair(float2 ql, float2 dq, float2 kl, float2 dk, float2 c_sign,
                                             float2 c_q, float2 c_k, float2 c_qk) {
    const float2 t1 = __fmul2_rn(ql, kl), t2 = __fmul2_rn(dq, kl), t3 = __fmul2_rn(ql, dk);
    const float2 t4 = __fmul2_rn(__fmul2_rn(dq, dk), c_qk);
    return __ffma2_rn(t1, c_sign, __ffma2_rn(t2, c_q, __ffma2_rn(t3, c_k, t4)));
}

// Shared-memory matrix descriptor, no swizzle, K-major: 8-row x 16-byte core
// matrices of 128 contiguous bytes; the next 16 bytes along K sit 128 bytes on,
// the next 8 rows 256 bytes on.  Version 1 in bits 46-47.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t addr) {
    return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(128 >> 4) << 16) |
           (static_cast<uint64_t>(256 >> 4) << 32) | (1ull << 46);
}
__device__ __forceinline__ uint32_t kblock_offset(int row, int c16) {
    return static_cast<uint32_t>((row >> 3) * 256 + c16 * 128 + (row & 7) * 16);
}

// Instruction descriptor of kind::f8f6f4: fp32 D (bits 4-5 = 1), e4m3 A and B
// (bits 7-9, 10-12 = 0), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
template <int N>
constexpr uint32_t idesc() {
    return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(kTile >> 4) << 24);
}

__device__ __forceinline__ void mma_f8(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t id,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n\t}\n"
        :: "r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(id), "r"(accumulate) : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* mbar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_addr(mbar)) : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 8 consecutive tensor-memory columns of this thread's lane.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
                 :: "r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]),
                    "r"(v[7]) : "memory");
}

// X consecutive tensor-memory columns of this thread's lane, as X/2 pairs.
template <int X>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float2 (&v)[X / 2]);

template <>
__device__ __forceinline__ void tmem_ld<2>(uint32_t taddr, float2 (&v)[1]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0,%1}, [%2];"
                 : "=f"(v[0].x), "=f"(v[0].y) : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_ld<4>(uint32_t taddr, float2 (&v)[2]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v[0].x), "=f"(v[0].y), "=f"(v[1].x), "=f"(v[1].y) : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t taddr, float2 (&v)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=f"(v[0].x), "=f"(v[0].y), "=f"(v[1].x), "=f"(v[1].y), "=f"(v[2].x), "=f"(v[2].y),
                   "=f"(v[3].x), "=f"(v[3].y) : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, float2 (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=f"(v[0].x), "=f"(v[0].y), "=f"(v[1].x), "=f"(v[1].y), "=f"(v[2].x), "=f"(v[2].y),
                   "=f"(v[3].x), "=f"(v[3].y), "=f"(v[4].x), "=f"(v[4].y), "=f"(v[5].x), "=f"(v[5].y),
                   "=f"(v[6].x), "=f"(v[6].y), "=f"(v[7].x), "=f"(v[7].y) : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// fp8 A rows of one key word: register s holds, in byte e, dim 8e + 7 - s of the
// word; `sgn` = s_k, `mag` = km s_k.
__device__ __forceinline__ void expand_word(uint32_t ks, uint32_t km, uint32_t (&sgn)[8], uint32_t (&mag)[8]) {
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        sgn[s] = pm_one(ks << s);
        mag[s] = sgn[s] & byte_masks(km << s);
    }
}

}  // namespace tc8

// Bounded waits of the tensor-core scorer that gave up (read by popkv_score_tc_timeouts()).
__device__ unsigned int g_score_tc8_timeouts = 0;



__device__ __forceinline__ void tc8_wait(uint64_t* bar, uint32_t parity) {
    if (!mbar_wait(bar, parity)) atomicAdd(&g_score_tc8_timeouts, 1u);
}

// Grid: x = chunks of one (batch, GQA group)'s tiles, y = batch * groups; at
// most kMaxHeads query heads per KV head.  With HIST the kernel also counts
// every score's top 11 key bits (order_key16 >> 5) per query row into `hist`
// [rows][2048] (zeros on entry): per-CTA shared-memory histograms, flushed with
// one global atomic per non-empty bin (the top-k's first radix pass).
template <int G, typename QT, bool RAW, bool HIST>
__global__ void __launch_bounds__(tc8::kThreads, 2) score128_tc8_kernel(
    const QT* __restrict__ queries, const int32_t* __restrict__ q_sign, const int32_t* __restrict__ q_mag,
    const float* __restrict__ q_low, const float* __restrict__ q_delta, const int32_t* __restrict__ k_sign,
    const int32_t* __restrict__ k_mag, const uint16_t* __restrict__ k_low, const uint16_t* __restrict__ k_delta,
    const int64_t* __restrict__ head_to_kv, uint16_t* __restrict__ scores, int q_heads, int group_heads,
    int64_t capacity, int64_t tokens, float scale, int64_t score_stride, const int64_t* __restrict__ dyn_tokens,
    int chunks, uint32_t* __restrict__ hist) {
    using L = tc8::Layout<G>;
    constexpr int R = L::R, N = L::N, S = tc8::kStages;
    extern __shared__ __align__(1024) unsigned char tc8_smem[];
    unsigned char* sB = tc8_smem + L::kRingBytes;
    uint32_t* shist = reinterpret_cast<uint32_t*>(tc8_smem + L::kHistOffset);  // [head][2048], with `hist`
    __shared__ QueryState<G> states[tc8::kMaxHeads];
    __shared__ float enc_scratch[tc8::kMaxHeads][2 * 32 * 4];
    __shared__ float4 qdq[tc8::kMaxHeads][R / 2];  // {ql_r, ql_r+1, dq_r, dq_r+1}
    __shared__ __align__(8) uint64_t full_bar[S];
    __shared__ __align__(8) uint64_t mma_bar;
    __shared__ uint32_t tmem_base;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int groups = q_heads / group_heads;
    const int64_t b = blockIdx.y / groups;
    const int grp = blockIdx.y % groups;
    const int qh0 = grp * group_heads;
    const int64_t row0 = b * q_heads + qh0;

    // Set-up that reads nothing a predecessor kernel writes runs before the
    // dependency wait: the head mapping (a read-only argument) and the stage
    // barriers.  Tensor memory is allocated only after the wait: a predecessor
    // that triggers this launch before allocating its own columns must never
    // find them taken by a CTA that is waiting for it.  Lane 0 of the last
    // warp streams the plane tiles; it issues the first kStages after the wait
    // while warps 0-3 encode the queries.
    const bool streamer = threadIdx.x == (tc8::kWarps - 1) * 32;
    const int64_t kvh = streamer ? head_to_kv[qh0] : 0;
    if (streamer) {
        for (int s = 0; s < S; ++s) mbar_init(&full_bar[s], 1);
        mbar_init(&mma_bar, 1);
    }
    pdl_wait();
    if (dyn_tokens) {
        const int64_t t = *dyn_tokens;
        tokens = t < 0 ? 0 : (t < tokens ? t : tokens);
    }
    const int64_t tiles = (tokens + tc8::kTile - 1) / tc8::kTile;
    const int64_t tile_begin = static_cast<int64_t>(blockIdx.x) * tiles / chunks;
    const int64_t tile_end = static_cast<int64_t>(blockIdx.x + 1) * tiles / chunks;
    if (tile_begin >= tile_end) {
        pdl_launch_dependents();
        return;
    }
    const int ntiles = static_cast<int>(tile_end - tile_begin);
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_addr(&tmem_base)), "r"(tc8::kTmemCols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }

    const unsigned char* sign_src = reinterpret_cast<const unsigned char*>(k_sign) + kvh * capacity * 16;
    const unsigned char* mag_src = reinterpret_cast<const unsigned char*>(k_mag) + kvh * capacity * 16;
    const unsigned char* low_src = reinterpret_cast<const unsigned char*>(k_low) + kvh * capacity * 2 * R;
    const unsigned char* delta_src = reinterpret_cast<const unsigned char*>(k_delta) + kvh * capacity * 2 * R;
    auto issue = [&](int i) {
        const int s = i % S;
        const int64_t t0 = (tile_begin + i) * tc8::kTile;
        const int64_t left = capacity - t0;
        const uint32_t n = static_cast<uint32_t>(left < tc8::kTile ? left : tc8::kTile);
        unsigned char* stage = tc8_smem + s * L::kStageBytes;
        mbar_arrive_expect_tx(&full_bar[s], n * (32u + 4u * R));
        bulk_copy_g2s(stage, sign_src + t0 * 16, n * 16u, &full_bar[s]);
        bulk_copy_g2s(stage + tc8::kTile * 16, mag_src + t0 * 16, n * 16u, &full_bar[s]);
        bulk_copy_g2s(stage + tc8::kTile * 32, low_src + t0 * 2 * R, n * 2u * R, &full_bar[s]);
        bulk_copy_g2s(stage + tc8::kTile * (32 + 2 * R), delta_src + t0 * 2 * R, n * 2u * R, &full_bar[s]);
    };
    if (streamer)
        for (int i = 0; i < ntiles && i < S; ++i) issue(i);

    if constexpr (HIST) {
        for (int i = threadIdx.x; i < group_heads * 512; i += tc8::kThreads)
            reinterpret_cast<uint4*>(shist)[i] = make_uint4(0u, 0u, 0u, 0u);
    }

    // ---- query side: states, then B (K-major fp8) and the {ql, dq} pairs ----
    if constexpr (RAW) {
        if (warp < group_heads) {
            encode_query_row<QT, 4>(queries + (row0 + warp) * 128, 128, G, lane, enc_scratch[warp],
                                    states[warp].qs, states[warp].qm, states[warp].ql, states[warp].dq);
        }
    } else {
        for (int i = threadIdx.x; i < group_heads * (8 + 2 * R); i += tc8::kThreads) {
            const int h = i / (8 + 2 * R), j = i % (8 + 2 * R);
            const int64_t qrow = row0 + h;
            if (j < 4) states[h].qs[j] = static_cast<uint32_t>(q_sign[qrow * 4 + j]);
            else if (j < 8) states[h].qm[j - 4] = static_cast<uint32_t>(q_mag[qrow * 4 + j - 4]);
            else if (j < 8 + R) states[h].ql[j - 8] = q_low[qrow * R + j - 8];
            else states[h].dq[j - 8 - R] = q_delta[qrow * R + j - 8 - R];
        }
    }
    __syncthreads();
    // B column n = P*4R + (hh*2 + qt)*R + r: head 2P + hh, s_q (qt 0) or qm s_q
    // (qt 1), restricted to group r.  K-block kb = word kb; the row's 32 bytes are
    // 8 words built like the A rows (word s, byte e: dim 32 kb + 8e + 7 - s).
    for (int item = threadIdx.x; item < 4 * N; item += tc8::kThreads) {
        const int kb = item / N, n = item % N;
        const int Pn = n / (4 * R), rem = n % (4 * R), hq = rem / R, r = rem % R;
        const int h = 2 * Pn + (hq >> 1), qt = hq & 1;
        uint32_t w[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
        if (h < group_heads) {
            uint32_t rep_bits;
            if constexpr (G == 16) rep_bits = r == 2 * kb ? 0x0000FFFFu : (r == 2 * kb + 1 ? 0xFFFF0000u : 0u);
            else if constexpr (G == 32) rep_bits = r == kb ? 0xFFFFFFFFu : 0u;
            else rep_bits = r == (kb >> 1) ? 0xFFFFFFFFu : 0u;
            const uint32_t qs = states[h].qs[kb];
            const uint32_t keep = qt ? (states[h].qm[kb] & rep_bits) : rep_bits;
#pragma unroll
            for (int sh = 0; sh < 8; ++sh) w[sh] = tc8::pm_one(qs << sh) & tc8::byte_masks(keep << sh);
        }
        unsigned char* dst = sB + kb * L::kBBlockBytes;
        *reinterpret_cast<uint4*>(dst + tc8::kblock_offset(n, 0)) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4*>(dst + tc8::kblock_offset(n, 1)) = make_uint4(w[4], w[5], w[6], w[7]);
    }
    if (threadIdx.x < tc8::kMaxHeads * (R / 2)) {
        const int h = threadIdx.x / (R / 2), p = threadIdx.x % (R / 2);
        qdq[h][p] = h < group_heads ? make_float4(states[h].ql[2 * p], states[h].ql[2 * p + 1],
                                                  states[h].dq[2 * p], states[h].dq[2 * p + 1])
                                    : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    fence_async_smem();  // B is read by the tensor core (async proxy)
    tc8::fence_before();
    __syncthreads();
    tc8::fence_after();
    const uint32_t tmem = tmem_base;
    const uint32_t b_addr = smem_addr(sB);

    // ---- per-thread roles: token `row` of the tile, words 2P, 2P+1, heads 2P, 2P+1 ----
    const int quarter = warp & 3, P = warp >> 2;
    const int row = 32 * quarter + lane;  // tensor-memory lane
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(32 * quarter) << 16);
    constexpr uint32_t kId = tc8::idesc<N>();

    // Expand tile j into A buffer `abuf`; keep the token's representative words.
    auto expand = [&](int j, uint32_t abuf, uint32_t (&lw)[R / 2], uint32_t (&dw)[R / 2]) {
        const int s = j % S;
        tc8_wait(&full_bar[s], (j / S) & 1);
        const unsigned char* stage = tc8_smem + s * L::kStageBytes;
        const uint2 ks = reinterpret_cast<const uint2*>(stage + row * 16)[P];
        const uint2 km = reinterpret_cast<const uint2*>(stage + tc8::kTile * 16 + row * 16)[P];
        const uint32_t* lo = reinterpret_cast<const uint32_t*>(stage + tc8::kTile * 32 + row * 2 * R);
        const uint32_t* de = reinterpret_cast<const uint32_t*>(stage + tc8::kTile * (32 + 2 * R) + row * 2 * R);
#pragma unroll
        for (int p = 0; p < R / 2; ++p) {
            lw[p] = lo[p];
            dw[p] = de[p];
        }
        uint32_t sg[8], mg[8];
        __syncwarp();  // converged for the .aligned tensor-memory stores
        tc8::expand_word(ks.x, km.x, sg, mg);
        tc8::tmem_st8(t_lane + abuf + 8 * (2 * P), sg);
        tc8::tmem_st8(t_lane + abuf + 32 + 8 * (2 * P), mg);
        tc8::expand_word(ks.y, km.y, sg, mg);
        tc8::tmem_st8(t_lane + abuf + 8 * (2 * P + 1), sg);
        tc8::tmem_st8(t_lane + abuf + 32 + 8 * (2 * P + 1), mg);
        tc8::tmem_wait_st();
    };
    // Thread 0: the eight MMAs of a tile (two planes x four K-blocks) and their commit.
    auto issue_mma = [&](uint32_t abuf) {
#pragma unroll
        for (int p = 0; p < 2; ++p) {
#pragma unroll
            for (int kb = 0; kb < 4; ++kb) {
                tc8::mma_f8(tmem + tc8::kColD + p * N, tmem + abuf + p * 32 + 8 * kb,
                            tc8::kmajor_desc(b_addr + kb * L::kBBlockBytes), kId, kb > 0 ? 1u : 0u);
            }
        }
        tc8::mma_commit(&mma_bar);
    };
    // Chains of heads 2P and 2P+1 for this thread's token of tile i.
    auto epilogue = [&](int i, const uint32_t (&lw)[R / 2], const uint32_t (&dw)[R / 2]) {
        float2 kl[R / 2], dk[R / 2];  // groups (2p, 2p+1)
#pragma unroll
        for (int p = 0; p < R / 2; ++p) {
            kl[p].x = tc8::half_of(lw[p], 0);
            kl[p].y = tc8::half_of(lw[p], 1);
            dk[p].x = tc8::half_of(dw[p], 0);
            dk[p].y = tc8::half_of(dw[p], 1);
        }
        const int64_t tok = (tile_begin + i) * tc8::kTile + row;
        const int h0 = 2 * P, h1 = 2 * P + 1;
        if (h0 >= group_heads) return;  // uniform over the warp
        __syncwarp();  // converged for the .aligned tensor-memory loads
        // Both heads' chains interleaved (independent dependency chains); each
        // head's groups are still summed in order.  Columns of head hh:
        // [qt 0: groups 0..R-1][qt 1: groups 0..R-1] from kColD + P*4R + hh*2R.
        // A missing second head (odd group) reads zero columns and is not stored.
        const uint32_t c0 = t_lane + tc8::kColD + P * 4 * R, c1 = c0 + 2 * R;
        float t0 = 0.0f, t1 = 0.0f;
        constexpr int H = R == 8 ? 2 : 1;  // column halves (register budget)
        constexpr int PP = R / 2 / H;      // group pairs per half
#pragma unroll
        for (int half = 0; half < H; ++half) {
            // [head][plane][qt] pairs of the half's groups
            float2 s0a[PP], s0b[PP], m0a[PP], m0b[PP], s1a[PP], s1b[PP], m1a[PP], m1b[PP];
            const uint32_t off = half * 2 * PP;  // first column of the half
            tc8::tmem_ld<2 * PP>(c0 + off, s0a);
            tc8::tmem_ld<2 * PP>(c0 + R + off, s0b);
            tc8::tmem_ld<2 * PP>(c0 + N + off, m0a);
            tc8::tmem_ld<2 * PP>(c0 + N + R + off, m0b);
            tc8::tmem_ld<2 * PP>(c1 + off, s1a);
            tc8::tmem_ld<2 * PP>(c1 + R + off, s1b);
            tc8::tmem_ld<2 * PP>(c1 + N + off, m1a);
            tc8::tmem_ld<2 * PP>(c1 + N + R + off, m1b);
            tc8::tmem_wait_ld();
#pragma unroll
            for (int pp = 0; pp < PP; ++pp) {
                const int p = half * PP + pp;
                const float4 q0 = qdq[h0][p], q1 = qdq[h1][p];
                const float2 ch0 = tc8::chain_pair(make_float2(q0.x, q0.y), make_float2(q0.z, q0.w), kl[p], dk[p],
                                                   s0a[pp], s0b[pp], m0a[pp], m0b[pp]);
                const float2 ch1 = tc8::chain_pair(make_float2(q1.x, q1.y), make_float2(q1.z, q1.w), kl[p], dk[p],
                                                   s1a[pp], s1b[pp], m1a[pp], m1b[pp]);
                t0 = __fadd_rn(__fadd_rn(t0, ch0.x), ch0.y);  // groups in order
                t1 = __fadd_rn(__fadd_rn(t1, ch1.x), ch1.y);
            }
        }
        if (tok < tokens) {
            const uint16_t b0 = float_to_half_bits(__fmul_rn(t0, scale));
            scores[(row0 + h0) * score_stride + tok] = b0;
            if constexpr (HIST) atomicAdd(&shist[h0 * 2048 + (order_key16(b0) >> 5)], 1u);
            if (h1 < group_heads) {
                const uint16_t b1 = float_to_half_bits(__fmul_rn(t1, scale));
                scores[(row0 + h1) * score_stride + tok] = b1;
                if constexpr (HIST) atomicAdd(&shist[h1 * 2048 + (order_key16(b1) >> 5)], 1u);
            }
        }
    };

    // ---- pipeline: expand i+1 while the MMAs of i run, then read i back ----
    uint32_t cur_l[R / 2], cur_d[R / 2];
    expand(0, tc8::kColA0, cur_l, cur_d);
    tc8::fence_before();
    __syncthreads();
    tc8::fence_after();
    if (threadIdx.x == 0) issue_mma(tc8::kColA0);
    if (streamer && S < ntiles) {
        fence_async_smem();
        issue(S);  // tile 0's stage is in registers and tensor memory now
    }
    for (int i = 0; i < ntiles; ++i) {
        const bool more = i + 1 < ntiles;
        const uint32_t next_buf = ((i + 1) & 1) ? tc8::kColA1 : tc8::kColA0;
        uint32_t nxt_l[R / 2], nxt_d[R / 2];
        if (more) expand(i + 1, next_buf, nxt_l, nxt_d);  // the MMAs of i-1 read this buffer and are done
        tc8_wait(&mma_bar, i & 1);
        tc8::fence_after();
        epilogue(i, cur_l, cur_d);
        tc8::fence_before();
        __syncthreads();  // D read by every thread; A of i+1 written by every thread
        tc8::fence_after();
        if (more) {
            if (threadIdx.x == 0) issue_mma(next_buf);
            if (streamer && i + 1 + S < ntiles) {
                fence_async_smem();
                issue(i + 1 + S);
            }
#pragma unroll
            for (int p = 0; p < R / 2; ++p) {
                cur_l[p] = nxt_l[p];
                cur_d[p] = nxt_d[p];
            }
        }
    }
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(tc8::kTmemCols) : "memory");
    if constexpr (HIST) {
        // Every epilogue count landed before the loop's last block barrier:
        // one global atomic per non-empty bin.
        for (int i = threadIdx.x; i < group_heads * 2048; i += tc8::kThreads) {
            const uint32_t c = shist[i];
            if (c) atomicAdd(&hist[(row0 + (i >> 11)) * 2048 + (i & 2047)], c);
        }
    }
    pdl_launch_dependents();
}

// The tensor-core scorer needs every tile's low/delta rows 16-byte aligned
// (capacity * 2R bytes a multiple of 16) and at most four query heads per KV head.
inline bool score_tc8_eligible(int G, int64_t capacity, int group_heads) {
    const int64_t row_bytes = capacity * 2 * (128 / G);
    return group_heads <= tc8::kMaxHeads && (row_bytes % 16) == 0;
}

// Whether the tensor-core scorer is the faster of the two for `rows` (batch x
// KV heads) rows of `tokens` keys.  Below about one 128-token tile per SM its
// per-CTA prologue (query encoding, B operand, first plane tile) dominates and
// the popcount kernel (4 CTAs per SM, lighter prologue) wins; the crossover is
// later for the coarser groups, whose popcount kernel needs fewer popcounts.
// Measured on B200 at head_dim 128, 4 query heads per KV head (both kernels
// give the same bits): G16 from 1024 tiles, G32 and G64 from 4096 tiles.
inline bool score_tc8_pays(int G, int64_t rows, int64_t tokens) {
    const int64_t tiles = rows * ((tokens + tc8::kTile - 1) / tc8::kTile);
    return tiles >= (G == 16 ? 1024 : 4096);
}

int score_sm_count();

template <int G, typename QT, bool RAW, bool HIST = false>
int launch_score128_tc8(const QT* queries, const int32_t* q_sign, const int32_t* q_mag, const float* q_low,
                        const float* q_delta, int64_t batch, int64_t q_heads, const int32_t* k_sign,
                        const int32_t* k_mag, const uint16_t* k_low, const uint16_t* k_delta, int64_t kv_heads,
                        int64_t capacity, const int64_t* head_to_kv, int64_t tokens, uint16_t* scores,
                        cudaStream_t stream, int64_t score_stride, const int64_t* dyn_tokens,
                        uint32_t* hist = nullptr) {
    const int group_heads = static_cast<int>(q_heads / kv_heads);
    const int64_t rows = batch * kv_heads;
    const int64_t tiles = (tokens + tc8::kTile - 1) / tc8::kTile;
    // Two CTAs per SM (two 256-column tensor-memory allocations fill an SM's 512):
    // at most one resident wave of chunks, since every CTA of a row runs the same
    // number of tiles and a second wave would double the kernel's time.
    const int64_t target = static_cast<int64_t>(score_sm_count()) * 2;
    int64_t chunks = target / rows;
    if (chunks > tiles) chunks = tiles;
    if (chunks < 1) chunks = 1;
    const dim3 grid(static_cast<unsigned>(chunks), static_cast<unsigned>(rows));
    constexpr int smem = tc8::Layout<G>::kSmemBytes;
    auto kernel = score128_tc8_kernel<G, QT, RAW, HIST>;
    const int st = allow_dynamic_smem(kernel, smem);
    if (st != POPKV_OK) return st;
    const cudaError_t err = launch_pdl(kernel, grid, dim3(tc8::kThreads), smem, stream, 1, queries, q_sign, q_mag,
                                       q_low, q_delta, k_sign, k_mag, k_low, k_delta, head_to_kv, scores,
                                       static_cast<int>(q_heads), group_heads, capacity, tokens, score_scale_for(128),
                                       score_stride, dyn_tokens, static_cast<int>(chunks), hist);
    if (err != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_score: %s", cudaGetErrorString(err));
    return check_launch("popkv_score");
}

}  // namespace popkv
