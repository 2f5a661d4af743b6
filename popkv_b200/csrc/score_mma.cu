// head_dim-128 popcount scorer on the 5th-generation tensor cores (tcgen05,
// kind::i8, accumulators in tensor memory).
//
// The four counts of one (query head, key token, representative group r) are
// small-integer dot products over the group's G dimensions
// (csrc/popkv_ext.cu:502-515 forms them with popcounts):
//   c_sign = sum_d uq(d) uk(d)          c_q  = sum_d [uq qm](d) uk(d)
//   c_k    = sum_d uq(d) [uk km](d)     c_qk = sum_d [uq qm](d) [uk km](d)
// with uq, uk = +1 where the sign bit is set and -1 elsewhere, and qm, km the
// magnitude bits.  So for a tile of 128 key tokens the counts are one int8
// matrix product per group: A = the tile's [uk | uk*km] bytes (128 x 2G,
// K-major, expanded from the bit planes into shared memory), B = the query
// coefficients (16 columns: 4 heads x 4 counts, 2G deep), D = 128 x 16 int32
// in tensor memory.  Every count is exact; the epilogue then applies the
// reference's fp32 chain unchanged (fma(ql*kl, c_sign, fma(dq*kl, c_q,
// fma(ql*dk, c_k, (dq*dk)*c_qk))) summed over r in order, times the scale,
// rounded to fp16), so the scores equal the popcount kernel's bit for bit.
//
// This moves the count work off the popcount pipe, which bounds the popcount
// kernel, onto the tensor cores.
#include <cstdint>

#include "common.cuh"
#include "mbarrier.cuh"
#include "score_impl.cuh"
#include "score_mma.cuh"

// Phase timestamps for profiling builds (-DPOPKV_SCORE_TIMING): thread 0 of
// each CTA records %globaltimer at its phase boundaries (first tile in detail).
#ifdef POPKV_SCORE_TIMING
__device__ unsigned long long g_score_phase_ns[1024][8];
#define POPKV_SCORE_PHASE(i)                                                             \
    do {                                                                                 \
        const unsigned cta_ = blockIdx.y * gridDim.x + blockIdx.x;                       \
        if (threadIdx.x == 0 && cta_ < 1024) {                                           \
            unsigned long long t_;                                                       \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                      \
            g_score_phase_ns[cta_][i] = t_;                                              \
        }                                                                                \
    } while (0)
#define POPKV_SCORE_PHASE_T(i, thread)                                                    \
    do {                                                                                 \
        const unsigned cta_ = blockIdx.y * gridDim.x + blockIdx.x;                       \
        if (threadIdx.x == (thread) && cta_ < 1024) {                                    \
            unsigned long long t_;                                                       \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                      \
            g_score_phase_ns[cta_][i] = t_;                                              \
        }                                                                                \
    } while (0)
extern "C" __attribute__((visibility("default"))) int popkv_score_phase_ns(unsigned long long* host, int ctas) {
    return static_cast<int>(cudaMemcpyFromSymbol(host, g_score_phase_ns, sizeof(unsigned long long) * 8 * ctas));
}
#else
#define POPKV_SCORE_PHASE(i) \
    do {                     \
    } while (0)
#define POPKV_SCORE_PHASE_T(i, thread) \
    do {                               \
    } while (0)
#endif

namespace popkv {
namespace {

constexpr int kMmaTile = 128;     // MMA M
constexpr int kMmaN = 16;         // 4 query heads x 4 counts
constexpr int kKBlocks = 8;       // 128 dims x {uk, uk*km} bytes / 32 bytes per MMA
constexpr int kABlockBytes = kMmaTile * 32;  // one k-block of A: 4 KB
constexpr int kBBlockBytes = kMmaN * 32;     // one k-block of B: 512 B
constexpr int kABytes = kKBlocks * kABlockBytes;

// ---------------------------------------------------------------------------
// PTX wrappers.
// ---------------------------------------------------------------------------

// Shared-memory matrix descriptor, no swizzle, K-major: core matrices of 8 rows
// x 16 bytes stored as 128 contiguous bytes; the next 16 bytes along K sit 128
// bytes on (leading byte offset), the next 8 rows 256 bytes on (stride byte
// offset).  Bits 46-47 hold the descriptor version (1).
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t addr) {
    return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(128 >> 4) << 16) |
           (static_cast<uint64_t>(256 >> 4) << 32) | (1ull << 46);
}

// Instruction descriptor of kind::i8: s32 accumulator (bits 4-5 = 2), signed
// A and B (bits 7-9, 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) |
                            (static_cast<uint32_t>(kMmaN >> 3) << 17) |
                            (static_cast<uint32_t>(kMmaTile >> 4) << 24);

__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_addr(dst)), "r"(cols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(cols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}


__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    const uint32_t mask0 = 0, mask1 = 0, mask2 = 0, mask3 = 0;  // no output lane disabled
    asm volatile(
        "{\n\t"
        ".reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t"
        "}\n"
        :: "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(mask0), "r"(mask1),
           "r"(mask2), "r"(mask3)
        : "memory");
}

// Arrives on the mbarrier once every MMA this thread issued has completed.
__device__ __forceinline__ void mma_commit(uint64_t* mbar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_addr(mbar)) : "memory");
}


// Byte offset of (row, 16-byte chunk c16 of a 32-byte k-block row) inside a
// k-block laid out as described at kmajor_desc.
__device__ __forceinline__ uint32_t kblock_offset(int row, int c16) {
    return static_cast<uint32_t>((row >> 3) * 256 + c16 * 128 + (row & 7) * 16);
}

// Position of the 16 bytes for dims [16q, 16q + 16) of plane p (0: uk, 1: uk*km)
// in the k-block sequence: group r = 16q / G keeps [uk (G bytes) | uk*km (G
// bytes)] in k-blocks [r*G/16, (r+1)*G/16).
template <int G>
__device__ __forceinline__ void plane_slot(int q, int p, int& kb, int& c16) {
    const int r = (16 * q) / G;
    const int li = p * G + (16 * q) % G;  // byte inside the group's 2G bytes
    kb = r * (G / 16) + li / 32;
    c16 = (li % 32) / 16;
}

// ---------------------------------------------------------------------------
// Warp-specialised, pipelined form.  384 threads: warps 8-11 produce (load a
// tile's sign/magnitude planes, expand them into one of two A stages; thread
// 256 then issues the tile's MMAs into one of two TMEM buffers), warps 0-7
// consume (TMEM counts -> fp32 chain -> fp16 scores): warp w reads TMEM lane
// quarter w % 4 (token rows 32(w%4)..) for query heads 2(w/4) and 2(w/4)+1,
// with those heads' query constants in registers.  mbarriers hand the stages
// around:
//   a_empty[s]  MMAs reading A stage s are done           (tcgen05.commit)
//   t_full[b]   counts of TMEM buffer b are ready           (tcgen05.commit)
//   t_empty[b]  the eight epilogue warps have read buffer b (one arrive per warp)
// so tile i+1 is expanded and multiplied while tile i's epilogue runs.
// ---------------------------------------------------------------------------
constexpr int kWsThreads = 384;   // warps 0-7 epilogue (two per TMEM lane quarter), 8-11 producers
constexpr int kWsEpilogueWarps = 8;
constexpr int kWsProducer0 = kWsEpilogueWarps * 32;  // first producer thread
constexpr int kWsStages = 2;
// 2 x 32 KB A stages + 4 KB B, padded so that at most two CTAs share an SM:
// two 256-column TMEM allocations fill its 512 columns.
constexpr size_t kWsDynSmem = 100 * 1024;
constexpr uint32_t kWsTmemCols = 256;
static_assert(kWsStages * kABytes + kKBlocks * kBBlockBytes <= 100 * 1024, "A stages and B fit");

// Count of threads whose bounded wait on an mbarrier gave up (0 in a healthy
// run); read with popkv_score_tc_timeouts().
__device__ unsigned int g_score_tc_timeouts = 0;

__device__ __forceinline__ void producer_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// 8 consecutive TMEM columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&c)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3]), "=r"(c[4]), "=r"(c[5]), "=r"(c[6]),
                   "=r"(c[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}


template <int G, typename QT>
__global__ void __launch_bounds__(kWsThreads, 2) score128_ws_kernel(
    const QT* __restrict__ queries, const int32_t* __restrict__ k_sign, const int32_t* __restrict__ k_mag,
    const uint16_t* __restrict__ k_low, const uint16_t* __restrict__ k_delta,
    const int64_t* __restrict__ head_to_kv, uint16_t* __restrict__ scores, int q_heads, int group_heads,
    int64_t capacity, int64_t tokens, int tiles_per_cta, float scale) {
    constexpr int R = 128 / G;
    extern __shared__ __align__(1024) unsigned char ws_smem[];
    unsigned char* sA = ws_smem;                          // kWsStages x kKBlocks x [128 rows x 32 B]
    unsigned char* sB = ws_smem + kWsStages * kABytes;    // kKBlocks x [16 rows x 32 B]
    __shared__ QueryState<G> states[4];
    __shared__ float scratch[4][2 * 32 * 4];
    __shared__ uint32_t u_table[16], m_table[16];
    __shared__ __align__(8) uint64_t a_empty[kWsStages], t_full[kWsStages], t_empty[kWsStages];
    __shared__ uint32_t tmem_base;

    POPKV_SCORE_PHASE_T(0, 0);
    pdl_wait();
    pdl_launch_dependents();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int groups = q_heads / group_heads;
    const int64_t b = blockIdx.y / groups;
    const int grp = blockIdx.y % groups;
    const int qh0 = grp * group_heads;
    const int64_t row0 = b * q_heads + qh0;
    const int64_t kvh = head_to_kv[qh0];

    if (warp == 0) tmem_alloc(&tmem_base, kWsTmemCols);
    if (tid == 0) {
        for (int st = 0; st < kWsStages; ++st) {
            mbar_init(&a_empty[st], 1);
            mbar_init(&t_full[st], 1);
            mbar_init(&t_empty[st], kWsEpilogueWarps);
        }
    }
    if (tid < 16) {
        uint32_t u = 0, m = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            u |= (((tid >> j) & 1) ? 0x01u : 0xFFu) << (8 * j);
            m |= (((tid >> j) & 1) ? 0xFFu : 0x00u) << (8 * j);
        }
        u_table[tid] = u;
        m_table[tid] = m;
    }
    if (warp < group_heads && warp < 4)
        encode_query_row<QT, 4>(queries + (row0 + warp) * 128, 128, G, lane, scratch[warp], states[warp].qs,
                                states[warp].qm, states[warp].ql, states[warp].dq);
    __syncthreads();
    if (tid < 128) {  // B: thread t fills column t / 8 (head, count) of k-block t % 8
        const int n = tid >> 3, kb = tid & 7, h = n >> 2, cnt = n & 3;
        const bool wants_k = cnt >= 2;
        const bool wants_qm = cnt & 1;
        const int r = kb / (G / 16);
        unsigned char* dstB = sB + kb * kBBlockBytes;
#pragma unroll
        for (int c16 = 0; c16 < 2; ++c16) {
            const int li = (kb % (G / 16)) * 32 + 16 * c16;
            const int p = li / G;
            const int d0 = r * G + li % G;
            uint32_t w[4] = {0u, 0u, 0u, 0u};
            if (h < group_heads && (p == 1) == wants_k) {
                const uint32_t qs = states[h].qs[d0 >> 5] >> (d0 & 31);
                const uint32_t qm = states[h].qm[d0 >> 5] >> (d0 & 31);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t u = u_table[(qs >> (4 * j)) & 15u];
                    w[j] = wants_qm ? (u & m_table[(qm >> (4 * j)) & 15u]) : u;
                }
            }
            *reinterpret_cast<uint4*>(dstB + kblock_offset(n, c16)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    const uint32_t a_base = smem_addr(sA), b_base = smem_addr(sB);
    POPKV_SCORE_PHASE_T(1, 0);

    const int64_t tiles = (tokens + kMmaTile - 1) / kMmaTile;
    const int64_t first = static_cast<int64_t>(blockIdx.x) * tiles_per_cta;
    const int ntiles = static_cast<int>(first >= tiles ? 0 : (tiles - first < tiles_per_cta ? tiles - first : tiles_per_cta));
    const uint4* sign4 = reinterpret_cast<const uint4*>(k_sign) + kvh * capacity;
    const uint4* mag4 = reinterpret_cast<const uint4*>(k_mag) + kvh * capacity;
    const uint16_t* lowp = k_low + kvh * capacity * R;
    const uint16_t* deltap = k_delta + kvh * capacity * R;
    bool ok = true;

    if (warp >= kWsEpilogueWarps) {
        // ---------------- producers ----------------
        const int row = tid - kWsProducer0;
        uint4 cs = make_uint4(0, 0, 0, 0), cm = cs, ns = cs, nm = cs;
        if (ntiles > 0) {
            const int64_t t0 = first * kMmaTile + row;
            cs = __ldg(sign4 + (t0 < tokens ? t0 : 0));
            cm = __ldg(mag4 + (t0 < tokens ? t0 : 0));
        }
        for (int i = 0; i < ntiles; ++i) {
            const int st = i & 1, n = i >> 1;
            const int64_t t = (first + i) * kMmaTile + row;
            const bool live = t < tokens;
            if (i + 1 < ntiles) {
                const int64_t tn = t + kMmaTile;
                ns = __ldg(sign4 + (tn < tokens ? tn : 0));
                nm = __ldg(mag4 + (tn < tokens ? tn : 0));
            }
            if (n >= 1) ok = mbar_wait(&a_empty[st], (n - 1) & 1) && ok;
            unsigned char* stage = sA + st * kABytes;
            const uint32_t ks[4] = {cs.x, cs.y, cs.z, cs.w}, km[4] = {cm.x, cm.y, cm.z, cm.w};
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const uint32_t sw = ks[q >> 1] >> ((q & 1) * 16);
                const uint32_t mw = km[q >> 1] >> ((q & 1) * 16);
                uint32_t u[4], w[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    u[j] = live ? u_table[(sw >> (4 * j)) & 15u] : 0u;
                    w[j] = u[j] & m_table[(mw >> (4 * j)) & 15u];
                }
                int kb, c16;
                plane_slot<G>(q, 0, kb, c16);
                *reinterpret_cast<uint4*>(stage + kb * kABlockBytes + kblock_offset(row, c16)) = make_uint4(u[0], u[1], u[2], u[3]);
                plane_slot<G>(q, 1, kb, c16);
                *reinterpret_cast<uint4*>(stage + kb * kABlockBytes + kblock_offset(row, c16)) = make_uint4(w[0], w[1], w[2], w[3]);
            }
            fence_async_smem();
            if (i == 0) POPKV_SCORE_PHASE_T(2, kWsProducer0);
            producer_sync();
            if (row == 0) {
                if (n >= 1) ok = mbar_wait(&t_empty[st], (n - 1) & 1) && ok;
                tc_fence_after();
#pragma unroll
                for (int r = 0; r < R; ++r) {
#pragma unroll
                    for (int j = 0; j < G / 16; ++j) {
                        const int kb = r * (G / 16) + j;
                        mma_i8(tmem + static_cast<uint32_t>(st * 128 + r * kMmaN),
                               kmajor_desc(a_base + static_cast<uint32_t>(st * kABytes + kb * kABlockBytes)),
                               kmajor_desc(b_base + static_cast<uint32_t>(kb * kBBlockBytes)), kIdesc, j > 0 ? 1u : 0u);
                    }
                }
                mma_commit(&t_full[st]);
                mma_commit(&a_empty[st]);
                if (i == 0) POPKV_SCORE_PHASE_T(3, kWsProducer0);
                if (i + 1 == ntiles) POPKV_SCORE_PHASE_T(4, kWsProducer0);
            }
            cs = ns;
            cm = nm;
        }
    } else {
        // ---------------- epilogue ----------------
        const int quarter = warp & 3, pair = warp >> 2;
        const int row = quarter * 32 + lane;
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        float qlr[2][R], dqr[2][R];  // this warp's two heads' query constants
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int h = 2 * pair + hh;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                qlr[hh][r] = h < group_heads ? states[h].ql[r] : 0.0f;
                dqr[hh][r] = h < group_heads ? states[h].dq[r] : 0.0f;
            }
        }
        uint32_t cl[R / 2], cd[R / 2], nl[R / 2], nd[R / 2];
        auto fetch = [&](int64_t t, uint32_t* l, uint32_t* d) {
            if constexpr (R == 8) {
                const uint4 l4 = __ldg(reinterpret_cast<const uint4*>(lowp) + t);
                const uint4 d4 = __ldg(reinterpret_cast<const uint4*>(deltap) + t);
                l[0] = l4.x; l[1] = l4.y; l[2] = l4.z; l[3] = l4.w;
                d[0] = d4.x; d[1] = d4.y; d[2] = d4.z; d[3] = d4.w;
            } else if constexpr (R == 4) {
                const uint2 l2 = __ldg(reinterpret_cast<const uint2*>(lowp) + t);
                const uint2 d2 = __ldg(reinterpret_cast<const uint2*>(deltap) + t);
                l[0] = l2.x; l[1] = l2.y;
                d[0] = d2.x; d[1] = d2.y;
            } else {
                l[0] = __ldg(reinterpret_cast<const uint32_t*>(lowp) + t);
                d[0] = __ldg(reinterpret_cast<const uint32_t*>(deltap) + t);
            }
        };
        if (ntiles > 0) {
            const int64_t t0 = first * kMmaTile + row;
            fetch(t0 < tokens ? t0 : 0, cl, cd);
        }
        for (int i = 0; i < ntiles; ++i) {
            const int bf = i & 1, n = i >> 1;
            const int64_t t = (first + i) * kMmaTile + row;
            const bool live = t < tokens;
            if (i + 1 < ntiles) {
                const int64_t tn = t + kMmaTile;
                fetch(tn < tokens ? tn : 0, nl, nd);
            }
            float kl[R], dk[R];
#pragma unroll
            for (int j = 0; j < R / 2; ++j) {
                kl[2 * j] = half_bits_to_float(static_cast<uint16_t>(cl[j] & 0xFFFFu));
                kl[2 * j + 1] = half_bits_to_float(static_cast<uint16_t>(cl[j] >> 16));
                dk[2 * j] = half_bits_to_float(static_cast<uint16_t>(cd[j] & 0xFFFFu));
                dk[2 * j + 1] = half_bits_to_float(static_cast<uint16_t>(cd[j] >> 16));
            }
            ok = mbar_wait(&t_full[bf], n & 1) && ok;
            if (i == 0) POPKV_SCORE_PHASE_T(5, 0);
            tc_fence_after();
            float total[2] = {0.0f, 0.0f};
#pragma unroll
            for (int r = 0; r < R; ++r) {
                uint32_t c[8];  // (head 2*pair, head 2*pair+1) x (sign, q, k, qk)
                tmem_ld8(tmem + lane_base + static_cast<uint32_t>(bf * 128 + r * kMmaN + 8 * pair), c);
                if (r + 1 == R) {  // every count of this buffer is in registers: hand it back
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&t_empty[bf]);
                }
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    const int* cc = reinterpret_cast<const int*>(c) + hh * 4;
                    const float ql = qlr[hh][r], dq = dqr[hh][r];
                    const float t1 = __fmul_rn(ql, kl[r]);
                    const float t2 = __fmul_rn(dq, kl[r]);
                    const float t3 = __fmul_rn(ql, dk[r]);
                    const float t4 = __fmul_rn(__fmul_rn(dq, dk[r]), small_int_to_float(cc[3]));
                    const float chain = __fmaf_rn(t1, small_int_to_float(cc[0]),
                                                  __fmaf_rn(t2, small_int_to_float(cc[1]),
                                                            __fmaf_rn(t3, small_int_to_float(cc[2]), t4)));
                    total[hh] = __fadd_rn(total[hh], chain);
                }
            }
            if (live) {
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    const int h = 2 * pair + hh;
                    if (h < group_heads)
                        scores[(row0 + h) * tokens + t] = float_to_half_bits(__fmul_rn(total[hh], scale));
                }
            }
#pragma unroll
            for (int j = 0; j < R / 2; ++j) {
                cl[j] = nl[j];
                cd[j] = nd[j];
            }
            if (i == 0) POPKV_SCORE_PHASE_T(6, 0);
        }
        POPKV_SCORE_PHASE_T(7, 0);
    }
    if (!ok) atomicAdd(&g_score_tc_timeouts, 1u);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kWsTmemCols);
    }
}

template <int G, typename QT>
int launch_mma(const void* queries, int64_t batch, int64_t q_heads, const int32_t* k_sign,
               const int32_t* k_mag, const uint16_t* k_low, const uint16_t* k_delta, int64_t kv_heads,
               int64_t capacity, const int64_t* head_to_kv, int64_t tokens, uint16_t* scores,
               cudaStream_t stream) {
    auto kernel = score128_ws_kernel<G, QT>;
    int st = allow_dynamic_smem(kernel, static_cast<int>(kWsDynSmem));
    if (st != POPKV_OK) return st;
    const int group_heads = static_cast<int>(q_heads / kv_heads);
    const int64_t tiles = (tokens + kMmaTile - 1) / kMmaTile;
    const int64_t units = batch * kv_heads;
    // About one wave of two CTAs per SM: each CTA pipelines a run of tiles.
    const int64_t target = 2 * 148;
    int64_t per = (tiles * units + target - 1) / target;
    if (per < 1) per = 1;
    const int64_t ctas_x = (tiles + per - 1) / per;
    const cudaError_t err = launch_pdl(kernel, dim3(static_cast<unsigned>(ctas_x), static_cast<unsigned>(units)),
                                       dim3(kWsThreads), kWsDynSmem, stream, 1,
                                       static_cast<const QT*>(queries), k_sign, k_mag, k_low, k_delta,
                                       head_to_kv, scores, static_cast<int>(q_heads), group_heads, capacity,
                                       tokens, static_cast<int>(per), score_scale_for(128));
    if (err != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_score: %s", cudaGetErrorString(err));
    return check_launch("popkv_score");
}

template <typename QT>
int dispatch_mma(int64_t g, const void* queries, int64_t batch, int64_t q_heads, const int32_t* k_sign,
                 const int32_t* k_mag, const uint16_t* k_low, const uint16_t* k_delta, int64_t kv_heads,
                 int64_t capacity, const int64_t* head_to_kv, int64_t tokens, uint16_t* scores,
                 cudaStream_t stream) {
    if (g == 16)
        return launch_mma<16, QT>(queries, batch, q_heads, k_sign, k_mag, k_low, k_delta, kv_heads,
                                  capacity, head_to_kv, tokens, scores, stream);
    if (g == 32)
        return launch_mma<32, QT>(queries, batch, q_heads, k_sign, k_mag, k_low, k_delta, kv_heads,
                                  capacity, head_to_kv, tokens, scores, stream);
    return launch_mma<64, QT>(queries, batch, q_heads, k_sign, k_mag, k_low, k_delta, kv_heads, capacity,
                              head_to_kv, tokens, scores, stream);
}

}  // namespace

bool score_mma_applies(int64_t q_heads, int64_t kv_heads, int64_t dim_group_size, int64_t batch,
                       int64_t tokens) {
    const int64_t gh = q_heads / kv_heads;
    return gh >= 1 && gh <= 4 && (dim_group_size == 16 || dim_group_size == 32 || dim_group_size == 64) &&
           batch * kv_heads <= 65535 && tokens > 0 && (tokens + kMmaTile - 1) / kMmaTile < 0x7FFFFFFFll;
}

int launch_score_mma(const void* queries, int queries_dtype, int64_t batch, int64_t q_heads,
                     const int32_t* k_sign, const int32_t* k_mag, const uint16_t* k_low,
                     const uint16_t* k_delta, int64_t kv_heads, int64_t capacity,
                     const int64_t* head_to_kv, int64_t tokens, int64_t dim_group_size, uint16_t* scores,
                     cudaStream_t stream) {
    if (queries_dtype == POPKV_DTYPE_F32)
        return dispatch_mma<float>(dim_group_size, queries, batch, q_heads, k_sign, k_mag, k_low, k_delta,
                                   kv_heads, capacity, head_to_kv, tokens, scores, stream);
    if (queries_dtype == POPKV_DTYPE_F16)
        return dispatch_mma<__half>(dim_group_size, queries, batch, q_heads, k_sign, k_mag, k_low, k_delta,
                                    kv_heads, capacity, head_to_kv, tokens, scores, stream);
    return dispatch_mma<__nv_bfloat16>(dim_group_size, queries, batch, q_heads, k_sign, k_mag, k_low,
                                       k_delta, kv_heads, capacity, head_to_kv, tokens, scores, stream);
}

}  // namespace popkv

extern "C" int popkv_score_tc(const void* queries, int queries_dtype, int64_t batch, int64_t q_heads,
                              int64_t head_dim, const int32_t* k_sign, const int32_t* k_mag,
                              const uint16_t* k_low, const uint16_t* k_delta, int64_t kv_heads,
                              int64_t capacity, const int64_t* head_to_kv, int64_t tokens,
                              int64_t dim_group_size, void* scores, int scores_dtype, void* stream) {
    using namespace popkv;
    if (!valid_dtype(queries_dtype)) return fail(POPKV_ERR_INVALID, "queries must be fp32/fp16/bf16");
    int st = check_score_common(batch, q_heads, kv_heads, capacity, tokens, dim_group_size, head_to_kv);
    if (st != POPKV_OK) return st;
    if (head_dim != 128)
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_score_tc: head_dim must be 128");
    if (scores_dtype != POPKV_DTYPE_F16) return fail(POPKV_ERR_INVALID, "head_dim 128 scores are fp16");
    if (!score_mma_applies(q_heads, kv_heads, dim_group_size, batch, tokens))
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_score_tc: at most 4 query heads per KV head");
    if (batch == 0) return POPKV_OK;
    if (!queries || !k_sign || !k_mag || !k_low || !k_delta || !scores)
        return fail(POPKV_ERR_INVALID, "popkv_score_tc: null pointer");
    if (!aligned(k_sign, 16) || !aligned(k_mag, 16) || !aligned(k_low, 16) || !aligned(k_delta, 16))
        return fail(POPKV_ERR_INVALID, "packed planes must be 16-byte aligned");
    return launch_score_mma(queries, queries_dtype, batch, q_heads, k_sign, k_mag, k_low, k_delta, kv_heads,
                            capacity, head_to_kv, tokens, dim_group_size, static_cast<uint16_t*>(scores),
                            static_cast<cudaStream_t>(stream));
}

extern "C" int popkv_score_tc_timeouts(uint32_t* count) {
    using namespace popkv;
    if (!count) return fail(POPKV_ERR_INVALID, "popkv_score_tc_timeouts: null pointer");
    uint32_t tc = 0, f8 = 0;
    const cudaError_t e = cudaMemcpyFromSymbol(&tc, g_score_tc_timeouts, sizeof(uint32_t));
    if (e != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_score_tc_timeouts: %s", cudaGetErrorString(e));
    const int st = read_score_tc8_timeouts(&f8);
    if (st != POPKV_OK) return st;
    *count = tc + f8;
    return POPKV_OK;
}
