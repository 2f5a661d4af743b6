// Fused decode-time retrieval: popcount score -> top-k with the current slot
// reserved -> sparse attention -> log-sum-exp merge, in one launch.
//
// Reference path (one eager launch per stage there): popkv.py:1076-1115 --
// query_encode + score_encoded (csrc/popkv_ext.cu:911-957, :757-876),
// torch.topk(sorted=False) + _append_current (popkv.py:1094-1098, :287-291),
// indexed_attention_split_partial / _merge (sparse_kernels.py:237-318).
//
// One thread-block cluster of C CTAs (16, or 8 where 16 cannot be scheduled)
// serves one (batch row, KV head) and the QPG query heads that read it.
// CTA q owns the token slice [q*slice, (q+1)*slice):
//
//  A. every CTA encodes the group's queries into shared memory;
//  B. it scores its slice for all QPG heads (the popcount arithmetic of
//     score_impl.cuh, bit-identical to popkv_score) and keeps the fp16 scores in
//     shared memory, building per-head histograms of the top 11 key bits;
//  C. radix select across the cluster: CTAs add their histograms into the
//     leader CTA's through distributed shared memory, the leader picks the digit
//     holding the k-th largest score; a second 5-bit pass resolves the exact
//     threshold; each CTA publishes its (greater, equal) counts so that ties at
//     the threshold are taken in token order -- the same selection, bit for bit,
//     as popkv_topk (higher score first, then lower index);
//  D. the CTA gathers the union of its selected tokens once (a token chosen by
//     several heads of the group is read once) through a cp.async ring, and
//     folds each row into the online-softmax state of every head that chose it;
//     rank 0 also folds in the current token;
//  E. CTA h merges head h's C partial states through distributed shared memory
//     and writes the output row.
//
// Scores and indices can also be written to global memory for inspection;
// nothing else leaves the chip.
#include <cooperative_groups.h>

#include <cstdint>
#include <type_traits>

#include "common.cuh"
#include "score_impl.cuh"

// Phase timestamps for profiling builds (-DPOPKV_RETRIEVE_TIMING): thread 0 of
// each CTA records %globaltimer at the phase boundaries into g_retrieve_phase_ns.
#ifdef POPKV_RETRIEVE_TIMING
__device__ unsigned long long g_retrieve_phase_ns[2048][16];
#define POPKV_PHASE(i)                                                                  \
    do {                                                                                \
        if (threadIdx.x == 0 && blockIdx.x < 2048) {                                    \
            unsigned long long t_;                                                      \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                     \
            g_retrieve_phase_ns[blockIdx.x][i] = t_;                                    \
        }                                                                               \
    } while (0)
#else
#define POPKV_PHASE(i) \
    do {               \
    } while (0)
#endif

namespace popkv {
namespace {

namespace cg = cooperative_groups;

constexpr int kRetThreads = 512;
constexpr int kRetWarps = kRetThreads / 32;
constexpr int kHist1Bins = 2048;  // key bits 15..5
constexpr int kHist2Bins = 32;    // key bits 4..0
constexpr int kRingRows = 32;     // rows per stage: 32 row groups of 16 threads
constexpr int kRowBytes128 = 256; // 128 x 16-bit
constexpr int kMaxSlice = 8192;
constexpr uint16_t kCurrentEntry = 0xFFFF;
constexpr float kLog2eF = 1.4426950408889634f;

__device__ __forceinline__ uint32_t score_key(uint16_t h) {
    if ((h & 0x7FFFu) == 0) h = 0;  // -0 == +0
    if ((h & 0x7C00u) == 0x7C00u && (h & 0x3FFu)) return 0xFFFFu;
    return (h & 0x8000u) ? (~static_cast<uint32_t>(h) & 0xFFFFu) : (static_cast<uint32_t>(h) | 0x8000u);
}

__device__ __forceinline__ void cp_async16_ret(void* smem, const void* gmem) {
    const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit_ret() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_ret() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

template <typename V>
__device__ __forceinline__ V ret_exclusive_scan(V x, V* warp_sums, V& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    V incl = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        V y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        V w = lane < kRetWarps ? warp_sums[lane] : V(0);
        V wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            V y = __shfl_up_sync(0xFFFFFFFFu, wi, o);
            if (lane >= o) wi += y;
        }
        if (lane < kRetWarps) warp_sums[lane] = wi - w;
        if (lane == kRetWarps - 1) warp_sums[kRetWarps] = wi;
    }
    __syncthreads();
    V result = warp_sums[warp] + incl - x;
    total = warp_sums[kRetWarps];
    __syncthreads();
    return result;
}

template <typename KT>
__device__ __forceinline__ void unpack8_ret(const uint4& u, float* f) {
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

template <typename T>
__device__ __forceinline__ void store_elem(T* p, float v) {
    if constexpr (std::is_same<T, float>::value) *p = v;
    else if constexpr (std::is_same<T, __half>::value) *p = __float2half_rn(v);
    else *p = __float2bfloat16_rn(v);
}

struct RetrieveArgs {
    const void* queries;
    const int32_t* k_sign;
    const int32_t* k_mag;
    const uint16_t* k_low;
    const uint16_t* k_delta;
    int64_t capacity;
    int64_t plane_batch_stride;  // rows between batch entries of the planes
    const void* prefix_k;
    const void* prefix_v;
    int64_t kbs, khs, kts, vbs, vhs, vts;  // elements
    const void* cur_k;
    const void* cur_v;
    const int64_t* head_to_kv;
    int q_heads;
    int kv_heads;
    int64_t tokens;
    int64_t k;      // winners per head (excluding the current slot)
    int64_t slice;  // tokens per CTA
    void* out;
    uint16_t* scores_out;   // nullable
    int64_t* indices_out;   // nullable, [B, QH, k + 1]
    float score_scale;
    float attn_scale;
};

// Dynamic shared memory layout (bytes), computed identically on host and device.
struct RetrieveSmem {
    size_t scores, mask, ulist, region, total;
    static __host__ __device__ RetrieveSmem make(int qpg, int64_t slice, int stages) {
        RetrieveSmem s;
        const size_t sc = static_cast<size_t>(qpg) * slice * 2;
        s.scores = 0;
        s.mask = (sc + 15) / 16 * 16;
        s.ulist = s.mask + (static_cast<size_t>(slice) + 15) / 16 * 16;
        s.region = s.ulist + (static_cast<size_t>(slice + 1) * 2 + 15) / 16 * 16;
        const size_t hist = static_cast<size_t>(qpg) * kHist1Bins * 4;
        const size_t ring = static_cast<size_t>(stages) * kRingRows * 2 * kRowBytes128;
        const size_t red = static_cast<size_t>(qpg) * kRetWarps * (2 + 16 * 8) * 4;
        size_t region = hist > ring ? hist : ring;
        region = region > red ? region : red;
        s.total = s.region + region;
        return s;
    }
};

template <int G, int QPG, typename QT, typename KT, int STAGES>
__global__ void __launch_bounds__(kRetThreads, 1) retrieve_kernel(const RetrieveArgs a) {
    constexpr int kRingStages = STAGES;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ QueryState<G> states[QPG];
    __shared__ float scratch[QPG][2 * 32 * 4];
    __shared__ uint32_t hist2[QPG][kHist2Bins];
    __shared__ uint32_t sel_b1[QPG];
    __shared__ unsigned long long sel_above1[QPG];
    __shared__ uint32_t sel_thr[QPG];
    __shared__ unsigned long long sel_need[QPG];
    __shared__ unsigned long long cta_gt[QPG], cta_eq[QPG];
    __shared__ unsigned long long scan_a[kRetWarps + 1], scan_b[kRetWarps + 1];
    __shared__ float part_m[QPG], part_s[QPG];
    __shared__ float part_acc[QPG][128];
    __shared__ int s_nu;
    __shared__ float s_w[16], s_den;
    __shared__ uint32_t loc_b1[QPG], loc_thr[QPG];
    __shared__ unsigned long long loc_need[QPG], loc_cgt[QPG], loc_ceq[QPG];
    __shared__ float s_part_s[16];

    cg::cluster_group cluster = cg::this_cluster();
    const int C = static_cast<int>(cluster.num_blocks());
    const int rank = static_cast<int>(cluster.block_rank());
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t cid = blockIdx.x / C;
    const int64_t b = cid / a.kv_heads;
    const int slot = static_cast<int>(cid % a.kv_heads);
    const int qh0 = slot * QPG;
    const int64_t row0 = b * a.q_heads + qh0;
    const int64_t kvh = a.head_to_kv[qh0];
    const int64_t t_begin = static_cast<int64_t>(rank) * a.slice;
    const int64_t t_end = min(t_begin + a.slice, a.tokens);
    const int n_local = t_end > t_begin ? static_cast<int>(t_end - t_begin) : 0;
    const RetrieveSmem lay = RetrieveSmem::make(QPG, a.slice, STAGES);
    uint16_t* scores16 = reinterpret_cast<uint16_t*>(smem + lay.scores);   // [QPG][slice]
    uint8_t* sel_mask = smem + lay.mask;                                    // [slice]
    uint16_t* ulist = reinterpret_cast<uint16_t*>(smem + lay.ulist);       // [slice + 1]
    uint32_t* hist1 = reinterpret_cast<uint32_t*>(smem + lay.region);      // [QPG][2048]
    unsigned char* ring = smem + lay.region;                               // aliases hist1
    float* red = reinterpret_cast<float*>(smem + lay.region);              // aliases both

    POPKV_PHASE(0);
    // ---- A: zero the histograms, encode the queries ----------------------------
    for (int i = tid; i < QPG * kHist1Bins; i += kRetThreads) hist1[i] = 0;
    for (int i = tid; i < QPG * kHist2Bins; i += kRetThreads) (&hist2[0][0])[i] = 0;
    if (warp < QPG) {
        const QT* qp = static_cast<const QT*>(a.queries) + (row0 + warp) * 128;
        encode_query_row<QT, 4>(qp, 128, G, lane, scratch[warp], states[warp].qs, states[warp].qm,
                                states[warp].ql, states[warp].dq);
    }
    __syncthreads();
    if (tid < QPG) finish_state<G>(states[tid]);
    cluster.sync();  // histograms zeroed cluster-wide before any remote add; states visible

    POPKV_PHASE(1);
    // ---- B: score the slice ---------------------------------------------------
    {
        constexpr int R = 128 / G;
        const int64_t prow = b * a.plane_batch_stride + kvh * a.capacity;
        const uint4* sign4 = reinterpret_cast<const uint4*>(a.k_sign) + prow;
        const uint4* mag4 = reinterpret_cast<const uint4*>(a.k_mag) + prow;
        const uint16_t* lowp = a.k_low + prow * R;
        const uint16_t* deltap = a.k_delta + prow * R;
        for (int base = 0; base < n_local; base += 2 * kRetThreads) {
            TokenPlanes<G> tp[2];
            bool live[2];
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int li = base + tid + i * kRetThreads;
                live[i] = li < n_local;
                load_token<G>(sign4, mag4, lowp, deltap, t_begin + (live[i] ? li : 0), tp[i]);
            }
#pragma unroll
            for (int h = 0; h < QPG; ++h) {
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const float total = score_token<G>(states[h], tp[i]);
                    if (live[i]) {
                        const int li = base + tid + i * kRetThreads;
                        const uint16_t bits = float_to_half_bits(__fmul_rn(total, a.score_scale));
                        scores16[h * a.slice + li] = bits;
                        atomicAdd(&hist1[h * kHist1Bins + (score_key(bits) >> 5)], 1u);
                        if (a.scores_out) a.scores_out[(row0 + h) * a.tokens + t_begin + li] = bits;
                    }
                }
            }
        }
    }
    __syncthreads();

    POPKV_PHASE(2);
    // ---- C: radix select across the cluster -------------------------------------
    // CTA h owns head h's selection: pass 1 pulls head h's 2048-bin histograms
    // (key bits 15..5) from every CTA through DSMEM, sums them and finds the digit
    // holding the k-th largest key; pass 2 counts the few keys inside that digit
    // by their low 5 bits into CTA h's 32-bin histogram, which gives the exact
    // threshold and the number of ties at it to take.
    const int64_t k = a.k;
    if (k > 0) {
        cluster.sync();  // all local histograms complete
        if (rank < QPG) {
            const int h = rank;
            constexpr int kPer = kHist1Bins / kRetThreads;  // 4 positions per thread
            uint32_t cnt[kPer];
            unsigned long long local = 0;
#pragma unroll
            for (int q = 0; q < kPer; ++q) {
                const int bin = kHist1Bins - 1 - (tid * kPer + q);  // descending key order
                const uint32_t* src = hist1 + h * kHist1Bins + bin;
                uint32_t v[16];
#pragma unroll
                for (int r = 0; r < 16; ++r) v[r] = r < C ? *cluster.map_shared_rank(src, r) : 0u;
                cnt[q] = 0;
#pragma unroll
                for (int r = 0; r < 16; ++r) cnt[q] += v[r];
                local += cnt[q];
            }
            unsigned long long total;
            unsigned long long run = ret_exclusive_scan<unsigned long long>(local, scan_a, total);
#pragma unroll
            for (int q = 0; q < kPer; ++q) {
                if (run < static_cast<unsigned long long>(k) && run + cnt[q] >= static_cast<unsigned long long>(k)) {
                    sel_b1[h] = kHist1Bins - 1 - (tid * kPer + q);
                    sel_above1[h] = run;
                }
                run += cnt[q];
            }
        }
        cluster.sync();  // digits chosen; pulls of every peer's histogram done
        if (tid < QPG) loc_b1[tid] = *cluster.map_shared_rank(&sel_b1[tid], tid);
        __syncthreads();
        for (int i = tid; i < n_local; i += kRetThreads) {
#pragma unroll
            for (int h = 0; h < QPG; ++h) {
                const uint32_t key = score_key(scores16[h * a.slice + i]);
                if ((key >> 5) == loc_b1[h])
                    atomicAdd(cluster.map_shared_rank(&hist2[h][0], h) + (key & 31u), 1u);
            }
        }
        cluster.sync();
        if (rank < QPG && warp == 0) {
            const int h = rank;
            const unsigned long long remaining = static_cast<unsigned long long>(k) - sel_above1[h];
            // Descending: lane j holds digit 31 - j.
            const uint32_t c2 = hist2[h][31 - lane];
            uint32_t incl = c2;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
                if (lane >= o) incl += y;
            }
            const uint32_t excl = incl - c2;
            if (excl < remaining && incl >= remaining) {
                sel_thr[h] = (sel_b1[h] << 5) | (31u - lane);
                sel_need[h] = remaining - excl;  // ties at the threshold to take
            }
        }
        cluster.sync();
        if (tid < QPG) {
            loc_thr[tid] = *cluster.map_shared_rank(&sel_thr[tid], tid);
            loc_need[tid] = *cluster.map_shared_rank(&sel_need[tid], tid);
        }
        __syncthreads();
    }

    POPKV_PHASE(3);
    // Selection of this slice, in token order.  Thread t owns local tokens
    // [t*per, (t+1)*per); per-head (greater, equal) counts travel as four
    // 16-bit fields of one 64-bit scan (per <= 16, slice <= 8192).
    {
        uint32_t thr[QPG];
        unsigned long long need[QPG];
#pragma unroll
        for (int h = 0; h < QPG; ++h) {
            thr[h] = k > 0 ? loc_thr[h] : 0u;
            need[h] = k > 0 ? loc_need[h] : 0ull;
        }
        const int per = (n_local + kRetThreads - 1) / kRetThreads;
        const int lo = min(n_local, tid * per), hi = min(n_local, lo + per);
        unsigned long long gt_pack = 0, eq_pack = 0;
        if (k > 0) {
            for (int i = lo; i < hi; ++i) {
#pragma unroll
                for (int h = 0; h < QPG; ++h) {
                    const uint32_t key = score_key(scores16[h * a.slice + i]);
                    gt_pack += static_cast<unsigned long long>(key > thr[h]) << (16 * (h & 3));
                    eq_pack += static_cast<unsigned long long>(key == thr[h]) << (16 * (h & 3));
                }
            }
        }
        // QPG <= 4 heads fit one 64-bit word per quantity.
        unsigned long long gt_tot, eq_tot;
        const unsigned long long gt_ex = ret_exclusive_scan<unsigned long long>(gt_pack, scan_a, gt_tot);
        const unsigned long long eq_ex = ret_exclusive_scan<unsigned long long>(eq_pack, scan_b, eq_tot);
        if (tid < QPG) {
            cta_gt[tid] = (gt_tot >> (16 * (tid & 3))) & 0xFFFFull;
            cta_eq[tid] = (eq_tot >> (16 * (tid & 3))) & 0xFFFFull;
        }
        cluster.sync();
        // Carries from lower ranks: lane c of warp h reads rank c's counts of head h.
        if (warp < QPG) {
            unsigned long long tg = 0, te = 0;
            if (k > 0 && lane < rank) {
                tg = *cluster.map_shared_rank(&cta_gt[warp], lane);
                te = *cluster.map_shared_rank(&cta_eq[warp], lane);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                tg += __shfl_xor_sync(0xFFFFFFFFu, tg, o);
                te += __shfl_xor_sync(0xFFFFFFFFu, te, o);
            }
            if (lane == 0) {
                loc_cgt[warp] = tg;
                loc_ceq[warp] = te;
            }
        }
        __syncthreads();
        unsigned long long gt_before[QPG], eq_before[QPG];
#pragma unroll
        for (int h = 0; h < QPG; ++h) {
            gt_before[h] = loc_cgt[h] + ((gt_ex >> (16 * (h & 3))) & 0xFFFFull);
            eq_before[h] = loc_ceq[h] + ((eq_ex >> (16 * (h & 3))) & 0xFFFFull);
        }
        for (int i = lo; i < hi; ++i) {
            uint32_t m = 0;
            if (k > 0) {
#pragma unroll
                for (int h = 0; h < QPG; ++h) {
                    const uint32_t key = score_key(scores16[h * a.slice + i]);
                    int64_t pos = -1;
                    if (key > thr[h]) {
                        pos = static_cast<int64_t>(gt_before[h] + min(eq_before[h], need[h]));
                        ++gt_before[h];
                    } else if (key == thr[h]) {
                        if (eq_before[h] < need[h]) pos = static_cast<int64_t>(gt_before[h] + eq_before[h]);
                        ++eq_before[h];
                    }
                    if (pos >= 0) {
                        m |= 1u << h;
                        if (a.indices_out) a.indices_out[(row0 + h) * (k + 1) + pos] = t_begin + i;
                    }
                }
            }
            sel_mask[i] = static_cast<uint8_t>(m);
        }
        if (rank == 0 && tid < QPG && a.indices_out) a.indices_out[(row0 + tid) * (k + 1) + k] = a.tokens;
        __syncthreads();
        // Union list of this slice's selected tokens (+ the current token on rank 0).
        int cnt = 0;
        for (int i = lo; i < hi; ++i) cnt += sel_mask[i] != 0;
        int tot;
        int pos = ret_exclusive_scan<int>(cnt, reinterpret_cast<int*>(scan_a), tot);
        for (int i = lo; i < hi; ++i)
            if (sel_mask[i]) ulist[pos++] = static_cast<uint16_t>(i);
        if (tid == 0) {
            int nu = tot;
            if (rank == 0) ulist[nu++] = kCurrentEntry;
            s_nu = nu;
        }
        __syncthreads();
    }

    POPKV_PHASE(4);
    // ---- D: attention over the union rows ---------------------------------------
    const int nu = s_nu;
#ifdef POPKV_RETRIEVE_TIMING
    if (threadIdx.x == 0 && blockIdx.x < 2048) g_retrieve_phase_ns[blockIdx.x][8] = static_cast<unsigned long long>(nu);
#endif
    const int g = tid >> 4, c = tid & 15;  // row group, 16-byte unit (dims 8c..8c+7)
    float qv[QPG][8];
#pragma unroll
    for (int h = 0; h < QPG; ++h) {
        const QT* qp = static_cast<const QT*>(a.queries) + (row0 + h) * 128 + 8 * c;
        const float qs = a.attn_scale * kLog2eF;
#pragma unroll
        for (int j = 0; j < 8; ++j) qv[h][j] = load_float(qp + j) * qs;
    }
    float m_[QPG], s_[QPG], acc[QPG][8];
#pragma unroll
    for (int h = 0; h < QPG; ++h) {
        m_[h] = -INFINITY;
        s_[h] = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[h][j] = 0.0f;
    }
    const unsigned char* kbase = reinterpret_cast<const unsigned char*>(
        static_cast<const KT*>(a.prefix_k) + b * a.kbs + kvh * a.khs + t_begin * a.kts) + c * 16;
    const unsigned char* vbase = reinterpret_cast<const unsigned char*>(
        static_cast<const KT*>(a.prefix_v) + b * a.vbs + kvh * a.vhs + t_begin * a.vts) + c * 16;
    const unsigned char* ckp = reinterpret_cast<const unsigned char*>(
        static_cast<const KT*>(a.cur_k) + (b * a.kv_heads + kvh) * 128) + c * 16;
    const unsigned char* cvp = reinterpret_cast<const unsigned char*>(
        static_cast<const KT*>(a.cur_v) + (b * a.kv_heads + kvh) * 128) + c * 16;
    const int64_t kstride = a.kts * 2, vstride = a.vts * 2;
    const int nstage = (nu + kRingRows - 1) / kRingRows;
    auto stage_k = [&](int st) { return ring + ((st * 2 + 0) * kRingRows + g) * kRowBytes128 + c * 16; };
    auto stage_v = [&](int st) { return ring + ((st * 2 + 1) * kRingRows + g) * kRowBytes128 + c * 16; };
    auto issue = [&](int i) {
        if (i < nstage) {
            const int u = i * kRingRows + g;
            if (u < nu) {
                const uint16_t e = ulist[u];
                const unsigned char* ks = e == kCurrentEntry ? ckp : kbase + static_cast<int64_t>(e) * kstride;
                const unsigned char* vs = e == kCurrentEntry ? cvp : vbase + static_cast<int64_t>(e) * vstride;
                cp_async16_ret(stage_k(i % kRingStages), ks);
                cp_async16_ret(stage_v(i % kRingStages), vs);
            }
        }
        cp_async_commit_ret();
    };
#pragma unroll
    for (int i = 0; i < kRingStages - 1; ++i) issue(i);
    for (int i = 0; i < nstage; ++i) {
        issue(i + kRingStages - 1);
        cp_async_wait_ret<kRingStages - 1>();
        const int u = i * kRingRows + g;
        const bool has = u < nu;
        uint32_t mask = 0;
        float kf[8], vf[8];
        if (has) {
            const uint16_t e = ulist[u];
            mask = e == kCurrentEntry ? ((1u << QPG) - 1u) : sel_mask[e];
            unpack8_ret<KT>(*reinterpret_cast<const uint4*>(stage_k(i % kRingStages)), kf);
            unpack8_ret<KT>(*reinterpret_cast<const uint4*>(stage_v(i % kRingStages)), vf);
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) kf[j] = vf[j] = 0.0f;
        }
        // The 16 lanes of a row group share `mask`, so a head's dot product and
        // its shuffles run only in the groups that selected the row.
        const unsigned group = 0xFFFFu << (lane & 16);
#pragma unroll
        for (int h = 0; h < QPG; ++h) {
            if (mask & (1u << h)) {
                float dot = 0.0f;
#pragma unroll
                for (int j = 0; j < 8; ++j) dot = __fmaf_rn(kf[j], qv[h][j], dot);
#pragma unroll
                for (int o = 8; o > 0; o >>= 1) dot += __shfl_xor_sync(group, dot, o);
                if (dot > m_[h]) {
                    const float alpha = exp2f(m_[h] - dot);
                    s_[h] = __fmaf_rn(s_[h], alpha, 1.0f);
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[h][j] = __fmaf_rn(acc[h][j], alpha, vf[j]);
                    m_[h] = dot;
                } else {
                    const float p = exp2f(dot - m_[h]);
                    s_[h] += p;
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[h][j] = __fmaf_rn(p, vf[j], acc[h][j]);
                }
            }
        }
    }
    cp_async_wait_ret<0>();
    __syncthreads();  // the ring is reused below

    POPKV_PHASE(5);
    // Combine the two row groups of each warp, then the 16 warps, per head.
    float* red_m = red;                                       // [QPG][16]
    float* red_s = red + QPG * kRetWarps;                     // [QPG][16]
    float* red_acc = red + 2 * QPG * kRetWarps;               // [QPG][16 warps][16 c][8]
#pragma unroll
    for (int h = 0; h < QPG; ++h) {
        const float m2 = __shfl_xor_sync(0xFFFFFFFFu, m_[h], 16);
        const float s2 = __shfl_xor_sync(0xFFFFFFFFu, s_[h], 16);
        const float M = fmaxf(m_[h], m2);
        const float f1 = m_[h] == -INFINITY ? 0.0f : exp2f(m_[h] - M);
        const float f2 = m2 == -INFINITY ? 0.0f : exp2f(m2 - M);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float a2 = __shfl_xor_sync(0xFFFFFFFFu, acc[h][j], 16);
            acc[h][j] = acc[h][j] * f1 + a2 * f2;
        }
        s_[h] = s_[h] * f1 + s2 * f2;
        m_[h] = M;
        if (lane < 16) {
#pragma unroll
            for (int j = 0; j < 8; ++j) red_acc[((h * kRetWarps + warp) * 16 + lane) * 8 + j] = acc[h][j];
            if (lane == 0) {
                red_m[h * kRetWarps + warp] = m_[h];
                red_s[h * kRetWarps + warp] = s_[h];
            }
        }
    }
    __syncthreads();
    for (int idx = tid; idx < QPG * 128; idx += kRetThreads) {
        const int h = idx / 128, d = idx % 128;
        float M = -INFINITY;
        for (int w = 0; w < kRetWarps; ++w) M = fmaxf(M, red_m[h * kRetWarps + w]);
        float accd = 0.0f, sum = 0.0f;
        if (M != -INFINITY) {
            for (int w = 0; w < kRetWarps; ++w) {
                const float mw = red_m[h * kRetWarps + w];
                if (mw == -INFINITY) continue;
                const float f = exp2f(mw - M);
                accd = __fmaf_rn(red_acc[((h * kRetWarps + w) * 16 + (d >> 3)) * 8 + (d & 7)], f, accd);
                sum = __fmaf_rn(red_s[h * kRetWarps + w], f, sum);
            }
        }
        part_acc[h][d] = accd;
        if (d == 0) {
            part_m[h] = M;  // log2 units
            part_s[h] = sum;
        }
    }
    cluster.sync();  // partial states of every CTA visible

    POPKV_PHASE(6);
    // ---- E: CTA h merges head h ---------------------------------------------------
    if (rank < QPG) {
        const int h = rank;
        if (tid < C) {
            s_w[tid] = *cluster.map_shared_rank(&part_m[h], tid);
            s_part_s[tid] = *cluster.map_shared_rank(&part_s[h], tid);
        }
        __syncthreads();
        if (tid == 0) {
            float M = -INFINITY;
            for (int q = 0; q < C; ++q) M = fmaxf(M, s_w[q]);
            float den = 0.0f;
            for (int q = 0; q < C; ++q) {
                const float w = s_w[q] == -INFINITY ? 0.0f : exp2f(s_w[q] - M);
                den = __fmaf_rn(s_part_s[q], w, den);
                s_w[q] = w;
            }
            s_den = den;
        }
        __syncthreads();
        if (tid < 128) {
            float v[16];
#pragma unroll
            for (int q = 0; q < 16; ++q) v[q] = q < C ? cluster.map_shared_rank(&part_acc[h][0], q)[tid] : 0.0f;
            float num = 0.0f;
#pragma unroll
            for (int q = 0; q < 16; ++q)
                if (q < C) num = __fmaf_rn(v[q], s_w[q], num);
            store_elem(static_cast<QT*>(a.out) + (row0 + h) * 128 + tid, num / s_den);
        }
    }
    cluster.sync();  // keep this CTA's shared memory alive until every peer has read it
    POPKV_PHASE(7);
}

constexpr size_t kSmemLimit = 227 * 1024 - 16 * 1024;  // dynamic budget beside static smem

template <int G, int QPG, typename QT, typename KT, int STAGES>
int launch_retrieve_s(const RetrieveArgs& args, int64_t clusters, cudaStream_t stream, bool* tried) {
    auto kernel = retrieve_kernel<G, QPG, QT, KT, STAGES>;
    cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    cudaLaunchConfig_t config = {};
    config.blockDim = dim3(kRetThreads, 1, 1);
    config.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    config.attrs = attr;
    config.numAttrs = 1;
    // Pick the cluster size minimising (waves x tokens per CTA): every cluster of
    // a wave must fit on the GPCs at once (one CTA per SM).
    int best_cs = 0;
    double best_cost = 0.0;
    int64_t best_slice = 0;
    for (int cs = 16; cs >= 8; --cs) {
        int64_t slice = ((args.tokens + cs - 1) / cs + 63) / 64 * 64;
        if (slice < 64) slice = 64;
        if (slice > kMaxSlice) continue;
        const RetrieveSmem lay = RetrieveSmem::make(QPG, slice, STAGES);
        if (lay.total > kSmemLimit) continue;
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(lay.total)) != cudaSuccess) {
            cudaGetLastError();
            continue;
        }
        attr[0].val.clusterDim.x = cs;
        config.gridDim = dim3(static_cast<unsigned>(clusters * cs), 1, 1);
        config.dynamicSmemBytes = lay.total;
        int active = 0;
        if (cudaOccupancyMaxActiveClusters(&active, kernel, &config) != cudaSuccess || active < 1) {
            cudaGetLastError();
            continue;
        }
        const double waves = static_cast<double>((clusters + active - 1) / active);
        const double cost = waves * static_cast<double>(slice);
        if (best_cs == 0 || cost < best_cost) {
            best_cs = cs;
            best_cost = cost;
            best_slice = slice;
        }
    }
    if (best_cs == 0) return POPKV_ERR_UNSUPPORTED;
    *tried = true;
    RetrieveArgs a = args;
    a.slice = best_slice;
    const RetrieveSmem lay = RetrieveSmem::make(QPG, best_slice, STAGES);
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(lay.total));
    if (err != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_retrieve: %s", cudaGetErrorString(err));
    attr[0].val.clusterDim.x = best_cs;
    config.gridDim = dim3(static_cast<unsigned>(clusters * best_cs), 1, 1);
    config.dynamicSmemBytes = lay.total;
    err = cudaLaunchKernelEx(&config, kernel, a);
    if (err != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_retrieve: %s", cudaGetErrorString(err));
    return check_launch("popkv_retrieve");
}

template <int G, int QPG, typename QT, typename KT>
int launch_retrieve_t(const RetrieveArgs& args, int64_t clusters, cudaStream_t stream) {
    bool tried = false;
    int st = launch_retrieve_s<G, QPG, QT, KT, 8>(args, clusters, stream, &tried);
    if (tried || st != POPKV_ERR_UNSUPPORTED) return st;
    st = launch_retrieve_s<G, QPG, QT, KT, 4>(args, clusters, stream, &tried);
    if (tried || st != POPKV_ERR_UNSUPPORTED) return st;
    return fail(POPKV_ERR_UNSUPPORTED, "popkv_retrieve: no cluster size can be scheduled for %lld tokens",
                static_cast<long long>(args.tokens));
}

template <int G, typename QT, typename KT>
int dispatch_qpg(int qpg, const RetrieveArgs& args, int64_t clusters, cudaStream_t stream) {
    switch (qpg) {
        case 1: return launch_retrieve_t<G, 1, QT, KT>(args, clusters, stream);
        case 2: return launch_retrieve_t<G, 2, QT, KT>(args, clusters, stream);
        case 4: return launch_retrieve_t<G, 4, QT, KT>(args, clusters, stream);
        default:
            return fail(POPKV_ERR_UNSUPPORTED, "popkv_retrieve: %d query heads per KV head (1, 2 or 4 supported)", qpg);
    }
}

template <typename QT, typename KT>
int dispatch_g(int64_t g, int qpg, const RetrieveArgs& args, int64_t clusters, cudaStream_t stream) {
    if (g == 16) return dispatch_qpg<16, QT, KT>(qpg, args, clusters, stream);
    if (g == 32) return dispatch_qpg<32, QT, KT>(qpg, args, clusters, stream);
    return dispatch_qpg<64, QT, KT>(qpg, args, clusters, stream);
}

}  // namespace
}  // namespace popkv

extern "C" int popkv_retrieve(
    const void* queries, int queries_dtype, int64_t batch, int64_t q_heads, int64_t head_dim,
    const int32_t* k_sign, const int32_t* k_mag, const uint16_t* k_low, const uint16_t* k_delta,
    int64_t kv_heads, int64_t capacity, int64_t plane_batch_stride, int64_t tokens,
    int64_t dim_group_size, const int64_t* head_to_kv, const void* prefix_keys,
    const void* prefix_values, int kv_dtype, int64_t k_batch_stride, int64_t k_head_stride,
    int64_t k_token_stride, int64_t v_batch_stride, int64_t v_head_stride, int64_t v_token_stride,
    const void* current_keys, const void* current_values, int64_t budget, void* out,
    uint16_t* scores_out, int64_t* indices_out, void* stream) {
    using namespace popkv;
    if (head_dim != 128) return fail(POPKV_ERR_UNSUPPORTED, "popkv_retrieve: head_dim must be 128");
    if (queries_dtype != kv_dtype || (kv_dtype != POPKV_DTYPE_BF16 && kv_dtype != POPKV_DTYPE_F16))
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_retrieve: queries and K/V must both be bf16 or both fp16");
    if (dim_group_size != 16 && dim_group_size != 32 && dim_group_size != 64)
        return fail(POPKV_ERR_INVALID, "dim_group_size must be 16, 32, or 64");
    if (batch < 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads)
        return fail(POPKV_ERR_INVALID, "invalid GQA head mapping");
    if (budget <= 1)
        return fail(POPKV_ERR_INVALID, "budget must reserve at least one retrieved and one current token");
    if (tokens < 0 || tokens > capacity) return fail(POPKV_ERR_INVALID, "invalid score token count");
    if (tokens > 16 * popkv::kMaxSlice)
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_retrieve: at most %d tokens", 16 * popkv::kMaxSlice);
    if (batch == 0) return POPKV_OK;
    if (!queries || !k_sign || !k_mag || !k_low || !k_delta || !head_to_kv || !prefix_keys ||
        !prefix_values || !current_keys || !current_values || !out)
        return fail(POPKV_ERR_INVALID, "popkv_retrieve: null pointer");
    if (!aligned(k_sign, 16) || !aligned(k_mag, 16) || !aligned(k_low, 16) || !aligned(k_delta, 16) ||
        !aligned(prefix_keys, 16) || !aligned(prefix_values, 16) || !aligned(current_keys, 16) ||
        !aligned(current_values, 16) || (k_batch_stride % 8) || (k_head_stride % 8) ||
        (k_token_stride % 8) || (v_batch_stride % 8) || (v_head_stride % 8) || (v_token_stride % 8))
        return fail(POPKV_ERR_INVALID, "popkv_retrieve: planes and K/V rows must be 16-byte aligned");
    const int qpg = static_cast<int>(q_heads / kv_heads);
    RetrieveArgs args;
    args.queries = queries;
    args.k_sign = k_sign;
    args.k_mag = k_mag;
    args.k_low = k_low;
    args.k_delta = k_delta;
    args.capacity = capacity;
    args.plane_batch_stride = plane_batch_stride;
    args.prefix_k = prefix_keys;
    args.prefix_v = prefix_values;
    args.kbs = k_batch_stride; args.khs = k_head_stride; args.kts = k_token_stride;
    args.vbs = v_batch_stride; args.vhs = v_head_stride; args.vts = v_token_stride;
    args.cur_k = current_keys;
    args.cur_v = current_values;
    args.head_to_kv = head_to_kv;
    args.q_heads = static_cast<int>(q_heads);
    args.kv_heads = static_cast<int>(kv_heads);
    args.tokens = tokens;
    args.k = budget - 1 < tokens ? budget - 1 : tokens;
    args.slice = 0;  // set per cluster size by the launcher
    args.out = out;
    args.scores_out = scores_out;
    args.indices_out = indices_out;
    args.score_scale = score_scale_for(128);
    args.attn_scale = score_scale_for(128);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t clusters = batch * kv_heads;
    if (kv_dtype == POPKV_DTYPE_BF16)
        return dispatch_g<__nv_bfloat16, __nv_bfloat16>(dim_group_size, qpg, args, clusters, s);
    return dispatch_g<__half, __half>(dim_group_size, qpg, args, clusters, s);
}

#ifdef POPKV_RETRIEVE_TIMING
extern "C" __attribute__((visibility("default"))) int popkv_retrieve_phase_reset() {
    static unsigned long long zeros[2048 * 16];
    return static_cast<int>(cudaMemcpyToSymbol(g_retrieve_phase_ns, zeros, sizeof(zeros)));
}

extern "C" __attribute__((visibility("default"))) int popkv_retrieve_phase_ns(unsigned long long* host, int ctas) {
    return static_cast<int>(cudaMemcpyFromSymbol(host, g_retrieve_phase_ns,
                                                  sizeof(unsigned long long) * 16 * static_cast<size_t>(ctas)));
}

extern "C" __attribute__((visibility("default"))) int popkv_retrieve_max_clusters(int cluster, int slice) {
    using namespace popkv;
    auto kernel = retrieve_kernel<16, 4, __nv_bfloat16, __nv_bfloat16, 8>;
    const RetrieveSmem lay = RetrieveSmem::make(4, slice, 8);
    cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(lay.total));
    cudaLaunchConfig_t config = {};
    config.blockDim = dim3(kRetThreads, 1, 1);
    config.gridDim = dim3(static_cast<unsigned>(8 * cluster), 1, 1);
    config.dynamicSmemBytes = lay.total;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    config.attrs = attr;
    config.numAttrs = 1;
    int active = -1;
    cudaError_t e = cudaOccupancyMaxActiveClusters(&active, kernel, &config);
    return e == cudaSuccess ? active : -100 - static_cast<int>(e);
}
#endif
