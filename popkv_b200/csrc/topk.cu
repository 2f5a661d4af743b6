// Per-query-head top-k with the current-token slot reserved (PopKV subsystem 3).
//
// Replaces torch.topk(scores, k, dim=-1, sorted=False).indices followed by
// _append_current (reference popkv.py:1094-1098, :287-291).  torch.topk leaves
// the order among equal scores unspecified; this kernel fixes it: higher score
// first, then lower token index, and the k winners are written in ascending
// token order (the order the attention gather reads the cache in).
//
// Radix select on an order-preserving integer key of each score, one CTA per
// row.  The row's keys are staged in shared memory when they fit.  Each pass
// builds a shared-memory histogram of the next digit of the keys that still
// match the threshold prefix (fp16: 11 + 5 bits; fp32: 11 + 11 + 10 bits) and
// a block-wide scan picks the digit holding the k-th largest key.  The final
// pass gives every thread a contiguous slice of the row: a block scan of its
// (greater, equal) counts yields each winner's output position, taking equal
// keys in index order until the quota is filled.
#include <cooperative_groups.h>

#include <cstdint>
#include <type_traits>

#include "common.cuh"

// Phase timestamps for profiling builds (-DPOPKV_TOPK_TIMING): thread 0 of each
// CTA of the cluster kernel records %globaltimer at its phase boundaries.
#ifdef POPKV_TOPK_TIMING
__device__ unsigned long long g_topk_phase_ns[1024][8];
#define POPKV_TOPK_PHASE(i)                                                              \
    do {                                                                                 \
        if (threadIdx.x == 0 && blockIdx.x < 1024) {                                     \
            unsigned long long t_;                                                       \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                      \
            g_topk_phase_ns[blockIdx.x][i] = t_;                                         \
        }                                                                                \
    } while (0)
extern "C" __attribute__((visibility("default"))) int popkv_topk_phase_ns(unsigned long long* host, int ctas) {
    return static_cast<int>(cudaMemcpyFromSymbol(host, g_topk_phase_ns, sizeof(unsigned long long) * 8 * ctas));
}
#else
#define POPKV_TOPK_PHASE(i) \
    do {                    \
    } while (0)
#endif

namespace popkv {
namespace {

constexpr int kTopkThreads = 1024;
constexpr int kTopkWarps = kTopkThreads / 32;
constexpr int kHistBins = 2048;
constexpr size_t kStageBytes = 96 * 1024;

// -0 == +0, NaN ranks highest (the key the score kernels' histograms use).
__device__ __forceinline__ uint32_t key16(uint16_t h) { return order_key16(h); }

__device__ __forceinline__ uint32_t key32(uint32_t u) {
    if ((u & 0x7FFFFFFFu) == 0) u = 0;
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return 0xFFFFFFFFu;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <bool F32>
__device__ __forceinline__ uint32_t load_key(const void* row, int64_t i) {
    if constexpr (F32) return key32(static_cast<const uint32_t*>(row)[i]);
    else return key16(static_cast<const uint16_t*>(row)[i]);
}

// Block-wide exclusive scan of one value per thread; `total` receives the sum.
template <typename V>
__device__ __forceinline__ V block_exclusive_scan(V x, V* warp_sums, V& total) {
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
        V w = lane < kTopkWarps ? warp_sums[lane] : V(0);
        V wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            V y = __shfl_up_sync(0xFFFFFFFFu, wi, o);
            if (lane >= o) wi += y;
        }
        if (lane < kTopkWarps) warp_sums[lane] = wi - w;
        if (lane == kTopkWarps - 1) warp_sums[kTopkWarps] = wi;
    }
    __syncthreads();
    V result = warp_sums[warp] + incl - x;
    total = warp_sums[kTopkWarps];
    __syncthreads();
    return result;
}

template <bool F32, bool STAGED>
__global__ void __launch_bounds__(kTopkThreads) topk_kernel(
    const void* __restrict__ scores, int64_t tokens, int64_t row_stride, int64_t k,
    int64_t current_index, int64_t* __restrict__ out, int64_t out_stride) {
    extern __shared__ __align__(16) unsigned char staged_raw[];
    __shared__ uint32_t hist[kHistBins];
    __shared__ unsigned long long scan_sums[kTopkWarps + 1];
    __shared__ uint32_t sel_bin;
    __shared__ unsigned long long sel_above;

    using KeyT = typename std::conditional<F32, uint32_t, uint16_t>::type;
    KeyT* staged = reinterpret_cast<KeyT*>(staged_raw);
    const int64_t row = blockIdx.x;
    const void* src = F32 ? static_cast<const void*>(static_cast<const float*>(scores) + row * row_stride)
                          : static_cast<const void*>(static_cast<const uint16_t*>(scores) + row * row_stride);
    int64_t* dst = out + row * out_stride;
    const int tid = threadIdx.x;

    if (current_index >= 0 && tid == 0) dst[k] = current_index;
    if (k <= 0) return;

    auto key_at = [&](int64_t i) -> uint32_t {
        if constexpr (STAGED) return staged[i];
        else return load_key<F32>(src, i);
    };
    if constexpr (STAGED) {
        for (int64_t i = tid; i < tokens; i += kTopkThreads) staged[i] = static_cast<KeyT>(load_key<F32>(src, i));
        __syncthreads();
    }

    // Radix passes: find the threshold key (the k-th largest).
    constexpr int kPasses = F32 ? 3 : 2;
    const int shifts[3] = {F32 ? 21 : 5, F32 ? 10 : 0, 0};
    const int widths[3] = {11, F32 ? 11 : 5, 10};
    uint32_t prefix = 0, prefix_mask = 0;
    unsigned long long above = 0;  // keys strictly above the current prefix range
#pragma unroll 1
    for (int p = 0; p < kPasses; ++p) {
        const int shift = shifts[p], width = widths[p];
        const uint32_t nbins = 1u << width;
        const uint32_t digit_mask = nbins - 1u;
        for (uint32_t b = tid; b < nbins; b += kTopkThreads) hist[b] = 0;
        __syncthreads();
        for (int64_t i = tid; i < tokens; i += kTopkThreads) {
            const uint32_t key = key_at(i);
            if ((key & prefix_mask) == prefix) atomicAdd(&hist[(key >> shift) & digit_mask], 1u);
        }
        __syncthreads();
        // Descending-digit scan: position j holds digit nbins - 1 - j.
        const unsigned long long remaining = static_cast<unsigned long long>(k) - above;
        const uint32_t per = (nbins + kTopkThreads - 1) / kTopkThreads;  // 1 or 2
        unsigned long long local = 0;
        for (uint32_t j = tid * per; j < min(nbins, (tid + 1) * per); ++j) local += hist[nbins - 1 - j];
        unsigned long long total;
        unsigned long long excl = block_exclusive_scan<unsigned long long>(local, scan_sums, total);
        unsigned long long run = excl;
        for (uint32_t j = tid * per; j < min(nbins, (tid + 1) * per); ++j) {
            const uint32_t cnt = hist[nbins - 1 - j];
            if (run < remaining && run + cnt >= remaining) {
                sel_bin = nbins - 1 - j;
                sel_above = run;
            }
            run += cnt;
        }
        __syncthreads();
        prefix |= sel_bin << shift;
        prefix_mask |= digit_mask << shift;
        above += sel_above;
        __syncthreads();
    }
    const uint32_t threshold = prefix;
    const unsigned long long need = static_cast<unsigned long long>(k) - above;  // ties to take

    // Compaction over contiguous slices, in token order.
    const int64_t chunk = (tokens + kTopkThreads - 1) / kTopkThreads;
    const int64_t lo = min(tokens, tid * chunk), hi = min(tokens, lo + chunk);
    unsigned int gt = 0, eq = 0;
    for (int64_t i = lo; i < hi; ++i) {
        const uint32_t key = key_at(i);
        gt += key > threshold;
        eq += key == threshold;
    }
    unsigned long long packed = (static_cast<unsigned long long>(gt) << 32) | eq;
    unsigned long long total;
    unsigned long long excl = block_exclusive_scan<unsigned long long>(packed, scan_sums, total);
    unsigned long long gt_before = excl >> 32, eq_before = excl & 0xFFFFFFFFull;
    for (int64_t i = lo; i < hi; ++i) {
        const uint32_t key = key_at(i);
        if (key > threshold) {
            const unsigned long long pos = gt_before + min(eq_before, need);
            if (pos < static_cast<unsigned long long>(k)) dst[pos] = i;
            ++gt_before;
        } else if (key == threshold) {
            const unsigned long long pos = gt_before + eq_before;
            if (eq_before < need && pos < static_cast<unsigned long long>(k)) dst[pos] = i;
            ++eq_before;
        }
    }
}

// Register-resident variant for rows of up to kTopkThreads * kVec * CHUNKS
// scores: one vectorised pass over the row puts every key in registers (chunk
// c = tid + kTopkThreads * j holds elements [c * kVec, (c + 1) * kVec)); the
// histogram passes and the compaction then run on registers only.  Round j of
// the compaction covers a contiguous slice of the row in thread order, so a
// block scan per round (carrying the previous rounds' totals) yields the
// ascending-index output positions.
template <bool F32, int CHUNKS>
__global__ void __launch_bounds__(kTopkThreads) topk_reg_kernel(
    const void* __restrict__ scores, int64_t tokens, int64_t row_stride, int64_t k,
    int64_t current_index, int64_t* __restrict__ out, int64_t out_stride, bool vec_ok) {
    constexpr int kVec = F32 ? 4 : 8;
    __shared__ uint32_t hist[kHistBins];
    __shared__ unsigned long long scan_sums[kTopkWarps + 1];
    __shared__ uint32_t sel_bin;
    __shared__ unsigned long long sel_above;

    const int64_t row = blockIdx.x;
    const int tid = threadIdx.x;
    int64_t* dst = out + row * out_stride;
    if (current_index >= 0 && tid == 0) dst[k] = current_index;
    if (k <= 0) return;

    // Four registers per chunk: fp32 keys one per register, fp16 keys two per register.
    uint32_t packed[CHUNKS][4];
#pragma unroll
    for (int j = 0; j < CHUNKS; ++j) {
        const int64_t base = (static_cast<int64_t>(tid) + static_cast<int64_t>(kTopkThreads) * j) * kVec;
        if (vec_ok && base + kVec <= tokens) {
            if constexpr (F32) {
                const uint4 v = __ldg(reinterpret_cast<const uint4*>(
                    static_cast<const float*>(scores) + row * row_stride + base));
                packed[j][0] = key32(v.x); packed[j][1] = key32(v.y);
                packed[j][2] = key32(v.z); packed[j][3] = key32(v.w);
            } else {
                const uint4 v = __ldg(reinterpret_cast<const uint4*>(
                    static_cast<const uint16_t*>(scores) + row * row_stride + base));
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    packed[j][e] = key16(static_cast<uint16_t>(w[e] & 0xFFFFu)) |
                                   (key16(static_cast<uint16_t>(w[e] >> 16)) << 16);
            }
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) packed[j][e] = 0;
#pragma unroll
            for (int e = 0; e < kVec; ++e) {
                const int64_t i = base + e;
                if (i < tokens) {
                    if constexpr (F32) packed[j][e] = key32(static_cast<const uint32_t*>(scores)[row * row_stride + i]);
                    else packed[j][e >> 1] |= key16(static_cast<const uint16_t*>(scores)[row * row_stride + i]) << (16 * (e & 1));
                }
            }
        }
    }
    auto key_of = [&](int j, int e) -> uint32_t {
        if constexpr (F32) return packed[j][e];
        else return (packed[j][e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
    };
    auto valid = [&](int j, int e) -> bool {
        return (static_cast<int64_t>(tid) + static_cast<int64_t>(kTopkThreads) * j) * kVec + e < tokens;
    };

    constexpr int kPasses = F32 ? 3 : 2;
    const int shifts[3] = {F32 ? 21 : 5, F32 ? 10 : 0, 0};
    const int widths[3] = {11, F32 ? 11 : 5, 10};
    uint32_t prefix = 0, prefix_mask = 0;
    unsigned long long above = 0;
#pragma unroll 1
    for (int p = 0; p < kPasses; ++p) {
        const int shift = shifts[p], width = widths[p];
        const uint32_t nbins = 1u << width;
        const uint32_t digit_mask = nbins - 1u;
        for (uint32_t b = tid; b < nbins; b += kTopkThreads) hist[b] = 0;
        __syncthreads();
#pragma unroll
        for (int j = 0; j < CHUNKS; ++j)
#pragma unroll
            for (int e = 0; e < kVec; ++e)
                if (valid(j, e) && (key_of(j, e) & prefix_mask) == prefix)
                    atomicAdd(&hist[(key_of(j, e) >> shift) & digit_mask], 1u);
        __syncthreads();
        const unsigned long long remaining = static_cast<unsigned long long>(k) - above;
        const uint32_t per = (nbins + kTopkThreads - 1) / kTopkThreads;
        unsigned long long local = 0;
        for (uint32_t jj = tid * per; jj < min(nbins, (tid + 1) * per); ++jj) local += hist[nbins - 1 - jj];
        unsigned long long total;
        unsigned long long run = block_exclusive_scan<unsigned long long>(local, scan_sums, total);
        for (uint32_t jj = tid * per; jj < min(nbins, (tid + 1) * per); ++jj) {
            const uint32_t cnt = hist[nbins - 1 - jj];
            if (run < remaining && run + cnt >= remaining) {
                sel_bin = nbins - 1 - jj;
                sel_above = run;
            }
            run += cnt;
        }
        __syncthreads();
        prefix |= sel_bin << shift;
        prefix_mask |= digit_mask << shift;
        above += sel_above;
        __syncthreads();
    }
    const uint32_t threshold = prefix;
    const unsigned long long need = static_cast<unsigned long long>(k) - above;

    unsigned long long gt_carry = 0, eq_carry = 0;
#pragma unroll
    for (int j = 0; j < CHUNKS; ++j) {
        unsigned int gt = 0, eq = 0;
#pragma unroll
        for (int e = 0; e < kVec; ++e) {
            if (valid(j, e)) {
                gt += key_of(j, e) > threshold;
                eq += key_of(j, e) == threshold;
            }
        }
        unsigned long long total;
        const unsigned long long excl = block_exclusive_scan<unsigned long long>(
            (static_cast<unsigned long long>(gt) << 32) | eq, scan_sums, total);
        unsigned long long gt_before = gt_carry + (excl >> 32);
        unsigned long long eq_before = eq_carry + (excl & 0xFFFFFFFFull);
        const int64_t base = (static_cast<int64_t>(tid) + static_cast<int64_t>(kTopkThreads) * j) * kVec;
#pragma unroll
        for (int e = 0; e < kVec; ++e) {
            if (!valid(j, e)) continue;
            const uint32_t key = key_of(j, e);
            if (key > threshold) {
                const unsigned long long pos = gt_before + min(eq_before, need);
                if (pos < static_cast<unsigned long long>(k)) dst[pos] = base + e;
                ++gt_before;
            } else if (key == threshold) {
                const unsigned long long pos = gt_before + eq_before;
                if (eq_before < need && pos < static_cast<unsigned long long>(k)) dst[pos] = base + e;
                ++eq_before;
            }
        }
        gt_carry += total >> 32;
        eq_carry += total & 0xFFFFFFFFull;
    }
}

// ---------------------------------------------------------------------------
// Cluster variant: CPR CTAs (a thread-block cluster) share one row, so a few
// dozen rows still occupy every SM.  CTA q of the cluster holds the keys of
// row slice [q * slice, (q + 1) * slice) in registers; after each local
// histogram pass the cluster barrier makes the CPR shared-memory histograms
// visible and every CTA sums them through distributed shared memory, so all
// CTAs pick the same digit.  For the compaction each CTA publishes its
// (greater, equal) totals; a CTA's output offset is the sum over lower ranks.
// ---------------------------------------------------------------------------
namespace cg = cooperative_groups;
constexpr int kClusterThreads = 512;
constexpr int kClusterWarps = kClusterThreads / 32;

template <typename V>
__device__ __forceinline__ V cta_exclusive_scan(V x, V* warp_sums, V& total) {
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
        V w = lane < kClusterWarps ? warp_sums[lane] : V(0);
        V wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            V y = __shfl_up_sync(0xFFFFFFFFu, wi, o);
            if (lane >= o) wi += y;
        }
        if (lane < kClusterWarps) warp_sums[lane] = wi - w;
        if (lane == kClusterWarps - 1) warp_sums[kClusterWarps] = wi;
    }
    __syncthreads();
    V result = warp_sums[warp] + incl - x;
    total = warp_sums[kClusterWarps];
    __syncthreads();
    return result;
}

template <bool F32, int CPR, int CHUNKS>
__global__ void __launch_bounds__(kClusterThreads) topk_cluster_kernel(
    const void* __restrict__ scores, int64_t tokens, int64_t row_stride, int64_t k,
    int64_t current_index, int64_t* __restrict__ out, int64_t out_stride, bool vec_ok) {
    constexpr int kVec = F32 ? 4 : 8;
    constexpr int64_t kSlice = static_cast<int64_t>(kClusterThreads) * kVec * CHUNKS;
    __shared__ uint32_t hist[kHistBins];
    __shared__ unsigned long long scan_sums[kClusterWarps + 1];
    __shared__ uint32_t sel_bin;
    __shared__ unsigned long long sel_above;
    __shared__ unsigned long long cta_totals;  // (gt << 32) | eq of this CTA

    POPKV_TOPK_PHASE(0);
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = static_cast<int>(cluster.block_rank());
    const int64_t row = blockIdx.x / CPR;
    const int tid = threadIdx.x;
    int64_t* dst = out + row * out_stride;
    if (current_index >= 0 && tid == 0 && rank == 0) dst[k] = current_index;
    if (k <= 0) return;  // uniform across the cluster: no CTA reaches a cluster barrier

    const int64_t slice0 = static_cast<int64_t>(rank) * kSlice;
    uint32_t packed[CHUNKS][4];
    int lim[CHUNKS];  // valid elements of each chunk (0..kVec)
#pragma unroll
    for (int j = 0; j < CHUNKS; ++j) {
        const int64_t base = slice0 + (static_cast<int64_t>(tid) + static_cast<int64_t>(kClusterThreads) * j) * kVec;
        const int64_t left = tokens - base;
        lim[j] = left <= 0 ? 0 : (left >= kVec ? kVec : static_cast<int>(left));
        if (vec_ok && lim[j] == kVec) {
            if constexpr (F32) {
                const uint4 v = __ldg(reinterpret_cast<const uint4*>(
                    static_cast<const float*>(scores) + row * row_stride + base));
                packed[j][0] = key32(v.x); packed[j][1] = key32(v.y);
                packed[j][2] = key32(v.z); packed[j][3] = key32(v.w);
            } else {
                const uint4 v = __ldg(reinterpret_cast<const uint4*>(
                    static_cast<const uint16_t*>(scores) + row * row_stride + base));
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    packed[j][e] = key16(static_cast<uint16_t>(w[e] & 0xFFFFu)) |
                                   (key16(static_cast<uint16_t>(w[e] >> 16)) << 16);
            }
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) packed[j][e] = 0;
#pragma unroll
            for (int e = 0; e < kVec; ++e) {
                if (e < lim[j]) {
                    if constexpr (F32) packed[j][e] = key32(static_cast<const uint32_t*>(scores)[row * row_stride + base + e]);
                    else packed[j][e >> 1] |= key16(static_cast<const uint16_t*>(scores)[row * row_stride + base + e]) << (16 * (e & 1));
                }
            }
        }
    }
    auto key_of = [&](int j, int e) -> uint32_t {
        if constexpr (F32) return packed[j][e];
        else return (packed[j][e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
    };

    constexpr int kPasses = F32 ? 3 : 2;
    uint32_t prefix = 0, prefix_mask = 0;
    unsigned long long above = 0;
    POPKV_TOPK_PHASE(1);
#pragma unroll
    for (int p = 0; p < kPasses; ++p) {
        const int shift = p == 0 ? (F32 ? 21 : 5) : (p == 1 ? (F32 ? 10 : 0) : 0);
        const int width = p == 0 ? 11 : (p == 1 ? (F32 ? 11 : 5) : 10);
        const uint32_t nbins = 1u << width;
        const uint32_t digit_mask = nbins - 1u;
        for (uint32_t b = tid; b < nbins; b += kClusterThreads) hist[b] = 0;
        __syncthreads();
#pragma unroll
        for (int j = 0; j < CHUNKS; ++j)
#pragma unroll
            for (int e = 0; e < kVec; ++e) {
                const uint32_t key = key_of(j, e);
                if (e < lim[j] && (key & prefix_mask) == prefix)
                    atomicAdd(&hist[(key >> shift) & digit_mask], 1u);
            }
        if (p == 0) POPKV_TOPK_PHASE(2);
        cluster.sync();  // every CTA's histogram is complete
        if (p == 0) POPKV_TOPK_PHASE(3);
        const unsigned long long remaining = static_cast<unsigned long long>(k) - above;
        const uint32_t per = (nbins + kClusterThreads - 1) / kClusterThreads;
        uint32_t counts[4];
        unsigned long long local = 0;
#pragma unroll
        for (uint32_t q = 0; q < 4; ++q) {
            counts[q] = 0;
            const uint32_t jj = tid * per + q;
            if (q < per && jj < nbins) {
                const uint32_t bin = nbins - 1 - jj;
                uint32_t v[CPR];
#pragma unroll
                for (int c = 0; c < CPR; ++c) v[c] = cluster.map_shared_rank(hist, c)[bin];  // all in flight
#pragma unroll
                for (int c = 0; c < CPR; ++c) counts[q] += v[c];
                local += counts[q];
            }
        }
        unsigned long long total;
        unsigned long long run = cta_exclusive_scan<unsigned long long>(local, scan_sums, total);
#pragma unroll
        for (uint32_t q = 0; q < 4; ++q) {
            const uint32_t jj = tid * per + q;
            if (q < per && jj < nbins) {
                if (run < remaining && run + counts[q] >= remaining) {
                    sel_bin = nbins - 1 - jj;
                    sel_above = run;
                }
                run += counts[q];
            }
        }
        cluster.sync();  // remote reads done; sel_* visible
        if (p == 0) POPKV_TOPK_PHASE(4);
        prefix |= sel_bin << shift;
        prefix_mask |= digit_mask << shift;
        above += sel_above;
    }
    const uint32_t threshold = prefix;
    const unsigned long long need = static_cast<unsigned long long>(k) - above;
    POPKV_TOPK_PHASE(5);

    unsigned long long round_counts[CHUNKS];
    unsigned long long mine = 0;
#pragma unroll
    for (int j = 0; j < CHUNKS; ++j) {
        unsigned int gt = 0, eq = 0;
#pragma unroll
        for (int e = 0; e < kVec; ++e) {
            const uint32_t key = key_of(j, e);
            if (e < lim[j]) {
                gt += key > threshold;
                eq += key == threshold;
            }
        }
        round_counts[j] = (static_cast<unsigned long long>(gt) << 32) | eq;
        mine += round_counts[j];
    }
    unsigned long long cta_sum;
    (void)cta_exclusive_scan<unsigned long long>(mine, scan_sums, cta_sum);
    if (tid == 0) cta_totals = cta_sum;
    cluster.sync();  // totals published
    if (tid < 32) {  // lane c < rank reads rank c's totals; one warp reduction
        unsigned long long t = (tid < rank) ? *cluster.map_shared_rank(&cta_totals, tid) : 0ull;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xFFFFFFFFu, t, o);
        if (tid == 0) scan_sums[kClusterWarps] = t;
    }
    cluster.sync();  // nobody exits while a peer may still read its totals
    POPKV_TOPK_PHASE(6);
    const unsigned long long carry = scan_sums[kClusterWarps];
    unsigned long long gt_carry = carry >> 32, eq_carry = carry & 0xFFFFFFFFull;
#pragma unroll
    for (int j = 0; j < CHUNKS; ++j) {
        unsigned long long total;
        const unsigned long long excl = cta_exclusive_scan<unsigned long long>(round_counts[j], scan_sums, total);
        unsigned long long gt_before = gt_carry + (excl >> 32);
        unsigned long long eq_before = eq_carry + (excl & 0xFFFFFFFFull);
        const int64_t base = slice0 + (static_cast<int64_t>(tid) + static_cast<int64_t>(kClusterThreads) * j) * kVec;
#pragma unroll
        for (int e = 0; e < kVec; ++e) {
            if (e >= lim[j]) continue;
            const uint32_t key = key_of(j, e);
            if (key > threshold) {
                const unsigned long long pos = gt_before + min(eq_before, need);
                if (pos < static_cast<unsigned long long>(k)) dst[pos] = base + e;
                ++gt_before;
            } else if (key == threshold) {
                const unsigned long long pos = gt_before + eq_before;
                if (eq_before < need && pos < static_cast<unsigned long long>(k)) dst[pos] = base + e;
                ++eq_before;
            }
        }
        gt_carry += total >> 32;
        eq_carry += total & 0xFFFFFFFFull;
    }
    POPKV_TOPK_PHASE(7);
}

template <bool F32, int CPR, int CHUNKS>
int launch_cluster(const void* scores, int64_t rows, int64_t tokens, int64_t row_stride, int64_t k,
                   int64_t current_index, int64_t* out, int64_t out_stride, bool vec_ok,
                   cudaStream_t stream) {
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3(static_cast<unsigned>(rows * CPR), 1, 1);
    config.blockDim = dim3(kClusterThreads, 1, 1);
    config.dynamicSmemBytes = 0;
    config.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CPR;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    config.attrs = attr;
    config.numAttrs = 1;
    cudaError_t err = cudaLaunchKernelEx(&config, topk_cluster_kernel<F32, CPR, CHUNKS>, scores, tokens,
                                         row_stride, k, current_index, out, out_stride, vec_ok);
    if (err != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_topk: %s", cudaGetErrorString(err));
    return check_launch("popkv_topk");
}

// Picks the cluster size (CTAs per row) so that rows * CPR is about one wave
// of the 148 SMs, then the smallest register footprint that holds the slice.
template <bool F32>
int try_launch_cluster(const void* scores, int64_t rows, int64_t tokens, int64_t row_stride,
                       int64_t k, int64_t current_index, int64_t* out, int64_t out_stride,
                       bool vec_ok, cudaStream_t stream) {
    constexpr int64_t kVec = F32 ? 4 : 8;
    int cpr = 1;
    while (cpr < 8 && rows * cpr * 2 <= 160) cpr *= 2;
    while (cpr < 8 && tokens > cpr * kClusterThreads * kVec * 4) cpr *= 2;
    if (tokens > cpr * kClusterThreads * kVec * 4) return -1;
    const int64_t per_cta = (tokens + cpr - 1) / cpr;
    int chunks = 1;
    while (per_cta > chunks * kClusterThreads * kVec) chunks *= 2;
#define POPKV_CLUSTER(CPR_, CH_)                                                                   \
    if (cpr == CPR_ && chunks == CH_)                                                              \
        return launch_cluster<F32, CPR_, CH_>(scores, rows, tokens, row_stride, k, current_index, \
                                              out, out_stride, vec_ok, stream);
#define POPKV_CLUSTER_CPR(CPR_) POPKV_CLUSTER(CPR_, 1) POPKV_CLUSTER(CPR_, 2) POPKV_CLUSTER(CPR_, 4)
    POPKV_CLUSTER_CPR(1)
    POPKV_CLUSTER_CPR(2)
    POPKV_CLUSTER_CPR(4)
    POPKV_CLUSTER_CPR(8)
#undef POPKV_CLUSTER_CPR
#undef POPKV_CLUSTER
    return -1;
}

// ---------------------------------------------------------------------------
// Top-k from a precomputed first-pass histogram (fp16 scores).
//
// The score kernel (popkv_score_hist) already counted every score's top 11
// key bits per row, so one CTA per row only has to: read and re-zero its row of
// the histogram and pick the digit of the k-th largest key; count the keys
// inside that digit by their low 5 bits; and compact.  Thread t owns the
// contiguous elements [t*PER, (t+1)*PER), held in registers (two keys per
// register), so a single block scan gives the ascending-index output positions.
// ---------------------------------------------------------------------------
constexpr int kHistThreads = 1024;
constexpr int kHistWarps = kHistThreads / 32;

template <typename V>
__device__ __forceinline__ V hist_exclusive_scan(V x, V* warp_sums, V& total) {
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
        V w = lane < kHistWarps ? warp_sums[lane] : V(0);
        V wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            V y = __shfl_up_sync(0xFFFFFFFFu, wi, o);
            if (lane >= o) wi += y;
        }
        if (lane < kHistWarps) warp_sums[lane] = wi - w;
        if (lane == kHistWarps - 1) warp_sums[kHistWarps] = wi;
    }
    __syncthreads();
    V result = warp_sums[warp] + incl - x;
    total = warp_sums[kHistWarps];
    __syncthreads();
    return result;
}

template <int PER>
__global__ void __launch_bounds__(kHistThreads) topk_hist_kernel(
    const uint16_t* __restrict__ scores, uint32_t* __restrict__ hist, int64_t tokens,
    int64_t row_stride, int64_t k, int64_t current_index, int64_t* __restrict__ out,
    int64_t out_stride, bool vec_ok) {
    __shared__ unsigned long long scan_sums[kHistWarps + 1];
    __shared__ uint32_t hist2[32];
    __shared__ uint32_t sel_b1, sel_thr;
    __shared__ unsigned long long sel_above, sel_need;
    const int64_t row = blockIdx.x;
    const int tid = threadIdx.x;
    int64_t* dst = out + row * out_stride;
    if (tid == 0) {
        if (current_index >= 0) dst[k] = current_index;
        // Defaults if the histogram does not hold this row's counts (all writes
        // stay inside the row's k slots regardless).
        sel_b1 = 0;
        sel_above = 0;
        sel_thr = 0;
        sel_need = 0;
    }
    uint32_t* hrow = hist + row * 2048;

    // Histogram of this row: positions 2*tid, 2*tid+1 in descending key order.
    const uint2 hv = *reinterpret_cast<const uint2*>(hrow + 2048 - 2 - 2 * tid);
    // hv.y is bin 2047 - 2*tid, hv.x is bin 2046 - 2*tid.
    // Keys: elements [tid*PER, tid*PER + PER), two per register.
    const int64_t base = static_cast<int64_t>(tid) * PER;
    const uint16_t* src = scores + row * row_stride + base;
    uint32_t packed[PER / 2];
    const int64_t left = tokens - base;
    const int lim = left <= 0 ? 0 : (left >= PER ? PER : static_cast<int>(left));
    if (vec_ok && lim == PER) {
#pragma unroll
        for (int j = 0; j < PER / 8; ++j) {
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(src) + j);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int e = 0; e < 4; ++e)
                packed[4 * j + e] = order_key16(static_cast<uint16_t>(w[e] & 0xFFFFu)) |
                                    (order_key16(static_cast<uint16_t>(w[e] >> 16)) << 16);
        }
    } else {
#pragma unroll
        for (int j = 0; j < PER / 2; ++j) packed[j] = 0;
#pragma unroll
        for (int e = 0; e < PER; ++e)
            if (e < lim) packed[e >> 1] |= order_key16(src[e]) << (16 * (e & 1));
    }
    auto key_of = [&](int e) -> uint32_t { return (packed[e >> 1] >> (16 * (e & 1))) & 0xFFFFu; };
    __syncthreads();  // every thread has read its histogram entries
    *reinterpret_cast<uint2*>(hrow + 2048 - 2 - 2 * tid) = make_uint2(0u, 0u);  // leave zeros for the next call
    if (tid < 32) hist2[tid] = 0;

    if (k > 0) {
        const unsigned long long kk = static_cast<unsigned long long>(k);
        unsigned long long total;
        const unsigned long long run0 =
            hist_exclusive_scan<unsigned long long>(static_cast<unsigned long long>(hv.x) + hv.y, scan_sums, total);
        const unsigned long long run1 = run0 + hv.y;
        if (run0 < kk && run1 >= kk) {
            sel_b1 = 2047u - 2u * tid;
            sel_above = run0;
        } else if (run1 < kk && run1 + hv.x >= kk) {
            sel_b1 = 2046u - 2u * tid;
            sel_above = run1;
        }
        __syncthreads();
        const uint32_t b1 = sel_b1;
#pragma unroll
        for (int e = 0; e < PER; ++e)
            if (e < lim && (key_of(e) >> 5) == b1) atomicAdd(&hist2[key_of(e) & 31u], 1u);
        __syncthreads();
        if (tid < 32) {
            const unsigned long long remaining = kk - sel_above;
            const uint32_t c2 = hist2[31 - tid];
            uint32_t incl = c2;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
                if (tid >= o) incl += y;
            }
            const uint32_t excl = incl - c2;
            if (excl < remaining && incl >= remaining) {
                sel_thr = (b1 << 5) | (31u - tid);
                sel_need = remaining - excl;
            }
        }
        __syncthreads();
        const uint32_t thr = sel_thr;
        const unsigned long long need = sel_need;
        unsigned int gt = 0, eq = 0;
#pragma unroll
        for (int e = 0; e < PER; ++e) {
            if (e < lim) {
                gt += key_of(e) > thr;
                eq += key_of(e) == thr;
            }
        }
        const unsigned long long ex = hist_exclusive_scan<unsigned long long>(
            (static_cast<unsigned long long>(gt) << 32) | eq, scan_sums, total);
        unsigned long long gt_before = ex >> 32, eq_before = ex & 0xFFFFFFFFull;
#pragma unroll
        for (int e = 0; e < PER; ++e) {
            if (e >= lim) continue;
            const uint32_t key = key_of(e);
            if (key > thr) {
                const unsigned long long pos = gt_before + min(eq_before, need);
                if (pos < kk) dst[pos] = base + e;
                ++gt_before;
            } else if (key == thr) {
                const unsigned long long pos = gt_before + eq_before;
                if (eq_before < need && pos < kk) dst[pos] = base + e;
                ++eq_before;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// fp16 top-k, one thread-block cluster of CPR CTAs per row, two cluster
// barriers in all.
//
// Thread t of rank r owns the contiguous keys [r*S + t*PER, r*S + (t+1)*PER),
// S = 512*PER, held in registers two to a word.
// (1) Every CTA counts its keys' top 11 bits in shared memory; barrier A.
//     Every CTA then reads all CPR histograms (one 16-byte DSMEM load per rank
//     and thread: thread t sums the four bins at descending positions
//     4t..4t+3) and scans them itself, so all CTAs pick the same digit b1.
// (2) Each CTA counts its keys above b1 and, by their low 5 bits, its keys in
//     b1 (a 32-bin histogram), and stores both into every CTA's shared memory
//     (its own row of `hist2_all`); barrier B.  Warp 0 of every CTA then
//     reads its local copy of the CPR rows, picks the threshold key and how
//     many keys equal to it are taken, and sums how many keys above and equal
//     to the threshold the lower ranks hold: the CTA's output offset, with no
//     further exchange.
// (3) A block scan of each thread's (greater, equal) counts gives positions
//     inside the CTA.  A thread's winners (from bit masks of its keys above and
//     equal to the threshold) take consecutive output positions, so each
//     thread stores its few winners directly; a warp's stores cover one short
//     contiguous range.
// Every DSMEM access (the reads of the 11-bit histograms, the stores of the
// small ones) comes before barrier B, the last cluster-wide wait, so no CTA
// exits while a peer may still touch its shared memory.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t popcount_mask(uint32_t m) { return static_cast<uint32_t>(__popc(m)); }
__device__ __forceinline__ uint32_t popcount_mask(unsigned long long m) { return static_cast<uint32_t>(__popcll(m)); }
__device__ __forceinline__ int lowest_bit(uint32_t m) { return __ffs(m) - 1; }
__device__ __forceinline__ int lowest_bit(unsigned long long m) { return __ffsll(m) - 1; }

__device__ __forceinline__ uint32_t cta_exclusive_scan32(uint32_t x, uint32_t* warp_sums, uint32_t& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t incl = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const uint32_t w = lane < kClusterWarps ? warp_sums[lane] : 0u;
        uint32_t wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, wi, o);
            if (lane >= o) wi += y;
        }
        if (lane < kClusterWarps) warp_sums[lane] = wi - w;
        if (lane == kClusterWarps - 1) warp_sums[kClusterWarps] = wi;
    }
    __syncthreads();
    const uint32_t result = warp_sums[warp] + incl - x;
    total = warp_sums[kClusterWarps];
    return result;
}

template <int CPR, int PER>
__global__ void __launch_bounds__(kClusterThreads, PER <= 16 ? 4 : 1) topk16_cluster_kernel(
    const uint16_t* __restrict__ scores, int64_t tokens, int64_t row_stride, int64_t k,
    int64_t current_index, int64_t* __restrict__ out, int64_t out_stride, bool vec_ok,
    const int64_t* __restrict__ dyn_tokens, uint32_t* __restrict__ ghist) {
    static_assert(PER % 8 == 0 && PER <= 64, "PER keys per thread, whole uint4 loads");
    static_assert(CPR <= 8, "at most 8 ranks per cluster");
    constexpr int64_t kSlice = static_cast<int64_t>(kClusterThreads) * PER;
    constexpr int kRow2 = 33;
    __shared__ __align__(16) uint32_t hist[kHistBins];
    __shared__ uint32_t hist2[kRow2];  // bins 0..31: keys in digit b1 by low 5 bits; [32]: keys above b1
    __shared__ uint32_t hist2_all[CPR * kRow2];  // row c: rank c's `hist2`
    __shared__ uint32_t warp_sums[kClusterWarps + 1];
    __shared__ uint32_t sel_b1, sel_above, sel_thr, sel_need, sel_gt_before, sel_eq_before;

    POPKV_TOPK_PHASE(0);
    pdl_wait();
    pdl_launch_dependents();
    if (dyn_tokens) {
        // Device-resident token count: `tokens` and `k` are upper bounds, the
        // current token's index is the count itself.
        const int64_t t = *dyn_tokens;
        tokens = t < 0 ? 0 : (t < tokens ? t : tokens);
        k = k < tokens ? k : tokens;
        current_index = tokens;
    }
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = static_cast<int>(cluster.block_rank());
    const int64_t row = blockIdx.x / CPR;
    const int tid = threadIdx.x;
    int64_t* dst = out + row * out_stride;
    if (current_index >= 0 && tid == 0 && rank == 0) dst[k] = current_index;
    uint32_t* grow = ghist ? ghist + row * kHistBins : nullptr;  // the row's first-pass histogram, if given
    if (k <= 0) {  // uniform across the cluster: no CTA reaches a cluster barrier
        if (grow && rank == 0)
            reinterpret_cast<uint4*>(grow)[tid] = make_uint4(0u, 0u, 0u, 0u);  // leave zeros for the next call
        return;
    }
    const uint32_t kk = static_cast<uint32_t>(k);
    uint4 gbins = make_uint4(0u, 0u, 0u, 0u);
    if (grow) gbins = __ldcg(reinterpret_cast<const uint4*>(grow) + (kHistBins / 4 - 1) - tid);  // 2047-4t..2044-4t

    if (!grow)
        for (int b = tid; b < kHistBins; b += kClusterThreads) hist[b] = 0;
    if (tid < kRow2) hist2[tid] = 0;
    if (tid == 0) {  // defaults; the scans below always overwrite them when k <= tokens
        sel_b1 = 0;
        sel_above = 0;
        sel_thr = 0;
        sel_need = 0;
        sel_gt_before = 0;
        sel_eq_before = 0;
    }

    const int64_t base = static_cast<int64_t>(rank) * kSlice + static_cast<int64_t>(tid) * PER;
    const uint16_t* src = scores + row * row_stride + base;
    const int64_t left = tokens - base;
    const int lim = left <= 0 ? 0 : (left >= PER ? PER : static_cast<int>(left));
    uint32_t packed[PER / 2];
    if (vec_ok && lim == PER) {
#pragma unroll
        for (int j = 0; j < PER / 8; ++j) {
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(src) + j);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int e = 0; e < 4; ++e)
                packed[4 * j + e] = key16(static_cast<uint16_t>(w[e] & 0xFFFFu)) |
                                    (key16(static_cast<uint16_t>(w[e] >> 16)) << 16);
        }
    } else {
#pragma unroll
        for (int j = 0; j < PER / 2; ++j) packed[j] = 0;
#pragma unroll
        for (int e = 0; e < PER; ++e)
            if (e < lim) packed[e >> 1] |= key16(src[e]) << (16 * (e & 1));
    }
    auto key_of = [&](int e) -> uint32_t { return (packed[e >> 1] >> (16 * (e & 1))) & 0xFFFFu; };
    POPKV_TOPK_PHASE(1);
    __syncthreads();  // histograms zeroed

    // (1) top 11 bits: counted here, or by the kernel that wrote the scores.
    uint32_t cnt[4] = {gbins.w, gbins.z, gbins.y, gbins.x};  // bins 2047 - 4t - q
    if (!grow) {
#pragma unroll
        for (int e = 0; e < PER; ++e)
            if (e < lim) atomicAdd(&hist[key_of(e) >> 5], 1u);
        POPKV_TOPK_PHASE(2);
        cluster.sync();  // A: every CTA's histogram is complete
        POPKV_TOPK_PHASE(3);
        uint4 v[CPR];
#pragma unroll
        for (int c = 0; c < CPR; ++c)  // all loads in flight at once
            v[c] = *reinterpret_cast<const uint4*>(cluster.map_shared_rank(hist, c) + (kHistBins - 4) - 4 * tid);
#pragma unroll
        for (int c = 0; c < CPR; ++c) {
            cnt[0] += v[c].w;  // bin 2047 - 4t (descending position 4t)
            cnt[1] += v[c].z;
            cnt[2] += v[c].y;
            cnt[3] += v[c].x;
        }
    }
    {
        uint32_t total;
        uint32_t run = cta_exclusive_scan32(cnt[0] + cnt[1] + cnt[2] + cnt[3], warp_sums, total);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if (run < kk && run + cnt[q] >= kk) {
                sel_b1 = static_cast<uint32_t>(kHistBins - 1 - 4 * tid - q);
                sel_above = run;
            }
            run += cnt[q];
        }
    }
    __syncthreads();
    const uint32_t b1 = sel_b1;
    POPKV_TOPK_PHASE(4);

    // (2) keys above digit b1, and the low 5 bits of the keys in it.
    uint32_t above_b1 = 0;
#pragma unroll
    for (int e = 0; e < PER; ++e) {
        if (e < lim) {
            above_b1 += (key_of(e) >> 5) > b1;
            if ((key_of(e) >> 5) == b1) atomicAdd(&hist2[key_of(e) & 31u], 1u);
        }
    }
    above_b1 = __reduce_add_sync(0xFFFFFFFFu, above_b1);
    if ((tid & 31) == 0 && above_b1) atomicAdd(&hist2[32], above_b1);
    __syncthreads();
    if (tid < CPR * kRow2)  // thread (c, i): entry i into rank c's copy
        cluster.map_shared_rank(hist2_all, tid / kRow2)[rank * kRow2 + tid % kRow2] = hist2[tid % kRow2];
    cluster.sync();  // B: every rank's row has arrived in every CTA
    if (grow && rank == 0)  // every CTA read the row's histogram before B: leave zeros for the next call
        reinterpret_cast<uint4*>(grow)[tid] = make_uint4(0u, 0u, 0u, 0u);
    if (tid < 32) {
        // Lane i: bin 31 - i, over all ranks and over the lower ranks.
        uint32_t c2 = 0, low = 0, low_above = 0;
#pragma unroll
        for (int c = 0; c < CPR; ++c) {
            const uint32_t h = hist2_all[c * kRow2 + 31 - tid];
            c2 += h;
            if (c < rank) {
                low += h;
                low_above += hist2_all[c * kRow2 + 32];
            }
        }
        uint32_t incl = c2, low_incl = low;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
            const uint32_t z = __shfl_up_sync(0xFFFFFFFFu, low_incl, o);
            if (tid >= o) {
                incl += y;
                low_incl += z;
            }
        }
        const uint32_t remaining = kk - sel_above;
        if (incl - c2 < remaining && incl >= remaining) {
            sel_thr = (b1 << 5) | (31u - static_cast<uint32_t>(tid));
            sel_need = remaining - (incl - c2);
            // Keys of lower ranks above the threshold: above digit b1, or in b1
            // with a higher low part; equal to it: this lane's bin.
            sel_gt_before = low_above + (low_incl - low);
            sel_eq_before = low;
        }
    }
    __syncthreads();
    const uint32_t thr = sel_thr, need = sel_need;
    POPKV_TOPK_PHASE(5);

    // (3) positions.  Bit e of `gtm` / `eqm`: key e is above / equal to the
    // threshold; the counts come from their population counts.
    using Mask = typename std::conditional<(PER > 32), unsigned long long, uint32_t>::type;
    Mask gtm = 0, eqm = 0;
#pragma unroll
    for (int e = 0; e < PER; ++e) {
        if (e < lim) {
            gtm |= static_cast<Mask>(key_of(e) > thr) << e;
            eqm |= static_cast<Mask>(key_of(e) == thr) << e;
        }
    }
    const uint32_t gt = popcount_mask(gtm), eq = popcount_mask(eqm);
    uint32_t cta_total;
    const uint32_t excl = cta_exclusive_scan32((gt << 16) | eq, warp_sums, cta_total);
    const uint32_t rank_gt = sel_gt_before, rank_eq = sel_eq_before;
    const uint32_t gt_before = rank_gt + (excl >> 16), eq_before = rank_eq + (excl & 0xFFFFu);
    POPKV_TOPK_PHASE(6);
    // This thread's winners: every key above the threshold and its first
    // `take` keys equal to it, at consecutive positions from `pos` on (the
    // winners before them: all keys above, and the equal keys taken, of the
    // lower threads and ranks).
    Mask win = gtm, rest = eqm;
    const uint32_t take = need > eq_before ? min(need - eq_before, eq) : 0u;
    for (uint32_t i = 0; i < take; ++i) {
        win |= rest & (~rest + 1);  // lowest remaining equal key
        rest &= rest - 1;
    }
    uint32_t pos = gt_before + min(eq_before, need);
    while (win) {
        const int e = lowest_bit(win);
        win &= win - 1;
        if (pos < kk) dst[pos] = base + e;
        ++pos;
    }
    POPKV_TOPK_PHASE(7);
}

template <int CPR, int PER>
int launch_cluster16(const void* scores, int64_t rows, int64_t tokens, int64_t row_stride, int64_t k,
                     int64_t current_index, int64_t* out, int64_t out_stride, bool vec_ok,
                     cudaStream_t stream, const int64_t* dyn_tokens, uint32_t* ghist) {
    const cudaError_t err = launch_pdl(topk16_cluster_kernel<CPR, PER>,
                                       dim3(static_cast<unsigned>(rows * CPR)), dim3(kClusterThreads), 0,
                                       stream, CPR, static_cast<const uint16_t*>(scores), tokens,
                                       row_stride, k, current_index, out, out_stride, vec_ok, dyn_tokens,
                                       ghist);
    if (err != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_topk: %s", cudaGetErrorString(err));
    return check_launch("popkv_topk");
}

// fp16 rows of up to 8 * 512 * 64 keys (64 keys per thread with 8 CTAs per row,
// or with 4 when many rows would overflow a wave) with 0 < k <= tokens and
// fewer than 2^16 keys per CTA
// slice: about one wave of CTAs (rows * CPR near 148), the fewest keys per
// thread that cover the row.  Returns -1 when the shape does not apply.
int try_launch_cluster16(const void* scores, int64_t rows, int64_t tokens, int64_t row_stride,
                         int64_t k, int64_t current_index, int64_t* out, int64_t out_stride,
                         bool vec_ok, cudaStream_t stream, const int64_t* dyn_tokens = nullptr,
                         uint32_t* ghist = nullptr) {
    if (k <= 0 || k > tokens || rows > 0x7FFFFFF) return -1;
    // Up to 4 CTAs per row while the rows leave SMs idle (larger clusters cost
    // more in DSMEM reads and barrier latency than they save), 8 for at most 8
    // rows (a sharded step: 7.5 against 8.0 us at 4 rows of 32768 keys), more
    // only when a row does not fit 4 x 512 x 32 keys.
    int cpr = 1;
    while (cpr < (rows <= 8 ? 8 : 4) && rows * cpr * 2 <= 160) cpr *= 2;
    while (cpr < 8 && tokens > static_cast<int64_t>(cpr) * kClusterThreads * 32) cpr *= 2;
    int per = 8;
    while (per < (cpr == 8 ? 64 : 32) && tokens > static_cast<int64_t>(cpr) * kClusterThreads * per) per *= 2;
    if (tokens > static_cast<int64_t>(cpr) * kClusterThreads * per) return -1;
    // A row just past 4 x 512 x 16 keys (e.g. 33K tokens) would take 32 keys per
    // thread in 4 CTAs and leave the last CTA of each cluster idle.  With 32 rows
    // or more, 24 keys per thread in 4 CTAs is fastest (11.5 against 13.3 us for
    // 6 CTAs at 16 keys, 32 rows of 32771 keys); fewer rows take the 6-CTA form.
    if (cpr == 4 && per == 32 && rows >= 32 && tokens <= static_cast<int64_t>(4) * kClusterThreads * 24) {
        per = 24;
    } else if (cpr == 4 && per == 32 && tokens <= static_cast<int64_t>(6) * kClusterThreads * 16) {
        cpr = 6;
        per = 16;
    }
    // Many long rows: 8-CTA clusters would need more than one resident wave
    // (4 CTAs of 512 threads per SM); 4 CTAs at 64 keys per thread fit in one.
    constexpr int64_t kWaveCtas = 4 * 148;  // resident 512-thread CTAs on a B200 (4 per SM)
    if (cpr == 8 && per == 32 && rows * 8 > kWaveCtas && tokens <= static_cast<int64_t>(4) * kClusterThreads * 64) {
        cpr = 4;
        per = 64;
    }
    // Likewise a row of 64K-96K keys fills 6 CTAs at 32 keys per thread.
    if (cpr == 8 && per == 32 && tokens <= static_cast<int64_t>(6) * kClusterThreads * 32) cpr = 6;
#define POPKV_C16(CPR_, PER_)                                                                      \
    if (cpr == CPR_ && per == PER_)                                                                \
        return launch_cluster16<CPR_, PER_>(scores, rows, tokens, row_stride, k, current_index, out, \
                                            out_stride, vec_ok, stream, dyn_tokens, ghist);
#define POPKV_C16_CPR(CPR_) POPKV_C16(CPR_, 8) POPKV_C16(CPR_, 16) POPKV_C16(CPR_, 32)
    POPKV_C16_CPR(1)
    POPKV_C16_CPR(2)
    POPKV_C16_CPR(4)
    POPKV_C16(4, 64)
    POPKV_C16(6, 16)
    POPKV_C16(4, 24)
    POPKV_C16(6, 32)
    POPKV_C16_CPR(8)
    POPKV_C16(8, 64)
#undef POPKV_C16_CPR
#undef POPKV_C16
    return -1;
}

template <bool F32>
int launch_topk(const void* scores, int64_t rows, int64_t tokens, int64_t row_stride, int64_t k,
                int64_t current_index, int64_t* out, int64_t out_stride, cudaStream_t stream) {
    const size_t key_bytes = F32 ? 4 : 2;
    constexpr int64_t kVec = F32 ? 4 : 8;
    const bool vec_ok = aligned(scores, 16) && (row_stride * static_cast<int64_t>(key_bytes)) % 16 == 0;
    const int64_t per_chunk = kTopkThreads * kVec;
    const unsigned grid = static_cast<unsigned>(rows);
    if constexpr (!F32) {
        const int st = try_launch_cluster16(scores, rows, tokens, row_stride, k, current_index, out,
                                            out_stride, vec_ok, stream);
        if (st >= 0) return st;
    }
    if (rows <= 0x7FFFFFF && k > 0) {
        const int st = try_launch_cluster<F32>(scores, rows, tokens, row_stride, k, current_index,
                                               out, out_stride, vec_ok, stream);
        if (st >= 0) return st;
    }
#define POPKV_TOPK_REG(C)                                                                      \
    if (tokens <= per_chunk * (C)) {                                                           \
        topk_reg_kernel<F32, C><<<grid, kTopkThreads, 0, stream>>>(                            \
            scores, tokens, row_stride, k, current_index, out, out_stride, vec_ok);            \
        return check_launch("popkv_topk");                                                     \
    }
    POPKV_TOPK_REG(1)
    POPKV_TOPK_REG(2)
    POPKV_TOPK_REG(4)
    if constexpr (F32) { POPKV_TOPK_REG(8) }
#undef POPKV_TOPK_REG
    const size_t stage = static_cast<size_t>(tokens) * key_bytes;
    if (stage <= kStageBytes) {
        auto kernel = topk_kernel<F32, true>;
        const int st = allow_dynamic_smem(kernel, static_cast<int>(kStageBytes));
        if (st != POPKV_OK) return st;
        kernel<<<grid, kTopkThreads, stage, stream>>>(scores, tokens, row_stride, k, current_index,
                                                      out, out_stride);
    } else {
        topk_kernel<F32, false><<<grid, kTopkThreads, 0, stream>>>(scores, tokens, row_stride, k,
                                                                   current_index, out, out_stride);
    }
    return check_launch("popkv_topk");
}

}  // namespace
}  // namespace popkv

extern "C" int popkv_topk(const void* scores, int scores_dtype, int64_t rows, int64_t tokens,
                          int64_t row_stride, int64_t k, int64_t current_index, int64_t* out,
                          int64_t out_stride, void* stream) {
    using namespace popkv;
    if (scores_dtype != POPKV_DTYPE_F16 && scores_dtype != POPKV_DTYPE_F32)
        return fail(POPKV_ERR_INVALID, "popkv_topk: scores must be fp16 or fp32");
    if (rows < 0 || tokens < 0) return fail(POPKV_ERR_INVALID, "popkv_topk: negative shape");
    if (k < 0 || k > tokens)
        return fail(POPKV_ERR_INVALID, "popkv_topk: k must be between 0 and the token count");
    if (row_stride < tokens) return fail(POPKV_ERR_INVALID, "popkv_topk: row_stride < tokens");
    const int64_t width = k + (current_index >= 0 ? 1 : 0);
    if (out_stride < width) return fail(POPKV_ERR_INVALID, "popkv_topk: out_stride too small");
    if (tokens > 0x7FFFFFFFll) return fail(POPKV_ERR_UNSUPPORTED, "popkv_topk: more than 2^31 tokens");
    if (rows == 0 || width == 0) return POPKV_OK;
    if (!out || (k > 0 && !scores)) return fail(POPKV_ERR_INVALID, "popkv_topk: null pointer");
    if (rows > 0x7FFFFFFFll) return fail(POPKV_ERR_UNSUPPORTED, "popkv_topk: too many rows");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (scores_dtype == POPKV_DTYPE_F32)
        return launch_topk<true>(scores, rows, tokens, row_stride, k, current_index, out, out_stride, s);
    return launch_topk<false>(scores, rows, tokens, row_stride, k, current_index, out, out_stride, s);
}

extern "C" int popkv_topk_hist(const uint16_t* scores, uint32_t* hist, int64_t rows, int64_t tokens,
                               int64_t row_stride, int64_t k, int64_t current_index, int64_t* out,
                               int64_t out_stride, void* stream) {
    using namespace popkv;
    if (rows < 0 || tokens < 0) return fail(POPKV_ERR_INVALID, "popkv_topk_hist: negative shape");
    if (k < 0 || k > tokens)
        return fail(POPKV_ERR_INVALID, "popkv_topk_hist: k must be between 0 and the token count");
    if (row_stride < tokens) return fail(POPKV_ERR_INVALID, "popkv_topk_hist: row_stride < tokens");
    const int64_t width = k + (current_index >= 0 ? 1 : 0);
    if (out_stride < width) return fail(POPKV_ERR_INVALID, "popkv_topk_hist: out_stride too small");
    if (rows == 0) return POPKV_OK;
    if (!out || !hist || !scores) return fail(POPKV_ERR_INVALID, "popkv_topk_hist: null pointer");
    if (!aligned(hist, 16)) return fail(POPKV_ERR_INVALID, "popkv_topk_hist: hist must be 16-byte aligned");
    const bool vec_ok = aligned(scores, 16) && (row_stride * 2) % 16 == 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // The cluster kernel finishes from the histogram when the row fits it.
    const int st = try_launch_cluster16(scores, rows, tokens, row_stride, k, current_index, out, out_stride,
                                        vec_ok, s, nullptr, hist);
    if (st >= 0) return st;
    if (tokens > 64 * kHistThreads)
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_topk_hist: at most %d tokens", 64 * kHistThreads);
    const unsigned grid = static_cast<unsigned>(rows);
    if (tokens <= 8 * kHistThreads)
        topk_hist_kernel<8><<<grid, kHistThreads, 0, s>>>(scores, hist, tokens, row_stride, k, current_index, out, out_stride, vec_ok);
    else if (tokens <= 16 * kHistThreads)
        topk_hist_kernel<16><<<grid, kHistThreads, 0, s>>>(scores, hist, tokens, row_stride, k, current_index, out, out_stride, vec_ok);
    else if (tokens <= 32 * kHistThreads)
        topk_hist_kernel<32><<<grid, kHistThreads, 0, s>>>(scores, hist, tokens, row_stride, k, current_index, out, out_stride, vec_ok);
    else
        topk_hist_kernel<64><<<grid, kHistThreads, 0, s>>>(scores, hist, tokens, row_stride, k, current_index, out, out_stride, vec_ok);
    return check_launch("popkv_topk_hist");
}

extern "C" int popkv_topk_dyn(const uint16_t* scores, int64_t rows, const int64_t* tokens_dev,
                              int64_t max_tokens, int64_t row_stride, int64_t k_max, int64_t* out,
                              int64_t out_stride, void* stream) {
    using namespace popkv;
    if (rows < 0 || max_tokens <= 0) return fail(POPKV_ERR_INVALID, "popkv_topk_dyn: invalid shape");
    if (k_max <= 0 || k_max > max_tokens)
        return fail(POPKV_ERR_INVALID, "popkv_topk_dyn: k_max must be between 1 and max_tokens");
    if (row_stride < max_tokens) return fail(POPKV_ERR_INVALID, "popkv_topk_dyn: row_stride < max_tokens");
    if (out_stride < k_max + 1) return fail(POPKV_ERR_INVALID, "popkv_topk_dyn: out_stride too small");
    if (rows == 0) return POPKV_OK;
    if (!scores || !out || !tokens_dev) return fail(POPKV_ERR_INVALID, "popkv_topk_dyn: null pointer");
    const bool vec_ok = aligned(scores, 16) && (row_stride * 2) % 16 == 0;
    const int st = try_launch_cluster16(scores, rows, max_tokens, row_stride, k_max, max_tokens, out,
                                        out_stride, vec_ok, static_cast<cudaStream_t>(stream), tokens_dev);
    if (st < 0)
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_topk_dyn: at most %d tokens and %d rows per launch",
                    8 * kClusterThreads * 64, 0x7FFFFFF);
    return st;
}
