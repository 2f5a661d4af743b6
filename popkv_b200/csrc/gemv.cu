// Weight-streaming matrix-vector products of the decode step (batch <= 4),
// with the step's element-wise work fused into their prologues/epilogues.
//
// A decode step of a Llama-shaped model reads every weight matrix once for a
// handful of activation rows: the products are HBM-bound (2 bytes of weight
// per multiply-add pair per row of the batch).  One kernel streams W [rows, k]
// (bf16, row-major) into shared memory with bulk asynchronous copies while x
// [batch, k] sits in shared memory; each warp owns whole output units (a row,
// or the two rows an epilogue needs together), streams their rows in 8 KB
// pieces through its own ring of up to three slots, and accumulates in fp32
// (fused multiply-add per element, lanes over 8-element chunks, shuffle tree),
// then rounds to bf16 as the reference model's nn.Linear output is.
//
// Grid: one CTA of 8 warps per SM.  The units are dealt to
// ceil(units / ceil(units / warps)) warps so every active warp gets the same
// number of units (no partial last round that would run below HBM
// bandwidth).  The rings are filled before waiting on the previous kernel
// (programmatic dependent launch): the weights do not depend on it, so their
// streaming overlaps its tail.
//
// Prologues (x in shared memory):
//   plain   x = the input rows;
//   norm    h = hidden (or embed[token] for the first layer) [+ delta], rounded
//           to bf16 (the residual add), CTA 0 stores h; x = RMSNorm(h) with
//           the rounding points of transformers' LlamaRMSNorm (popkv.py:1011).
// Epilogues:
//   store   out[b, row] = bf16(acc);
//   swiglu  units pair gate row j with up row I + j: act = silu(g) * up with
//           the LlamaMLP rounding points;
//   rope    units pair dims (d, d + 64) of a q/k/v head: rotary embedding at
//           the device-resident position (_apply_rope, popkv.py:745-749) into
//           the step's q / current k / current v buffers and row `position` of
//           the caches (append_kv, popkv.py:965-972);
//   argmax  logits[b, row] = bf16(acc) and the greedy choice (torch.argmax:
//           largest logit, lowest index among equals, NaN largest); the last
//           CTA writes the token id, clears the reduction state and advances
//           the position by one.
#include "common.cuh"
#include "mbarrier.cuh"

namespace popkv {
namespace {

constexpr int kMaxBatch = 4;

enum Prologue { kPlain = 0, kNorm = 1 };
enum Epilogue { kStore = 0, kSwiglu = 1, kRope = 2, kArgmax = 3 };

struct GemvArgs {
    const __nv_bfloat16* w;  // [rows, k]
    int64_t units;
    int k;
    int batch;
    int active_warps;
    // prologue
    const __nv_bfloat16* x;       // plain: [batch, k]; norm: hidden in [batch, k]
    const __nv_bfloat16* delta;   // norm: residual delta [batch, k] or null
    const __nv_bfloat16* embed;   // norm: embedding rows replace hidden (first layer) or null
    const int64_t* token;         // [batch] embedding row ids
    const __nv_bfloat16* norm_w;  // [k]
    float eps;
    __nv_bfloat16* hidden_out;    // norm: h [batch, k] (CTA 0), or null
    // epilogue
    __nv_bfloat16* out;           // store / argmax: [batch, out_stride]; swiglu: act [batch, out_stride]
    int64_t out_stride;
    int64_t pair_offset;          // swiglu: row of the up half (= units)
    // rope
    int q_heads, kv_heads;
    const __nv_bfloat16* cos_tab;
    const __nv_bfloat16* sin_tab;
    const int64_t* position;
    int64_t max_position;
    __nv_bfloat16* q_out;
    __nv_bfloat16* k_cur;
    __nv_bfloat16* v_cur;
    __nv_bfloat16* k_cache;
    __nv_bfloat16* v_cache;
    int64_t kbs, khs, kts, vbs, vhs, vts;
    // argmax
    unsigned long long* argmax_key;  // [batch], zero between launches
    unsigned int* done;              // zero between launches
    int64_t* token_next;             // [batch]
    int64_t* advance;                // position to advance by one, or null
};

__device__ __forceinline__ float lo_bf(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float hi_bf(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }
__device__ __forceinline__ float round_bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// acc += dot(w chunk, x chunk) over 8 bf16 pairs, two chains (even/odd elements).
__device__ __forceinline__ void dot8(const uint4& w, const uint4& x, float& a0, float& a1) {
    a0 = __fmaf_rn(lo_bf(w.x), lo_bf(x.x), a0);
    a1 = __fmaf_rn(hi_bf(w.x), hi_bf(x.x), a1);
    a0 = __fmaf_rn(lo_bf(w.y), lo_bf(x.y), a0);
    a1 = __fmaf_rn(hi_bf(w.y), hi_bf(x.y), a1);
    a0 = __fmaf_rn(lo_bf(w.z), lo_bf(x.z), a0);
    a1 = __fmaf_rn(hi_bf(w.z), hi_bf(x.z), a1);
    a0 = __fmaf_rn(lo_bf(w.w), lo_bf(x.w), a0);
    a1 = __fmaf_rn(hi_bf(w.w), hi_bf(x.w), a1);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

// Orderable key of a bf16 logit (NaN above everything) with the lower index
// winning among equal values.
__device__ __forceinline__ unsigned long long argmax_key(__nv_bfloat16 v, int64_t row) {
    const float f = __bfloat162float(v);
    uint32_t bits = __float_as_uint(f);
    uint32_t ord = (f != f) ? 0xFFFFFFFFu : ((bits & 0x80000000u) ? ~bits : (bits | 0x80000000u));
    return (static_cast<unsigned long long>(ord) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(row));
}

template <int MB, int THREADS>
__device__ void load_x_plain(const GemvArgs& a, uint4* xs) {
    const int nch = a.k / 8;
    for (int i = threadIdx.x; i < MB * nch; i += THREADS) {
        const int m = i / nch, c = i % nch;
        xs[i] = *(reinterpret_cast<const uint4*>(a.x + static_cast<int64_t>(m) * a.k) + c);
    }
    __syncthreads();
}

template <int MB, int THREADS, int WARPS>
__device__ void load_x_norm(const GemvArgs& a, uint4* xs, float* red) {
    const int nch = a.k / 8;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float ss[MB];
#pragma unroll
    for (int m = 0; m < MB; ++m) ss[m] = 0.0f;
    for (int i = tid; i < MB * nch; i += THREADS) {
        const int m = i / nch, c = i % nch;
        uint4 h;
        if (a.embed) {
            h = *(reinterpret_cast<const uint4*>(a.embed + a.token[m] * a.k) + c);
        } else {
            h = *(reinterpret_cast<const uint4*>(a.x + static_cast<int64_t>(m) * a.k) + c);
        }
        if (a.delta) {
            const uint4 d = *(reinterpret_cast<const uint4*>(a.delta + static_cast<int64_t>(m) * a.k) + c);
            uint32_t* hw = reinterpret_cast<uint32_t*>(&h);
            const uint32_t* dw = reinterpret_cast<const uint32_t*>(&d);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const __nv_bfloat16 l = __float2bfloat16_rn(lo_bf(hw[j]) + lo_bf(dw[j]));
                const __nv_bfloat16 u = __float2bfloat16_rn(hi_bf(hw[j]) + hi_bf(dw[j]));
                hw[j] = static_cast<uint32_t>(__bfloat16_as_ushort(l)) |
                        (static_cast<uint32_t>(__bfloat16_as_ushort(u)) << 16);
            }
        }
        xs[i] = h;
        if (blockIdx.x == 0 && a.hidden_out)
            *(reinterpret_cast<uint4*>(a.hidden_out + static_cast<int64_t>(m) * a.k) + c) = h;
        const uint32_t* hw = reinterpret_cast<const uint32_t*>(&h);
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            s = __fmaf_rn(lo_bf(hw[j]), lo_bf(hw[j]), s);
            s = __fmaf_rn(hi_bf(hw[j]), hi_bf(hw[j]), s);
        }
#pragma unroll
        for (int mm = 0; mm < MB; ++mm)
            if (mm == m) ss[mm] += s;
    }
#pragma unroll
    for (int m = 0; m < MB; ++m) {
        const float v = warp_sum(ss[m]);
        if (lane == 0) red[m * WARPS + warp] = v;
    }
    __syncthreads();
    float inv[MB];
#pragma unroll
    for (int m = 0; m < MB; ++m) {
        float t = 0.0f;
#pragma unroll
        for (int w = 0; w < WARPS; ++w) t += red[m * WARPS + w];
        inv[m] = rsqrtf(t / static_cast<float>(a.k) + a.eps);
    }
    for (int i = tid; i < MB * nch; i += THREADS) {
        const int m = i / nch, c = i % nch;
        uint4 h = xs[i];
        const uint4 nw = *(reinterpret_cast<const uint4*>(a.norm_w) + c);
        uint32_t* hw = reinterpret_cast<uint32_t*>(&h);
        const uint32_t* ww = reinterpret_cast<const uint32_t*>(&nw);
        float im = inv[0];
#pragma unroll
        for (int mm = 1; mm < MB; ++mm)
            if (mm == m) im = inv[mm];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const __nv_bfloat16 l = __float2bfloat16_rn(lo_bf(ww[j]) * round_bf(lo_bf(hw[j]) * im));
            const __nv_bfloat16 u = __float2bfloat16_rn(hi_bf(ww[j]) * round_bf(hi_bf(hw[j]) * im));
            hw[j] = static_cast<uint32_t>(__bfloat16_as_ushort(l)) |
                    (static_cast<uint32_t>(__bfloat16_as_ushort(u)) << 16);
        }
        xs[i] = h;
    }
    __syncthreads();
}

// Rows of unit u: r0 and (pairs) r1.
template <int EPI>
__device__ __forceinline__ void unit_rows(const GemvArgs& a, int64_t u, int64_t& r0, int64_t& r1) {
    if constexpr (EPI == kSwiglu) {
        r0 = u;
        r1 = a.pair_offset + u;
    } else if constexpr (EPI == kRope) {
        r0 = (u >> 6) * 128 + (u & 63);
        r1 = r0 + 64;
    } else {
        r0 = u;
        r1 = u;
    }
}

__device__ unsigned int g_gemv_timeouts = 0;

// Epilogue of one unit (lane 0 holds the warp sums y[r][m], rounded to bf16).
template <int MB, int EPI, int R>
__device__ __forceinline__ void unit_epilogue(const GemvArgs& a, int64_t u, int64_t r0, const float (&y)[R][MB],
                                              int64_t pos, unsigned long long* cta_key) {
#pragma unroll
    for (int m = 0; m < MB; ++m) {
        if (m >= a.batch) break;
        if constexpr (EPI == kStore) {
            a.out[m * a.out_stride + r0] = __float2bfloat16_rn(y[0][m]);
        } else if constexpr (EPI == kSwiglu) {
            const float g = y[0][m];
            const float s = round_bf(g / (1.0f + expf(-g)));
            a.out[m * a.out_stride + u] = __float2bfloat16_rn(s * y[R - 1][m]);
        } else if constexpr (EPI == kRope) {
            const int h = static_cast<int>(u >> 6), d = static_cast<int>(u & 63);
            const float x0 = y[0][m], x1 = y[R - 1][m];
            if (h < a.q_heads + a.kv_heads) {
                const float c = __bfloat162float(a.cos_tab[pos * 64 + d]);
                const float s = __bfloat162float(a.sin_tab[pos * 64 + d]);
                const __nv_bfloat16 o0 = __float2bfloat16_rn(round_bf(x0 * c) + round_bf(-x1 * s));
                const __nv_bfloat16 o1 = __float2bfloat16_rn(round_bf(x1 * c) + round_bf(x0 * s));
                if (h < a.q_heads) {
                    __nv_bfloat16* q = a.q_out + (static_cast<int64_t>(m) * a.q_heads + h) * 128;
                    q[d] = o0;
                    q[d + 64] = o1;
                } else {
                    const int kh = h - a.q_heads;
                    __nv_bfloat16* kc = a.k_cur + (static_cast<int64_t>(m) * a.kv_heads + kh) * 128;
                    __nv_bfloat16* kr = a.k_cache + m * a.kbs + kh * a.khs + pos * a.kts;
                    kc[d] = o0;
                    kc[d + 64] = o1;
                    kr[d] = o0;
                    kr[d + 64] = o1;
                }
            } else {
                const int vh = h - a.q_heads - a.kv_heads;
                __nv_bfloat16* vc = a.v_cur + (static_cast<int64_t>(m) * a.kv_heads + vh) * 128;
                __nv_bfloat16* vr = a.v_cache + m * a.vbs + vh * a.vhs + pos * a.vts;
                const __nv_bfloat16 o0 = __float2bfloat16_rn(x0), o1 = __float2bfloat16_rn(x1);
                vc[d] = o0;
                vc[d + 64] = o1;
                vr[d] = o0;
                vr[d + 64] = o1;
            }
        } else {  // argmax
            const __nv_bfloat16 v = __float2bfloat16_rn(y[0][m]);
            a.out[m * a.out_stride + r0] = v;
            atomicMax(&cta_key[m], argmax_key(v, r0));
        }
    }
}

// The greedy choice over all CTAs: each CTA folds its best key into the global
// one; the last CTA to arrive writes the token ids, clears the state and
// advances the position.
__device__ __forceinline__ void argmax_finish(const GemvArgs& a, unsigned long long* cta_key, unsigned int& s_last) {
    const int tid = threadIdx.x;
    __syncthreads();
    if (tid < a.batch && cta_key[tid]) atomicMax(a.argmax_key + tid, cta_key[tid]);
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(a.done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (s_last) {
        __threadfence();
        if (tid < a.batch) {
            const unsigned long long key = atomicExch(a.argmax_key + tid, 0ull);
            a.token_next[tid] = static_cast<int64_t>(0xFFFFFFFFu - static_cast<uint32_t>(key & 0xFFFFFFFFull));
        }
        if (tid == 0) {
            *a.done = 0u;
            if (a.advance) *a.advance += 1;
        }
    }
}

// Weights move in pieces of up to kPieceElems elements of one row; each warp
// streams its own pieces through a private ring of S shared-memory slots with
// bulk asynchronous copies (lane 0 issues, every lane waits on the slot's
// mbarrier), so a warp keeps S pieces in flight without holding registers.
constexpr int kTmaWarps = 8;
constexpr int kTmaThreads = kTmaWarps * 32;
constexpr int kPieceElems = 4096;
constexpr int kPieceBytes = kPieceElems * 2;
// Loaded HBM latency is several microseconds: a full SM's worth of slots in
// flight (~190 KB) is what keeps the stream near peak, so one CTA per SM.
constexpr int kSmemBudget = 227 * 1024;

// Walks a warp's pieces in order without divisions: the warp's unit t, row r
// of the unit, piece p of the row.
struct PieceCursor {
    int t = 0, r = 0, p = 0;
    __device__ __forceinline__ void next(int rows, int npieces) {
        if (++p == npieces) {
            p = 0;
            if (++r == rows) {
                r = 0;
                ++t;
            }
        }
    }
};

template <int MB, int PRO, int EPI, int S>
__global__ void __launch_bounds__(kTmaThreads, 1) gemv_kernel(const GemvArgs a) {
    constexpr int R = (EPI == kSwiglu || EPI == kRope) ? 2 : 1;  // rows per unit
    extern __shared__ __align__(128) uint4 smem[];
    uint4* ring = smem;                                            // [warps][S][kPieceBytes / 16]
    uint4* xs = smem + kTmaWarps * S * (kPieceBytes / 16);         // [MB][k / 8]
    __shared__ __align__(8) uint64_t bars[kTmaWarps][S];
    __shared__ float red[kMaxBatch * kTmaWarps];
    __shared__ unsigned long long cta_key[kMaxBatch];
    __shared__ unsigned int s_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t gw = static_cast<int64_t>(blockIdx.x) * kTmaWarps + warp;
    const int nch = a.k / 8;
    const int64_t k = a.k;
    const int npieces = (a.k + kPieceElems - 1) / kPieceElems;
    const int ppu = R * npieces;
    const int my_units =
        (gw < a.active_warps && gw < a.units) ? static_cast<int>((a.units - 1 - gw) / a.active_warps + 1) : 0;
    const int total = my_units * ppu;
    uint4* my_ring = ring + static_cast<int64_t>(warp) * S * (kPieceBytes / 16);

    // Piece j of this warp (issued in order, lane 0): unit gw + t * active_warps,
    // row r of the unit, elements [p * kPieceElems, ...) of that row.
    PieceCursor produced;
    auto issue = [&](int j) {
        int64_t r0, r1;
        unit_rows<EPI>(a, gw + static_cast<int64_t>(produced.t) * a.active_warps, r0, r1);
        const int64_t row = produced.r == 0 ? r0 : r1;
        const int64_t off = static_cast<int64_t>(produced.p) * kPieceElems;
        const int64_t elems = k - off < kPieceElems ? k - off : kPieceElems;
        const int st = j % S;
        mbar_arrive_expect_tx(&bars[warp][st], static_cast<uint32_t>(elems * 2));
        bulk_copy_g2s(my_ring + st * (kPieceBytes / 16), a.w + row * k + off, static_cast<uint32_t>(elems * 2),
                      &bars[warp][st]);
        produced.next(R, npieces);
    };

    // The weights do not depend on the previous kernel: fill the ring first.
    if (lane == 0) {
#pragma unroll
        for (int st = 0; st < S; ++st) mbar_init(&bars[warp][st], 1);
        fence_async_smem();
        for (int j = 0; j < S && j < total; ++j) issue(j);
    }
    if constexpr (EPI == kArgmax) {
        if (tid < kMaxBatch) cta_key[tid] = 0ull;
    }
    __syncwarp();
    pdl_wait();
    // The previous kernel is complete: let the next one start filling its rings.
    pdl_launch_dependents();
    if constexpr (PRO == kNorm) load_x_norm<MB, kTmaThreads, kTmaWarps>(a, xs, red);
    else load_x_plain<MB, kTmaThreads>(a, xs);

    int64_t pos = 0;
    if constexpr (EPI == kRope) {
        pos = *a.position;
        pos = pos < 0 ? 0 : (pos > a.max_position ? a.max_position : pos);
    }

    float acc0[R][MB], acc1[R][MB];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int m = 0; m < MB; ++m) acc0[r][m] = acc1[r][m] = 0.0f;
    bool failed = false;
    int j = 0;
    PieceCursor cur;
    for (; j < total; ++j) {
        const int st = j % S;
        const bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(&bars[warp][st], static_cast<uint32_t>((j / S) & 1)));
        if (!ok) {
            failed = true;
            break;
        }
        const int r = cur.r, p = cur.p;
        const bool unit_end = r == R - 1 && p == npieces - 1;
        const int64_t u = gw + static_cast<int64_t>(cur.t) * a.active_warps;
        cur.next(R, npieces);
        const int pch = (a.k - p * kPieceElems < kPieceElems ? a.k - p * kPieceElems : kPieceElems) / 8;
        const uint4* wp = my_ring + st * (kPieceBytes / 16);
        const uint4* xp = xs + p * (kPieceElems / 8);
        if (r == 0) {
#pragma unroll 4
            for (int c = lane; c < pch; c += 32) {
                const uint4 wv = wp[c];
#pragma unroll
                for (int m = 0; m < MB; ++m) dot8(wv, xp[m * nch + c], acc0[0][m], acc1[0][m]);
            }
        } else {
#pragma unroll 4
            for (int c = lane; c < pch; c += 32) {
                const uint4 wv = wp[c];
#pragma unroll
                for (int m = 0; m < MB; ++m) dot8(wv, xp[m * nch + c], acc0[R - 1][m], acc1[R - 1][m]);
            }
        }
        __syncwarp();
        if (lane == 0 && j + S < total) {
            fence_async_smem();  // this slot's reads come before the copy that overwrites it
            issue(j + S);
        }
        if (unit_end) {
            int64_t r0, r1;
            unit_rows<EPI>(a, u, r0, r1);
            float y[R][MB];
#pragma unroll
            for (int rr = 0; rr < R; ++rr)
#pragma unroll
                for (int m = 0; m < MB; ++m) {
                    y[rr][m] = round_bf(warp_sum(acc0[rr][m] + acc1[rr][m]));
                    acc0[rr][m] = acc1[rr][m] = 0.0f;
                }
            if (lane == 0) unit_epilogue<MB, EPI, R>(a, u, r0, y, pos, cta_key);
        }
    }
    if (failed) {
        // Record the stall and wait (bounded) for this warp's copies still in flight.
        if (lane == 0) {
            atomicAdd(&g_gemv_timeouts, 1u);
            for (int jj = j; jj < total && jj < j + S; ++jj)
                mbar_wait(&bars[warp][jj % S], static_cast<uint32_t>((jj / S) & 1));
        }
        __syncwarp();
    }
    if constexpr (EPI == kArgmax) argmax_finish(a, cta_key, s_last);
}

// ---------------------------------------------------------------------------
// Layer tail (batch 1): o_proj -> gate/up + SwiGLU -> down -> the next layer's
// q/k/v + RoPE, or the LM head + greedy argmax after the last layer, in one
// persistent launch of one CTA per SM.  Each warp's ring streams its pieces of
// all four phases back to back, so HBM stays busy across the phase boundaries;
// only the compute of phase p + 1 waits for every CTA to finish phase p (its
// input is phase p's output): a bounded grid barrier, then the CTA rebuilds x
// in shared memory.  One CTA per SM (220 KB of shared memory) and a grid of at
// most one CTA per SM make every CTA co-resident once earlier kernels drain.
// ---------------------------------------------------------------------------
constexpr int kTailPhases = 4;
constexpr int kTailSlots = 3;
constexpr int kGridPolls = 1 << 22;

struct TailArgs {
    GemvArgs ph[kTailPhases];
    unsigned long long* barrier;  // ticket counter, zero at setup
};

__device__ unsigned int g_tail_timeouts = 0;

#ifdef POPKV_TAIL_TIMING
// Phase timestamps (globaltimer ns) of thread 0 of each CTA: start, after the
// dependency wait, then per phase: compute start, CTA done, barrier released.
constexpr int kTailStamps = 14;
__device__ unsigned long long g_tail_stamp_ns[160 * kTailStamps];
#define POPKV_TAIL_STAMP(i)                                                           \
    do {                                                                              \
        if (threadIdx.x == 0 && blockIdx.x < 160) {                                  \
            unsigned long long t_;                                                   \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                   \
            g_tail_stamp_ns[blockIdx.x * kTailStamps + (i)] = t_;                    \
        }                                                                             \
    } while (0)
#else
#define POPKV_TAIL_STAMP(i) \
    do {                    \
    } while (0)
#endif

// Grid-wide barrier of co-resident CTAs on a monotonic ticket counter (never
// reset, so consecutive launches of the same grid size share it): arrival n
// waits until the count reaches the next multiple of the grid size.  False if
// the bounded wait gave up.
__device__ __forceinline__ bool grid_barrier(unsigned long long* count) {
    __shared__ int s_ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned long long ticket = atomicAdd(count, 1ull);
        const unsigned long long target = (ticket / gridDim.x + 1) * gridDim.x;
        volatile unsigned long long* vc = count;
        int ok = 0;
        for (int i = 0; i < kGridPolls; ++i) {
            if (*vc >= target) {
                ok = 1;
                break;
            }
        }
        __threadfence();
        s_ok = ok;
    }
    __syncthreads();
    return s_ok != 0;
}

template <int LAST>
__device__ __forceinline__ int tail_rows_per_unit(int p) {
    return (p == 1 || (p == 3 && LAST == kRope)) ? 2 : 1;
}

template <int LAST>
__device__ __forceinline__ void tail_rows(int p, const GemvArgs& a, int64_t u, int64_t& r0, int64_t& r1) {
    if (p == 1) unit_rows<kSwiglu>(a, u, r0, r1);
    else if (p == 3 && LAST == kRope) unit_rows<kRope>(a, u, r0, r1);
    else unit_rows<kStore>(a, u, r0, r1);
}

template <int LAST>
__global__ void __launch_bounds__(kTmaThreads, 1) layer_tail_kernel(const TailArgs t) {
    constexpr int S = kTailSlots;
    extern __shared__ __align__(128) uint4 smem[];
    uint4* ring = smem;
    uint4* xs = smem + kTmaWarps * S * (kPieceBytes / 16);
    __shared__ __align__(8) uint64_t bars[kTmaWarps][S];
    __shared__ float red[kMaxBatch * kTmaWarps];
    __shared__ unsigned long long cta_key[kMaxBatch];
    __shared__ unsigned int s_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t gw = static_cast<int64_t>(blockIdx.x) * kTmaWarps + warp;
    uint4* my_ring = ring + static_cast<int64_t>(warp) * S * (kPieceBytes / 16);

    // This warp's units per phase; pieces walk the phases in order.
    int units[kTailPhases], rows[kTailPhases], npieces[kTailPhases];
    int total = 0;
#pragma unroll
    for (int p = 0; p < kTailPhases; ++p) {
        const GemvArgs& a = t.ph[p];
        npieces[p] = (a.k + kPieceElems - 1) / kPieceElems;
        rows[p] = tail_rows_per_unit<LAST>(p);
        units[p] = (gw < a.active_warps && gw < a.units) ? static_cast<int>((a.units - 1 - gw) / a.active_warps + 1) : 0;
        total += units[p] * rows[p] * npieces[p];
    }

    int prod_phase = 0;
    PieceCursor produced;
    auto issue = [&](int j) {
        while (produced.t == units[prod_phase]) {  // next phase with work for this warp
            ++prod_phase;
            produced = PieceCursor{};
        }
        const int p = prod_phase;
        const GemvArgs& a = t.ph[p];
        int64_t r0, r1;
        tail_rows<LAST>(p, a, gw + static_cast<int64_t>(produced.t) * a.active_warps, r0, r1);
        const int64_t k = a.k;
        const int64_t row = produced.r == 0 ? r0 : r1;
        const int64_t off = static_cast<int64_t>(produced.p) * kPieceElems;
        const int64_t elems = k - off < kPieceElems ? k - off : kPieceElems;
        const int st = j % S;
        mbar_arrive_expect_tx(&bars[warp][st], static_cast<uint32_t>(elems * 2));
        bulk_copy_g2s(my_ring + st * (kPieceBytes / 16), a.w + row * k + off, static_cast<uint32_t>(elems * 2),
                      &bars[warp][st]);
        produced.next(rows[p], npieces[p]);
    };

    if (lane == 0) {
#pragma unroll
        for (int st = 0; st < S; ++st) mbar_init(&bars[warp][st], 1);
        fence_async_smem();
        for (int jj = 0; jj < S && jj < total; ++jj) issue(jj);
    }
    if (tid < kMaxBatch) cta_key[tid] = 0ull;
    POPKV_TAIL_STAMP(0);
    __syncwarp();
    pdl_wait();
    pdl_launch_dependents();
    POPKV_TAIL_STAMP(1);

    bool failed = false;
    int j = 0, j_fail = 0;
    for (int p = 0; p < kTailPhases; ++p) {
        const GemvArgs& a = t.ph[p];
        if (p > 0) {
            __syncthreads();
            POPKV_TAIL_STAMP(3 * p);  // every warp of the CTA is done with phase p - 1
            if (!grid_barrier(t.barrier) && tid == 0) atomicAdd(&g_tail_timeouts, 1u);
            POPKV_TAIL_STAMP(3 * p + 1);
        }
        if (p == 1 || p == 3) load_x_norm<1, kTmaThreads, kTmaWarps>(a, xs, red);
        else load_x_plain<1, kTmaThreads>(a, xs);
        POPKV_TAIL_STAMP(3 * p + 2);
        int64_t pos = 0;
        if (p == 3 && LAST == kRope) {
            pos = *a.position;
            pos = pos < 0 ? 0 : (pos > a.max_position ? a.max_position : pos);
        }
        const int R = rows[p], np = npieces[p];
        const int count = units[p] * R * np;
        float acc0[2] = {0.0f, 0.0f}, acc1[2] = {0.0f, 0.0f};
        PieceCursor cur;
        for (int q = 0; q < count; ++q, ++j) {
            if (failed) continue;
            const int st = j % S;
            if (!__all_sync(0xFFFFFFFFu, mbar_wait(&bars[warp][st], static_cast<uint32_t>((j / S) & 1)))) {
                failed = true;
                j_fail = j;
                if (lane == 0) atomicAdd(&g_tail_timeouts, 1u);
                continue;
            }
            const int r = cur.r, pc = cur.p;
            const bool unit_end = r == R - 1 && pc == np - 1;
            const int64_t u = gw + static_cast<int64_t>(cur.t) * a.active_warps;
            cur.next(R, np);
            const int pch = (a.k - pc * kPieceElems < kPieceElems ? a.k - pc * kPieceElems : kPieceElems) / 8;
            const uint4* wp = my_ring + st * (kPieceBytes / 16);
            const uint4* xp = xs + pc * (kPieceElems / 8);
            if (r == 0) {
#pragma unroll 4
                for (int c = lane; c < pch; c += 32) dot8(wp[c], xp[c], acc0[0], acc1[0]);
            } else {
#pragma unroll 4
                for (int c = lane; c < pch; c += 32) dot8(wp[c], xp[c], acc0[1], acc1[1]);
            }
            __syncwarp();
            if (lane == 0 && j + S < total) {
                fence_async_smem();
                issue(j + S);
            }
            if (unit_end) {
                int64_t r0, r1;
                tail_rows<LAST>(p, a, u, r0, r1);
                float y[2][1];
                y[0][0] = round_bf(warp_sum(acc0[0] + acc1[0]));
                y[1][0] = round_bf(warp_sum(acc0[1] + acc1[1]));
                acc0[0] = acc0[1] = acc1[0] = acc1[1] = 0.0f;
                if (lane == 0) {
                    if (p == 1) {
                        unit_epilogue<1, kSwiglu, 2>(a, u, r0, y, pos, cta_key);
                    } else if (p == 3) {
                        if constexpr (LAST == kRope) {
                            unit_epilogue<1, kRope, 2>(a, u, r0, y, pos, cta_key);
                        } else {
                            const float y1[1][1] = {{y[0][0]}};
                            unit_epilogue<1, kArgmax, 1>(a, u, r0, y1, pos, cta_key);
                        }
                    } else {
                        const float y1[1][1] = {{y[0][0]}};
                        unit_epilogue<1, kStore, 1>(a, u, r0, y1, pos, cta_key);
                    }
                }
            }
        }
    }
    __syncthreads();
    POPKV_TAIL_STAMP(12);
    if (failed && lane == 0) {  // the copies still in flight land before the CTA exits
        for (int jj = j_fail; jj < total && jj < j_fail + S; ++jj)
            mbar_wait(&bars[warp][jj % S], static_cast<uint32_t>((jj / S) & 1));
    }
    __syncwarp();
    if constexpr (LAST == kArgmax) argmax_finish(t.ph[kTailPhases - 1], cta_key, s_last);
}

int g_sm_count[64] = {0};

int sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!g_sm_count[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        g_sm_count[dev] = n > 0 ? n : 148;
    }
    return g_sm_count[dev];
}

template <int MB, int PRO, int EPI, int S>
int launch_gemv_s(GemvArgs a, cudaStream_t stream, const char* name) {
    const int sms = sm_count();
    const int64_t warps = static_cast<int64_t>(sms) * kTmaWarps;
    const int64_t rounds = (a.units + warps - 1) / warps;
    const int64_t active = rounds > 0 ? (a.units + rounds - 1) / rounds : 1;
    a.active_warps = static_cast<int>(active);
    const int64_t ctas = (active + kTmaWarps - 1) / kTmaWarps;
    const size_t smem = static_cast<size_t>(kTmaWarps) * S * kPieceBytes + static_cast<size_t>(MB) * a.k * 2;
    const int st = allow_dynamic_smem(gemv_kernel<MB, PRO, EPI, S>, static_cast<int>(smem));
    if (st != POPKV_OK) return st;
    const cudaError_t err = launch_pdl(gemv_kernel<MB, PRO, EPI, S>, dim3(static_cast<unsigned>(ctas)),
                                       dim3(kTmaThreads), smem, stream, 1, a);
    if (err != cudaSuccess) return fail(POPKV_ERR_CUDA, "%s: %s", name, cudaGetErrorString(err));
    return check_launch(name);
}

// Ring depth: as many slots per warp (up to 3) as shared memory leaves beside x.
template <int MB, int PRO, int EPI>
int launch_gemv(const GemvArgs& a, cudaStream_t stream, const char* name) {
    const int64_t x_bytes = static_cast<int64_t>(MB) * a.k * 2;
    const int64_t slot = static_cast<int64_t>(kTmaWarps) * kPieceBytes;
    const int64_t depth = (kSmemBudget - 1024 - x_bytes) / slot;
    if (depth >= 3) return launch_gemv_s<MB, PRO, EPI, 3>(a, stream, name);
    if (depth == 2) return launch_gemv_s<MB, PRO, EPI, 2>(a, stream, name);
    if (depth == 1) return launch_gemv_s<MB, PRO, EPI, 1>(a, stream, name);
    return fail(POPKV_ERR_UNSUPPORTED, "%s: batch * k too large for shared memory", name);
}

template <int PRO, int EPI>
int dispatch_gemv(const GemvArgs& a, cudaStream_t s, const char* name) {
    switch (a.batch) {
        case 1: return launch_gemv<1, PRO, EPI>(a, s, name);
        case 2: return launch_gemv<2, PRO, EPI>(a, s, name);
        case 3: return launch_gemv<3, PRO, EPI>(a, s, name);
        default: return launch_gemv<4, PRO, EPI>(a, s, name);
    }
}

int check_common(const void* w, int64_t rows, int64_t k, int64_t batch, const char* name) {
    if (batch < 1 || batch > kMaxBatch) return fail(POPKV_ERR_UNSUPPORTED, "%s: batch must be 1..%d", name, kMaxBatch);
    if (rows <= 0 || k <= 0 || k % 8) return fail(POPKV_ERR_INVALID, "%s: k must be a positive multiple of 8", name);
    if (k * batch * 2 > kSmemBudget - 1024 - kTmaWarps * kPieceBytes)
        return fail(POPKV_ERR_UNSUPPORTED, "%s: batch * k too large for shared memory", name);
    if (rows > 0x7FFFFFFFll) return fail(POPKV_ERR_UNSUPPORTED, "%s: too many rows", name);
    if (!w || !aligned(w, 16)) return fail(POPKV_ERR_INVALID, "%s: weights must be 16-byte aligned", name);
    return POPKV_OK;
}

GemvArgs norm_args(const void* w, int64_t units, int64_t k, int64_t batch, const void* hidden, const void* delta,
                   const void* embed, const int64_t* token, const void* norm_w, float eps, void* hidden_out) {
    GemvArgs a{};
    a.w = static_cast<const __nv_bfloat16*>(w);
    a.units = units;
    a.k = static_cast<int>(k);
    a.batch = static_cast<int>(batch);
    a.x = static_cast<const __nv_bfloat16*>(hidden);
    a.delta = static_cast<const __nv_bfloat16*>(delta);
    a.embed = static_cast<const __nv_bfloat16*>(embed);
    a.token = token;
    a.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
    a.eps = eps;
    a.hidden_out = static_cast<__nv_bfloat16*>(hidden_out);
    return a;
}

int check_norm(const void* hidden, const void* delta, const void* embed, const int64_t* token,
               const void* norm_w, const void* hidden_out, const char* name) {
    if (!norm_w || (!hidden && !embed) || (embed && !token))
        return fail(POPKV_ERR_INVALID, "%s: null pointer", name);
    if ((hidden && !aligned(hidden, 16)) || (delta && !aligned(delta, 16)) || (embed && !aligned(embed, 16)) ||
        !aligned(norm_w, 16) || (hidden_out && !aligned(hidden_out, 16)))
        return fail(POPKV_ERR_INVALID, "%s: activations must be 16-byte aligned", name);
    return POPKV_OK;
}

}  // namespace
}  // namespace popkv

extern "C" int popkv_linear(const void* w, int64_t rows, int64_t k, const void* x, int64_t batch, void* out,
                            int64_t out_stride, void* stream) {
    using namespace popkv;
    int st = check_common(w, rows, k, batch, "popkv_linear");
    if (st != POPKV_OK) return st;
    if (!x || !out || !aligned(x, 16)) return fail(POPKV_ERR_INVALID, "popkv_linear: null or unaligned input");
    if (out_stride < rows) return fail(POPKV_ERR_INVALID, "popkv_linear: out_stride < rows");
    GemvArgs a{};
    a.w = static_cast<const __nv_bfloat16*>(w);
    a.units = rows;
    a.k = static_cast<int>(k);
    a.batch = static_cast<int>(batch);
    a.x = static_cast<const __nv_bfloat16*>(x);
    a.out = static_cast<__nv_bfloat16*>(out);
    a.out_stride = out_stride;
    return dispatch_gemv<kPlain, kStore>(a, static_cast<cudaStream_t>(stream), "popkv_linear");
}

extern "C" int popkv_norm_qkv_rope(const void* w, int64_t q_heads, int64_t kv_heads, int64_t k, int64_t batch,
                                   const void* hidden, const void* delta, const void* embed, const int64_t* token,
                                   const void* norm_w, float eps, void* hidden_out, const void* cos_table,
                                   const void* sin_table, const int64_t* position_dev, int64_t max_position,
                                   void* q_out, void* k_cur, void* v_cur, void* k_cache, void* v_cache,
                                   int64_t k_batch_stride, int64_t k_head_stride, int64_t k_token_stride,
                                   int64_t v_batch_stride, int64_t v_head_stride, int64_t v_token_stride,
                                   void* stream) {
    using namespace popkv;
    if (q_heads <= 0 || kv_heads <= 0 || q_heads + 2 * kv_heads > (1 << 20))
        return fail(POPKV_ERR_INVALID, "popkv_norm_qkv_rope: invalid head counts");
    const int64_t rows = (q_heads + 2 * kv_heads) * 128;
    int st = check_common(w, rows, k, batch, "popkv_norm_qkv_rope");
    if (st == POPKV_OK) st = check_norm(hidden, delta, embed, token, norm_w, hidden_out, "popkv_norm_qkv_rope");
    if (st != POPKV_OK) return st;
    if (!cos_table || !sin_table || !position_dev || !q_out || !k_cur || !v_cur || !k_cache || !v_cache ||
        max_position < 0)
        return fail(POPKV_ERR_INVALID, "popkv_norm_qkv_rope: null pointer");
    GemvArgs a = norm_args(w, (q_heads + 2 * kv_heads) * 64, k, batch, hidden, delta, embed, token, norm_w, eps,
                           hidden_out);
    a.q_heads = static_cast<int>(q_heads);
    a.kv_heads = static_cast<int>(kv_heads);
    a.cos_tab = static_cast<const __nv_bfloat16*>(cos_table);
    a.sin_tab = static_cast<const __nv_bfloat16*>(sin_table);
    a.position = position_dev;
    a.max_position = max_position;
    a.q_out = static_cast<__nv_bfloat16*>(q_out);
    a.k_cur = static_cast<__nv_bfloat16*>(k_cur);
    a.v_cur = static_cast<__nv_bfloat16*>(v_cur);
    a.k_cache = static_cast<__nv_bfloat16*>(k_cache);
    a.v_cache = static_cast<__nv_bfloat16*>(v_cache);
    a.kbs = k_batch_stride;
    a.khs = k_head_stride;
    a.kts = k_token_stride;
    a.vbs = v_batch_stride;
    a.vhs = v_head_stride;
    a.vts = v_token_stride;
    return dispatch_gemv<kNorm, kRope>(a, static_cast<cudaStream_t>(stream), "popkv_norm_qkv_rope");
}

extern "C" int popkv_norm_gate_up_swiglu(const void* w, int64_t inter, int64_t k, int64_t batch, const void* hidden,
                                         const void* delta, const void* norm_w, float eps, void* hidden_out,
                                         void* act, void* stream) {
    using namespace popkv;
    int st = check_common(w, 2 * inter, k, batch, "popkv_norm_gate_up_swiglu");
    if (st == POPKV_OK) st = check_norm(hidden, delta, nullptr, nullptr, norm_w, hidden_out, "popkv_norm_gate_up_swiglu");
    if (st != POPKV_OK) return st;
    if (!act) return fail(POPKV_ERR_INVALID, "popkv_norm_gate_up_swiglu: null pointer");
    GemvArgs a = norm_args(w, inter, k, batch, hidden, delta, nullptr, nullptr, norm_w, eps, hidden_out);
    a.out = static_cast<__nv_bfloat16*>(act);
    a.out_stride = inter;
    a.pair_offset = inter;
    return dispatch_gemv<kNorm, kSwiglu>(a, static_cast<cudaStream_t>(stream), "popkv_norm_gate_up_swiglu");
}

extern "C" int popkv_norm_lm_head_argmax(const void* w, int64_t vocab, int64_t k, int64_t batch, const void* hidden,
                                         const void* delta, const void* norm_w, float eps, void* hidden_out,
                                         void* logits, unsigned long long* argmax_state, int64_t* token_next,
                                         int64_t* position_dev, void* stream) {
    using namespace popkv;
    int st = check_common(w, vocab, k, batch, "popkv_norm_lm_head_argmax");
    if (st == POPKV_OK) st = check_norm(hidden, delta, nullptr, nullptr, norm_w, hidden_out, "popkv_norm_lm_head_argmax");
    if (st != POPKV_OK) return st;
    if (!logits || !argmax_state || !token_next)
        return fail(POPKV_ERR_INVALID, "popkv_norm_lm_head_argmax: null pointer");
    GemvArgs a = norm_args(w, vocab, k, batch, hidden, delta, nullptr, nullptr, norm_w, eps, hidden_out);
    a.out = static_cast<__nv_bfloat16*>(logits);
    a.out_stride = vocab;
    a.argmax_key = argmax_state;
    a.done = reinterpret_cast<unsigned int*>(argmax_state + batch);
    a.token_next = token_next;
    a.advance = position_dev;
    return dispatch_gemv<kNorm, kArgmax>(a, static_cast<cudaStream_t>(stream), "popkv_norm_lm_head_argmax");
}

extern "C" int popkv_gemv_timeouts(uint32_t* count) {
    using namespace popkv;
    if (!count) return fail(POPKV_ERR_INVALID, "popkv_gemv_timeouts: null pointer");
    const cudaError_t err = cudaMemcpyFromSymbol(count, g_gemv_timeouts, sizeof(uint32_t));
    if (err != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_gemv_timeouts: %s", cudaGetErrorString(err));
    return POPKV_OK;
}

namespace popkv {
namespace {

template <int LAST>
int launch_tail(TailArgs t, cudaStream_t stream) {
    const int sms = sm_count();
    const int64_t warps = static_cast<int64_t>(sms) * kTmaWarps;
    for (int p = 0; p < kTailPhases; ++p) {
        const int64_t rounds = (t.ph[p].units + warps - 1) / warps;
        t.ph[p].active_warps = static_cast<int>(rounds > 0 ? (t.ph[p].units + rounds - 1) / rounds : 1);
    }
    int64_t kmax = 0;
    for (int p = 0; p < kTailPhases; ++p) kmax = t.ph[p].k > kmax ? t.ph[p].k : kmax;
    const size_t smem = static_cast<size_t>(kTmaWarps) * kTailSlots * kPieceBytes + static_cast<size_t>(kmax) * 2;
    if (smem + 4096 > static_cast<size_t>(kSmemBudget))
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_layer_tail: k too large for shared memory");
    const int st = allow_dynamic_smem(layer_tail_kernel<LAST>, static_cast<int>(smem));
    if (st != POPKV_OK) return st;
    const cudaError_t err = launch_pdl(layer_tail_kernel<LAST>, dim3(static_cast<unsigned>(sms)), dim3(kTmaThreads),
                                       smem, stream, 1, t);
    if (err != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_layer_tail: %s", cudaGetErrorString(err));
    return check_launch("popkv_layer_tail");
}

}  // namespace
}  // namespace popkv

extern "C" int popkv_layer_tail(int64_t hidden_size, int64_t inter, int64_t attn_width, const void* o_w,
                                const void* attn, void* o_out, const void* gate_up_w, const void* post_norm,
                                const void* hidden_mid, void* hidden, void* act, float eps, const void* down_w,
                                void* down_out, const void* next_qkv_w, int64_t q_heads, int64_t kv_heads,
                                const void* next_input_norm, void* hidden_mid_out, const void* cos_table,
                                const void* sin_table, const int64_t* position_dev, int64_t max_position,
                                void* q_out, void* k_cur, void* v_cur, void* k_cache, void* v_cache,
                                int64_t k_batch_stride, int64_t k_head_stride, int64_t k_token_stride,
                                int64_t v_batch_stride, int64_t v_head_stride, int64_t v_token_stride,
                                const void* lm_head_w, int64_t vocab, const void* final_norm, void* logits,
                                unsigned long long* argmax_state, int64_t* token_next, unsigned int* barrier,
                                void* stream) {
    using namespace popkv;
    const char* name = "popkv_layer_tail";
    const int64_t H = hidden_size;
    int st = check_common(o_w, H, attn_width, 1, name);
    if (st == POPKV_OK) st = check_common(gate_up_w, 2 * inter, H, 1, name);
    if (st == POPKV_OK) st = check_common(down_w, H, inter, 1, name);
    if (st != POPKV_OK) return st;
    if (!attn || !o_out || !act || !down_out || !barrier || !aligned(attn, 16) || !aligned(o_out, 16) ||
        !aligned(act, 16) || !aligned(down_out, 16))
        return fail(POPKV_ERR_INVALID, "%s: null or unaligned buffer", name);
    st = check_norm(hidden_mid, o_out, nullptr, nullptr, post_norm, hidden, name);
    if (st != POPKV_OK) return st;
    if (!aligned(barrier, 8)) return fail(POPKV_ERR_INVALID, "%s: barrier must be 8-byte aligned", name);
    TailArgs t{};
    t.barrier = reinterpret_cast<unsigned long long*>(barrier);
    GemvArgs& o = t.ph[0];
    o.w = static_cast<const __nv_bfloat16*>(o_w);
    o.units = H;
    o.k = static_cast<int>(attn_width);
    o.batch = 1;
    o.x = static_cast<const __nv_bfloat16*>(attn);
    o.out = static_cast<__nv_bfloat16*>(o_out);
    o.out_stride = H;
    t.ph[1] = norm_args(gate_up_w, inter, H, 1, hidden_mid, o_out, nullptr, nullptr, post_norm, eps, hidden);
    t.ph[1].out = static_cast<__nv_bfloat16*>(act);
    t.ph[1].out_stride = inter;
    t.ph[1].pair_offset = inter;
    GemvArgs& d = t.ph[2];
    d.w = static_cast<const __nv_bfloat16*>(down_w);
    d.units = H;
    d.k = static_cast<int>(inter);
    d.batch = 1;
    d.x = static_cast<const __nv_bfloat16*>(act);
    d.out = static_cast<__nv_bfloat16*>(down_out);
    d.out_stride = H;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (next_qkv_w) {
        if (q_heads <= 0 || kv_heads <= 0 || !cos_table || !sin_table || !position_dev || !q_out || !k_cur ||
            !v_cur || !k_cache || !v_cache || max_position < 0)
            return fail(POPKV_ERR_INVALID, "%s: null pointer or invalid heads for the q/k/v phase", name);
        st = check_common(next_qkv_w, (q_heads + 2 * kv_heads) * 128, H, 1, name);
        if (st == POPKV_OK) st = check_norm(hidden, down_out, nullptr, nullptr, next_input_norm, hidden_mid_out, name);
        if (st != POPKV_OK) return st;
        GemvArgs& q = t.ph[3];
        q = norm_args(next_qkv_w, (q_heads + 2 * kv_heads) * 64, H, 1, hidden, down_out, nullptr, nullptr,
                      next_input_norm, eps, hidden_mid_out);
        q.q_heads = static_cast<int>(q_heads);
        q.kv_heads = static_cast<int>(kv_heads);
        q.cos_tab = static_cast<const __nv_bfloat16*>(cos_table);
        q.sin_tab = static_cast<const __nv_bfloat16*>(sin_table);
        q.position = position_dev;
        q.max_position = max_position;
        q.q_out = static_cast<__nv_bfloat16*>(q_out);
        q.k_cur = static_cast<__nv_bfloat16*>(k_cur);
        q.v_cur = static_cast<__nv_bfloat16*>(v_cur);
        q.k_cache = static_cast<__nv_bfloat16*>(k_cache);
        q.v_cache = static_cast<__nv_bfloat16*>(v_cache);
        q.kbs = k_batch_stride;
        q.khs = k_head_stride;
        q.kts = k_token_stride;
        q.vbs = v_batch_stride;
        q.vhs = v_head_stride;
        q.vts = v_token_stride;
        return launch_tail<kRope>(t, s);
    }
    if (!lm_head_w || !final_norm || !logits || !argmax_state || !token_next)
        return fail(POPKV_ERR_INVALID, "%s: null pointer for the LM-head phase", name);
    st = check_common(lm_head_w, vocab, H, 1, name);
    if (st != POPKV_OK) return st;
    GemvArgs& l = t.ph[3];
    l = norm_args(lm_head_w, vocab, H, 1, hidden, down_out, nullptr, nullptr, final_norm, eps, nullptr);
    l.out = static_cast<__nv_bfloat16*>(logits);
    l.out_stride = vocab;
    l.argmax_key = argmax_state;
    l.done = reinterpret_cast<unsigned int*>(argmax_state + 1);
    l.token_next = token_next;
    l.advance = const_cast<int64_t*>(position_dev);
    return launch_tail<kArgmax>(t, s);
}

extern "C" int popkv_layer_tail_timeouts(uint32_t* count) {
    using namespace popkv;
    if (!count) return fail(POPKV_ERR_INVALID, "popkv_layer_tail_timeouts: null pointer");
    const cudaError_t err = cudaMemcpyFromSymbol(count, g_tail_timeouts, sizeof(uint32_t));
    if (err != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_layer_tail_timeouts: %s", cudaGetErrorString(err));
    return POPKV_OK;
}

#ifdef POPKV_TAIL_TIMING
extern "C" __attribute__((visibility("default"))) int popkv_tail_stamps(unsigned long long* host, int ctas) {
    return static_cast<int>(cudaMemcpyFromSymbol(host, popkv::g_tail_stamp_ns,
                                                  sizeof(unsigned long long) * popkv::kTailStamps * ctas));
}
#endif
