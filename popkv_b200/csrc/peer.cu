// Cross-GPU exchange of the attention output over NVLink peer memory.
//
// With KV heads sharded over `world` GPUs, rank r merges the split partials of
// its local query-head rows and every rank needs all rows.  The reference
// plan gathers them with one NCCL all-gather per layer after the merge.  Here
// the merge kernel itself does the exchange: each CTA merges one row, stores it
// into every peer's receive area, polls its own area for the same row of every
// peer, and writes the gathered rows to the output.  Merge and all-gather are
// one kernel.
//
// Each element crosses NVLink as one 8-byte word, (value bits, epoch), written
// with a single aligned store.  The receiver polls the word until its epoch is
// the current one, and a 64-bit aligned access is observed whole, so no fence
// or separate signal is needed.  The epoch is the launch count, kept in this
// rank's memory.  Receive slots alternate by launch parity: a rank that is one
// step ahead writes the other parity, and it cannot get two steps ahead,
// because finishing a step needs every peer's rows of that step.
//
// The memory is a plain cudaMalloc allocation exported with cudaIpcGetMemHandle:
// no NVLS object, no TMA.
#include <cstdint>
#include <cstring>

#include "common.cuh"

namespace popkv {
namespace {

constexpr int kGatherThreads = 128;      // one thread per output element (head_dim 128)
constexpr int kGatherMaxSplits = 1024;
constexpr long long kPolls = 1ll << 20;  // bounded wait for a peer's word (about a second)

// Poll limit of a launch: state[3] when nonzero (a test can make waits run out
// quickly), else kPolls.
__device__ __forceinline__ long long poll_limit(const unsigned int* state) {
    const unsigned int v = state[3];
    return v ? static_cast<long long>(v) : kPolls;
}

__device__ __forceinline__ unsigned long long load_relaxed_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void store_relaxed_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" :: "l"(p), "l"(v) : "memory");
}

template <typename OT>
__device__ __forceinline__ uint32_t out_bits(float v) {
    if constexpr (std::is_same<OT, float>::value) return __float_as_uint(v);
    else if constexpr (std::is_same<OT, __half>::value) return __half_as_ushort(__float2half_rn(v));
    else return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

template <typename OT>
__device__ __forceinline__ OT from_bits(uint32_t b) {
    if constexpr (std::is_same<OT, float>::value) return __uint_as_float(b);
    else if constexpr (std::is_same<OT, __half>::value) return __ushort_as_half(static_cast<unsigned short>(b));
    else return __ushort_as_bfloat16(static_cast<unsigned short>(b));
}

// Receive area of each rank: [2 parities][world source ranks][rows][128] words.
// state[0]: launches completed (the epoch), state[1]: CTAs done in this launch,
// state[2]: set to 1 when a wait for a peer gave up (sticky), state[3]: poll
// limit override (0: about a second).  After a wait gave up the ranks' epochs
// may disagree; every rank must then reset its area and state together
// (sharding._PeerArea.reset) before the next launch.
template <typename OT>
__global__ void __launch_bounds__(kGatherThreads) merge_gather_kernel(
    const float* __restrict__ partials, int64_t splits, int rows, int rank, int world,
    unsigned long long* const* __restrict__ peer_recv, const unsigned long long* own_recv,
    unsigned int* state, OT* __restrict__ out) {
    __shared__ float s_w[kGatherMaxSplits];
    __shared__ float s_red[kGatherThreads / 32];
    __shared__ float s_den;
    __shared__ int s_failed;
    pdl_wait();
    const unsigned int epoch = state[0] + 1u;
    const int64_t par = epoch & 1u;
    const long long limit = poll_limit(state);

    // Log-sum-exp merge of row `blockIdx.x`, in the order of attn_merge_kernel.
    const int64_t row = blockIdx.x;
    constexpr int D = 128;
    const int64_t state_len = D + 2;
    const float* p = partials + row * splits * state_len;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int nwarps = kGatherThreads / 32;
    if (tid == 0) s_failed = 0;
    // Up to 16 splits: this thread's dim of every split's accumulator is loaded
    // up front, overlapping the max/sum pass.
    constexpr int kPre = 16;
    const bool pre = splits <= kPre;
    float acc_pre[kPre];
    if (pre) {
#pragma unroll
        for (int sp = 0; sp < kPre; ++sp) acc_pre[sp] = sp < splits ? p[sp * state_len + 2 + tid] : 0.0f;
    }
    float gm = -INFINITY;
    for (int64_t sp = tid; sp < splits; sp += kGatherThreads) gm = fmaxf(gm, p[sp * state_len]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) gm = fmaxf(gm, __shfl_xor_sync(0xFFFFFFFFu, gm, o));
    if (lane == 0) s_red[warp] = gm;
    __syncthreads();
    gm = s_red[0];
    for (int w = 1; w < nwarps; ++w) gm = fmaxf(gm, s_red[w]);
    __syncthreads();
    float den = 0.0f;
    for (int64_t sp = tid; sp < splits; sp += kGatherThreads) {
        const float w = expf(p[sp * state_len] - gm);
        s_w[sp] = w;
        den = __fmaf_rn(p[sp * state_len + 1], w, den);
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
    float num = 0.0f;
    if (pre) {
#pragma unroll
        for (int sp = 0; sp < kPre; ++sp)
            if (sp < splits) num = __fmaf_rn(acc_pre[sp], s_w[sp], num);
    } else {
#pragma unroll 4
        for (int64_t sp = 0; sp < splits; ++sp) num = __fmaf_rn(p[sp * state_len + 2 + tid], s_w[sp], num);
    }
    const uint32_t bits = out_bits<OT>(num / den);

    // Send: this row to every peer, as (bits, epoch) words.
    const unsigned long long word = (static_cast<unsigned long long>(epoch) << 32) | bits;
    const int64_t send = ((par * world + rank) * rows + row) * D + tid;
    for (int r = 0; r < world; ++r)
        if (r != rank) store_relaxed_sys(peer_recv[r] + send, word);
    out[(static_cast<int64_t>(rank) * rows + row) * D + tid] = from_bits<OT>(bits);

    // Receive: the same row of every peer.
    bool ok = true;
    for (int r = 0; r < world; ++r) {
        if (r == rank) continue;
        const unsigned long long* src = own_recv + ((par * world + r) * rows + row) * D + tid;
        unsigned long long w = load_relaxed_sys(src);
        long long polls = 0;
        while (static_cast<unsigned int>(w >> 32) != epoch) {
            if (++polls > limit) {
                ok = false;
                break;
            }
            w = load_relaxed_sys(src);
        }
        out[(static_cast<int64_t>(r) * rows + row) * D + tid] = from_bits<OT>(static_cast<uint32_t>(w));
    }
    if (!ok) s_failed = 1;
    __syncthreads();
    if (tid == 0) {
        if (s_failed) state[2] = 1u;
        __threadfence();
        if (atomicAdd(&state[1], 1u) == gridDim.x - 1) {  // the last CTA advances the epoch
            state[1] = 0u;
            state[0] = epoch;
        }
    }
}

// One-shot all-reduce (sum) of a short vector over peer memory: the partial
// products of a tensor-parallel layer.  Each thread owns one 32-bit word of the
// vector (two 16-bit values or one fp32), stores it with the launch epoch into
// every peer's receive area, then polls its own area for the same word of
// every peer.  The sum runs in fp32 in rank order 0..world-1 and is rounded
// once, so every rank computes identical bits.  Receive area:
// [2 parities][world source ranks][words] 8-byte words; state as above.
constexpr int kSumThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kSumThreads) peer_sum_kernel(
    uint32_t* data, int64_t words, int rank, int world, unsigned long long* const* __restrict__ peer_recv,
    const unsigned long long* own_recv, unsigned int* state) {
    constexpr int V = 4 / static_cast<int>(sizeof(T));
    __shared__ int s_failed;
    pdl_wait();
    // The next product may fill its weight ring while the words cross NVLink.
    pdl_launch_dependents();
    if (threadIdx.x == 0) s_failed = 0;
    __syncthreads();
    const unsigned int epoch = state[0] + 1u;
    const int64_t par = epoch & 1u;
    const long long limit = poll_limit(state);
    const int64_t i = static_cast<int64_t>(blockIdx.x) * kSumThreads + threadIdx.x;
    if (i < words) {
        const uint32_t mine = data[i];
        const unsigned long long word = (static_cast<unsigned long long>(epoch) << 32) | mine;
        const int64_t send = (par * world + rank) * words + i;
        for (int r = 0; r < world; ++r)
            if (r != rank) store_relaxed_sys(peer_recv[r] + send, word);
        float acc[V];
#pragma unroll
        for (int v = 0; v < V; ++v) acc[v] = 0.0f;
        bool ok = true;
        for (int r = 0; r < world; ++r) {
            uint32_t bits = mine;
            if (r != rank) {
                const unsigned long long* src = own_recv + (par * world + r) * words + i;
                unsigned long long w = load_relaxed_sys(src);
                long long polls = 0;
                while (static_cast<unsigned int>(w >> 32) != epoch) {
                    if (++polls > limit) {
                        ok = false;
                        break;
                    }
                    w = load_relaxed_sys(src);
                }
                bits = static_cast<uint32_t>(w);
            }
#pragma unroll
            for (int v = 0; v < V; ++v)
                acc[v] += to_float(from_bits<T>(V == 1 ? bits : (bits >> (16 * v)) & 0xFFFFu));
        }
        uint32_t out = 0;
#pragma unroll
        for (int v = 0; v < V; ++v) out |= out_bits<T>(acc[v]) << (16 * v);
        data[i] = out;
        if (!ok) s_failed = 1;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (s_failed) state[2] = 1u;
        __threadfence();
        if (atomicAdd(&state[1], 1u) == gridDim.x - 1) {  // the last CTA advances the epoch
            state[1] = 0u;
            state[0] = epoch;
        }
    }
}

}  // namespace
}  // namespace popkv

extern "C" int popkv_peer_alloc(int64_t bytes, void** ptr, unsigned char* handle) {
    using namespace popkv;
    if (bytes <= 0 || !ptr || !handle) return fail(POPKV_ERR_INVALID, "popkv_peer_alloc: invalid arguments");
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, static_cast<size_t>(bytes));
    if (e != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_peer_alloc: cudaMalloc: %s", cudaGetErrorString(e));
    e = cudaMemset(p, 0, static_cast<size_t>(bytes));
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(p);
        return fail(POPKV_ERR_CUDA, "popkv_peer_alloc: %s", cudaGetErrorString(e));
    }
    std::memcpy(handle, &h, sizeof(h));
    *ptr = p;
    return POPKV_OK;
}

extern "C" int popkv_peer_open(const unsigned char* handle, void** ptr) {
    using namespace popkv;
    if (!handle || !ptr) return fail(POPKV_ERR_INVALID, "popkv_peer_open: invalid arguments");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_peer_open: %s", cudaGetErrorString(e));
    *ptr = p;
    return POPKV_OK;
}

extern "C" int popkv_peer_close(void* ptr) {
    using namespace popkv;
    const cudaError_t e = cudaIpcCloseMemHandle(ptr);
    if (e != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_peer_close: %s", cudaGetErrorString(e));
    return POPKV_OK;
}

extern "C" int popkv_peer_clear(void* ptr, int64_t bytes, void* stream) {
    using namespace popkv;
    if (!ptr || bytes <= 0) return fail(POPKV_ERR_INVALID, "popkv_peer_clear: invalid arguments");
    const cudaError_t e = cudaMemsetAsync(ptr, 0, static_cast<size_t>(bytes), static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_peer_clear: %s", cudaGetErrorString(e));
    return POPKV_OK;
}

extern "C" int popkv_peer_free(void* ptr) {
    using namespace popkv;
    const cudaError_t e = cudaFree(ptr);
    if (e != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_peer_free: %s", cudaGetErrorString(e));
    return POPKV_OK;
}

extern "C" int popkv_attn_merge_gather(const float* partials, int64_t rows, int64_t splits, int64_t head_dim,
                                       int out_dtype, int64_t rank, int64_t world, uint64_t* const* peer_recv,
                                       const uint64_t* own_recv, uint32_t* state, void* out, void* stream) {
    using namespace popkv;
    if (!valid_dtype(out_dtype)) return fail(POPKV_ERR_INVALID, "popkv_attn_merge_gather: output must be fp32/fp16/bf16");
    if (head_dim != 128) return fail(POPKV_ERR_UNSUPPORTED, "popkv_attn_merge_gather: head_dim must be 128");
    if (rows <= 0 || rows > 65535 || splits <= 0 || splits > kGatherMaxSplits)
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_attn_merge_gather: rows or splits out of range");
    if (world < 1 || world > 64 || rank < 0 || rank >= world)
        return fail(POPKV_ERR_INVALID, "popkv_attn_merge_gather: invalid rank/world");
    if (!partials || !peer_recv || !own_recv || !state || !out)
        return fail(POPKV_ERR_INVALID, "popkv_attn_merge_gather: null pointer");
    if (!aligned(own_recv, 8)) return fail(POPKV_ERR_INVALID, "popkv_attn_merge_gather: receive area must be 8-byte aligned");
    // Every CTA waits for a peer's CTA of the same row, so the whole grid must be
    // resident at once on every rank: at most one wave.
    int device = 0, sms = 0, per_sm = 0;
    cudaError_t qerr = cudaGetDevice(&device);
    if (qerr == cudaSuccess) qerr = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (qerr == cudaSuccess)
        qerr = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, merge_gather_kernel<float>, kGatherThreads, 0);
    if (qerr != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_attn_merge_gather: %s", cudaGetErrorString(qerr));
    if (rows > static_cast<int64_t>(sms) * per_sm)
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_attn_merge_gather: %lld rows exceed one resident wave (%d)",
                    static_cast<long long>(rows), sms * per_sm);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const dim3 grid(static_cast<unsigned>(rows)), block(kGatherThreads);
    const int r = static_cast<int>(rank), w = static_cast<int>(world), n = static_cast<int>(rows);
    auto peers = reinterpret_cast<unsigned long long* const*>(peer_recv);
    auto own = reinterpret_cast<const unsigned long long*>(own_recv);
    cudaError_t err;
    if (out_dtype == POPKV_DTYPE_F32)
        err = launch_pdl(merge_gather_kernel<float>, grid, block, 0, s, 1, partials, splits, n, r, w, peers, own,
                         state, static_cast<float*>(out));
    else if (out_dtype == POPKV_DTYPE_F16)
        err = launch_pdl(merge_gather_kernel<__half>, grid, block, 0, s, 1, partials, splits, n, r, w, peers, own,
                         state, static_cast<__half*>(out));
    else
        err = launch_pdl(merge_gather_kernel<__nv_bfloat16>, grid, block, 0, s, 1, partials, splits, n, r, w, peers,
                         own, state, static_cast<__nv_bfloat16*>(out));
    if (err != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_attn_merge_gather: %s", cudaGetErrorString(err));
    return check_launch("popkv_attn_merge_gather");
}

extern "C" int popkv_peer_sum(void* data, int dtype, int64_t count, int64_t rank, int64_t world,
                              uint64_t* const* peer_recv, const uint64_t* own_recv, uint32_t* state, void* stream) {
    using namespace popkv;
    if (!valid_dtype(dtype)) return fail(POPKV_ERR_INVALID, "popkv_peer_sum: data must be fp32/fp16/bf16");
    if (world < 1 || world > 64 || rank < 0 || rank >= world)
        return fail(POPKV_ERR_INVALID, "popkv_peer_sum: invalid rank/world");
    if (!data || !peer_recv || !own_recv || !state) return fail(POPKV_ERR_INVALID, "popkv_peer_sum: null pointer");
    const int64_t elem = dtype == POPKV_DTYPE_F32 ? 4 : 2;
    if (count <= 0 || (count * elem) % 4)
        return fail(POPKV_ERR_INVALID, "popkv_peer_sum: count must be positive and fill whole 4-byte words");
    if (!aligned(data, 4) || !aligned(own_recv, 8))
        return fail(POPKV_ERR_INVALID, "popkv_peer_sum: data must be 4-byte and the receive area 8-byte aligned");
    const int64_t words = count * elem / 4;
    const int64_t ctas = (words + kSumThreads - 1) / kSumThreads;
    // Every CTA waits for the peers' CTAs of the same words: one resident wave.
    int device = 0, sms = 0, per_sm = 0;
    cudaError_t qerr = cudaGetDevice(&device);
    if (qerr == cudaSuccess) qerr = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (qerr == cudaSuccess)
        qerr = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, peer_sum_kernel<float>, kSumThreads, 0);
    if (qerr != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_peer_sum: %s", cudaGetErrorString(qerr));
    if (ctas > static_cast<int64_t>(sms) * per_sm)
        return fail(POPKV_ERR_UNSUPPORTED, "popkv_peer_sum: %lld values exceed one resident wave",
                    static_cast<long long>(count));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const dim3 grid(static_cast<unsigned>(ctas)), block(kSumThreads);
    const int r = static_cast<int>(rank), w = static_cast<int>(world);
    auto peers = reinterpret_cast<unsigned long long* const*>(peer_recv);
    auto own = reinterpret_cast<const unsigned long long*>(own_recv);
    auto d = static_cast<uint32_t*>(data);
    cudaError_t err;
    if (dtype == POPKV_DTYPE_F32)
        err = launch_pdl(peer_sum_kernel<float>, grid, block, 0, s, 1, d, words, r, w, peers, own, state);
    else if (dtype == POPKV_DTYPE_F16)
        err = launch_pdl(peer_sum_kernel<__half>, grid, block, 0, s, 1, d, words, r, w, peers, own, state);
    else
        err = launch_pdl(peer_sum_kernel<__nv_bfloat16>, grid, block, 0, s, 1, d, words, r, w, peers, own, state);
    if (err != cudaSuccess) return fail(POPKV_ERR_CUDA, "popkv_peer_sum: %s", cudaGetErrorString(err));
    return check_launch("popkv_peer_sum");
}
