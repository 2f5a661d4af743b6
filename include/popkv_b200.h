/*
 * popkv_b200.h -- C ABI of the B200 (sm_100a) PopKV retrieval kernels.
 *
 * Every entry point takes plain device pointers, element counts and strides,
 * a CUDA stream (cudaStream_t passed as void*, NULL = legacy default stream)
 * and returns a status code (POPKV_OK on success).  On failure
 * popkv_last_error() returns a message describing the most recent failing
 * call on the calling host thread.  All work is enqueued asynchronously on
 * the given stream; no entry point synchronises the device or allocates
 * device memory.
 *
 * Each declaration names the reference interface it replaces (file:line in
 * kw78999/PopKV).  The reference binds its kernels through pybind11 + torch
 * (csrc/popkv_ext.cpp:39-52) and the Python wrappers in popkv_cuda.py and
 * sparse_kernels.py; the Python package popkv_b200 keeps those Python
 * signatures and calls these functions through ctypes.
 *
 * Layouts (token-major, as in the reference's PopKVCache.packed,
 * popkv.py:89-96 and csrc/popkv_ext.cu:1166-1171):
 *   k_sign, k_mag   int32  [kv_heads, capacity, W]    W = ceil(head_dim / 32)
 *   k_low, k_delta  fp16   [kv_heads, capacity, R]    R = ceil(head_dim / G)
 *   q_sign, q_mag   int32  [batch, q_heads, W]
 *   q_low, q_delta  fp32   [batch, q_heads, R]
 * Bit l of word w holds dimension 32*w + l.  G (dim_group_size) is 16, 32 or 64.
 */
#ifndef POPKV_B200_H
#define POPKV_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define POPKV_API __attribute__((visibility("default")))
#else
#define POPKV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element types of floating-point operands. */
#define POPKV_DTYPE_F32 0
#define POPKV_DTYPE_F16 1
#define POPKV_DTYPE_BF16 2

/* Status codes. */
#define POPKV_OK 0
#define POPKV_ERR_INVALID 1     /* an argument failed validation */
#define POPKV_ERR_CAPACITY 2    /* token_offset + tokens exceeds the planes' capacity */
#define POPKV_ERR_UNSUPPORTED 3 /* a valid request this build does not implement */
#define POPKV_ERR_CUDA 4        /* the CUDA runtime reported an error */

#define POPKV_ABI_VERSION 1

/* Message of the last failing call on this host thread ("" if none). */
POPKV_API const char* popkv_last_error(void);

/* POPKV_ABI_VERSION of the loaded library. */
POPKV_API int popkv_abi_version(void);

/*
 * Key bit-planes and low/delta representatives for `tokens` keys, written to
 * rows [token_offset, token_offset + tokens) of the planes.
 *
 * Replaces ext.pack / ext.pack_dim (prepack; csrc/popkv_ext.cu:1058-1073,
 * :1153-1175) and ext.pack_into / ext.pack_into_dim (append;
 * csrc/popkv_ext.cu:1075-1092, :1177-1206), reached from popkv_cuda.pack_keys
 * (popkv_cuda.py:53) and popkv_cuda.pack_keys_into (popkv_cuda.py:72).
 * Token groups of `token_group_size` are counted from keys' first token.
 * keys[h, t, d] is read at keys + h*key_head_stride + t*key_token_stride + d
 * (strides in elements; d is contiguous).
 */
POPKV_API int popkv_pack(const void* keys, int keys_dtype, int64_t kv_heads, int64_t tokens,
               int64_t head_dim, int64_t key_head_stride, int64_t key_token_stride,
               int32_t* k_sign, int32_t* k_mag, uint16_t* k_low, uint16_t* k_delta,
               int64_t capacity, int64_t token_offset, int64_t token_group_size,
               int64_t dim_group_size, void* stream);

/*
 * Append of one decoded token fused with its metadata re-encode (head_dim
 * 128, token groups of at most 128).
 *
 * What one launch does:
 * - It writes new_keys[h] and new_values[h] ([kv_heads, 128], contiguous)
 *   into the static caches at row `position`. cache_keys[h, t, d] is at
 *   cache_keys + h*k_head_stride + t*k_token_stride + d; likewise the values.
 * - It re-encodes the open token group, rows [sealed, position] of the key
 *   cache, into the planes at the same token rows. The new key comes straight
 *   from registers.
 *
 * `sealed` is the first row of the open group, a multiple of
 * token_group_size, and position - sealed < token_group_size. The planes
 * equal popkv_pack over the same rows.
 *
 * Replaces append_popkv's staging of active_keys (torch.cat) and
 * pack_keys_into (popkv.py:438-459, popkv_cuda.py:72-87,
 * csrc/popkv_ext.cu:1177-1206), together with the KV-cache append of the same
 * token.
 */
POPKV_API int popkv_append_kv(const void* new_keys, const void* new_values, int dtype, int64_t kv_heads,
                              int64_t head_dim, void* cache_keys, void* cache_values, int64_t k_head_stride,
                              int64_t k_token_stride, int64_t v_head_stride, int64_t v_token_stride,
                              int64_t position, int32_t* k_sign, int32_t* k_mag, uint16_t* k_low,
                              uint16_t* k_delta, int64_t capacity, int64_t sealed, int64_t token_group_size,
                              int64_t dim_group_size, void* stream);

/*
 * Query bit-planes and representatives of `rows` = batch*q_heads queries
 * [rows, head_dim] (contiguous).
 *
 * Replaces ext.query_encode_out (csrc/popkv_ext.cu:1315-1358), reached from
 * popkv_cuda.query_encode (popkv_cuda.py:157).
 */
POPKV_API int popkv_query_encode(const void* queries, int queries_dtype, int64_t rows, int64_t head_dim,
                       int64_t dim_group_size, int32_t* q_sign, int32_t* q_mag, float* q_low,
                       float* q_delta, void* stream);

/*
 * Popcount scores of the first `tokens` cached keys against pre-encoded
 * queries, for head_dim 128: scores fp16 [batch, q_heads, tokens].
 * head_to_kv int64 [q_heads]; query heads that share a KV head must be
 * consecutive (GQA layout arange(q_heads) // group).
 *
 * Replaces ext.score_encoded (csrc/popkv_ext.cu:1533-1593), reached from
 * popkv_cuda.score_encoded (popkv_cuda.py:170).
 */
POPKV_API int popkv_score_encoded(const int32_t* q_sign, const int32_t* q_mag, const float* q_low,
                        const float* q_delta, int64_t batch, int64_t q_heads,
                        const int32_t* k_sign, const int32_t* k_mag, const uint16_t* k_low,
                        const uint16_t* k_delta, int64_t kv_heads, int64_t capacity,
                        const int64_t* head_to_kv, int64_t tokens, int64_t dim_group_size,
                        uint16_t* scores, void* stream);

/*
 * Encode raw queries [batch, q_heads, head_dim] and score them.  For
 * head_dim 128 the scores are fp16 (scores_dtype must be POPKV_DTYPE_F16);
 * otherwise fp32 (POPKV_DTYPE_F32).
 *
 * head_dim 128 with at most 8 query heads per KV head and 16-byte aligned
 * tile rows (capacity * 2 * 128/dim_group_size bytes a multiple of 16) runs
 * the fp8 tensor-core scorer: the four counts per representative group are
 * exact products of +-1/0 fp8 vectors (mma.sync e4m3, fp32 accumulate) and
 * the fp32 reconstruction is the reference's, so the scores are bit-identical
 * to the popcount path.  Other shapes run the popcount scorer.
 *
 * Replaces ext.score and ext.score_dim (csrc/popkv_ext.cu:1208-1313), reached
 * from popkv_cuda.score (popkv_cuda.py:190).
 */
POPKV_API int popkv_score(const void* queries, int queries_dtype, int64_t batch, int64_t q_heads,
                int64_t head_dim, const int32_t* k_sign, const int32_t* k_mag,
                const uint16_t* k_low, const uint16_t* k_delta, int64_t kv_heads,
                int64_t capacity, const int64_t* head_to_kv, int64_t tokens,
                int64_t dim_group_size, void* scores, int scores_dtype, void* stream);

/*
 * Which head_dim-128 scorer the score entry points (popkv_score,
 * popkv_score_encoded, popkv_score_dyn, popkv_score_hist) use, for the whole
 * process: 0 (default) the faster one for the shape -- the fp8 tensor-core
 * scorer from about one 128-token tile per SM up (G16: 1024 tiles of
 * batch x KV heads x tokens/128; G32/G64: 4096), the popcount scorer below --
 * 1 always the popcount scorer, 2 the fp8 tensor-core scorer wherever it
 * applies (at most 4 query heads per KV head, 16-byte aligned representative
 * rows).  All give the same bits; this is a tuning and testing switch.
 * No reference counterpart.
 */
POPKV_API int popkv_score_dispatch(int mode);

/*
 * popkv_score on the popcount scorer only (one token per thread, __popc per
 * count), whatever the shape; bit-identical to popkv_score.  Kept for
 * comparison with the fp8 tensor-core scorer.
 *
 * Same interface and reference functions as popkv_score (ext.score,
 * csrc/popkv_ext.cu:1208-1313, via popkv_cuda.score, popkv_cuda.py:190).
 */
POPKV_API int popkv_score_popcount(const void* queries, int queries_dtype, int64_t batch,
                int64_t q_heads, int64_t head_dim, const int32_t* k_sign, const int32_t* k_mag,
                const uint16_t* k_low, const uint16_t* k_delta, int64_t kv_heads,
                int64_t capacity, const int64_t* head_to_kv, int64_t tokens,
                int64_t dim_group_size, void* scores, int scores_dtype, void* stream);

/*
 * popkv_score for head_dim 128 on the 5th-generation tensor cores: the four
 * per-group counts come from int8 matrix products (tcgen05.mma kind::i8,
 * accumulators in tensor memory) of the key bit planes expanded to +-1/0
 * bytes against the query coefficients, and the fp32 reconstruction is the
 * same as popkv_score's, so the scores are bit-identical.  At most 4 query
 * heads per KV head; POPKV_ERR_UNSUPPORTED otherwise or for other head dims.
 *
 * Same interface as popkv_score (and the same reference functions it replaces:
 * ext.score, csrc/popkv_ext.cu:1208-1313, via popkv_cuda.score).
 */
POPKV_API int popkv_score_tc(const void* queries, int queries_dtype, int64_t batch, int64_t q_heads,
                int64_t head_dim, const int32_t* k_sign, const int32_t* k_mag,
                const uint16_t* k_low, const uint16_t* k_delta, int64_t kv_heads,
                int64_t capacity, const int64_t* head_to_kv, int64_t tokens,
                int64_t dim_group_size, void* scores, int scores_dtype, void* stream);

/*
 * popkv_score plus the first radix pass of the top-k, for head_dim 128 and at
 * most 4 query heads per KV head: besides the fp16 scores it adds, for every
 * query row, the count of scores per top-11-bit key digit into hist
 * (uint32 [batch*q_heads, 2048]), which must hold zeros on entry.
 * popkv_topk_hist consumes the histogram and leaves it zeroed again.
 * No reference counterpart: the reference runs torch.topk on the scores.
 */
POPKV_API int popkv_score_hist(const void* queries, int queries_dtype, int64_t batch,
                               int64_t q_heads, const int32_t* k_sign, const int32_t* k_mag,
                               const uint16_t* k_low, const uint16_t* k_delta, int64_t kv_heads,
                               int64_t capacity, const int64_t* head_to_kv, int64_t tokens,
                               int64_t dim_group_size, uint16_t* scores, uint32_t* hist,
                               void* stream);

/*
 * popkv_topk for fp16 scores whose first-pass histogram popkv_score_hist has
 * already produced (rows of up to 262144 scores; `hist` 16-byte aligned).
 * Same output contract as popkv_topk; resets the rows of `hist` it reads to
 * zero, also when k is 0.
 */
POPKV_API int popkv_topk_hist(const uint16_t* scores, uint32_t* hist, int64_t rows, int64_t tokens,
                              int64_t row_stride, int64_t k, int64_t current_index, int64_t* out,
                              int64_t out_stride, void* stream);

/*
 * Per-row top-k with the current-token slot reserved.
 *
 * For each of `rows` rows of `tokens` scores (fp16 or fp32, row r at
 * scores + r*row_stride elements) writes the k highest-scoring token indices
 * in ascending index order to out[r*out_stride + 0 .. k-1] (int64).  Ties
 * rank by lower token index; +0 and -0 are equal; NaN ranks highest.  When
 * current_index >= 0 it is written to out[r*out_stride + k].
 *
 * Replaces torch.topk(scores, k, dim=-1, sorted=False).indices followed by
 * _append_current (popkv.py:1094-1098, :287-291), whose order among equal
 * scores is unspecified; also serves LlamaSparseDecoder.experimental_topk
 * (popkv.py:1091-1093).
 */
POPKV_API int popkv_topk(const void* scores, int scores_dtype, int64_t rows, int64_t tokens,
               int64_t row_stride, int64_t k, int64_t current_index, int64_t* out,
               int64_t out_stride, void* stream);

/*
 * Split-token sparse attention partial states.
 *
 * queries [batch, q_heads, head_dim] (contiguous); prefix K/V element (b, h, t, d)
 * at base + b*batch_stride + h*head_stride + t*token_stride + d; current K/V
 * [batch, kv_heads, head_dim] (contiguous); indices int64 [batch, q_heads,
 * selected]; valid uint8 [batch, q_heads, selected] or NULL; head_to_kv int64
 * [q_heads].  Slot j of split s = j / split_tokens reads the current key/value
 * when indices == prefix_tokens, else prefix row clamp(index, 0,
 * prefix_tokens - 1); masked slots are skipped.  partials fp32
 * [batch, q_heads, splits, head_dim + 2] = (max logit, sum exp, sum exp*v).
 *
 * Replaces sparse_kernels.indexed_attention_split_partial and its Triton
 * kernel (sparse_kernels.py:321-364, :237-294), which are batch-1.
 */
POPKV_API int popkv_attn_partial(const void* queries, int queries_dtype, int64_t batch, int64_t q_heads,
                       int64_t head_dim, const void* prefix_keys, const void* prefix_values,
                       int kv_dtype, int64_t kv_heads, int64_t prefix_tokens,
                       int64_t k_batch_stride, int64_t k_head_stride, int64_t k_token_stride,
                       int64_t v_batch_stride, int64_t v_head_stride, int64_t v_token_stride,
                       const void* current_keys, const void* current_values,
                       const int64_t* indices, int64_t selected, const uint8_t* valid,
                       const int64_t* head_to_kv, int64_t split_tokens, float* partials,
                       void* stream);

/*
 * Log-sum-exp merge of split partial states into one output row per query
 * head: out[r, d] = sum_s exp(m_s - M) acc_s[d] / sum_s exp(m_s - M) sum_s.
 *
 * Replaces sparse_kernels.indexed_attention_split_merge and its Triton kernel
 * (sparse_kernels.py:367-387, :297-318).
 */
POPKV_API int popkv_attn_merge(const float* partials, int64_t rows, int64_t splits, int64_t head_dim,
                     void* out, int out_dtype, void* stream);

/*
 * Split partials and their log-sum-exp merge in one call: the arguments of
 * popkv_attn_partial plus `counters` (int32 [batch*q_heads], zero before the
 * first call; every call leaves them zero again) and the merged output
 * `out` [batch, q_heads, head_dim] of `out_dtype`.  For bf16 queries/K/V with
 * head_dim 128, split_tokens <= 256 and at most 64 splits this is one launch
 * (the last CTA of each row merges it); otherwise it runs popkv_attn_partial
 * then popkv_attn_merge.  `partials` is scratch of popkv_attn_partial's size.
 *
 * Replaces sparse_kernels.indexed_attention_split (sparse_kernels.py:390-401).
 */
POPKV_API int popkv_attn_partial_merge(
    const void* queries, int queries_dtype, int64_t batch, int64_t q_heads, int64_t head_dim,
    const void* prefix_keys, const void* prefix_values, int kv_dtype, int64_t kv_heads,
    int64_t prefix_tokens, int64_t k_batch_stride, int64_t k_head_stride, int64_t k_token_stride,
    int64_t v_batch_stride, int64_t v_head_stride, int64_t v_token_stride,
    const void* current_keys, const void* current_values, const int64_t* indices, int64_t selected,
    const uint8_t* valid, const int64_t* head_to_kv, int64_t split_tokens, float* partials,
    int32_t* counters, void* out, int out_dtype, void* stream);

/*
 * popkv_attn_partial_merge with its scratch in a fixed device array of the
 * library instead of caller buffers: the call allocates no memory (no
 * cudaMalloc / cudaFree, no allocator of the caller).  No counterpart in the
 * reference, whose split attention allocates its partials with torch on every
 * call (sparse_kernels.py:321-364).
 *
 * For callers that cannot allocate device memory at the point of the call: a
 * C, Go or Java host that binds only this C ABI and owns no device allocator,
 * and serving loops whose device memory is already reserved up front for the
 * KV cache (there may be no free memory left), where a cudaMalloc / cudaFree
 * pair per token would also synchronise the device.
 *
 * Limits (POPKV_ERR_CAPACITY beyond them, checked before any CUDA call):
 * batch*q_heads <= 65536 and batch*q_heads*splits*(head_dim + 2) <= 2^20 fp32
 * (4 MiB), splits = ceil(selected / split_tokens); head_dim <= 256.
 *
 * The first call on a device (with that device current) sets up: it looks up
 * the array's address with cudaGetSymbolAddress and clears the completion
 * counters with cudaMemset + cudaDeviceSynchronize.  Make that first call
 * before any stream capture.  Every call leaves the counters zero.  All calls
 * on one device share the one array: calls that overlap in time (other
 * streams, other host threads) race on it and must be serialised by the
 * caller.  Other arguments and results as for popkv_attn_partial_merge.
 */
POPKV_API int popkv_attn_partial_merge_static(
    const void* queries, int queries_dtype, int64_t batch, int64_t q_heads, int64_t head_dim,
    const void* prefix_keys, const void* prefix_values, int kv_dtype, int64_t kv_heads,
    int64_t prefix_tokens, int64_t k_batch_stride, int64_t k_head_stride, int64_t k_token_stride,
    int64_t v_batch_stride, int64_t v_head_stride, int64_t v_token_stride,
    const void* current_keys, const void* current_values, const int64_t* indices, int64_t selected,
    const uint8_t* valid, const int64_t* head_to_kv, int64_t split_tokens, void* out, int out_dtype,
    void* stream);

/*
 * Fused decode-time retrieval for head_dim 128: popcount score of the first
 * `tokens` cached keys, per-head top-(budget-1) with the current slot
 * reserved, sparse attention over the selected rows plus the current token,
 * and the merge -- one launch, no global intermediates.
 *
 * queries [batch, q_heads, 128] and K/V share one dtype (bf16 or fp16); the
 * packed planes are laid out as for popkv_score_encoded with batch entry b at
 * row offset b*plane_batch_stride; prefix/current K/V as for
 * popkv_attn_partial; q_heads/kv_heads in {1, 2, 4}; tokens <= 131072.
 * out [batch, q_heads, 128] (queries' dtype).  Optional outputs (NULL to skip):
 * scores_out fp16 [batch, q_heads, tokens] (identical to popkv_score) and
 * indices_out int64 [batch, q_heads, k + 1], k = min(budget - 1, tokens)
 * (identical to popkv_topk with current_index = tokens).
 *
 * Replaces the PopKV branch of LlamaSparseDecoder.decode (popkv.py:1076-1115):
 * query_encode + score_encoded + torch.topk + _append_current +
 * indexed_attention_split_partial + indexed_attention_split_merge.
 */
POPKV_API int popkv_retrieve(
    const void* queries, int queries_dtype, int64_t batch, int64_t q_heads, int64_t head_dim,
    const int32_t* k_sign, const int32_t* k_mag, const uint16_t* k_low, const uint16_t* k_delta,
    int64_t kv_heads, int64_t capacity, int64_t plane_batch_stride, int64_t tokens,
    int64_t dim_group_size, const int64_t* head_to_kv, const void* prefix_keys,
    const void* prefix_values, int kv_dtype, int64_t k_batch_stride, int64_t k_head_stride,
    int64_t k_token_stride, int64_t v_batch_stride, int64_t v_head_stride, int64_t v_token_stride,
    const void* current_keys, const void* current_values, int64_t budget, void* out,
    uint16_t* scores_out, int64_t* indices_out, void* stream);

/*
 * Number of popkv_score_tc threads, since the library was loaded on the current
 * device, whose bounded wait for the tensor cores gave up (0 in a healthy
 * run).  A nonzero count means those launches' scores are incomplete.
 * Synchronises with the device.  No counterpart in the reference.
 */
POPKV_API int popkv_score_tc_timeouts(uint32_t* count);

/*
 * Copy `bytes` (a multiple of 16) from `src` to `dst` with a kernel, so that
 * the copy chains to the next kernel of the step by programmatic dependent
 * launch.  `src` may be pinned host memory (device-addressable under unified
 * addressing); both 16-byte aligned.  The captured decode step uses it to
 * bring a step's q | current k | current v in from host staging.
 *
 * No counterpart in the reference (its inputs are device tensors already).
 */
POPKV_API int popkv_stage(const void* src, void* dst, int64_t bytes, void* stream);

/*
 * Peer memory for the cross-GPU exchange (setup time, not per step).
 * popkv_peer_alloc: cudaMalloc `bytes` (zeroed) on the current device and
 * export it: `handle` receives the 64-byte CUDA IPC handle.  popkv_peer_open
 * maps another process's handle on the current device (peer access enabled
 * lazily); popkv_peer_close unmaps it; popkv_peer_free frees an allocation of
 * popkv_peer_alloc.  A process cannot open its own handle.  popkv_peer_clear
 * zeroes `bytes` of this process's area on `stream` (asynchronous): after a
 * wait for a peer gave up, every rank clears its area and its state words with
 * no launch in flight on any rank, then all ranks continue from epoch 0.
 *
 * No counterpart in the reference, which gathers with NCCL.
 */
POPKV_API int popkv_peer_alloc(int64_t bytes, void** ptr, unsigned char* handle);
POPKV_API int popkv_peer_open(const unsigned char* handle, void** ptr);
POPKV_API int popkv_peer_close(void* ptr);
POPKV_API int popkv_peer_clear(void* ptr, int64_t bytes, void* stream);
POPKV_API int popkv_peer_free(void* ptr);

/*
 * Merge of split partials (as popkv_attn_merge, head_dim 128) fused with the
 * all-gather of the merged rows across `world` GPUs over peer memory.
 *
 * Rank `rank` merges its `rows` local rows (one CTA per row).  Each element is
 * stored into every peer's receive area as one 8-byte word (value bits, launch
 * epoch).  The CTA then polls its own area for the same row of every peer,
 * with a bounded wait, and writes the world*rows gathered rows, rank-major, to
 * `out` [world*rows, 128] of `out_dtype`.
 *
 * Arguments:
 * - peer_recv: device array [world] of each rank's receive area. An area is
 *   2 x world x rows x 128 uint64, zero at setup, 8-byte aligned.
 * - own_recv: this rank's area.
 * - state: 4 uint32 in this rank's memory, zero at setup. state[0] counts
 *   launches, state[1] is scratch, state[2] becomes 1 when a wait for a peer
 *   gave up (the output is then incomplete; sticky until cleared), state[3]
 *   overrides the poll limit of each wait when nonzero (0: about a second).
 *
 * Every rank must issue the same sequence of these calls on one set of
 * buffers.
 *
 * Replaces popkv_attn_merge followed by a per-layer NCCL all-gather of the
 * KV-head shards' attention outputs (sparse_kernels.py:367-387 for the merge).
 */
POPKV_API int popkv_attn_merge_gather(const float* partials, int64_t rows, int64_t splits, int64_t head_dim,
                                      int out_dtype, int64_t rank, int64_t world, uint64_t* const* peer_recv,
                                      const uint64_t* own_recv, uint32_t* state, void* out, void* stream);

/*
 * One-shot all-reduce (sum) of `count` values of `dtype` in place across
 * `world` GPUs over peer memory: the partial products of a tensor-parallel
 * output projection or MLP down projection.  Each 32-bit word of `data` (two
 * fp16/bf16 values or one fp32) is stored into every peer's receive area with
 * the launch epoch; each rank polls its own area, with a bounded wait, and sums
 * in fp32 in rank order, rounded once, so every rank holds the same bits.
 *
 * Arguments:
 * - data: count values, 4-byte aligned; count * element size a multiple of 4.
 * - peer_recv / own_recv: as popkv_attn_merge_gather, areas of
 *   2 x world x (count * element size / 4) uint64, zero at setup.
 * - state: 4 uint32 in this rank's memory, as popkv_attn_merge_gather.
 *
 * Every rank must issue the same sequence of these calls on one set of
 * buffers.  The reference decodes on one GPU and has no counterpart; this
 * replaces torch.distributed.all_reduce in the tensor-parallel decode of
 * popkv_b200/decoder.py.
 */
POPKV_API int popkv_peer_sum(void* data, int dtype, int64_t count, int64_t rank, int64_t world,
                             uint64_t* const* peer_recv, const uint64_t* own_recv, uint32_t* state, void* stream);

/*
 * Device-resident step lengths.  The reference passes the cache length as a
 * Python integer on every decode call (popkv.py:1079-1099), so each token's
 * launches differ.  The *_dyn entry points read it from device memory at run
 * time instead (`tokens_dev` / `position_dev`: one int64, the number of cached
 * prefix tokens = the current token's position).  One captured CUDA graph then
 * serves every decode step while a kernel of the step advances the count.
 * Host-side arguments give the upper bounds the launch is sized for; a device
 * value outside [0, bound] is clamped to it.
 */

/*
 * popkv_score (raw queries, head_dim 128, fp16 scores) over the first
 * *tokens_dev <= max_tokens cached tokens.  Score row r starts at
 * scores + r * score_stride (score_stride >= max_tokens).
 * Replaces ext.score via popkv_cuda.score (csrc/popkv_ext.cu:1208-1313).
 */
POPKV_API int popkv_score_dyn(const void* queries, int queries_dtype, int64_t batch, int64_t q_heads,
                              const int32_t* k_sign, const int32_t* k_mag, const uint16_t* k_low,
                              const uint16_t* k_delta, int64_t kv_heads, int64_t capacity,
                              const int64_t* head_to_kv, const int64_t* tokens_dev, int64_t max_tokens,
                              int64_t dim_group_size, uint16_t* scores, int64_t score_stride, void* stream);

/*
 * popkv_topk over fp16 rows of t = *tokens_dev scores with k = min(k_max, t)
 * and the current slot t at out[r*out_stride + k] (out_stride >= k_max + 1).
 * max_tokens <= 262144.  Replaces torch.topk + _append_current
 * (popkv.py:1090-1099, :287-291).
 */
POPKV_API int popkv_topk_dyn(const uint16_t* scores, int64_t rows, const int64_t* tokens_dev,
                             int64_t max_tokens, int64_t row_stride, int64_t k_max, int64_t* out,
                             int64_t out_stride, void* stream);

/*
 * Split partials + merge (popkv_attn_partial + popkv_attn_merge) for
 * head_dim 128 and fp16/bf16 queries, K/V of the query dtype, with
 * t = *tokens_dev prefix tokens.
 *
 * With `indices` (rows of index_stride >= k_max + 1 int64, as written by
 * popkv_topk_dyn) a row attends over its min(k_max, t) + 1 selected slots;
 * with indices NULL it attends over every prefix token plus the current one
 * (the dense layers; as the reference's full-attention branch, popkv.py:1023-1036).
 * partials holds batch * q_heads * S * 130 fp32, S = ceil(m / split_tokens)
 * with m = min(k_max, max_tokens) + 1 (indices) or max_tokens + 1 (dense);
 * out [batch, q_heads, 128] of out_dtype, or NULL to leave the merge to the
 * caller (popkv_attn_merge_gather on several GPUs).
 * Replaces sparse_kernels.indexed_attention_split_partial + _merge
 * (sparse_kernels.py:321-387).
 */
POPKV_API int popkv_attn_dyn(const void* queries, int queries_dtype, int64_t batch, int64_t q_heads,
                             const void* prefix_keys, const void* prefix_values, int kv_dtype,
                             int64_t kv_heads, int64_t max_tokens, int64_t k_batch_stride,
                             int64_t k_head_stride, int64_t k_token_stride, int64_t v_batch_stride,
                             int64_t v_head_stride, int64_t v_token_stride, const void* current_keys,
                             const void* current_values, const int64_t* tokens_dev,
                             const int64_t* indices, int64_t index_stride, int64_t k_max,
                             const int64_t* head_to_kv, int64_t split_tokens, float* partials,
                             void* out, int out_dtype, void* stream);

/*
 * popkv_append_kv at position p = *position_dev (< max_tokens <= capacity):
 * re-encodes the open token group [p - p % token_group_size, p] of the key
 * cache into the packed planes.  With new_keys/new_values [kv_heads, 128] the
 * row p of the caches is written from them first; with both NULL the caller
 * has already written row p (popkv_rope_append does).
 * Replaces append_kv + append_retrieval_caches (popkv.py:965-972, :884-943).
 */
POPKV_API int popkv_append_kv_dyn(const void* new_keys, const void* new_values, int dtype,
                                  int64_t kv_heads, int64_t head_dim, void* cache_keys,
                                  void* cache_values, int64_t k_head_stride, int64_t k_token_stride,
                                  int64_t v_head_stride, int64_t v_token_stride,
                                  const int64_t* position_dev, int64_t max_tokens, int32_t* k_sign,
                                  int32_t* k_mag, uint16_t* k_low, uint16_t* k_delta,
                                  int64_t capacity, int64_t token_group_size,
                                  int64_t dim_group_size, void* stream);

/*
 * Decode-loop glue for a Llama-shaped model, bf16 only.
 *
 * popkv_rms_norm: per row of `dim`, with delta non-NULL hidden <- hidden +
 * delta first (the residual add, written back), then out = RMSNorm(hidden) *
 * weight.  Follows transformers' LlamaRMSNorm as called by the reference
 * decoder (popkv.py:1011, :1109; decode_runtime.py:39) with the rounding points
 * of its eager ops.
 *
 * popkv_rope_append: qkv [batch, (q_heads + 2 kv_heads) * 128] (q | k | v rows
 * of the fused projection); rotary embedding at position p = *position_dev
 * (clamped to max_position) from bf16 tables cos/sin [max_position + 1, 64];
 * writes the rotated queries to q_out [batch, q_heads, 128], the rotated keys
 * and the values to k_cur/v_cur [batch, kv_heads, 128] and to row p of the
 * caches.  Replaces _apply_rope (popkv.py:745-749) and append_kv
 * (popkv.py:965-972).
 *
 * popkv_silu_mul: act [rows, inter] = silu(gate) * up for gate_up
 * [rows, 2 * inter] = [gate | up] (the reference model's LlamaMLP).
 */
POPKV_API int popkv_rms_norm(const void* delta, void* hidden, const void* weight, int64_t rows,
                             int64_t dim, float eps, void* out, void* stream);
POPKV_API int popkv_rope_append(const void* qkv, int64_t batch, int64_t q_heads, int64_t kv_heads,
                                int64_t head_dim, const void* cos_table, const void* sin_table,
                                const int64_t* position_dev, int64_t max_position, void* q_out,
                                void* k_cur, void* v_cur, void* k_cache, void* v_cache,
                                int64_t k_batch_stride, int64_t k_head_stride, int64_t k_token_stride,
                                int64_t v_batch_stride, int64_t v_head_stride, int64_t v_token_stride,
                                void* stream);
POPKV_API int popkv_silu_mul(const void* gate_up, int64_t rows, int64_t inter, void* act, void* stream);


/*
 * Weight-streaming products of the decode step, bf16, batch 1..4 (the rows of
 * x), weights W [rows, k] row-major (k a multiple of 8, 16-byte aligned), fp32
 * accumulation, bf16 results; each fuses the element-wise work around it.  The
 * reference runs these as nn.Linear modules of the HF model plus separate
 * eager ops (popkv.py:1009-1016, :1103-1112; decode_runtime.py:37-40).
 *
 * popkv_linear: out[b, r] = sum_j W[r, j] x[b, j] (o_proj, down_proj).
 *
 * The popkv_norm_* products first form h = hidden[b] (or embed[token[b]] when
 * embed is non-NULL: the first layer) plus delta[b] when non-NULL (the
 * residual add, rounded to bf16), store h to hidden_out when non-NULL, and use
 * x = RMSNorm(h) * norm_w (LlamaRMSNorm rounding points, eps) as the vector:
 *
 * popkv_norm_qkv_rope: W = [q | k | v] rows of q_heads + 2 kv_heads heads of
 *   128; rotary embedding at p = *position_dev (clamped to max_position) from
 *   bf16 cos/sin tables [max_position + 1, 64]; rotated q to q_out [b, q_heads,
 *   128], rotated k and v to k_cur / v_cur [b, kv_heads, 128] and to row p of
 *   the caches (element (b, h, t, d) at base + b*batch_stride + h*head_stride +
 *   t*token_stride + d).  Replaces q/k/v_proj + _apply_rope + append_kv
 *   (popkv.py:1011-1016, :745-749, :965-972).
 * popkv_norm_gate_up_swiglu: W = [gate | up] ([2 inter, k]); act [b, inter] =
 *   silu(gate x) * (up x) (LlamaMLP without down_proj).
 * popkv_norm_lm_head_argmax: logits [b, vocab] = W x, and the greedy token
 *   (largest logit, lowest index among equals) to token_next[b]; argmax_state
 *   holds batch + 1 zeroed uint64 and is left zeroed; when position_dev is
 *   non-NULL the launch's last CTA adds 1 to it.  Replaces the final norm +
 *   lm_head (popkv.py:1109-1110) and the greedy argmax of the caller.
 */
/* Count of weight-streaming product warps whose bounded wait for a weight
 * copy gave up since the library was loaded (0 in a healthy run; their
 * outputs are incomplete).  Synchronises with the device. */
POPKV_API int popkv_gemv_timeouts(uint32_t* count);
POPKV_API int popkv_linear(const void* w, int64_t rows, int64_t k, const void* x, int64_t batch, void* out,
                           int64_t out_stride, void* stream);
POPKV_API int popkv_norm_qkv_rope(const void* w, int64_t q_heads, int64_t kv_heads, int64_t k, int64_t batch,
                                  const void* hidden, const void* delta, const void* embed, const int64_t* token,
                                  const void* norm_w, float eps, void* hidden_out, const void* cos_table,
                                  const void* sin_table, const int64_t* position_dev, int64_t max_position,
                                  void* q_out, void* k_cur, void* v_cur, void* k_cache, void* v_cache,
                                  int64_t k_batch_stride, int64_t k_head_stride, int64_t k_token_stride,
                                  int64_t v_batch_stride, int64_t v_head_stride, int64_t v_token_stride,
                                  void* stream);
POPKV_API int popkv_norm_gate_up_swiglu(const void* w, int64_t inter, int64_t k, int64_t batch,
                                        const void* hidden, const void* delta, const void* norm_w, float eps,
                                        void* hidden_out, void* act, void* stream);
/*
 * A layer's tail at batch 1 in one persistent launch (one CTA per SM):
 * o_out = o_w attn; act = SwiGLU(gate_up_w RMSNorm(hidden_mid + o_out)) with
 * hidden = hidden_mid + o_out stored; down_out = down_w act; then either the
 * next layer's popkv_norm_qkv_rope (next_qkv_w non-NULL: hidden + down_out,
 * stored to hidden_mid_out, normalised with next_input_norm, RoPE at
 * *position_dev into q_out / k_cur / v_cur and the caches) or, with next_qkv_w
 * NULL, popkv_norm_lm_head_argmax (final_norm, logits, argmax_state [2],
 * token_next, and *position_dev advanced by one).  Weight copies stream
 * across the phase boundaries; the phases meet at a bounded grid barrier on
 * `barrier` (2 uint32, zero at setup, left reusable).  Same results as the
 * separate products.  Replaces o_proj + MLP + the next layer's projections
 * (popkv.py:1103-1112, :1009-1016).
 */
POPKV_API int popkv_layer_tail(int64_t hidden_size, int64_t inter, int64_t attn_width, const void* o_w,
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
                               void* stream);
/* Count of layer-tail waits (a weight copy or the grid barrier) that gave up
 * since the library was loaded; 0 in a healthy run.  Synchronises. */
POPKV_API int popkv_layer_tail_timeouts(uint32_t* count);
POPKV_API int popkv_norm_lm_head_argmax(const void* w, int64_t vocab, int64_t k, int64_t batch,
                                        const void* hidden, const void* delta, const void* norm_w, float eps,
                                        void* hidden_out, void* logits, unsigned long long* argmax_state,
                                        int64_t* token_next, int64_t* position_dev, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* POPKV_B200_H */
