// Launcher of the tensor-core (tcgen05 kind::i8) head_dim-128 scorer.
#pragma once

#include <cstdint>

#include <cuda_runtime.h>

namespace popkv {

// Shape and pointer checks shared by the score entry points (score.cu).
int check_score_common(int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t capacity,
                       int64_t tokens, int64_t g, const void* head_to_kv);

// Whether the tensor-core scorer handles this shape (<= 4 query heads per KV
// head, dim group 16/32/64).
bool score_mma_applies(int64_t q_heads, int64_t kv_heads, int64_t dim_group_size, int64_t batch,
                       int64_t tokens);

// fp16 scores [batch, q_heads, tokens] of raw queries (head_dim 128).
int launch_score_mma(const void* queries, int queries_dtype, int64_t batch, int64_t q_heads,
                     const int32_t* k_sign, const int32_t* k_mag, const uint16_t* k_low,
                     const uint16_t* k_delta, int64_t kv_heads, int64_t capacity,
                     const int64_t* head_to_kv, int64_t tokens, int64_t dim_group_size, uint16_t* scores,
                     cudaStream_t stream);

// Bounded waits of the fp8 tensor-core scorer (score_tc8.cuh) that gave up since load.
int read_score_tc8_timeouts(uint32_t* count);

}  // namespace popkv
