/*
 * popkv_oracle.c -- CPU restatement of PopKV's decode-time retrieval path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * kernels in popkv_b200/csrc and the timed CPU baseline of bench.py.  Nothing
 * in the shipped library links, imports or calls it.
 *
 * Every routine restates the arithmetic of the reference implementation
 * (kw78999/PopKV) with IEEE-754 single precision and round-to-nearest-even:
 *
 *   - key packing            csrc/popkv_ext.cu:381-500 (fused G16/G64),
 *                            :79-143 (G32), :284-374 (generic head dim)
 *   - query encoding         csrc/popkv_ext.cu:911-957 (G16/G64), :235-281 (G32)
 *   - popcount scoring       csrc/popkv_ext.cu:757-876 (GQA tiled, fp16 out),
 *                            :502-515 (four-count reconstruction),
 *                            :517-675 and :145-230 (generic head dim, fp32 out)
 *   - top-k + current slot   popkv.py:1090-1099, :287-291
 *   - split attention        sparse_kernels.py:237-294 (partials), :297-318 (merge)
 *
 * Documented differences from the reference GPU build (which compiles with
 * --use_fast_math): divisions here are correctly rounded (the reference uses the
 * approximate fast-math divide), subnormals are kept (the reference flushes them),
 * and the score scale is fp32(1 / fp32(sqrt(D))) (0x3DB504F3 for D = 128).  The
 * CUDA kernels of this project follow exactly these semantics, so the two agree
 * bit for bit.
 *
 * Reduction orders that fix the rounding of fp32 sums:
 *   key representatives: per representative group, lane value x[l] (l = 0..31)
 *     is the bucket's |k| at dim r*G + l, plus the one at r*G + l + 32 when G = 64,
 *     and the 32 lane values are added by the tree
 *       s[i] += s[i + o] for o = 16, 8, 4, 2, 1        (result in s[0])
 *     which is the warp shuffle-down reduction of popkv_ext.cu:121-127/408-414/474-480.
 *   query representatives: sequential, increasing dim (popkv_ext.cu:938-947).
 *   score: per representative group in increasing order,
 *       total += fma(ql*kl, c_sign, fma(dq*kl, c_q, fma(ql*dk, c_k, (dq*dk)*c_qk)))
 *     (popkv_ext.cu:511-514), then total * scale, then fp16 round-to-nearest-even.
 *
 * Build: see oracle/Makefile (gcc -O2 -ffp-contract=off -fopenmp).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

enum { DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2 };

enum {
    OK = 0,
    ERR_ARG = 1,
};

/* ------------------------------------------------------------------------ */
/* fp16 / bf16 conversions (exact decode, round-to-nearest-even encode).     */
/* ------------------------------------------------------------------------ */

static float bits_to_float(uint32_t u) {
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

static uint32_t float_to_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, sizeof u);
    return u;
}

float oracle_half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    if (exp == 0x1Fu) return bits_to_float(sign | 0x7F800000u | (man << 13));
    if (exp == 0) {
        if (man == 0) return bits_to_float(sign);
        /* subnormal: value = man * 2^-24 */
        float v = (float)man * 5.9604644775390625e-08f;
        return sign ? -v : v;
    }
    return bits_to_float(sign | ((exp + 112u) << 23) | (man << 13));
}

uint16_t oracle_float_to_half(float f) {
    uint32_t u = float_to_bits(f);
    uint32_t sign = (u >> 16) & 0x8000u;
    uint32_t abs = u & 0x7FFFFFFFu;
    if (abs >= 0x7F800000u) {                      /* inf or nan */
        if (abs == 0x7F800000u) return (uint16_t)(sign | 0x7C00u);
        return (uint16_t)(sign | 0x7E00u | ((abs >> 13) & 0x3FFu));
    }
    if (abs >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  /* rounds to inf */
    if (abs < 0x38800000u) {                        /* result is subnormal or zero */
        if (abs < 0x33000000u) return (uint16_t)sign; /* below half of min subnormal */
        uint32_t exp = abs >> 23;
        uint32_t man = (abs & 0x7FFFFFu) | 0x800000u;
        uint32_t shift = 126u - exp;                /* 14..24 */
        uint32_t q = man >> shift;
        uint32_t rem = man & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t exp = (abs >> 23) - 112u;
    uint32_t man = abs & 0x7FFFFFu;
    uint32_t q = (exp << 10) | (man >> 13);
    uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return (uint16_t)(sign | q);
}

static float load_elem(const void* base, int dtype, int64_t idx) {
    if (dtype == DT_F32) return ((const float*)base)[idx];
    uint16_t h = ((const uint16_t*)base)[idx];
    if (dtype == DT_F16) return oracle_half_to_float(h);
    return bits_to_float((uint32_t)h << 16);
}

/* ------------------------------------------------------------------------ */
/* Bucket means (popkv_ext.cu:128-135, shared by every encoder).             */
/* ------------------------------------------------------------------------ */

static void bucket_means(float low_sum, int low_count, float high_sum, int high_count,
                         float* low_out, float* delta_out) {
    float low, high;
    if (low_count == 0) {
        low = high_count ? high_sum / (float)high_count : 0.0f;
        high = low;
    } else {
        low = low_sum / (float)low_count;
        high = high_count ? high_sum / (float)high_count : low;
    }
    *low_out = low;
    *delta_out = high - low;
}

static float tree32(float* s) {
    for (int o = 16; o > 0; o >>= 1)
        for (int i = 0; i < o; ++i) s[i] = s[i] + s[i + o];
    return s[0];
}

/* ------------------------------------------------------------------------ */
/* Key packing: prepack (pack_keys) and append (pack_keys_into).            */
/* popkv_ext.cu:381-500, :79-143, :284-374; popkv_cuda.py:53-87.            */
/*                                                                          */
/* keys[h, t, d] lives at keys + h*head_stride + t*token_stride + d.        */
/* Token groups are counted from token 0 of `keys`; outputs go to rows      */
/* token_offset + t of the [kv_heads, capacity, words|reps] planes.         */
/* ------------------------------------------------------------------------ */

int oracle_pack(const void* keys, int dtype, int64_t kv_heads, int64_t tokens,
                int64_t head_dim, int64_t head_stride, int64_t token_stride,
                int64_t token_group_size, int64_t dim_group_size,
                int64_t capacity, int64_t token_offset,
                int32_t* k_sign, int32_t* k_mag, uint16_t* k_low, uint16_t* k_delta) {
    if (kv_heads < 0 || tokens < 0 || head_dim <= 0 || token_group_size < 1 ||
        (dim_group_size != 16 && dim_group_size != 32 && dim_group_size != 64) ||
        token_offset < 0 || token_offset + tokens > capacity)
        return ERR_ARG;
    const int64_t words = (head_dim + 31) / 32;
    const int64_t reps = (head_dim + dim_group_size - 1) / dim_group_size;
    const int64_t groups = (tokens + token_group_size - 1) / token_group_size;

#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int64_t h = 0; h < kv_heads; ++h) {
        for (int64_t g = 0; g < groups; ++g) {
            float* vmin = (float*)malloc(sizeof(float) * (size_t)head_dim);
            float* vmax = (float*)malloc(sizeof(float) * (size_t)head_dim);
            float* row = (float*)malloc(sizeof(float) * (size_t)head_dim);
            unsigned char* mag = (unsigned char*)malloc((size_t)head_dim);
            const int64_t t0 = g * token_group_size;
            const int64_t t1 = t0 + token_group_size < tokens ? t0 + token_group_size : tokens;
            for (int64_t d = 0; d < head_dim; ++d) {
                float v = load_elem(keys, dtype, h * head_stride + t0 * token_stride + d);
                vmin[d] = v; vmax[d] = v;
                for (int64_t t = t0 + 1; t < t1; ++t) {
                    float x = load_elem(keys, dtype, h * head_stride + t * token_stride + d);
                    vmin[d] = fminf(vmin[d], x);
                    vmax[d] = fmaxf(vmax[d], x);
                }
            }
            for (int64_t t = t0; t < t1; ++t) {
                const int64_t out_row = h * capacity + token_offset + t;
                for (int64_t d = 0; d < head_dim; ++d)
                    row[d] = load_elem(keys, dtype, h * head_stride + t * token_stride + d);
                for (int64_t w = 0; w < words; ++w) {
                    uint32_t sw = 0, mw = 0;
                    for (int64_t l = 0; l < 32; ++l) {
                        int64_t d = w * 32 + l;
                        if (d >= head_dim) break;
                        float v = row[d];
                        int sign = v >= 0.0f;
                        int m = sign ? (v > vmax[d] * 0.5f) : (v < vmin[d] * 0.5f);
                        mag[d] = (unsigned char)m;
                        if (sign) sw |= 1u << l;
                        if (m) mw |= 1u << l;
                    }
                    k_sign[out_row * words + w] = (int32_t)sw;
                    k_mag[out_row * words + w] = (int32_t)mw;
                }
                for (int64_t r = 0; r < reps; ++r) {
                    float low_lane[32], high_lane[32];
                    int low_count = 0, high_count = 0;
                    for (int l = 0; l < 32; ++l) {
                        float lo = 0.0f, hi = 0.0f;
                        for (int64_t j = l; j < dim_group_size; j += 32) {
                            int64_t d = r * dim_group_size + j;
                            if (d >= head_dim) continue;
                            float a = fabsf(row[d]);
                            if (mag[d]) { hi = hi + a; ++high_count; }
                            else { lo = lo + a; ++low_count; }
                        }
                        low_lane[l] = lo;
                        high_lane[l] = hi;
                    }
                    float low_sum = tree32(low_lane);
                    float high_sum = tree32(high_lane);
                    float low, delta;
                    bucket_means(low_sum, low_count, high_sum, high_count, &low, &delta);
                    k_low[out_row * reps + r] = oracle_float_to_half(low);
                    k_delta[out_row * reps + r] = oracle_float_to_half(delta);
                }
            }
            free(vmin); free(vmax); free(row); free(mag);
        }
    }
    return OK;
}

/* ------------------------------------------------------------------------ */
/* Query encoding: whole-head thresholds, sequential representative sums.    */
/* popkv_ext.cu:911-957 (G16/G64) and :235-281 (G32); popkv_cuda.py:157-167. */
/* ------------------------------------------------------------------------ */

int oracle_query_encode(const void* queries, int dtype, int64_t rows, int64_t head_dim,
                        int64_t dim_group_size, int32_t* q_sign, int32_t* q_mag,
                        float* q_low, float* q_delta) {
    if (rows < 0 || head_dim <= 0 ||
        (dim_group_size != 16 && dim_group_size != 32 && dim_group_size != 64))
        return ERR_ARG;
    const int64_t words = (head_dim + 31) / 32;
    const int64_t reps = (head_dim + dim_group_size - 1) / dim_group_size;
#pragma omp parallel for schedule(static)
    for (int64_t row = 0; row < rows; ++row) {
        const int64_t base = row * head_dim;
        float mn = load_elem(queries, dtype, base), mx = mn;
        for (int64_t d = 1; d < head_dim; ++d) {
            float v = load_elem(queries, dtype, base + d);
            mn = fminf(mn, v);
            mx = fmaxf(mx, v);
        }
        const float neg = mn * 0.5f, pos = mx * 0.5f;
        for (int64_t w = 0; w < words; ++w) {
            uint32_t sw = 0, mw = 0;
            for (int64_t d = w * 32; d < head_dim && d < w * 32 + 32; ++d) {
                float v = load_elem(queries, dtype, base + d);
                int sign = v >= 0.0f;
                int m = sign ? (v > pos) : (v < neg);
                if (sign) sw |= 1u << (d - w * 32);
                if (m) mw |= 1u << (d - w * 32);
            }
            q_sign[row * words + w] = (int32_t)sw;
            q_mag[row * words + w] = (int32_t)mw;
        }
        for (int64_t r = 0; r < reps; ++r) {
            float low_sum = 0.0f, high_sum = 0.0f;
            int low_count = 0, high_count = 0;
            for (int64_t d = r * dim_group_size; d < head_dim && d < (r + 1) * dim_group_size; ++d) {
                float v = load_elem(queries, dtype, base + d);
                int sign = v >= 0.0f;
                int m = sign ? (v > pos) : (v < neg);
                if (m) { high_sum = high_sum + fabsf(v); ++high_count; }
                else { low_sum = low_sum + fabsf(v); ++low_count; }
            }
            bucket_means(low_sum, low_count, high_sum, high_count,
                         &q_low[row * reps + r], &q_delta[row * reps + r]);
        }
    }
    return OK;
}

/* ------------------------------------------------------------------------ */
/* Popcount scoring.  popkv_ext.cu:757-876 / :502-515 (head_dim 128, fp16)  */
/* and :517-675 / :145-230 (other head dims, fp32).                          */
/* ------------------------------------------------------------------------ */

static int popc32(uint32_t x) { return __builtin_popcount(x); }

float oracle_score_scale(int64_t head_dim) {
    float root = sqrtf((float)head_dim);
    return 1.0f / root;
}

/* Score one (query row, key row) pair; returns the fp32 value before scaling. */
static float score_pair(const int32_t* qs, const int32_t* qm, const float* ql, const float* qd,
                        const int32_t* ks, const int32_t* km, const uint16_t* kl,
                        const uint16_t* kd, int64_t head_dim, int64_t dim_group_size,
                        int64_t reps) {
    float total = 0.0f;
    for (int64_t r = 0; r < reps; ++r) {
        const int64_t start = r * dim_group_size;
        const int64_t end = start + dim_group_size < head_dim ? start + dim_group_size : head_dim;
        int c_sign = 0, c_q = 0, c_k = 0, c_qk = 0;
        for (int64_t w = start / 32; w <= (end - 1) / 32; ++w) {
            const int64_t ws = w * 32;
            const int begin = (int)((start > ws ? start : ws) - ws);
            const int finish = (int)((end < ws + 32 ? end : ws + 32) - ws);
            const int width = finish - begin;
            const uint32_t mask = width == 32 ? 0xFFFFFFFFu : (((1u << width) - 1u) << begin);
            const uint32_t qmm = (uint32_t)qm[w] & mask;
            const uint32_t kmm = (uint32_t)km[w] & mask;
            const uint32_t match = ~((uint32_t)qs[w] ^ (uint32_t)ks[w]) & mask;
            const uint32_t both = qmm & kmm;
            c_sign += 2 * popc32(match) - popc32(mask);
            c_q += 2 * popc32(match & qmm) - popc32(qmm);
            c_k += 2 * popc32(match & kmm) - popc32(kmm);
            c_qk += 2 * popc32(match & both) - popc32(both);
        }
        const float qlr = ql[r], dqr = qd[r];
        const float klr = oracle_half_to_float(kl[r]);
        const float dkr = oracle_half_to_float(kd[r]);
        const float t1 = qlr * klr;
        const float t2 = dqr * klr;
        const float t3 = qlr * dkr;
        const float t4 = (dqr * dkr) * (float)c_qk;
        const float chain = fmaf(t1, (float)c_sign, fmaf(t2, (float)c_q, fmaf(t3, (float)c_k, t4)));
        total = total + chain;
    }
    return total;
}

int oracle_score(const int32_t* q_sign, const int32_t* q_mag, const float* q_low,
                 const float* q_delta, int64_t batch, int64_t q_heads,
                 const int32_t* k_sign, const int32_t* k_mag, const uint16_t* k_low,
                 const uint16_t* k_delta, int64_t kv_heads, int64_t capacity,
                 int64_t head_dim, int64_t dim_group_size, const int64_t* head_to_kv,
                 int64_t tokens, float* out_f32, uint16_t* out_f16) {
    if (batch < 0 || q_heads <= 0 || kv_heads <= 0 || head_dim <= 0 || tokens < 0 ||
        tokens > capacity ||
        (dim_group_size != 16 && dim_group_size != 32 && dim_group_size != 64))
        return ERR_ARG;
    const int64_t words = (head_dim + 31) / 32;
    const int64_t reps = (head_dim + dim_group_size - 1) / dim_group_size;
    const float scale = oracle_score_scale(head_dim);
    for (int64_t h = 0; h < q_heads; ++h)
        if (head_to_kv[h] < 0 || head_to_kv[h] >= kv_heads) return ERR_ARG;
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t b = 0; b < batch; ++b) {
        for (int64_t h = 0; h < q_heads; ++h) {
            const int64_t row = b * q_heads + h;
            const int64_t kvh = head_to_kv[h];
            for (int64_t t = 0; t < tokens; ++t) {
                const int64_t key_row = kvh * capacity + t;
                float total = score_pair(q_sign + row * words, q_mag + row * words,
                                         q_low + row * reps, q_delta + row * reps,
                                         k_sign + key_row * words, k_mag + key_row * words,
                                         k_low + key_row * reps, k_delta + key_row * reps,
                                         head_dim, dim_group_size, reps);
                float scaled = total * scale;
                if (out_f32) out_f32[row * tokens + t] = scaled;
                if (out_f16) out_f16[row * tokens + t] = oracle_float_to_half(scaled);
            }
        }
    }
    return OK;
}

/* ------------------------------------------------------------------------ */
/* Top-k with a deterministic tie-break.  Replaces                           */
/*   torch.topk(scores, k, dim=-1, sorted=False).indices  (popkv.py:1094-1098) */
/* whose order among equal scores is unspecified.  Contract: a score ranks   */
/* higher when its value is larger; equal values (+0 and -0 are equal) rank  */
/* by lower token index; the k best tokens are returned in ascending index   */
/* order.  NaN ranks above every number, as in torch.topk.                   */
/* ------------------------------------------------------------------------ */

/* Order-preserving 16-bit key of an fp16 score (larger key = larger score). */
uint32_t oracle_key16(uint16_t h) {
    if ((h & 0x7FFFu) == 0) h = 0;                       /* -0 == +0 */
    if ((h & 0x7C00u) == 0x7C00u && (h & 0x3FFu)) return 0xFFFFu;  /* NaN on top */
    return (h & 0x8000u) ? (uint32_t)(~h & 0xFFFFu) : (uint32_t)(h | 0x8000u);
}

uint32_t oracle_key32(float f) {
    uint32_t u = float_to_bits(f);
    if ((u & 0x7FFFFFFFu) == 0) u = 0;
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return 0xFFFFFFFFu;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

typedef struct { uint32_t key; int64_t index; } rank_item;

static int rank_cmp(const void* a, const void* b) {
    const rank_item* x = (const rank_item*)a;
    const rank_item* y = (const rank_item*)b;
    if (x->key != y->key) return x->key > y->key ? -1 : 1;
    return x->index < y->index ? -1 : (x->index > y->index ? 1 : 0);
}

static int index_cmp(const void* a, const void* b) {
    int64_t x = *(const int64_t*)a, y = *(const int64_t*)b;
    return x < y ? -1 : (x > y ? 1 : 0);
}

/* scores: fp16 bits (is_f32 == 0) or fp32 (is_f32 == 1), row r at scores + r*row_stride. */
int oracle_topk(const void* scores, int is_f32, int64_t rows, int64_t tokens,
                int64_t row_stride, int64_t k, int64_t* out, int64_t out_stride) {
    if (rows < 0 || tokens < 0 || k < 0 || k > tokens) return ERR_ARG;
#pragma omp parallel for schedule(dynamic)
    for (int64_t r = 0; r < rows; ++r) {
        rank_item* items = (rank_item*)malloc(sizeof(rank_item) * (size_t)(tokens ? tokens : 1));
        for (int64_t t = 0; t < tokens; ++t) {
            uint32_t key = is_f32 ? oracle_key32(((const float*)scores)[r * row_stride + t])
                                  : oracle_key16(((const uint16_t*)scores)[r * row_stride + t]);
            items[t].key = key;
            items[t].index = t;
        }
        qsort(items, (size_t)tokens, sizeof(rank_item), rank_cmp);
        int64_t* dst = out + r * out_stride;
        for (int64_t i = 0; i < k; ++i) dst[i] = items[i].index;
        qsort(dst, (size_t)k, sizeof(int64_t), index_cmp);
        free(items);
    }
    return OK;
}

/* ------------------------------------------------------------------------ */
/* Split indexed attention: partial states and log-sum-exp merge.           */
/* sparse_kernels.py:237-294 (partials) and :297-318 (merge).                */
/*                                                                          */
/* Selected slot j of query head h reads token idx = indices[h, j]: the     */
/* current token when idx == prefix_tokens, else prefix row                  */
/* min(idx, prefix_tokens - 1) (sparse_kernels.py:267-274); slot j is masked */
/* when valid is given and valid[h, j] == 0.  Split s covers slots           */
/* [s*split, (s+1)*split).  State layout per (h, s): [max, sum, acc[D]] with */
/* max = max logit, sum = sum exp(logit - max), acc = sum exp(logit - max)*v. */
/* Arithmetic is double precision: this is the exact-math checker.  A split  */
/* with no valid slot has max = -inf, sum = 0, acc = 0.                      */
/* ------------------------------------------------------------------------ */

int oracle_attn_partial(const void* queries, int q_dtype, int64_t q_heads, int64_t head_dim,
                        const void* prefix_keys, const void* prefix_values, int kv_dtype,
                        int64_t prefix_tokens, int64_t k_head_stride, int64_t k_token_stride,
                        int64_t v_head_stride, int64_t v_token_stride,
                        const void* current_keys, const void* current_values,
                        const int64_t* indices, int64_t selected, const uint8_t* valid,
                        const int64_t* head_to_kv, int64_t split_tokens, double* partials) {
    if (q_heads <= 0 || head_dim <= 0 || prefix_tokens <= 0 || selected <= 0 || split_tokens <= 0)
        return ERR_ARG;
    const int64_t splits = (selected + split_tokens - 1) / split_tokens;
    const int64_t state = head_dim + 2;
    const double scale = 1.0 / sqrt((double)head_dim);
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t h = 0; h < q_heads; ++h) {
        for (int64_t s = 0; s < splits; ++s) {
            const int64_t kvh = head_to_kv[h];
            double* out = partials + (h * splits + s) * state;
            double* logits = (double*)malloc(sizeof(double) * (size_t)split_tokens);
            int64_t* rows = (int64_t*)malloc(sizeof(int64_t) * (size_t)split_tokens);
            double mx = -INFINITY;
            for (int64_t j = 0; j < split_tokens; ++j) {
                const int64_t slot = s * split_tokens + j;
                logits[j] = -INFINITY;
                rows[j] = -2;
                if (slot >= selected) continue;
                if (valid && !valid[h * selected + slot]) continue;
                int64_t idx = indices[h * selected + slot];
                double dot = 0.0;
                if (idx == prefix_tokens) {
                    rows[j] = -1;
                    for (int64_t d = 0; d < head_dim; ++d)
                        dot += (double)load_elem(queries, q_dtype, h * head_dim + d) *
                               (double)load_elem(current_keys, kv_dtype, kvh * head_dim + d);
                } else {
                    if (idx > prefix_tokens - 1) idx = prefix_tokens - 1;
                    if (idx < 0) idx = 0;
                    rows[j] = idx;
                    for (int64_t d = 0; d < head_dim; ++d)
                        dot += (double)load_elem(queries, q_dtype, h * head_dim + d) *
                               (double)load_elem(prefix_keys, kv_dtype,
                                                 kvh * k_head_stride + idx * k_token_stride + d);
                }
                logits[j] = dot * scale;
                if (logits[j] > mx) mx = logits[j];
            }
            double sum = 0.0;
            for (int64_t d = 0; d < head_dim; ++d) out[2 + d] = 0.0;
            if (mx != -INFINITY) {
                for (int64_t j = 0; j < split_tokens; ++j) {
                    if (rows[j] == -2) continue;
                    const double p = exp(logits[j] - mx);
                    sum += p;
                    for (int64_t d = 0; d < head_dim; ++d) {
                        double v = rows[j] == -1
                            ? (double)load_elem(current_values, kv_dtype, kvh * head_dim + d)
                            : (double)load_elem(prefix_values, kv_dtype,
                                                kvh * v_head_stride + rows[j] * v_token_stride + d);
                        out[2 + d] += p * v;
                    }
                }
            }
            out[0] = mx;
            out[1] = sum;
            free(logits);
            free(rows);
        }
    }
    return OK;
}

int oracle_attn_merge(const double* partials, int64_t q_heads, int64_t splits,
                      int64_t head_dim, double* out) {
    if (q_heads <= 0 || splits <= 0 || head_dim <= 0) return ERR_ARG;
    const int64_t state = head_dim + 2;
    for (int64_t h = 0; h < q_heads; ++h) {
        const double* p = partials + h * splits * state;
        double gm = -INFINITY;
        for (int64_t s = 0; s < splits; ++s)
            if (p[s * state] > gm) gm = p[s * state];
        double den = 0.0;
        for (int64_t s = 0; s < splits; ++s)
            den += p[s * state + 1] * exp(p[s * state] - gm);
        for (int64_t d = 0; d < head_dim; ++d) {
            double num = 0.0;
            for (int64_t s = 0; s < splits; ++s)
                num += p[s * state + 2 + d] * exp(p[s * state] - gm);
            out[h * head_dim + d] = num / den;
        }
    }
    return OK;
}

int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
