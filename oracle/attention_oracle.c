/*
 * CPU oracle for the InferLab attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This file restates, in plain C, the reference's
 * scalar CPU attention kernel and the worker's paged KV-cache gather so that
 * tests and the benchmark's CPU baseline have something to check the CUDA
 * library against. Nothing in the product (inferlab_b200/) links, loads or
 * calls it; the product fails loudly when its CUDA library is missing.
 *
 * Every function names the reference lines it follows (paths are relative to
 * the reference project root). The floating-point operation order of the
 * attention loops is kept identical to the reference so that, compiled with
 * the same flags (-O2, no FMA contraction), the oracle is bit-identical to a
 * build of kernels/attention_cpu.cpp; tests/test_oracle.py checks exactly that
 * against oracle/_ref/libref.so and against the reference's retained golden
 * vectors.
 */
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stddef.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_FP32 0u
#define ORACLE_FP16 1u
#define ORACLE_BF16 2u

#define ORACLE_MATERIALIZED 0u
#define ORACLE_ONLINE_TILED 1u

static void set_error(char* error, size_t capacity, const char* message) {
    if (error == NULL || capacity == 0) {
        return;
    }
    size_t count = strlen(message);
    if (count > capacity - 1) {
        count = capacity - 1;
    }
    memcpy(error, message, count);
    error[count] = '\0';
}

static uint32_t float_bits(float value) {
    uint32_t bits;
    memcpy(&bits, &value, sizeof bits);
    return bits;
}

static float bits_float(uint32_t bits) {
    float value;
    memcpy(&value, &bits, sizeof value);
    return value;
}

/*
 * IEEE binary32 -> binary16, round to nearest even, subnormals kept, overflow
 * to signed infinity, NaN to a quiet NaN.
 * Follows kernels/attention_cpu.cpp:15-67 (float_to_half_bits).
 */
uint16_t oracle_float_to_half_bits(float value) {
    const uint32_t bits = float_bits(value);
    const uint32_t sign = (bits >> 16) & 0x8000u;
    const uint32_t biased = (bits >> 23) & 0xFFu;
    const uint32_t fraction = bits & 0x7FFFFFu;
    if (biased == 0xFFu) {
        return (uint16_t)(sign | 0x7C00u | (fraction ? 0x0200u : 0u));
    }
    const int exponent = (int)biased - 127 + 15;
    if (exponent >= 31) {
        return (uint16_t)(sign | 0x7C00u);
    }
    if (exponent <= 0) {
        if (exponent < -10) {
            return (uint16_t)sign;
        }
        /* Subnormal half: shift the full significand right, round half even. */
        const uint32_t significand = fraction | 0x800000u;
        const int shift = 14 - exponent;
        uint32_t result = significand >> shift;
        const uint32_t dropped = significand & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1);
        if (dropped > half || (dropped == half && (result & 1u))) {
            result += 1u;
        }
        return (uint16_t)(sign | result);
    }
    /* Normal half: keep 10 fraction bits, round half even; a carry out of the
     * fraction bumps the exponent and may overflow to infinity. */
    uint32_t result = ((uint32_t)exponent << 10) | (fraction >> 13);
    const uint32_t dropped = fraction & 0x1FFFu;
    if (dropped > 0x1000u || (dropped == 0x1000u && (result & 1u))) {
        result += 1u;
    }
    if ((result >> 10) >= 31u) {
        return (uint16_t)(sign | 0x7C00u);
    }
    return (uint16_t)(sign | result);
}

/* binary16 -> binary32 as the reference does it (kernels/attention_cpu.cpp:69-97).
 * Its subnormal branch builds the exponent as 127 - 15 - shift (:86-88), one
 * below the exact 127 - 14 - shift, so fp16 subnormals come back at half
 * their value; restated as is, because round_attention_value depends on it
 * and the parity target is the reference's behaviour. Normal numbers, zero
 * and infinities are exact. */
float oracle_half_bits_to_float(uint16_t half) {
    const uint32_t sign = ((uint32_t)half & 0x8000u) << 16;
    const uint32_t exponent = ((uint32_t)half >> 10) & 0x1Fu;
    uint32_t fraction = (uint32_t)half & 0x3FFu;
    if (exponent == 0) {
        if (fraction == 0) {
            return bits_float(sign);
        }
        int shift = 0;
        while ((fraction & 0x400u) == 0) {
            fraction <<= 1;
            shift += 1;
        }
        fraction &= 0x3FFu;
        return bits_float(sign | ((uint32_t)(127 - 15 - shift) << 23) | (fraction << 13));
    }
    if (exponent == 0x1Fu) {
        return bits_float(sign | 0x7F800000u | (fraction << 13));
    }
    return bits_float(sign | ((exponent + 127u - 15u) << 23) | (fraction << 13));
}

/* binary32 -> bfloat16 bits by adding 0x7FFF plus the kept LSB (round half
 * even on finite values). Follows kernels/attention_cpu.cpp:412-416. */
uint16_t oracle_float_to_bf16_bits(float value) {
    const uint32_t bits = float_bits(value);
    return (uint16_t)((bits + 0x7FFFu + ((bits >> 16) & 1u)) >> 16);
}

/* Exact binary16 -> binary32 (IEEE), for values that are stored as real fp16
 * in the device pool: a subnormal h is h.fraction * 2^-24. */
float oracle_half_bits_to_float_ieee(uint16_t half) {
    const uint32_t exponent = ((uint32_t)half >> 10) & 0x1Fu;
    const uint32_t fraction = (uint32_t)half & 0x3FFu;
    if (exponent == 0) {
        const float magnitude = (float)fraction * 5.9604644775390625e-08f; /* 2^-24 */
        return (half & 0x8000u) ? -magnitude : magnitude;
    }
    return oracle_half_bits_to_float(half);
}

float oracle_bf16_bits_to_float(uint16_t bits) {
    return bits_float((uint32_t)bits << 16);
}

/* Storage-precision simulation. Follows kernels/attention_cpu.cpp:405-417. */
float oracle_round_value(float value, uint32_t precision) {
    if (precision == ORACLE_FP32) {
        return value;
    }
    if (precision == ORACLE_FP16) {
        return oracle_half_bits_to_float(oracle_float_to_half_bits(value));
    }
    return oracle_bf16_bits_to_float(oracle_float_to_bf16_bits(value));
}

/* Causal bound. Follows kernels/attention_cpu.cpp:113-123. */
static size_t legal_sources(size_t query, size_t kv_tokens, size_t start, int causal) {
    if (!causal) {
        return kv_tokens;
    }
    const size_t bound = start + query + 1;
    return bound < kv_tokens ? bound : kv_tokens;
}

static int mul_overflows(uint64_t a, uint64_t b) {
    return a != 0 && b > UINT64_MAX / a;
}

/*
 * Analytic statistics; the eight u64 fields in AttentionStats order
 * (kernels/attention_cpu.h:26-35). Follows kernels/attention_cpu.cpp:140-213.
 * Returns 0, or -1 when a product overflows u64.
 */
int oracle_attention_stats(size_t q_tokens, size_t kv_tokens, size_t heads, size_t head_dim,
                           size_t start, uint32_t algorithm, uint32_t precision, size_t tile,
                           int causal, uint64_t* stats) {
    uint64_t legal_pairs = 0;
    uint64_t key_tiles = 0;
    for (size_t query = 0; query < q_tokens; ++query) {
        const uint64_t legal = legal_sources(query, kv_tokens, start, causal);
        if (mul_overflows(legal, heads)) return -1;
        legal_pairs += legal * heads;
        const uint64_t tiles = (legal + tile - 1) / tile;
        if (mul_overflows(tiles, heads)) return -1;
        key_tiles += tiles * heads;
    }
    if (mul_overflows(q_tokens, kv_tokens) || mul_overflows((uint64_t)q_tokens * kv_tokens, heads))
        return -1;
    const uint64_t all_pairs = (uint64_t)q_tokens * kv_tokens * heads;
    const uint64_t scalar = precision == ORACLE_FP32 ? 4u : 2u;
    const uint64_t query_bytes = (uint64_t)q_tokens * heads * head_dim * scalar;
    const uint64_t kv_bytes = (uint64_t)kv_tokens * heads * head_dim * scalar;
    const uint64_t output_bytes = (uint64_t)q_tokens * heads * head_dim * 4u;
    memset(stats, 0, 8 * sizeof(uint64_t));
    stats[0] = legal_pairs;
    stats[1] = all_pairs - legal_pairs;
    stats[7] = key_tiles;
    if (algorithm == ORACLE_MATERIALIZED) {
        const uint64_t score_bytes = all_pairs * 4u;
        stats[2] = score_bytes;
        stats[3] = score_bytes;
        stats[4] = query_bytes + kv_bytes * 2u + score_bytes * 2u;
        stats[5] = score_bytes * 2u + output_bytes;
    } else {
        stats[2] = (uint64_t)tile * 4u;
        stats[3] = stats[2] + (uint64_t)head_dim * 4u;
        const uint64_t query_tiles = (q_tokens + tile - 1) / tile;
        stats[4] = query_bytes + query_tiles * kv_bytes * 2u;
        stats[5] = output_bytes;
    }
    stats[6] = stats[4] + stats[5];
    return 0;
}

/* Three-pass attention over a full score buffer.
 * Follows kernels/attention_cpu.cpp:215-304. */
static int materialized(const float* q, const float* k, const float* v, size_t tq, size_t tkv,
                        size_t heads, size_t d, size_t start, int causal, float* out) {
    const size_t rows = tq * heads;
    float* scores = (float*)malloc(rows * tkv * sizeof(float));
    if (scores == NULL) return -1;
    for (size_t i = 0; i < rows * tkv; ++i) scores[i] = -INFINITY;
    const float scale = 1.0f / sqrtf((float)d);
    const size_t width = heads * d;
    for (size_t query = 0; query < tq; ++query) {
        const size_t sources = legal_sources(query, tkv, start, causal);
        for (size_t head = 0; head < heads; ++head) {
            const size_t row = query * heads + head;
            for (size_t source = 0; source < sources; ++source) {
                float score = 0.0f;
                for (size_t c = 0; c < d; ++c) {
                    score += q[query * width + head * d + c] * k[source * width + head * d + c];
                }
                scores[row * tkv + source] = score * scale;
            }
        }
    }
    for (size_t query = 0; query < tq; ++query) {
        const size_t sources = legal_sources(query, tkv, start, causal);
        for (size_t head = 0; head < heads; ++head) {
            float* row = scores + (query * heads + head) * tkv;
            float maximum = -INFINITY;
            for (size_t s = 0; s < sources; ++s) maximum = maximum < row[s] ? row[s] : maximum;
            float denominator = 0.0f;
            for (size_t s = 0; s < sources; ++s) {
                row[s] = expf(row[s] - maximum);
                denominator += row[s];
            }
            for (size_t s = 0; s < sources; ++s) row[s] /= denominator;
        }
    }
    for (size_t query = 0; query < tq; ++query) {
        const size_t sources = legal_sources(query, tkv, start, causal);
        for (size_t head = 0; head < heads; ++head) {
            const float* row = scores + (query * heads + head) * tkv;
            for (size_t c = 0; c < d; ++c) {
                float accumulated = 0.0f;
                for (size_t s = 0; s < sources; ++s) {
                    accumulated += row[s] * v[s * width + head * d + c];
                }
                out[query * width + head * d + c] = accumulated;
            }
        }
    }
    free(scores);
    return 0;
}

/* Online softmax over key tiles of `tile` tokens.
 * Follows kernels/attention_cpu.cpp:306-401. Returns -2 when a normalizer is
 * not finite or not positive (the reference's ":391" error). */
static int online_tiled(const float* q, const float* k, const float* v, size_t tq, size_t tkv,
                        size_t heads, size_t d, size_t start, size_t tile, int causal,
                        float* out) {
    const float scale = 1.0f / sqrtf((float)d);
    const size_t width = heads * d;
    float* tile_scores = (float*)malloc(tile * sizeof(float));
    float* numerator = (float*)malloc(d * sizeof(float));
    if (tile_scores == NULL || numerator == NULL) {
        free(tile_scores);
        free(numerator);
        return -1;
    }
    int status = 0;
    for (size_t query = 0; query < tq && status == 0; ++query) {
        const size_t sources = legal_sources(query, tkv, start, causal);
        for (size_t head = 0; head < heads; ++head) {
            for (size_t c = 0; c < d; ++c) numerator[c] = 0.0f;
            float running_max = -INFINITY;
            float running_den = 0.0f;
            for (size_t begin = 0; begin < sources; begin += tile) {
                const size_t end = begin + tile < sources ? begin + tile : sources;
                float tile_max = -INFINITY;
                for (size_t i = 0; i < end - begin; ++i) {
                    const size_t s = begin + i;
                    float score = 0.0f;
                    for (size_t c = 0; c < d; ++c) {
                        score += q[query * width + head * d + c] * k[s * width + head * d + c];
                    }
                    tile_scores[i] = score * scale;
                    tile_max = tile_max < tile_scores[i] ? tile_scores[i] : tile_max;
                }
                const float new_max = running_max < tile_max ? tile_max : running_max;
                const float previous = isinf(running_max) ? 0.0f : expf(running_max - new_max);
                running_den *= previous;
                for (size_t c = 0; c < d; ++c) numerator[c] *= previous;
                for (size_t i = 0; i < end - begin; ++i) {
                    const size_t s = begin + i;
                    const float p = expf(tile_scores[i] - new_max);
                    running_den += p;
                    for (size_t c = 0; c < d; ++c) numerator[c] += p * v[s * width + head * d + c];
                }
                running_max = new_max;
            }
            if (!isfinite(running_den) || running_den <= 0.0f) {
                status = -2;
                break;
            }
            for (size_t c = 0; c < d; ++c) {
                out[query * width + head * d + c] = numerator[c] / running_den;
            }
        }
    }
    free(tile_scores);
    free(numerator);
    return status;
}

static int size_product(size_t a, size_t b, size_t* out) {
    if (a != 0 && b > SIZE_MAX / a) return -1;
    *out = a * b;
    return 0;
}

/*
 * The C entry inferlab_attention_forward restated: validation order and
 * messages (worker/cpp/inferlab_runtime.cpp:2561-2619 and the config mapping
 * at :446-490), then attention_forward (kernels/attention_cpu.cpp:419-502):
 * pointer and shape checks, storage rounding with the finite check, zero
 * fill, algorithm dispatch, statistics.
 * config = {algorithm, precision, tile_tokens, causal} as in
 * InferlabAttentionConfig (worker/cpp/inferlab_runtime.h:67-72); stats is the
 * eight u64 fields of InferlabAttentionStats (:74-83).
 * Returns 0, or -1 with the reference's error text.
 */
int oracle_attention_forward(const float* q, const float* k, const float* v, size_t tq,
                             size_t tkv, size_t heads, size_t d, size_t start,
                             const uint32_t* config, float* out, size_t out_capacity,
                             uint64_t* stats, char* error, size_t error_capacity) {
    if (error != NULL && error_capacity > 0) error[0] = '\0';
    if (config == NULL || stats == NULL) {
        set_error(error, error_capacity, "attention config or stats pointer is null");
        return -1;
    }
    size_t nq = 0;
    size_t nkv = 0;
    size_t tmp = 0;
    if (size_product(tq, heads, &tmp) != 0 || size_product(tmp, d, &nq) != 0) {
        set_error(error, error_capacity, "attention shape product overflows");
        return -1;
    }
    if (out == NULL || out_capacity < nq) {
        set_error(error, error_capacity, "attention output buffer is too small");
        return -1;
    }
    const uint32_t algorithm = config[0];
    const uint32_t precision = config[1];
    const size_t tile = config[2];
    const int causal = config[3] != 0;
    if (tile == 0 || tile > 4096) {
        set_error(error, error_capacity, "attention tile_tokens must be between 1 and 4096");
        return -1;
    }
    if (algorithm > 1u) {
        set_error(error, error_capacity,
                  "attention algorithm must be 0 (materialized) or 1 (online tiled)");
        return -1;
    }
    if (precision > 2u) {
        set_error(error, error_capacity,
                  "attention precision must be 0 (FP32), 1 (FP16), or 2 (BF16)");
        return -1;
    }
    if (q == NULL || k == NULL || v == NULL) {
        set_error(error, error_capacity, "attention input or output pointer is null");
        return -1;
    }
    if (tq == 0 || tkv == 0 || heads == 0 || d == 0) {
        set_error(error, error_capacity, "attention dimensions must be positive");
        return -1;
    }
    if (causal && (start >= tkv || tq > tkv - start)) {
        set_error(error, error_capacity, "causal query positions exceed the KV sequence");
        return -1;
    }
    if (size_product(tkv, heads, &tmp) != 0 || size_product(tmp, d, &nkv) != 0) {
        set_error(error, error_capacity, "attention shape product overflows");
        return -1;
    }
    float* pq = (float*)malloc(nq * sizeof(float));
    float* pk = (float*)malloc(nkv * sizeof(float));
    float* pv = (float*)malloc(nkv * sizeof(float));
    int status = 0;
    if (pq == NULL || pk == NULL || pv == NULL) {
        status = -4;
        goto done;
    }
    /* prepare(): finite check on the raw value, then rounding
     * (kernels/attention_cpu.cpp:125-138), queries, keys, values in order. */
    for (size_t i = 0; i < nq; ++i) {
        if (!isfinite(q[i])) { status = -3; goto done; }
        pq[i] = oracle_round_value(q[i], precision);
    }
    for (size_t i = 0; i < nkv; ++i) {
        if (!isfinite(k[i])) { status = -3; goto done; }
        pk[i] = oracle_round_value(k[i], precision);
    }
    for (size_t i = 0; i < nkv; ++i) {
        if (!isfinite(v[i])) { status = -3; goto done; }
        pv[i] = oracle_round_value(v[i], precision);
    }
    for (size_t i = 0; i < nq; ++i) out[i] = 0.0f;
    if (algorithm == ORACLE_MATERIALIZED) {
        status = materialized(pq, pk, pv, tq, tkv, heads, d, start, causal, out) == 0 ? 0 : -4;
    } else {
        status = online_tiled(pq, pk, pv, tq, tkv, heads, d, start, tile, causal, out);
        if (status == -1) status = -4;
    }
    if (status == 0 &&
        oracle_attention_stats(tq, tkv, heads, d, start, algorithm, precision, tile, causal,
                               stats) != 0) {
        status = -5;
    }
done:
    if (status == -2) {
        set_error(error, error_capacity, "online attention normalizer is invalid");
    } else if (status == -3) {
        set_error(error, error_capacity, "attention input must be finite");
    } else if (status == -4) {
        set_error(error, error_capacity, "oracle allocation failed");
    } else if (status == -5) {
        set_error(error, error_capacity, "attention metric product overflows");
    }
    free(pq);
    free(pk);
    free(pv);
    return status == 0 ? 0 : -1;
}

/* ---------------------------------------------------------------------------
 * Paged KV cache.
 *
 * Arena layout of the device pool (one arena for keys, one for values):
 *   [num_blocks][kv_heads][block_tokens][head_dim], element type dtype
 *   (0 fp32, 1 f16 bits, 2 bf16 bits).
 * Block-table semantics follow worker/cpp/inferlab_runtime.cpp:769-803 and
 * docs/rfcs/0014-paged-kv-cache-prefix-ownership.md:149:
 *   logical block = pos / block_tokens, slot = pos % block_tokens,
 *   physical block = table[logical block].
 * ------------------------------------------------------------------------- */

static float arena_value(const void* arena, uint32_t dtype, size_t index) {
    if (dtype == ORACLE_FP32) return ((const float*)arena)[index];
    const uint16_t bits = ((const uint16_t*)arena)[index];
    return dtype == ORACLE_FP16 ? oracle_half_bits_to_float_ieee(bits)
                                : oracle_bf16_bits_to_float(bits);
}

/*
 * Gather `tokens` rows of one sequence into contiguous [tokens][kv_heads][head_dim]
 * fp32 (16-bit stored values widened exactly, IEEE, including fp16 subnormals). Restates PagedKvPool::materialize
 * (worker/cpp/inferlab_runtime.cpp:769-803): the table length must equal
 * ceil(tokens / block_tokens) (:776-780), ids must be in range (:931-936).
 */
int oracle_materialize(const void* arena, uint32_t dtype, size_t num_blocks, size_t kv_heads,
                       size_t block_tokens, size_t head_dim, const int32_t* table,
                       size_t table_len, size_t tokens, float* out) {
    const size_t expected = (tokens + block_tokens - 1) / block_tokens;
    if (table_len != expected) return -1;
    for (size_t t = 0; t < tokens; ++t) {
        const int32_t block = table[t / block_tokens];
        if (block < 0 || (size_t)block >= num_blocks) return -2;
        const size_t slot = t % block_tokens;
        for (size_t h = 0; h < kv_heads; ++h) {
            const size_t src = (((size_t)block * kv_heads + h) * block_tokens + slot) * head_dim;
            float* dst = out + (t * kv_heads + h) * head_dim;
            for (size_t c = 0; c < head_dim; ++c) dst[c] = arena_value(arena, dtype, src + c);
        }
    }
    return 0;
}

/*
 * Reference attention for one segment of a paged batch: query tokens at
 * positions [start, start + q_tokens) of a sequence whose KV is
 * [0, start + q_tokens), causal. GQA maps q-head h to kv-head
 * h / (q_heads / kv_heads); the reference has no GQA, so each q-head is one
 * attention_forward call with heads = 1 on that kv-head's slice
 * (worker/cpp/inferlab_runtime.cpp:1458-1470 is the decode call shape).
 * q: [q_tokens][q_heads][head_dim] fp32; out likewise.
 */
static int segment_attention(const void* k_arena, const void* v_arena, uint32_t dtype,
                             size_t num_blocks, size_t kv_heads, size_t block_tokens,
                             size_t head_dim, size_t q_heads, const int32_t* table,
                             size_t start, size_t q_tokens, const float* q, uint32_t algorithm,
                             size_t tile, float* out, float* kbuf, float* vbuf, float* hk,
                             float* hv, float* hq, float* ho) {
    const size_t tokens = start + q_tokens;
    const size_t table_len = (tokens + block_tokens - 1) / block_tokens;
    if (oracle_materialize(k_arena, dtype, num_blocks, kv_heads, block_tokens, head_dim, table,
                           table_len, tokens, kbuf) != 0)
        return -1;
    if (oracle_materialize(v_arena, dtype, num_blocks, kv_heads, block_tokens, head_dim, table,
                           table_len, tokens, vbuf) != 0)
        return -1;
    const size_t group = q_heads / kv_heads;
    for (size_t h = 0; h < q_heads; ++h) {
        const size_t kvh = h / group;
        for (size_t t = 0; t < tokens; ++t) {
            memcpy(hk + t * head_dim, kbuf + (t * kv_heads + kvh) * head_dim, head_dim * 4);
            memcpy(hv + t * head_dim, vbuf + (t * kv_heads + kvh) * head_dim, head_dim * 4);
        }
        for (size_t t = 0; t < q_tokens; ++t) {
            memcpy(hq + t * head_dim, q + (t * q_heads + h) * head_dim, head_dim * 4);
        }
        const uint32_t config[4] = {algorithm, ORACLE_FP32, (uint32_t)tile, 1u};
        uint64_t stats[8];
        if (oracle_attention_forward(hq, hk, hv, q_tokens, tokens, 1, head_dim, start, config, ho,
                                     q_tokens * head_dim, stats, NULL, 0) != 0)
            return -1;
        for (size_t t = 0; t < q_tokens; ++t) {
            memcpy(out + (t * q_heads + h) * head_dim, ho + t * head_dim, head_dim * 4);
        }
    }
    return 0;
}

typedef struct {
    const void* k_arena;
    const void* v_arena;
    uint32_t dtype;
    size_t num_blocks, kv_heads, block_tokens, head_dim, q_heads;
    const int32_t* tables;
    size_t max_blocks, num_segments;
    const int64_t* starts;
    const int64_t* q_counts;
    const int64_t* q_offsets;
    const float* q;
    uint32_t algorithm;
    size_t tile;
    float* out;
    atomic_long next;
    atomic_int failures;
} paged_job;

static void* paged_worker(void* arg) {
    paged_job* job = (paged_job*)arg;
    for (;;) {
        const long s = atomic_fetch_add(&job->next, 1);
        if (s >= (long)job->num_segments) break;
        const size_t tokens = (size_t)(job->starts[s] + job->q_counts[s]);
        const size_t nq = (size_t)job->q_counts[s];
        const size_t hd = job->head_dim;
        float* kbuf = (float*)malloc(tokens * job->kv_heads * hd * 4);
        float* vbuf = (float*)malloc(tokens * job->kv_heads * hd * 4);
        float* hk = (float*)malloc(tokens * hd * 4);
        float* hv = (float*)malloc(tokens * hd * 4);
        float* hq = (float*)malloc(nq * hd * 4);
        float* ho = (float*)malloc(nq * hd * 4);
        if (!kbuf || !vbuf || !hk || !hv || !hq || !ho ||
            (tokens + job->block_tokens - 1) / job->block_tokens > job->max_blocks ||
            segment_attention(job->k_arena, job->v_arena, job->dtype, job->num_blocks,
                              job->kv_heads, job->block_tokens, hd, job->q_heads,
                              job->tables + (size_t)s * job->max_blocks, (size_t)job->starts[s],
                              nq, job->q + (size_t)job->q_offsets[s] * job->q_heads * hd,
                              job->algorithm, job->tile,
                              job->out + (size_t)job->q_offsets[s] * job->q_heads * hd, kbuf,
                              vbuf, hk, hv, hq, ho) != 0) {
            atomic_fetch_add(&job->failures, 1);
        }
        free(kbuf);
        free(vbuf);
        free(hk);
        free(hv);
        free(hq);
        free(ho);
    }
    return NULL;
}

/*
 * Paged batch: `num_segments` segments; segment s has q_counts[s] query
 * tokens starting at position starts[s] (decode: q_counts = 1,
 * starts = context - 1). Its queries are rows [q_offsets[s], +q_counts[s])
 * of q ([total_q][q_heads][head_dim]); its block table is row s of
 * tables ([num_segments][max_blocks]). Queries are fp32 and already in the
 * pool precision (the caller rounds them), so each call runs in Fp32 mode on
 * the widened stored K/V values. Segments are independent and are spread over
 * `threads` host threads (0 = one).
 */
int oracle_paged_attention(const void* k_arena, const void* v_arena, uint32_t dtype,
                           size_t num_blocks, size_t kv_heads, size_t block_tokens,
                           size_t head_dim, size_t q_heads, const int32_t* tables,
                           size_t max_blocks, size_t num_segments, const int64_t* starts,
                           const int64_t* q_counts, const int64_t* q_offsets, const float* q,
                           uint32_t algorithm, size_t tile, float* out, int threads) {
    if (kv_heads == 0 || q_heads % kv_heads != 0) return -1;
    paged_job job = {k_arena, v_arena, dtype, num_blocks, kv_heads, block_tokens, head_dim,
                     q_heads, tables, max_blocks, num_segments, starts, q_counts, q_offsets,
                     q, algorithm, tile, out, 0, 0};
    atomic_init(&job.next, 0);
    atomic_init(&job.failures, 0);
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    pthread_t workers[256];
    int started = 0;
    for (int i = 1; i < threads; ++i) {
        if (pthread_create(&workers[started], NULL, paged_worker, &job) == 0) started += 1;
    }
    paged_worker(&job);
    for (int i = 0; i < started; ++i) pthread_join(workers[i], NULL);
    return atomic_load(&job.failures) == 0 ? 0 : -1;
}

/*
 * Log-sum-exp merge of split-KV partials in fixed order. For each row r and
 * part i: m[i][r] (natural-log running max of the scaled scores), l[i][r]
 * (sum of exp(score - m)), o[i][r][d] (unnormalised sum of exp(score - m) * v).
 * out[r] = sum_i o_i e^(m_i - M) / sum_i l_i e^(m_i - M), M = max_i m_i.
 * Parts with l = 0 (no keys) contribute nothing. This is the combine step the
 * split-KV decode needs; the reference has no split-KV, so it is checked
 * against whole-context attention_forward.
 */
void oracle_lse_merge(size_t parts, size_t rows, size_t head_dim, const float* m, const float* l,
                      const float* o, float* out) {
    for (size_t r = 0; r < rows; ++r) {
        float maximum = -INFINITY;
        for (size_t i = 0; i < parts; ++i) {
            const float mi = m[i * rows + r];
            if (l[i * rows + r] > 0.0f && mi > maximum) maximum = mi;
        }
        double den = 0.0;
        for (size_t c = 0; c < head_dim; ++c) out[r * head_dim + c] = 0.0f;
        double* acc = (double*)calloc(head_dim, sizeof(double));
        for (size_t i = 0; i < parts; ++i) {
            if (!(l[i * rows + r] > 0.0f)) continue;
            const double w = exp((double)m[i * rows + r] - (double)maximum);
            den += w * l[i * rows + r];
            for (size_t c = 0; c < head_dim; ++c) acc[c] += w * o[(i * rows + r) * head_dim + c];
        }
        for (size_t c = 0; c < head_dim; ++c) out[r * head_dim + c] = (float)(acc[c] / den);
        free(acc);
    }
}
