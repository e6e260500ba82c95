// generic_attention.cuh - fp32 CUDA-core attention for any head_dim, any
// block size and either contiguous or paged K/V.
//
// One warp owns one (query token, q-head) row. It walks the legal key range
// (legal_sources, kernels/attention_cpu.cpp:113-123) in chunks of 32 * kTpl
// keys: each lane scores kTpl keys (full dot product in fp32), the chunk max
// updates the running max, the probabilities go to shared memory, and the lanes
// then sweep the head dimensions accumulating p * v with the running rescale
// (the online-softmax recurrence of kernels/attention_cpu.cpp:306-401, with
// 256-key tiles instead of tile_tokens). Accumulators live in shared memory so
// head_dim is only bounded by the shared-memory budget.
#pragma once

#include "common.cuh"

namespace ilb {

constexpr int kGenericWarps = 4;
constexpr int kGenericTpl = 8;  // keys per lane per chunk
constexpr int kGenericChunk = 32 * kGenericTpl;
constexpr unsigned kGenericMaxHeadDim = 4096;

inline std::size_t generic_smem_bytes(unsigned head_dim) {
    return static_cast<std::size_t>(kGenericWarps) * (2u * head_dim + kGenericChunk) * sizeof(float);
}

// Key/value access for the contiguous layout [tokens][heads][head_dim] fp32
// with storage rounding applied on load.
struct ContiguousKv {
    const float* keys;
    const float* values;
    std::uint32_t precision;
    std::uint32_t heads;
    std::uint32_t head_dim;

    struct Row {
        const float* ptr;
    };
    __device__ __forceinline__ Row key_row(int, long long token, std::uint32_t head) const {
        return Row{keys + (static_cast<std::size_t>(token) * heads + head) * head_dim};
    }
    __device__ __forceinline__ Row value_row(int, long long token, std::uint32_t head) const {
        return Row{values + (static_cast<std::size_t>(token) * heads + head) * head_dim};
    }
    __device__ __forceinline__ float load(const Row& row, std::uint32_t dim) const {
        return round_reference(row.ptr[dim], precision);
    }
    // Four consecutive dimensions (dim a multiple of 4, head_dim too).
    __device__ __forceinline__ float4 load4(const Row& row, std::uint32_t dim) const {
        const float4 x = *reinterpret_cast<const float4*>(row.ptr + dim);
        return make_float4(round_reference(x.x, precision), round_reference(x.y, precision),
                           round_reference(x.z, precision), round_reference(x.w, precision));
    }
};

// Key/value access through a block table into a pool arena
// [num_blocks][kv_heads][block_tokens][head_dim] of T.
template <typename T>
struct PagedKv {
    const T* key_arena;
    const T* value_arena;
    const std::int32_t* tables;
    std::uint32_t max_blocks;
    std::uint32_t block_tokens;
    std::uint32_t kv_heads;
    std::uint32_t head_dim;
    std::uint64_t num_blocks;
    std::uint32_t* error_word;

    struct Row {
        const T* ptr;
    };
    __device__ __forceinline__ std::size_t offset(int segment, long long token,
                                                  std::uint32_t head) const {
        const long long logical = token / block_tokens;
        std::int32_t block = tables[static_cast<std::size_t>(segment) * max_blocks + logical];
        if (block < 0 || static_cast<std::uint64_t>(block) >= num_blocks) {
            flag_error(error_word, kErrBadBlock);
            block = 0;
        }
        return ((static_cast<std::size_t>(block) * kv_heads + head) * block_tokens +
                static_cast<std::size_t>(token % block_tokens)) *
               head_dim;
    }
    __device__ __forceinline__ Row key_row(int segment, long long token, std::uint32_t head) const {
        return Row{key_arena + offset(segment, token, head)};
    }
    __device__ __forceinline__ Row value_row(int segment, long long token,
                                             std::uint32_t head) const {
        return Row{value_arena + offset(segment, token, head)};
    }
    __device__ __forceinline__ float load(const Row& row, std::uint32_t dim) const {
        return Storage<T>::to_float(row.ptr[dim]);
    }
    // Four consecutive dimensions (dim a multiple of 4, head_dim too).
    __device__ __forceinline__ float4 load4(const Row& row, std::uint32_t dim) const {
        if constexpr (sizeof(T) == 4) {
            return *reinterpret_cast<const float4*>(row.ptr + dim);
        } else {
            const uint2 raw = *reinterpret_cast<const uint2*>(row.ptr + dim);
            const T* h = reinterpret_cast<const T*>(&raw);
            return make_float4(Storage<T>::to_float(h[0]), Storage<T>::to_float(h[1]),
                               Storage<T>::to_float(h[2]), Storage<T>::to_float(h[3]));
        }
    }
};

// Where each query row sits. Rows are numbered query_row * q_heads + head.
struct SegmentMap {
    // mode 0: one contiguous segment, host-known geometry.
    // mode 1: decode batch; segment = query row, kv = context_lens[row],
    //         start = kv - 1.
    // mode 2: prefill segments given by starts/counts/offsets (device arrays).
    int mode;
    long long start0;
    long long kv_tokens0;
    int causal;
    const std::int32_t* context_lens;
    const std::int32_t* starts;
    const std::int32_t* counts;
    const std::int32_t* offsets;
    int num_segments;
    long long max_kv;  // bound on kv tokens a segment may have (paged: table capacity)

    // Resolves query row `q_row` into (segment, kv tokens, legal sources).
    // Returns false (and flags) when the segment description is invalid.
    __device__ __forceinline__ bool resolve(long long q_row, int& segment, long long& legal,
                                            std::uint32_t* error_word) const {
        if (mode == 0) {
            segment = 0;
            legal = causal ? min(kv_tokens0, start0 + q_row + 1) : kv_tokens0;
            return true;
        }
        if (mode == 1) {
            segment = static_cast<int>(q_row);
            const long long kv = context_lens[q_row];
            if (kv < 1 || kv > max_kv) {
                flag_error(error_word, kErrContext);
                return false;
            }
            legal = kv;
            return true;
        }
        // mode 2: binary search the segment whose [offset, offset + count) holds q_row
        int lo = 0;
        int hi = num_segments - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (offsets[mid] <= q_row) lo = mid; else hi = mid - 1;
        }
        segment = lo;
        const long long index = q_row - offsets[lo];
        const long long start = starts[lo];
        const long long count = counts[lo];
        if (index < 0 || index >= count || start < 0 || start + count > max_kv) {
            flag_error(error_word, kErrSegment);
            return false;
        }
        legal = start + index + 1;
        return true;
    }
};

struct GenericParams {
    const float* queries;  // [rows / heads][q_heads][head_dim]
    std::uint32_t query_precision;
    int reference_rounding;  // 1: round_reference (drop-in entry), 0: round_storage
    float* out;
    long long query_rows;  // number of query tokens
    std::uint32_t q_heads;
    std::uint32_t kv_heads;
    std::uint32_t head_dim;
    float scale;
    std::uint32_t* error_word;
    int check_normalizer;
    // Optional finite check over raw fp32 inputs (contiguous entry only).
    const float* check_ptr[3];
    std::size_t check_count[3];
};

template <typename Kv>
__global__ void __launch_bounds__(kGenericWarps * 32)
    generic_attention_kernel(GenericParams p, Kv kv, SegmentMap segments) {
    extern __shared__ float generic_smem[];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const unsigned d = p.head_dim;
    float* q_s = generic_smem + warp * (2 * d + kGenericChunk);
    float* acc_s = q_s + d;
    float* p_s = acc_s + d;

    // Finite check of the raw inputs, spread over the whole grid
    // (kernels/attention_cpu.cpp:131-134 checks every element).
    // Four loads in flight per thread; the entry sizes the grid so that a
    // call with few query rows still spreads the check over enough CTAs.
    for (int t = 0; t < 3; ++t) {
        const float* ptr = p.check_ptr[t];
        if (ptr == nullptr) continue;
        bool bad = false;
        const std::size_t stride = static_cast<std::size_t>(gridDim.x) * blockDim.x;
        std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
        for (; i + 3 * stride < p.check_count[t]; i += 4 * stride) {
            const float a = ptr[i];
            const float b = ptr[i + stride];
            const float c = ptr[i + 2 * stride];
            const float e = ptr[i + 3 * stride];
            bad |= !(isfinite(a) && isfinite(b) && isfinite(c) && isfinite(e));
        }
        for (; i < p.check_count[t]; i += stride) bad |= !isfinite(ptr[i]);
        if (bad) flag_error(p.error_word, kErrNonFinite);
    }

    const long long row = static_cast<long long>(blockIdx.x) * kGenericWarps + warp;
    if (row >= p.query_rows * p.q_heads) return;
    const long long q_row = row / p.q_heads;
    const std::uint32_t head = static_cast<std::uint32_t>(row % p.q_heads);
    const std::uint32_t kv_head = head / (p.q_heads / p.kv_heads);
    float* out = p.out + static_cast<std::size_t>(row) * d;

    int segment = 0;
    long long legal = 0;
    if (!segments.resolve(q_row, segment, legal, p.error_word)) {
        for (unsigned c = lane; c < d; c += 32) out[c] = 0.0f;
        return;
    }

    const float* q_global = p.queries + static_cast<std::size_t>(row) * d;
    for (unsigned c = lane; c < d; c += 32) {
        q_s[c] = p.reference_rounding ? round_reference(q_global[c], p.query_precision)
                                      : round_storage(q_global[c], p.query_precision);
        acc_s[c] = 0.0f;
    }
    __syncwarp();

    float running_max = -INFINITY;
    float running_den = 0.0f;
    for (long long begin = 0; begin < legal; begin += kGenericChunk) {
        float score[kGenericTpl];
        float chunk_max = -INFINITY;
        // Scores of this lane's kTpl keys. The dot products keep the
        // reference's order and rounding (kernels/attention_cpu.cpp:245-251):
        // sequential over the head dimension, product and sum rounded
        // separately, so the scores - whose errors exp() amplifies - agree
        // exactly. The loads of all kTpl keys are issued together (four
        // dimensions at a time when head_dim allows), so a key costs one
        // memory round trip per four dimensions, not one per dimension.
        typename Kv::Row krow[kGenericTpl];
        bool valid[kGenericTpl];
#pragma unroll
        for (int j = 0; j < kGenericTpl; ++j) {
            const long long token = begin + j * 32 + lane;
            valid[j] = token < legal;
            krow[j] = kv.key_row(segment, valid[j] ? token : begin, kv_head);
            score[j] = 0.0f;
        }
        if ((d & 3u) == 0) {
#pragma unroll 2
            for (unsigned c = 0; c < d; c += 4) {
                float4 k4[kGenericTpl];
#pragma unroll
                for (int j = 0; j < kGenericTpl; ++j) {
                    k4[j] = valid[j] ? kv.load4(krow[j], c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                }
#pragma unroll
                for (int j = 0; j < kGenericTpl; ++j) {
                    float s_ = score[j];
                    s_ = __fadd_rn(s_, __fmul_rn(q_s[c], k4[j].x));
                    s_ = __fadd_rn(s_, __fmul_rn(q_s[c + 1], k4[j].y));
                    s_ = __fadd_rn(s_, __fmul_rn(q_s[c + 2], k4[j].z));
                    s_ = __fadd_rn(s_, __fmul_rn(q_s[c + 3], k4[j].w));
                    score[j] = s_;
                }
            }
        } else {
            for (unsigned c = 0; c < d; ++c) {
                float k1[kGenericTpl];
#pragma unroll
                for (int j = 0; j < kGenericTpl; ++j) k1[j] = valid[j] ? kv.load(krow[j], c) : 0.0f;
#pragma unroll
                for (int j = 0; j < kGenericTpl; ++j) {
                    score[j] = __fadd_rn(score[j], __fmul_rn(q_s[c], k1[j]));
                }
            }
        }
#pragma unroll
        for (int j = 0; j < kGenericTpl; ++j) {
            score[j] = valid[j] ? __fmul_rn(score[j], p.scale) : -INFINITY;
            chunk_max = fmaxf(chunk_max, score[j]);
        }
        chunk_max = warp_max(chunk_max);
        const float new_max = fmaxf(running_max, chunk_max);
        const float alpha = running_max == -INFINITY ? 0.0f : expf(running_max - new_max);
        float local_sum = 0.0f;
#pragma unroll
        for (int j = 0; j < kGenericTpl; ++j) {
            const float prob = score[j] == -INFINITY ? 0.0f : expf(score[j] - new_max);
            local_sum += prob;
            p_s[j * 32 + lane] = prob;
        }
        running_den = running_den * alpha + warp_sum(local_sum);
        running_max = new_max;
        __syncwarp();
        const long long count = min(static_cast<long long>(kGenericChunk), legal - begin);
        for (unsigned c = lane; c < d; c += 32) {
            float a = acc_s[c] * alpha;
            long long t = 0;
            // Eight value loads in flight, accumulated in token order.
            for (; t + 8 <= count; t += 8) {
                float v8[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    v8[u] = kv.load(kv.value_row(segment, begin + t + u, kv_head), c);
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) a = fmaf(p_s[t + u], v8[u], a);
            }
            for (; t < count; ++t) {
                const auto vrow = kv.value_row(segment, begin + t, kv_head);
                a = fmaf(p_s[t], kv.load(vrow, c), a);
            }
            acc_s[c] = a;
        }
        __syncwarp();
    }
    if (p.check_normalizer && !(isfinite(running_den) && running_den > 0.0f)) {
        flag_error(p.error_word, kErrNormalizer);
    }
    for (unsigned c = lane; c < d; c += 32) out[c] = acc_s[c] / running_den;
}

}  // namespace ilb
