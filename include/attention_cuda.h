// attention_cuda.h - C++ API of the B200 attention library.
//
// Same declarations as the reference's kernels/attention_cpu.h:1-53
// (namespace inferlab, C++ linkage), so C++ callers such as the worker's
// Model::forward_cached / forward_all (worker/cpp/inferlab_runtime.cpp:
// 1458-1470, 1327-1339) link against this library instead of
// attention_cpu.cpp without source changes.
#pragma once

#include <cstddef>
#include <cstdint>

namespace inferlab {

enum class AttentionAlgorithm : std::uint32_t {
    Materialized = 0,
    OnlineTiled = 1,
};

enum class AttentionPrecision : std::uint32_t {
    Fp32 = 0,
    Fp16 = 1,
    Bf16 = 2,
};

struct AttentionConfig {
    AttentionAlgorithm algorithm = AttentionAlgorithm::Materialized;
    AttentionPrecision precision = AttentionPrecision::Fp32;
    std::size_t tile_tokens = 16;
    bool causal = true;
};

struct AttentionStats {
    std::uint64_t score_elements = 0;
    std::uint64_t masked_score_elements = 0;
    std::uint64_t score_buffer_bytes = 0;
    std::uint64_t working_set_bytes = 0;
    std::uint64_t modeled_external_read_bytes = 0;
    std::uint64_t modeled_external_write_bytes = 0;
    std::uint64_t modeled_external_total_bytes = 0;
    std::uint64_t key_tiles = 0;
};

// Replaces kernels/attention_cpu.h:37 (round_attention_value): storage
// rounding to fp16/bf16 and back, round to nearest even.
float round_attention_value(float value, AttentionPrecision precision);

// Replaces kernels/attention_cpu.h:39-51. Host pointers; runs on the current
// CUDA device; throws std::runtime_error with the reference's messages. Same
// arithmetic and tolerances as inferlab_attention_forward (include/
// inferlab_attention.h), including its tensor-core route for large causal
// Fp16 / Bf16 calls with head_dimension 128.
void attention_forward(const float* queries, const float* keys, const float* values,
                       std::size_t query_tokens, std::size_t key_value_tokens,
                       std::size_t heads, std::size_t head_dimension,
                       std::size_t query_start_position, const AttentionConfig& config,
                       float* output, AttentionStats* stats);

}  // namespace inferlab
