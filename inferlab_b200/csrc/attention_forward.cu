// attention_forward.cu - the reference worker's attention entry on the GPU.
//
// inferlab_attention_forward keeps the C ABI of
// worker/cpp/inferlab_runtime.cpp:2561-2619 and inferlab::attention_forward
// the C++ API of kernels/attention_cpu.cpp:419-502: host fp32 buffers in and
// out, the same validation order and messages, the same analytic stats. The
// arithmetic runs on the current CUDA device: one packed host->device copy of
// Q|K|V from pinned staging, the generic online-softmax kernel (which also
// checks every input for finiteness and applies the storage rounding on
// load), one packed device->host copy of the error word and the output.
#include "common.cuh"
#include "generic_attention.cuh"

#include "../../include/attention_cuda.h"
#include "../../include/inferlab_attention.h"

#include <chrono>
#include <cmath>
#include <limits>
#include <mutex>
#include <thread>

namespace ilb {

void wait_stream(cudaStream_t stream, std::uint32_t timeout_ms) {
    const auto deadline = std::chrono::steady_clock::now() +
                          std::chrono::milliseconds(timeout_ms == 0 ? 10000u : timeout_ms);
    for (int spin = 0;; ++spin) {
        const cudaError_t status = cudaStreamQuery(stream);
        if (status == cudaSuccess) return;
        if (status != cudaErrorNotReady) cuda_check(status, "CUDA stream failed");
        if (std::chrono::steady_clock::now() > deadline) {
            throw std::runtime_error("CUDA stream wait timed out");
        }
        if (spin > 64) std::this_thread::yield();
    }
}

std::string describe_error_bits(std::uint32_t bits) {
    if (bits & kErrBadBlock) return "paged KV block table contains an invalid page";
    if (bits & kErrNonFinite) return "attention input must be finite";
    if (bits & kErrContext) return "paged KV context length is invalid";
    if (bits & kErrSegment) return "paged prefill segment is invalid";
    if (bits & kErrPosition) return "paged KV append position is outside the block table";
    if (bits & kErrNormalizer) return "online attention normalizer is invalid";
    if (bits & kErrWaitTimeout) return "device wait timed out";
    return "unknown device error";
}

namespace {

// Per-device resources for the host-buffer entry. One caller at a time per
// device (the mutex); the reference kernel is re-entrant, and so is this entry
// across threads, which simply serialise on the device they share.
struct DeviceContext {
    std::mutex mutex;
    int device = 0;
    cudaStream_t stream = nullptr;
    unsigned char* device_buffer = nullptr;
    std::size_t device_capacity = 0;
    unsigned char* host_buffer = nullptr;  // pinned
    std::size_t host_capacity = 0;
    bool smem_configured = false;
};

std::mutex registry_mutex;
DeviceContext* registry[128] = {};

DeviceContext& context_for(int device) {
    if (device < 0 || device >= 128) throw std::runtime_error("CUDA device index out of range");
    std::lock_guard<std::mutex> guard(registry_mutex);
    if (registry[device] == nullptr) {
        auto* ctx = new DeviceContext();
        ctx->device = device;
        cuda_check(cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking),
                   "cudaStreamCreate");
        registry[device] = ctx;
    }
    return *registry[device];
}

void reserve(DeviceContext& ctx, std::size_t bytes) {
    if (bytes > ctx.device_capacity) {
        if (ctx.device_buffer != nullptr) cudaFree(ctx.device_buffer);
        ctx.device_buffer = nullptr;
        ctx.device_capacity = 0;
        const std::size_t grown = bytes + bytes / 4;
        cuda_check(cudaMalloc(&ctx.device_buffer, grown), "cudaMalloc");
        ctx.device_capacity = grown;
    }
    if (bytes > ctx.host_capacity) {
        if (ctx.host_buffer != nullptr) cudaFreeHost(ctx.host_buffer);
        ctx.host_buffer = nullptr;
        ctx.host_capacity = 0;
        const std::size_t grown = bytes + bytes / 4;
        cuda_check(cudaMallocHost(&ctx.host_buffer, grown), "cudaMallocHost");
        ctx.host_capacity = grown;
    }
}

std::uint64_t checked_u64(std::uint64_t a, std::uint64_t b) {
    if (a != 0 && b > std::numeric_limits<std::uint64_t>::max() / a) {
        throw std::runtime_error("attention metric product overflows");
    }
    return a * b;
}

std::size_t legal_sources(std::size_t query, std::size_t kv_tokens, std::size_t start, bool causal) {
    if (!causal) return kv_tokens;
    return std::min(kv_tokens, start + query + 1);
}

// Analytic statistics of the reference CPU algorithm (kernels/attention_cpu.cpp:
// 140-213): integer formulae, reproduced exactly for ABI parity.
void compute_stats(std::size_t tq, std::size_t tkv, std::size_t heads, std::size_t d,
                   std::size_t start, const inferlab::AttentionConfig& config,
                   inferlab::AttentionStats& stats) {
    std::uint64_t legal_pairs = 0;
    std::uint64_t key_tiles = 0;
    for (std::size_t query = 0; query < tq; ++query) {
        const std::uint64_t legal = legal_sources(query, tkv, start, config.causal);
        legal_pairs += checked_u64(legal, heads);
        key_tiles += checked_u64((legal + config.tile_tokens - 1) / config.tile_tokens, heads);
    }
    const std::uint64_t all_pairs = checked_u64(checked_u64(tq, tkv), heads);
    stats.score_elements = legal_pairs;
    stats.masked_score_elements = all_pairs - legal_pairs;
    stats.key_tiles = key_tiles;
    const std::uint64_t scalar = config.precision == inferlab::AttentionPrecision::Fp32 ? 4 : 2;
    const std::uint64_t query_bytes = checked_u64(checked_u64(tq, heads), checked_u64(d, scalar));
    const std::uint64_t kv_bytes = checked_u64(checked_u64(tkv, heads), checked_u64(d, scalar));
    const std::uint64_t output_bytes = checked_u64(checked_u64(tq, heads), checked_u64(d, 4));
    if (config.algorithm == inferlab::AttentionAlgorithm::Materialized) {
        const std::uint64_t score_bytes = checked_u64(all_pairs, 4);
        stats.score_buffer_bytes = score_bytes;
        stats.working_set_bytes = score_bytes;
        stats.modeled_external_read_bytes =
            query_bytes + checked_u64(kv_bytes, 2) + checked_u64(score_bytes, 2);
        stats.modeled_external_write_bytes = checked_u64(score_bytes, 2) + output_bytes;
    } else {
        stats.score_buffer_bytes = checked_u64(config.tile_tokens, 4);
        stats.working_set_bytes = stats.score_buffer_bytes + checked_u64(d, 4);
        const std::uint64_t query_tiles = (tq + config.tile_tokens - 1) / config.tile_tokens;
        stats.modeled_external_read_bytes =
            query_bytes + checked_u64(checked_u64(query_tiles, kv_bytes), 2);
        stats.modeled_external_write_bytes = output_bytes;
    }
    stats.modeled_external_total_bytes =
        stats.modeled_external_read_bytes + stats.modeled_external_write_bytes;
}

inferlab::AttentionConfig map_config(std::uint32_t algorithm, std::uint32_t precision,
                                     std::uint32_t tile_tokens, bool causal) {
    // worker/cpp/inferlab_runtime.cpp:446-490: tile first, then the enums.
    if (tile_tokens == 0 || tile_tokens > 4096) {
        throw std::runtime_error("attention tile_tokens must be between 1 and 4096");
    }
    if (algorithm > 1) {
        throw std::runtime_error("attention algorithm must be 0 (materialized) or 1 (online tiled)");
    }
    if (precision > 2) {
        throw std::runtime_error("attention precision must be 0 (FP32), 1 (FP16), or 2 (BF16)");
    }
    inferlab::AttentionConfig config;
    config.algorithm = static_cast<inferlab::AttentionAlgorithm>(algorithm);
    config.precision = static_cast<inferlab::AttentionPrecision>(precision);
    config.tile_tokens = tile_tokens;
    config.causal = causal;
    return config;
}

}  // namespace
}  // namespace ilb

namespace inferlab {

float round_attention_value(float value, AttentionPrecision precision) {
    // The reference's storage simulation, including its widening of fp16
    // subnormals to half their value (see round_reference).
    return ilb::round_reference(value, static_cast<std::uint32_t>(precision));
}

void attention_forward(const float* queries, const float* keys, const float* values,
                       std::size_t query_tokens, std::size_t key_value_tokens, std::size_t heads,
                       std::size_t head_dimension, std::size_t query_start_position,
                       const AttentionConfig& config, float* output, AttentionStats* stats) {
    using namespace ilb;
    // kernels/attention_cpu.cpp:432-447, in order.
    if (queries == nullptr || keys == nullptr || values == nullptr || output == nullptr) {
        throw std::runtime_error("attention input or output pointer is null");
    }
    if (query_tokens == 0 || key_value_tokens == 0 || heads == 0 || head_dimension == 0) {
        throw std::runtime_error("attention dimensions must be positive");
    }
    if (config.tile_tokens == 0 || config.tile_tokens > 4096) {
        throw std::runtime_error("attention tile_tokens must be between 1 and 4096");
    }
    if (config.causal && (query_start_position >= key_value_tokens ||
                          query_tokens > key_value_tokens - query_start_position)) {
        throw std::runtime_error("causal query positions exceed the KV sequence");
    }
    const char* overflow = "attention shape product overflows";
    const std::size_t query_values = checked_mul(checked_mul(query_tokens, heads, overflow),
                                                 head_dimension, overflow);
    const std::size_t kv_values = checked_mul(checked_mul(key_value_tokens, heads, overflow),
                                              head_dimension, overflow);
    if (head_dimension > kGenericMaxHeadDim) {
        throw std::runtime_error("attention head_dimension exceeds the CUDA kernel limit of 4096");
    }
    if (query_values > static_cast<std::size_t>(std::numeric_limits<long long>::max() / 4)) {
        throw std::runtime_error(overflow);
    }

    int device = 0;
    cuda_check(cudaGetDevice(&device), "cudaGetDevice");
    DeviceContext& ctx = context_for(device);
    std::lock_guard<std::mutex> guard(ctx.mutex);

    // Device layout: [Q][K][V][error word (16 B)][out]; host staging mirrors it.
    const std::size_t q_bytes = query_values * sizeof(float);
    const std::size_t kv_bytes = kv_values * sizeof(float);
    const std::size_t in_bytes = q_bytes + 2 * kv_bytes;
    const std::size_t err_offset = (in_bytes + 15) & ~static_cast<std::size_t>(15);
    const std::size_t out_offset = err_offset + 16;
    const std::size_t total = out_offset + q_bytes;
    reserve(ctx, total);

    unsigned char* host = ctx.host_buffer;
    std::memcpy(host, queries, q_bytes);
    std::memcpy(host + q_bytes, keys, kv_bytes);
    std::memcpy(host + q_bytes + kv_bytes, values, kv_bytes);
    std::memset(host + in_bytes, 0, out_offset - in_bytes);

    unsigned char* dev = ctx.device_buffer;
    auto* d_q = reinterpret_cast<float*>(dev);
    auto* d_k = reinterpret_cast<float*>(dev + q_bytes);
    auto* d_v = reinterpret_cast<float*>(dev + q_bytes + kv_bytes);
    auto* d_err = reinterpret_cast<std::uint32_t*>(dev + err_offset);
    auto* d_out = reinterpret_cast<float*>(dev + out_offset);

    cuda_check(cudaMemcpyAsync(dev, host, out_offset, cudaMemcpyHostToDevice, ctx.stream),
               "cudaMemcpyAsync H2D");

    const std::size_t smem = generic_smem_bytes(static_cast<unsigned>(head_dimension));
    if (!ctx.smem_configured) {
        cuda_check(cudaFuncSetAttribute(generic_attention_kernel<ContiguousKv>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(generic_smem_bytes(kGenericMaxHeadDim))),
                   "cudaFuncSetAttribute");
        ctx.smem_configured = true;
    }
    GenericParams params{};
    params.queries = d_q;
    params.query_precision = static_cast<std::uint32_t>(config.precision);
    params.reference_rounding = 1;
    params.out = d_out;
    params.query_rows = static_cast<long long>(query_tokens);
    params.q_heads = static_cast<std::uint32_t>(heads);
    params.kv_heads = static_cast<std::uint32_t>(heads);
    params.head_dim = static_cast<std::uint32_t>(head_dimension);
    params.scale = 1.0f / std::sqrt(static_cast<float>(head_dimension));
    params.error_word = d_err;
    params.check_normalizer = config.algorithm == AttentionAlgorithm::OnlineTiled ? 1 : 0;
    params.check_ptr[0] = d_q;
    params.check_ptr[1] = d_k;
    params.check_ptr[2] = d_v;
    params.check_count[0] = query_values;
    params.check_count[1] = kv_values;
    params.check_count[2] = kv_values;
    ContiguousKv kv{d_k, d_v, static_cast<std::uint32_t>(config.precision),
                    static_cast<std::uint32_t>(heads), static_cast<std::uint32_t>(head_dimension)};
    SegmentMap segments{};
    segments.mode = 0;
    segments.start0 = static_cast<long long>(query_start_position);
    segments.kv_tokens0 = static_cast<long long>(key_value_tokens);
    segments.causal = config.causal ? 1 : 0;
    const std::size_t rows = query_tokens * heads;
    const unsigned grid = static_cast<unsigned>((rows + kGenericWarps - 1) / kGenericWarps);
    generic_attention_kernel<ContiguousKv>
        <<<grid, kGenericWarps * 32, smem, ctx.stream>>>(params, kv, segments);
    cuda_check(cudaGetLastError(), "attention kernel launch");

    cuda_check(cudaMemcpyAsync(host + err_offset, dev + err_offset, 16 + q_bytes,
                               cudaMemcpyDeviceToHost, ctx.stream),
               "cudaMemcpyAsync D2H");
    wait_stream(ctx.stream, 0);
    std::uint32_t bits = 0;
    std::memcpy(&bits, host + err_offset, sizeof bits);
    if (bits & kErrNonFinite) throw std::runtime_error("attention input must be finite");
    if (bits & kErrNormalizer) throw std::runtime_error("online attention normalizer is invalid");
    if (bits != 0) throw std::runtime_error(describe_error_bits(bits));
    std::memcpy(output, host + out_offset, q_bytes);
    if (stats != nullptr) {
        *stats = AttentionStats{};
        compute_stats(query_tokens, key_value_tokens, heads, head_dimension,
                      query_start_position, config, *stats);
    }
}

}  // namespace inferlab

extern "C" int inferlab_attention_forward(const float* queries, const float* keys,
                                          const float* values, std::size_t query_tokens,
                                          std::size_t key_value_tokens, std::size_t heads,
                                          std::size_t head_dimension,
                                          std::size_t query_start_position,
                                          const InferlabAttentionConfig* config, float* output,
                                          std::size_t output_capacity,
                                          InferlabAttentionStats* stats, char* error,
                                          std::size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        // worker/cpp/inferlab_runtime.cpp:2577-2617, in order.
        if (config == nullptr || stats == nullptr) {
            throw std::runtime_error("attention config or stats pointer is null");
        }
        const char* overflow = "attention shape product overflows";
        const std::size_t output_values = ilb::checked_mul(
            ilb::checked_mul(query_tokens, heads, overflow), head_dimension, overflow);
        if (output == nullptr || output_capacity < output_values) {
            throw std::runtime_error("attention output buffer is too small");
        }
        const auto native = ilb::map_config(config->algorithm, config->precision,
                                            config->tile_tokens, config->causal != 0);
        inferlab::AttentionStats native_stats{};
        inferlab::attention_forward(queries, keys, values, query_tokens, key_value_tokens, heads,
                                    head_dimension, query_start_position, native, output,
                                    &native_stats);
        *stats = InferlabAttentionStats{
            native_stats.score_elements,
            native_stats.masked_score_elements,
            native_stats.score_buffer_bytes,
            native_stats.working_set_bytes,
            native_stats.modeled_external_read_bytes,
            native_stats.modeled_external_write_bytes,
            native_stats.modeled_external_total_bytes,
            native_stats.key_tiles,
        };
    });
}

extern "C" const char* inferlab_cuda_version(void) { return "inferlab-b200 0.1 sm_100a"; }
