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
//
// Full-sequence calls in the Fp16 / Bf16 storage modes with head_dim 128
// (the shape of Model::forward_all, worker/cpp/inferlab_runtime.cpp:
// 1327-1339, on a real model) take the tensor cores instead: a preparation
// kernel checks and rounds the inputs like the reference (kernels/
// attention_cpu.cpp:125-138, 405-417), stores them in 16-bit form with K/V
// in 16-token blocks, and the paged tcgen05 prefill kernel computes the
// causal attention with fp32 accumulation and fp16 probabilities (within
// 2e-3 of the reference's fp32 arithmetic). Inputs whose rounded values leave
// the tensor path's range (an fp16 overflow to infinity, or a bf16 value
// beyond fp16's range in V, which the kernel widens to fp16) go back to the
// generic kernel, which reproduces the reference's handling of them.
#include "common.cuh"
#include "generic_attention.cuh"
#include "prefill_tc.cuh"

#include "../../include/attention_cuda.h"
#include "../../include/inferlab_attention.h"

#include <chrono>
#include <cmath>
#include <limits>
#include <mutex>
#include <thread>
#include <vector>

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

void wait_event(cudaEvent_t event, std::uint32_t timeout_ms) {
    const auto deadline = std::chrono::steady_clock::now() +
                          std::chrono::milliseconds(timeout_ms == 0 ? 10000u : timeout_ms);
    for (int spin = 0;; ++spin) {
        const cudaError_t status = cudaEventQuery(event);
        if (status == cudaSuccess) return;
        if (status != cudaErrorNotReady) cuda_check(status, "CUDA event failed");
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
    std::uint32_t* tc_words = nullptr;  // error word + work-queue counters of the tensor route
    unsigned char* device_buffer = nullptr;
    std::size_t device_capacity = 0;
    unsigned char* host_buffer = nullptr;  // pinned
    std::size_t host_capacity = 0;
    bool smem_configured = false;
    std::vector<cudaEvent_t> events;  // chunk completion of pipelined copies
};

// Host-side copies between the caller's arrays and the page-locked staging:
// 8 MB and more are split over up to 8 host threads, one per 2 MB (one thread
// copies about 10 GB/s, well below the bus; smaller copies do not repay the
// threads' start-up), and transfers move in 16 MB chunks so the DMA of one
// chunk overlaps the host copy of the next.
constexpr std::size_t kParallelCopyBytes = std::size_t(8) << 20;
constexpr std::size_t kChunkBytes = std::size_t(16) << 20;

// Copies bytes [begin, end) of the packed image of `parts` consecutive source
// arrays into image + begin, spread over host threads by bytes.
void copy_packed_range(unsigned char* image, const unsigned char* const* sources,
                       const std::size_t* sizes, int parts, std::size_t begin, std::size_t end) {
    auto copy_span = [&](std::size_t lo_all, std::size_t hi_all) {
        std::size_t base = 0;
        for (int i = 0; i < parts && lo_all < hi_all; ++i) {
            const std::size_t lo = std::max(lo_all, base);
            const std::size_t hi = std::min(hi_all, base + sizes[i]);
            if (lo < hi) std::memcpy(image + lo, sources[i] + (lo - base), hi - lo);
            base += sizes[i];
        }
    };
    const std::size_t bytes = end - begin;
    if (bytes < kParallelCopyBytes) {
        copy_span(begin, end);
        return;
    }
    const unsigned hw = std::max(2u, std::min(8u, std::thread::hardware_concurrency()));
    const unsigned threads = static_cast<unsigned>(std::min<std::size_t>(hw, bytes >> 21));
    const std::size_t slice = ((bytes + threads - 1) / threads + 63) & ~static_cast<std::size_t>(63);
    std::vector<std::thread> pool;
    pool.reserve(threads);
    for (unsigned t = 1; t < threads; ++t) {
        const std::size_t lo = std::min(end, begin + t * slice);
        const std::size_t hi = std::min(end, lo + slice);
        if (lo < hi) pool.emplace_back(copy_span, lo, hi);
    }
    copy_span(begin, std::min(end, begin + slice));
    for (auto& t : pool) t.join();
}

void parallel_copy(unsigned char* dst, const unsigned char* src, std::size_t bytes) {
    const unsigned char* sources[1] = {src};
    const std::size_t sizes[1] = {bytes};
    copy_packed_range(dst, sources, sizes, 1, 0, bytes);
}

cudaEvent_t chunk_event(DeviceContext& ctx, std::size_t index) {
    while (ctx.events.size() <= index) {
        cudaEvent_t event = nullptr;
        cuda_check(cudaEventCreateWithFlags(&event, cudaEventDisableTiming), "cudaEventCreate");
        ctx.events.push_back(event);
    }
    return ctx.events[index];
}

// Stages the packed sources into host[0, bytes) and copies them to dev,
// chunk by chunk for large images.
void stage_to_device(DeviceContext& ctx, unsigned char* host, unsigned char* dev,
                     const unsigned char* const* sources, const std::size_t* sizes, int parts,
                     std::size_t bytes) {
    const std::size_t chunk = bytes < kParallelCopyBytes ? bytes : kChunkBytes;
    for (std::size_t begin = 0; begin < bytes; begin += chunk) {
        const std::size_t end = std::min(bytes, begin + chunk);
        copy_packed_range(host, sources, sizes, parts, begin, end);
        cuda_check(cudaMemcpyAsync(dev + begin, host + begin, end - begin, cudaMemcpyHostToDevice,
                                   ctx.stream),
                   "cudaMemcpyAsync H2D");
    }
}

// Copies `words` (16 B of device error words) and then `bytes` of output
// from the device to host staging and on to `output`, chunk by chunk: the
// error words are checked (by `check`, which throws) before any output is
// copied.
template <typename Check>
void finish_from_device(DeviceContext& ctx, unsigned char* host, const unsigned char* d_words,
                        const unsigned char* d_out, std::size_t bytes, float* output, Check&& check) {
    const std::size_t chunk = bytes < kParallelCopyBytes ? std::max<std::size_t>(bytes, 1)
                                                         : kChunkBytes;
    // Words and output in one copy when they sit next to each other.
    const bool adjacent = d_out == d_words + 16;
    if (!adjacent) {
        cuda_check(cudaMemcpyAsync(host, d_words, 16, cudaMemcpyDeviceToHost, ctx.stream),
                   "cudaMemcpyAsync D2H");
    }
    std::size_t index = 0;
    for (std::size_t begin = 0; begin < bytes; begin += chunk, ++index) {
        const std::size_t end = std::min(bytes, begin + chunk);
        const std::size_t lead = adjacent && begin == 0 ? 16 : 0;
        cuda_check(cudaMemcpyAsync(host + 16 + begin - lead, d_out + begin - lead,
                                   end - begin + lead, cudaMemcpyDeviceToHost, ctx.stream),
                   "cudaMemcpyAsync D2H");
        cuda_check(cudaEventRecord(chunk_event(ctx, index), ctx.stream), "cudaEventRecord");
    }
    if (index == 0) {
        wait_stream(ctx.stream, 0);
    } else {
        wait_event(chunk_event(ctx, 0), 0);
    }
    std::uint32_t words[4];
    std::memcpy(words, host, sizeof words);
    bool copy_out = false;
    try {
        copy_out = check(words);
    } catch (...) {
        // Let the remaining copies into the staging land before it is reused.
        try {
            wait_stream(ctx.stream, 0);
        } catch (...) {
        }
        throw;
    }
    if (!copy_out) {
        wait_stream(ctx.stream, 0);
        return;
    }
    index = 0;
    for (std::size_t begin = 0; begin < bytes; begin += chunk, ++index) {
        const std::size_t end = std::min(bytes, begin + chunk);
        if (index > 0) wait_event(chunk_event(ctx, index), 0);
        parallel_copy(reinterpret_cast<unsigned char*>(output) + begin, host + 16 + begin,
                      end - begin);
    }
    wait_stream(ctx.stream, 0);
}

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

// Query rows (tokens x heads) from which a Fp16 / Bf16 call with head_dim 128
// takes the tensor cores; smaller calls are latency-bound either way.
constexpr std::size_t kTcMinRows = 1024;

// Tensor route inputs: Q as 16-bit [tokens][heads][128]; K and V as 16-bit
// blocks [token / 16][head][token % 16][128] (the pool layout the prefill
// kernel reads), the tail of the last block zeroed; an identity block table;
// segment {start, tokens, offset 0}. word[0] takes the reference's input
// errors, word[1] is set when a rounded value leaves the tensor path's range.
template <typename T>
__global__ void tc_prepare_kernel(const float* q, const float* k, const float* v,
                                  std::size_t q_values, std::size_t kv_values,
                                  std::size_t padded_kv_values, std::uint32_t heads,
                                  std::uint32_t precision, T* q16, T* k_arena, T* v_arena,
                                  std::int32_t* table, std::uint32_t blocks, std::int32_t* segment,
                                  long long start, long long q_tokens, std::uint32_t* word) {
    const std::size_t stride = static_cast<std::size_t>(gridDim.x) * blockDim.x;
    const std::size_t first = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    bool bad = false;
    bool out_of_range = false;
    for (std::size_t i = first; i < q_values; i += stride) {
        const float x = q[i];
        bad |= !isfinite(x);
        const float r = round_reference(x, precision);
        out_of_range |= !isfinite(r);
        q16[i] = Storage<T>::from_float(r);
    }
    const std::size_t row = static_cast<std::size_t>(heads) * 128;
    for (std::size_t i = first; i < padded_kv_values; i += stride) {
        const std::size_t token = i / row;
        const std::size_t head = (i / 128) % heads;
        const std::size_t dst = ((token >> 4) * heads + head) * 2048 + (token & 15) * 128 + (i & 127);
        if (i < kv_values) {
            const float a = k[i];
            const float b = v[i];
            bad |= !(isfinite(a) && isfinite(b));
            const float ra = round_reference(a, precision);
            const float rb = round_reference(b, precision);
            out_of_range |= !(isfinite(ra) && isfinite(rb));
            if (precision == kBf16) out_of_range |= fabsf(rb) > 65504.0f;
            k_arena[dst] = Storage<T>::from_float(ra);
            v_arena[dst] = Storage<T>::from_float(rb);
        } else {
            k_arena[dst] = Storage<T>::from_float(0.0f);
            v_arena[dst] = Storage<T>::from_float(0.0f);
        }
    }
    for (std::size_t b = first; b < blocks; b += stride) table[b] = static_cast<std::int32_t>(b);
    if (first == 0) {
        segment[0] = static_cast<std::int32_t>(start);
        segment[1] = static_cast<std::int32_t>(q_tokens);
        segment[2] = 0;
    }
    if (bad) flag_error(word, kErrNonFinite);
    if (out_of_range) atomicOr(word + 1, 1u);
}

// Tensor-core route of the drop-in entry: the fp32 inputs are already in
// HBM at dev (Q, K, V packed); this prepares the 16-bit copies, runs the
// paged prefill kernel and copies the output to `output`. Returns false
// (nothing written) when a rounded value leaves the tensor path's range, so
// the caller runs the generic kernel on the same staged inputs.
bool run_tensor_route(DeviceContext& ctx, std::size_t q_bytes, std::size_t kv_bytes,
                      std::size_t query_tokens, std::size_t kv_tokens, std::size_t heads,
                      std::size_t start, inferlab::AttentionPrecision precision, float* output) {
    const std::uint32_t dtype = precision == inferlab::AttentionPrecision::Fp16 ? kF16 : kBf16;
    const std::size_t q_values = q_bytes / 4;
    const std::size_t kv_values = kv_bytes / 4;
    const std::size_t blocks = (kv_tokens + 15) / 16;
    const std::size_t padded_kv_values = blocks * 16 * heads * 128;
    auto align = [](std::size_t x) { return (x + 255) & ~static_cast<std::size_t>(255); };
    // [raw Q|K|V fp32][q16][K blocks][V blocks][table][segment][out]
    const std::size_t q16_off = align(q_bytes + 2 * kv_bytes);
    const std::size_t k_off = q16_off + align(q_values * 2);
    const std::size_t v_off = k_off + align(padded_kv_values * 2);
    const std::size_t table_off = v_off + align(padded_kv_values * 2);
    const std::size_t seg_off = table_off + align(blocks * 4);
    const std::size_t out_off = seg_off + 256;
    const std::size_t total = out_off + q_bytes;
    if (total > ctx.device_capacity) {
        // Grow the device buffer, keeping the staged inputs.
        unsigned char* grown = nullptr;
        const std::size_t capacity = total + total / 4;
        cuda_check(cudaMalloc(&grown, capacity), "cudaMalloc");
        cuda_check(cudaMemcpyAsync(grown, ctx.device_buffer, q_bytes + 2 * kv_bytes,
                                   cudaMemcpyDeviceToDevice, ctx.stream),
                   "cudaMemcpyAsync D2D");
        cuda_check(cudaStreamSynchronize(ctx.stream), "cudaStreamSynchronize");
        cudaFree(ctx.device_buffer);
        ctx.device_buffer = grown;
        ctx.device_capacity = capacity;
    }
    unsigned char* dev = ctx.device_buffer;
    if (ctx.tc_words == nullptr) {
        cuda_check(cudaMalloc(&ctx.tc_words, kPoolWordBytes), "cudaMalloc");
    }
    cuda_check(cudaMemsetAsync(ctx.tc_words, 0, kPoolWordBytes, ctx.stream), "cudaMemsetAsync");
    const auto* d_q = reinterpret_cast<const float*>(dev);
    const auto* d_k = reinterpret_cast<const float*>(dev + q_bytes);
    const auto* d_v = reinterpret_cast<const float*>(dev + q_bytes + kv_bytes);
    auto* table = reinterpret_cast<std::int32_t*>(dev + table_off);
    auto* segment = reinterpret_cast<std::int32_t*>(dev + seg_off);
    auto* out = reinterpret_cast<float*>(dev + out_off);
    const std::size_t work = std::max(q_values, padded_kv_values);
    const unsigned grid = static_cast<unsigned>(std::min<std::size_t>((work + 255) / 256, 148 * 16));
    if (dtype == kF16) {
        tc_prepare_kernel<__half><<<grid, 256, 0, ctx.stream>>>(
            d_q, d_k, d_v, q_values, kv_values, padded_kv_values, static_cast<std::uint32_t>(heads),
            dtype, reinterpret_cast<__half*>(dev + q16_off), reinterpret_cast<__half*>(dev + k_off),
            reinterpret_cast<__half*>(dev + v_off), table, static_cast<std::uint32_t>(blocks),
            segment, static_cast<long long>(start), static_cast<long long>(query_tokens),
            ctx.tc_words);
    } else {
        tc_prepare_kernel<__nv_bfloat16><<<grid, 256, 0, ctx.stream>>>(
            d_q, d_k, d_v, q_values, kv_values, padded_kv_values, static_cast<std::uint32_t>(heads),
            dtype, reinterpret_cast<__nv_bfloat16*>(dev + q16_off),
            reinterpret_cast<__nv_bfloat16*>(dev + k_off),
            reinterpret_cast<__nv_bfloat16*>(dev + v_off), table,
            static_cast<std::uint32_t>(blocks), segment, static_cast<long long>(start),
            static_cast<long long>(query_tokens), ctx.tc_words);
    }
    cuda_check(cudaGetLastError(), "tensor route preparation launch");
    // A pool view over the prepared blocks: one segment, identity table.
    InferlabCudaKvPool view;
    view.device = ctx.device;
    view.dtype = dtype;
    view.element_bytes = 2;
    view.block_tokens = 16;
    view.kv_heads = static_cast<std::uint32_t>(heads);
    view.head_dim = 128;
    view.num_blocks = blocks;
    view.block_bytes = static_cast<std::uint64_t>(heads) * 16 * 128 * 2;
    view.arena_bytes = view.block_bytes * blocks;
    view.key_arena = dev + k_off;
    view.value_arena = dev + v_off;
    view.error_word = ctx.tc_words;
    run_tc_prefill(view, dev + q16_off, dtype, table, static_cast<std::uint32_t>(blocks), segment,
                   segment + 1, segment + 2, 1, static_cast<std::uint32_t>(heads),
                   static_cast<std::uint32_t>(query_tokens), static_cast<long long>(query_tokens),
                   out, ctx.stream);
    // The host staging holds at least the staged inputs (more than 16 + q_bytes).
    bool in_range = true;
    finish_from_device(ctx, ctx.host_buffer, reinterpret_cast<const unsigned char*>(ctx.tc_words),
                       reinterpret_cast<const unsigned char*>(out), q_bytes, output,
                       [&](const std::uint32_t* words) {
                           if (words[0] & kErrNonFinite) {
                               throw std::runtime_error("attention input must be finite");
                           }
                           if (words[1] != 0) {
                               in_range = false;
                               return false;
                           }
                           if (words[0] & kErrNormalizer) {
                               throw std::runtime_error("online attention normalizer is invalid");
                           }
                           if (words[0] != 0) throw std::runtime_error(describe_error_bits(words[0]));
                           return true;
                       });
    return in_range;
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

    unsigned char* dev = ctx.device_buffer;
    float* d_q = reinterpret_cast<float*>(dev);
    float* d_k = reinterpret_cast<float*>(dev + q_bytes);
    float* d_v = reinterpret_cast<float*>(dev + q_bytes + kv_bytes);
    std::uint32_t* d_err = reinterpret_cast<std::uint32_t*>(dev + err_offset);
    float* d_out = reinterpret_cast<float*>(dev + out_offset);

    // Inputs and a zeroed error word in one staged image.
    static const unsigned char kZeros[32] = {};
    const unsigned char* sources[4] = {reinterpret_cast<const unsigned char*>(queries),
                                       reinterpret_cast<const unsigned char*>(keys),
                                       reinterpret_cast<const unsigned char*>(values), kZeros};
    const std::size_t sizes[4] = {q_bytes, kv_bytes, kv_bytes, out_offset - in_bytes};
    stage_to_device(ctx, host, dev, sources, sizes, 4, out_offset);

    const bool tensor_route = config.precision != AttentionPrecision::Fp32 &&
                              head_dimension == 128 && config.causal &&
                              query_tokens * heads >= kTcMinRows &&
                              key_value_tokens <= 0x7FFFFFF0u && query_tokens <= 0x7FFFFFF0u;
    if (tensor_route && run_tensor_route(ctx, q_bytes, kv_bytes, query_tokens, key_value_tokens,
                                         heads, query_start_position, config.precision, output)) {
        if (stats != nullptr) {
            *stats = AttentionStats{};
            compute_stats(query_tokens, key_value_tokens, heads, head_dimension,
                          query_start_position, config, *stats);
        }
        return;
    }
    if (tensor_route) {
        // Back from the tensor route: the staged inputs are kept (the buffer
        // may have grown), the error word was overwritten by its 16-bit copies.
        dev = ctx.device_buffer;
        d_q = reinterpret_cast<float*>(dev);
        d_k = reinterpret_cast<float*>(dev + q_bytes);
        d_v = reinterpret_cast<float*>(dev + q_bytes + kv_bytes);
        d_err = reinterpret_cast<std::uint32_t*>(dev + err_offset);
        d_out = reinterpret_cast<float*>(dev + out_offset);
        cuda_check(cudaMemsetAsync(d_err, 0, 16, ctx.stream), "cudaMemsetAsync");
    }

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
    // One warp per (query, head) row, and at least one CTA per 8192 input
    // values for the finite check (CTAs past the last row only check).
    const std::size_t row_ctas = (rows + kGenericWarps - 1) / kGenericWarps;
    const std::size_t check_ctas = std::min<std::size_t>((query_values + 2 * kv_values + 8191) / 8192,
                                                         148 * 8);
    const unsigned grid = static_cast<unsigned>(std::max(row_ctas, check_ctas));
    generic_attention_kernel<ContiguousKv>
        <<<grid, kGenericWarps * 32, smem, ctx.stream>>>(params, kv, segments);
    cuda_check(cudaGetLastError(), "attention kernel launch");

    finish_from_device(ctx, host + err_offset, dev + err_offset, dev + out_offset, q_bytes, output,
                       [](const std::uint32_t* words) {
                           const std::uint32_t bits = words[0];
                           if (bits & kErrNonFinite) {
                               throw std::runtime_error("attention input must be finite");
                           }
                           if (bits & kErrNormalizer) {
                               throw std::runtime_error("online attention normalizer is invalid");
                           }
                           if (bits != 0) throw std::runtime_error(describe_error_bits(bits));
                           return true;
                       });
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
