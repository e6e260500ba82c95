// decode_step.cu - one continuous-batching decode step with host buffers.
//
// The reference's paged decode runs per sequence on the host: append the new
// token's K/V row (PagedKvPool::append, worker/cpp/inferlab_runtime.cpp:
// 713-767), gather the pages (materialize, :769-803) and call
// attention_forward (:1458-1470), once for every active sequence
// (worker/src/scheduler.rs:268-270). inferlab_cuda_decode_step_host is that
// whole step for a batch in one synchronous call: the step's inputs are packed
// into pinned staging and cross to HBM in one copy, kv_append writes every new
// row, one decode launch covers all sequences, and one copy brings the output
// and the pool's error word back. The K/V history stays in the HBM pool.
#include "common.cuh"
#include "internal.cuh"
#include "pool.cuh"

#include "../../include/inferlab_attention.h"

#include <algorithm>
#include <cstring>

namespace ilb {
namespace {

std::size_t align256(std::size_t n) { return (n + 255) & ~static_cast<std::size_t>(255); }

struct StepLayout {
    std::size_t q, k, v, tables, lens, pos, seq, out, err, inputs_end, total, workspace;
};

StepLayout layout_for(const InferlabCudaKvPool& p, std::uint32_t num_seqs, std::uint32_t q_heads,
                      std::uint32_t max_blocks, bool append, std::size_t workspace_bytes) {
    StepLayout l{};
    const std::size_t q_bytes = static_cast<std::size_t>(num_seqs) * q_heads * p.head_dim * 4;
    const std::size_t row_bytes =
        append ? static_cast<std::size_t>(num_seqs) * p.kv_heads * p.head_dim * 4 : 0;
    std::size_t at = 0;
    l.q = at;
    at = align256(at + q_bytes);
    l.k = at;
    at = align256(at + row_bytes);
    l.v = at;
    at = align256(at + row_bytes);
    l.tables = at;
    at = align256(at + static_cast<std::size_t>(num_seqs) * max_blocks * 4);
    l.lens = at;
    at = align256(at + static_cast<std::size_t>(num_seqs) * 4);
    l.pos = at;
    at = align256(at + static_cast<std::size_t>(num_seqs) * 4);
    l.seq = at;
    at = align256(at + static_cast<std::size_t>(num_seqs) * 4);
    l.inputs_end = at;
    l.err = at;  // error word copy (device -> host), 16 bytes
    at = align256(at + 16);
    l.out = at;
    at = align256(at + q_bytes);
    l.workspace = at;
    l.total = at + workspace_bytes;
    return l;
}

// Grow-only pinned + device staging (one allocation each, reused across steps).
// Page-locked host memory (cudaHostAlloc / cudaHostRegister): the DMA engine
// can read and write it directly, so the step skips the staging memcpy.
bool is_pinned(const void* ptr) {
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, ptr) != cudaSuccess) {
        cudaGetLastError();  // pageable memory on old runtimes reports an error; clear it
        return false;
    }
    return attr.type == cudaMemoryTypeHost;
}

void reserve_step(InferlabCudaKvPool& p, std::size_t bytes, cudaStream_t stream) {
    if (bytes <= p.step_capacity) return;
    wait_stream(stream, 0);  // no step may still be using the old buffers
    const std::size_t grown = bytes + bytes / 4;
    if (p.step_host != nullptr) cudaFreeHost(p.step_host);
    if (p.step_device != nullptr) cudaFree(p.step_device);
    p.step_host = nullptr;
    p.step_device = nullptr;
    p.step_capacity = 0;
    cuda_check(cudaMallocHost(&p.step_host, grown), "cudaMallocHost step staging");
    cuda_check(cudaMalloc(&p.step_device, grown), "cudaMalloc step staging");
    p.step_capacity = grown;
}

}  // namespace
}  // namespace ilb

extern "C" int inferlab_cuda_decode_step_host(
    InferlabCudaKvPool* pool, const float* queries, const float* new_keys, const float* new_values,
    const std::int32_t* block_tables, std::uint32_t max_blocks_per_seq,
    const std::int32_t* context_lens, std::uint32_t num_seqs, std::uint32_t q_heads, float* out,
    void* stream, std::uint32_t timeout_ms, char* error, std::size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        using namespace ilb;
        auto& p = checked_pool(pool);
        if (num_seqs == 0) return;
        if (queries == nullptr || block_tables == nullptr || context_lens == nullptr ||
            out == nullptr) {
            throw std::runtime_error("decode step pointer is null");
        }
        if ((new_keys == nullptr) != (new_values == nullptr)) {
            throw std::runtime_error("decode step needs both new key and value rows, or neither");
        }
        if (q_heads == 0 || q_heads % p.kv_heads != 0) {
            throw std::runtime_error("paged decode q_heads must be a positive multiple of kv_heads");
        }
        if (max_blocks_per_seq == 0) throw std::runtime_error("paged KV block table is empty");
        // Host-side checks of the step's block tables (the reference's
        // materialize checks, worker/cpp/inferlab_runtime.cpp:776-789).
        std::uint32_t max_context = 0;
        const std::uint64_t capacity = static_cast<std::uint64_t>(max_blocks_per_seq) * p.block_tokens;
        for (std::uint32_t s = 0; s < num_seqs; ++s) {
            const std::int32_t ctx = context_lens[s];
            if (ctx < 1 || static_cast<std::uint64_t>(ctx) > capacity) {
                throw std::runtime_error("paged KV context length is invalid");
            }
            const std::uint32_t nblk = (static_cast<std::uint32_t>(ctx) + p.block_tokens - 1) / p.block_tokens;
            const std::int32_t* row = block_tables + static_cast<std::size_t>(s) * max_blocks_per_seq;
            for (std::uint32_t b = 0; b < nblk; ++b) {
                if (row[b] < 0 || static_cast<std::uint64_t>(row[b]) >= p.num_blocks) {
                    throw std::runtime_error("paged KV block table contains an invalid page");
                }
            }
            max_context = std::max(max_context, static_cast<std::uint32_t>(ctx));
        }
        const bool append = new_keys != nullptr;
        const std::size_t ws_bytes = decode_workspace_bytes(p, num_seqs, q_heads, max_context);
        const StepLayout l = layout_for(p, num_seqs, q_heads, max_blocks_per_seq, append, ws_bytes);

        DeviceGuard guard(p.device);
        std::lock_guard<std::mutex> lock(p.step_mutex);
        auto s = static_cast<cudaStream_t>(stream);
        reserve_step(p, l.total, s);
        unsigned char* h = p.step_host;
        unsigned char* d = p.step_device;
        const std::size_t q_bytes = static_cast<std::size_t>(num_seqs) * q_heads * p.head_dim * 4;
        const std::size_t row_bytes = static_cast<std::size_t>(num_seqs) * p.kv_heads * p.head_dim * 4;
        const std::size_t table_bytes = static_cast<std::size_t>(num_seqs) * max_blocks_per_seq * 4;
        // Caller buffers already page-locked: copy them straight to HBM (and
        // the output straight back) instead of through the staging buffer.
        const bool direct = is_pinned(queries) && is_pinned(block_tables) &&
                            is_pinned(context_lens) && is_pinned(out) &&
                            (!append || (is_pinned(new_keys) && is_pinned(new_values)));
        auto* pos = reinterpret_cast<std::int32_t*>(h + l.pos);
        auto* seq = reinterpret_cast<std::int32_t*>(h + l.seq);
        for (std::uint32_t i = 0; i < num_seqs; ++i) {
            pos[i] = context_lens[i] - 1;  // the new token sits at the last position
            seq[i] = static_cast<std::int32_t>(i);
        }
        if (direct) {
            cuda_check(cudaMemcpyAsync(d + l.pos, h + l.pos, l.inputs_end - l.pos, cudaMemcpyHostToDevice, s),
                       "cudaMemcpyAsync step positions");
            cuda_check(cudaMemcpyAsync(d + l.tables, block_tables, table_bytes, cudaMemcpyHostToDevice, s),
                       "cudaMemcpyAsync step tables");
            cuda_check(cudaMemcpyAsync(d + l.lens, context_lens, static_cast<std::size_t>(num_seqs) * 4,
                                       cudaMemcpyHostToDevice, s),
                       "cudaMemcpyAsync step lengths");
            if (append) {
                cuda_check(cudaMemcpyAsync(d + l.k, new_keys, row_bytes, cudaMemcpyHostToDevice, s),
                           "cudaMemcpyAsync step keys");
                cuda_check(cudaMemcpyAsync(d + l.v, new_values, row_bytes, cudaMemcpyHostToDevice, s),
                           "cudaMemcpyAsync step values");
            }
            cuda_check(cudaMemcpyAsync(d + l.q, queries, q_bytes, cudaMemcpyHostToDevice, s),
                       "cudaMemcpyAsync step queries");
        } else {
            std::memcpy(h + l.q, queries, q_bytes);
            if (append) {
                std::memcpy(h + l.k, new_keys, row_bytes);
                std::memcpy(h + l.v, new_values, row_bytes);
            }
            std::memcpy(h + l.tables, block_tables, table_bytes);
            std::memcpy(h + l.lens, context_lens, static_cast<std::size_t>(num_seqs) * 4);
            cuda_check(cudaMemcpyAsync(d, h, l.inputs_end, cudaMemcpyHostToDevice, s),
                       "cudaMemcpyAsync step inputs");
        }
        // The split counters at the front of the workspace start at zero.
        cuda_check(cudaMemsetAsync(d + l.workspace, 0, decode_counter_bytes(p, num_seqs), s),
                   "cudaMemsetAsync step workspace");
        const auto* d_tables = reinterpret_cast<const std::int32_t*>(d + l.tables);
        if (append) {
            launch_kv_append(p, d + l.k, d + l.v, kFp32,
                             reinterpret_cast<const std::int32_t*>(d + l.seq),
                             reinterpret_cast<const std::int32_t*>(d + l.pos), num_seqs, d_tables,
                             max_blocks_per_seq, s);
        }
        launch_paged_decode(p, reinterpret_cast<const float*>(d + l.q), d_tables,
                            max_blocks_per_seq, reinterpret_cast<const std::int32_t*>(d + l.lens),
                            num_seqs, q_heads, max_context, reinterpret_cast<float*>(d + l.out),
                            d + l.workspace, p.step_capacity - l.workspace, s);
        cuda_check(cudaMemcpyAsync(d + l.err, p.error_word, 4, cudaMemcpyDeviceToDevice, s),
                   "cudaMemcpyAsync error word");
        if (direct) {
            cuda_check(cudaMemcpyAsync(h + l.err, d + l.err, 4, cudaMemcpyDeviceToHost, s),
                       "cudaMemcpyAsync step error word");
            cuda_check(cudaMemcpyAsync(out, d + l.out, q_bytes, cudaMemcpyDeviceToHost, s),
                       "cudaMemcpyAsync step output");
        } else {
            cuda_check(cudaMemcpyAsync(h + l.err, d + l.err, l.out + q_bytes - l.err,
                                       cudaMemcpyDeviceToHost, s),
                       "cudaMemcpyAsync step output");
        }
        wait_stream(s, timeout_ms);
        std::uint32_t bits = 0;
        std::memcpy(&bits, h + l.err, 4);
        if (bits != 0) {
            cuda_check(cudaMemsetAsync(p.error_word, 0, 4, s), "cudaMemsetAsync error word");
            wait_stream(s, timeout_ms);
            throw std::runtime_error(describe_error_bits(bits));
        }
        if (!direct) std::memcpy(out, h + l.out, q_bytes);
    });
}
