// decode_step.cu - one continuous-batching decode step with host buffers.
//
// The reference's paged decode runs per sequence on the host: append the new
// token's K/V row (PagedKvPool::append, worker/cpp/inferlab_runtime.cpp:
// 713-767), gather the pages (materialize, :769-803) and call
// attention_forward (:1458-1470), once for every active sequence
// (worker/src/scheduler.rs:268-270). inferlab_cuda_decode_step_host is that
// whole step for a batch in one synchronous call. When the caller's arrays are
// page-locked and mapped, a prologue kernel reads them over the bus (appending
// every new row and staging the decode's inputs), one decode launch covers all
// sequences and writes the output straight into the caller's array, and a
// 4-byte copy brings the pool's error word back. Otherwise the inputs cross to
// HBM by copies (packed into pinned staging for pageable arrays), kv_append
// writes the rows, and the output comes back by copy. The K/V history stays
// in the HBM pool.
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

// Device-accessible address of page-locked host memory (mapped into the
// current device's address space), or nullptr.
const void* mapped_host(const void* ptr) {
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, ptr) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return attr.type == cudaMemoryTypeHost ? attr.devicePointer : nullptr;
}

// The fused step prologue reads the caller's page-locked arrays over the bus
// itself (no copy calls): CTAs [0, num_seqs) append one sequence's new K/V
// row each, the rest copy the queries, tables and lengths into device staging
// for the decode launch and zero its split counters.
struct StepPrologue {
    const unsigned char* src[3];
    unsigned char* dst[3];
    std::size_t bytes[3];
    std::uint32_t* counters;
    std::size_t counter_words;
    const float* keys;    // host-mapped [num_seqs][kv_heads * head_dim]
    const float* values;
    const std::int32_t* lens;    // host-mapped [num_seqs]
    const std::int32_t* tables;  // host-mapped [num_seqs][max_blocks]
    const std::int32_t* block_copies;  // host-mapped [num_seqs][2] (from, to), or nullptr
    std::size_t block_bytes;           // one block of one arena, all kv-heads
    std::uint32_t max_blocks;
    void* key_arena;
    void* value_arena;
    std::uint64_t num_blocks;
    std::uint32_t kv_heads, block_tokens, head_dim;
    std::uint32_t append_ctas;  // num_seqs when rows are appended, else 0
    std::uint32_t copy_ctas;
    std::uint32_t* error_word;
};

constexpr int kPrologueThreads = 256;
constexpr int kPrologueCopyCtas = 64;

__device__ __forceinline__ void copy_range(const unsigned char* src, unsigned char* dst, std::size_t bytes,
                                           std::size_t t, std::size_t stride) {
    if (((reinterpret_cast<std::uintptr_t>(src) | reinterpret_cast<std::uintptr_t>(dst) | bytes) & 15) == 0) {
        const auto* s4 = reinterpret_cast<const uint4*>(src);
        auto* d4 = reinterpret_cast<uint4*>(dst);
        for (std::size_t i = t; i < bytes / 16; i += stride) d4[i] = s4[i];
    } else {
        // Every staged array is a whole number of 4-byte elements.
        const auto* s1 = reinterpret_cast<const std::uint32_t*>(src);
        auto* d1 = reinterpret_cast<std::uint32_t*>(dst);
        for (std::size_t i = t; i < bytes / 4; i += stride) d1[i] = s1[i];
    }
}

template <typename PoolT>
__global__ void __launch_bounds__(kPrologueThreads) step_prologue_kernel(const StepPrologue p) {
    if (blockIdx.x >= p.append_ctas) {
        const std::size_t t = static_cast<std::size_t>(blockIdx.x - p.append_ctas) * blockDim.x + threadIdx.x;
        const std::size_t stride = static_cast<std::size_t>(p.copy_ctas) * blockDim.x;
#pragma unroll
        for (int r = 0; r < 3; ++r) copy_range(p.src[r], p.dst[r], p.bytes[r], t, stride);
        for (std::size_t i = t; i < p.counter_words; i += stride) p.counters[i] = 0u;
        return;
    }
    const std::size_t s = blockIdx.x;
    // Copy on write first: the sequence's shared tail block is copied whole
    // into its private block (both arenas), then the new row goes there
    // (PagedKvPool::append, worker/cpp/inferlab_runtime.cpp:738-754).
    if (p.block_copies != nullptr) {
        const std::int32_t from = p.block_copies[s * 2];
        const std::int32_t to = p.block_copies[s * 2 + 1];
        if (from >= 0) {
            for (int arena = 0; arena < 2; ++arena) {
                const auto* src = reinterpret_cast<const uint4*>(
                    static_cast<const unsigned char*>(arena ? p.value_arena : p.key_arena) +
                    static_cast<std::size_t>(from) * p.block_bytes);
                auto* dst = reinterpret_cast<uint4*>(static_cast<unsigned char*>(arena ? p.value_arena : p.key_arena) +
                                                     static_cast<std::size_t>(to) * p.block_bytes);
                for (std::size_t i = threadIdx.x; i < p.block_bytes / 16; i += blockDim.x) dst[i] = src[i];
            }
            __syncthreads();
        }
    }
    // Append: the row lands in shared memory first, so a non-finite element
    // rejects the whole row before any of it is written (the reference's
    // prepare() rejects non-finite K/V, kernels/attention_cpu.cpp:131-134).
    extern __shared__ float row_buf[];  // [2][width]
    __shared__ std::int32_t block_slot[2];
    const std::size_t width = static_cast<std::size_t>(p.kv_heads) * p.head_dim;
    bool bad = false;
    for (std::size_t i = threadIdx.x; i < width; i += blockDim.x) {
        const float k = p.keys[s * width + i];
        const float v = p.values[s * width + i];
        bad |= !isfinite(k) || !isfinite(v);
        row_buf[i] = k;
        row_buf[width + i] = v;
    }
    if (threadIdx.x == 0) {
        // The new token sits at the last position of the context; the host
        // has checked 1 <= length <= max_blocks * block_tokens.
        const std::int32_t pos = p.lens[s] - 1;
        std::int32_t block = -1;
        if (pos >= 0 && static_cast<std::uint32_t>(pos) / p.block_tokens < p.max_blocks) {
            block = p.tables[s * p.max_blocks + static_cast<std::uint32_t>(pos) / p.block_tokens];
        }
        block_slot[0] = block;
        block_slot[1] = pos;
    }
    if (__syncthreads_or(bad)) {
        if (threadIdx.x == 0) flag_error(p.error_word, kErrNonFinite);
        return;
    }
    const std::int32_t block = block_slot[0];
    const std::int32_t pos = block_slot[1];
    if (pos < 0 || static_cast<std::uint32_t>(pos) / p.block_tokens >= p.max_blocks) {
        if (threadIdx.x == 0) flag_error(p.error_word, kErrPosition);
        return;
    }
    if (block < 0 || static_cast<std::uint64_t>(block) >= p.num_blocks) {
        if (threadIdx.x == 0) flag_error(p.error_word, kErrBadBlock);
        return;
    }
    const std::uint32_t slot = static_cast<std::uint32_t>(pos) % p.block_tokens;
    auto* karena = static_cast<PoolT*>(p.key_arena);
    auto* varena = static_cast<PoolT*>(p.value_arena);
    for (std::size_t i = threadIdx.x; i < width; i += blockDim.x) {
        const std::size_t head = i / p.head_dim;
        const std::size_t dim = i % p.head_dim;
        const std::size_t dst =
            ((static_cast<std::size_t>(block) * p.kv_heads + head) * p.block_tokens + slot) * p.head_dim + dim;
        karena[dst] = Storage<PoolT>::from_float(row_buf[i]);
        varena[dst] = Storage<PoolT>::from_float(row_buf[width + i]);
    }
}

}  // namespace
}  // namespace ilb

namespace ilb {
namespace {

int decode_step_host(InferlabCudaKvPool* pool, const float* queries, const float* new_keys,
                     const float* new_values, const std::int32_t* block_copies,
                     const std::int32_t* block_tables, std::uint32_t max_blocks_per_seq,
                     const std::int32_t* context_lens, std::uint32_t num_seqs, std::uint32_t q_heads,
                     float* out, void* stream, std::uint32_t timeout_ms, char* error,
                     std::size_t error_capacity) {
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
        // Host-side checks of the step's context lengths. The block ids are
        // checked where they are read, by the append and decode kernels (the
        // reference's materialize checks, worker/cpp/inferlab_runtime.cpp:776-789):
        // an id outside the pool is never dereferenced and fails the call with
        // the same message. Scanning every used table entry on the host cost
        // 115-200 us per call on the 256-sequence long-context step.
        std::uint32_t max_context = 0;
        const std::uint64_t capacity = static_cast<std::uint64_t>(max_blocks_per_seq) * p.block_tokens;
        for (std::uint32_t s = 0; s < num_seqs; ++s) {
            const std::int32_t ctx = context_lens[s];
            if (ctx < 1 || static_cast<std::uint64_t>(ctx) > capacity) {
                throw std::runtime_error("paged KV context length is invalid");
            }
            max_context = std::max(max_context, static_cast<std::uint32_t>(ctx));
        }
        const bool append = new_keys != nullptr;
        const std::size_t block_bytes =
            static_cast<std::size_t>(p.kv_heads) * p.block_tokens * p.head_dim * p.element_bytes;
        bool any_copy = false;
        if (block_copies != nullptr) {
            if (!append) throw std::runtime_error("decode step block copies need new key and value rows");
            for (std::uint32_t s = 0; s < num_seqs; ++s) {
                const std::int32_t from = block_copies[2 * s];
                const std::int32_t to = block_copies[2 * s + 1];
                if (from < 0 && to < 0) continue;
                if (from < 0 || to < 0 || static_cast<std::uint64_t>(from) >= p.num_blocks ||
                    static_cast<std::uint64_t>(to) >= p.num_blocks || from == to) {
                    throw std::runtime_error("paged KV block table contains an invalid page");
                }
                any_copy = true;
            }
        }
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
        // Caller buffers page-locked and mapped into the device's address
        // space: one prologue kernel reads them over the bus (appending the
        // new rows and staging the decode's inputs), the decode writes the
        // output straight into the caller's buffer, and only the error word
        // is copied back - two launches and one copy per step.
        const void* m_q = mapped_host(queries);
        const void* m_tables = mapped_host(block_tables);
        const void* m_lens = mapped_host(context_lens);
        void* m_out = const_cast<void*>(mapped_host(out));
        const void* m_k = append ? mapped_host(new_keys) : nullptr;
        const void* m_v = append ? mapped_host(new_values) : nullptr;
        const void* m_copies = any_copy ? mapped_host(block_copies) : nullptr;
        const std::size_t width_bytes = static_cast<std::size_t>(p.kv_heads) * p.head_dim * 8;
        if (m_q != nullptr && m_tables != nullptr && m_lens != nullptr && m_out != nullptr &&
            (!append || (m_k != nullptr && m_v != nullptr)) && (!any_copy || m_copies != nullptr) &&
            block_bytes % 16 == 0 && width_bytes <= 48 * 1024 &&
            reinterpret_cast<std::uintptr_t>(m_q) % 4 == 0 &&
            reinterpret_cast<std::uintptr_t>(m_out) % 4 == 0) {
            StepPrologue pr{};
            pr.src[0] = static_cast<const unsigned char*>(m_q);
            pr.dst[0] = d + l.q;
            pr.bytes[0] = q_bytes;
            pr.src[1] = static_cast<const unsigned char*>(m_tables);
            pr.dst[1] = d + l.tables;
            pr.bytes[1] = table_bytes;
            pr.src[2] = static_cast<const unsigned char*>(m_lens);
            pr.dst[2] = d + l.lens;
            pr.bytes[2] = static_cast<std::size_t>(num_seqs) * 4;
            pr.counters = reinterpret_cast<std::uint32_t*>(d + l.workspace);
            pr.counter_words = decode_counter_bytes(p, num_seqs) / 4;
            pr.keys = static_cast<const float*>(m_k);
            pr.values = static_cast<const float*>(m_v);
            pr.lens = static_cast<const std::int32_t*>(m_lens);
            pr.tables = static_cast<const std::int32_t*>(m_tables);
            pr.block_copies = static_cast<const std::int32_t*>(m_copies);
            pr.block_bytes = block_bytes;
            pr.max_blocks = max_blocks_per_seq;
            pr.key_arena = p.key_arena;
            pr.value_arena = p.value_arena;
            pr.num_blocks = p.num_blocks;
            pr.kv_heads = p.kv_heads;
            pr.block_tokens = p.block_tokens;
            pr.head_dim = p.head_dim;
            pr.append_ctas = append ? num_seqs : 0u;
            pr.copy_ctas = kPrologueCopyCtas;
            pr.error_word = p.error_word;
            const unsigned grid = pr.append_ctas + pr.copy_ctas;
            const std::size_t smem = append ? width_bytes : 0;
            if (p.dtype == kFp32) {
                step_prologue_kernel<float><<<grid, kPrologueThreads, smem, s>>>(pr);
            } else if (p.dtype == kF16) {
                step_prologue_kernel<__half><<<grid, kPrologueThreads, smem, s>>>(pr);
            } else {
                step_prologue_kernel<__nv_bfloat16><<<grid, kPrologueThreads, smem, s>>>(pr);
            }
            cuda_check(cudaGetLastError(), "step prologue launch");
            launch_paged_decode(p, reinterpret_cast<const float*>(d + l.q),
                                reinterpret_cast<const std::int32_t*>(d + l.tables), max_blocks_per_seq,
                                reinterpret_cast<const std::int32_t*>(d + l.lens), num_seqs, q_heads,
                                max_context, static_cast<float*>(m_out), d + l.workspace,
                                p.step_capacity - l.workspace, s);
            cuda_check(cudaMemcpyAsync(h + l.err, p.error_word, 4, cudaMemcpyDeviceToHost, s),
                       "cudaMemcpyAsync step error word");
            wait_stream(s, timeout_ms);
            std::uint32_t bits = 0;
            std::memcpy(&bits, h + l.err, 4);
            if (bits != 0) {
                cuda_check(cudaMemsetAsync(p.error_word, 0, 4, s), "cudaMemsetAsync error word");
                wait_stream(s, timeout_ms);
                throw std::runtime_error(describe_error_bits(bits));
            }
            return;
        }
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
        for (std::uint32_t i = 0; any_copy && i < num_seqs; ++i) {
            if (block_copies[2 * i] < 0) continue;
            for (unsigned char* arena : {static_cast<unsigned char*>(p.key_arena),
                                         static_cast<unsigned char*>(p.value_arena)}) {
                cuda_check(cudaMemcpyAsync(arena + static_cast<std::size_t>(block_copies[2 * i + 1]) * block_bytes,
                                           arena + static_cast<std::size_t>(block_copies[2 * i]) * block_bytes,
                                           block_bytes, cudaMemcpyDeviceToDevice, s),
                           "cudaMemcpyAsync block copy");
            }
        }
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

}  // namespace
}  // namespace ilb

extern "C" int inferlab_cuda_decode_step_host(
    InferlabCudaKvPool* pool, const float* queries, const float* new_keys, const float* new_values,
    const std::int32_t* block_tables, std::uint32_t max_blocks_per_seq,
    const std::int32_t* context_lens, std::uint32_t num_seqs, std::uint32_t q_heads, float* out,
    void* stream, std::uint32_t timeout_ms, char* error, std::size_t error_capacity) {
    return ilb::decode_step_host(pool, queries, new_keys, new_values, nullptr, block_tables,
                                 max_blocks_per_seq, context_lens, num_seqs, q_heads, out, stream,
                                 timeout_ms, error, error_capacity);
}

extern "C" int inferlab_cuda_decode_step_host_cow(
    InferlabCudaKvPool* pool, const float* queries, const float* new_keys, const float* new_values,
    const std::int32_t* block_copies, const std::int32_t* block_tables,
    std::uint32_t max_blocks_per_seq, const std::int32_t* context_lens, std::uint32_t num_seqs,
    std::uint32_t q_heads, float* out, void* stream, std::uint32_t timeout_ms, char* error,
    std::size_t error_capacity) {
    return ilb::decode_step_host(pool, queries, new_keys, new_values, block_copies, block_tables,
                                 max_blocks_per_seq, context_lens, num_seqs, q_heads, out, stream,
                                 timeout_ms, error, error_capacity);
}
