// kv_pool.cu - the HBM block pool: creation, error readback, and the two data
// movement kernels of PagedKvPool (worker/cpp/inferlab_runtime.cpp:649-1026):
//   K1 kv_append: token rows -> (table[pos / block_tokens], pos % block_tokens)
//   K2 kv_gather: a sequence's blocks -> contiguous [tokens][kv_heads][head_dim]
// The pool's allocation policy (free list, refcounts, prefix LRU, copy on
// write) stays on the host; only block ids cross to the device.
#include "common.cuh"
#include "internal.cuh"
#include "pool.cuh"

#include "../../include/inferlab_attention.h"

#include <memory>
#include <type_traits>

namespace ilb {
namespace {

constexpr int kAppendThreads = 128;

template <typename PoolT, typename RowT>
__global__ void __launch_bounds__(kAppendThreads)
    kv_append_kernel(PoolT* key_arena, PoolT* value_arena, const RowT* key_rows,
                     const RowT* value_rows, const std::int32_t* row_sequences,
                     const std::int32_t* positions, const std::int32_t* tables,
                     std::uint32_t max_blocks, std::uint64_t num_blocks, std::uint32_t kv_heads,
                     std::uint32_t block_tokens, std::uint32_t head_dim,
                     std::uint32_t* error_word) {
    const std::size_t row = blockIdx.x;
    const std::size_t width = static_cast<std::size_t>(kv_heads) * head_dim;
    const RowT* key_src = key_rows + row * width;
    const RowT* value_src = value_rows + row * width;

    // The reference's prepare() rejects non-finite K/V (kernels/attention_cpu.cpp:
    // 131-134); the pool rejects them when they arrive instead of on every read.
    bool bad = false;
    for (std::size_t i = threadIdx.x; i < width; i += blockDim.x) {
        bad |= !isfinite(Storage<RowT>::to_float(key_src[i]));
        bad |= !isfinite(Storage<RowT>::to_float(value_src[i]));
    }
    if (__syncthreads_or(bad)) {
        if (threadIdx.x == 0) flag_error(error_word, kErrNonFinite);
        return;
    }
    const std::int32_t seq = row_sequences[row];
    const std::int32_t pos = positions[row];
    if (seq < 0 || pos < 0 || static_cast<std::uint32_t>(pos) / block_tokens >= max_blocks) {
        if (threadIdx.x == 0) flag_error(error_word, kErrPosition);
        return;
    }
    const std::int32_t block =
        tables[static_cast<std::size_t>(seq) * max_blocks + static_cast<std::uint32_t>(pos) / block_tokens];
    if (block < 0 || static_cast<std::uint64_t>(block) >= num_blocks) {
        if (threadIdx.x == 0) flag_error(error_word, kErrBadBlock);
        return;
    }
    const std::uint32_t slot = static_cast<std::uint32_t>(pos) % block_tokens;
    for (std::size_t i = threadIdx.x; i < width; i += blockDim.x) {
        const std::size_t head = i / head_dim;
        const std::size_t dim = i % head_dim;
        const std::size_t dst =
            ((static_cast<std::size_t>(block) * kv_heads + head) * block_tokens + slot) * head_dim +
            dim;
        if constexpr (std::is_same<PoolT, RowT>::value) {
            key_arena[dst] = key_src[i];
            value_arena[dst] = value_src[i];
        } else {
            key_arena[dst] = Storage<PoolT>::from_float(Storage<RowT>::to_float(key_src[i]));
            value_arena[dst] = Storage<PoolT>::from_float(Storage<RowT>::to_float(value_src[i]));
        }
    }
}

// One CTA per token: copies its kv_heads rows (head_dim elements each) from the
// block the table names into the contiguous output, 16 bytes at a time when the
// row allows it. Bit-exact by construction (no conversion).
template <typename Word>
__global__ void kv_gather_kernel(const unsigned char* key_arena, const unsigned char* value_arena,
                                 const std::int32_t* table, std::uint64_t num_blocks,
                                 std::uint32_t kv_heads, std::uint32_t block_tokens,
                                 std::size_t row_bytes, unsigned char* keys_out,
                                 unsigned char* values_out, std::uint32_t* error_word) {
    const std::size_t token = blockIdx.x;
    std::int32_t block = table[token / block_tokens];
    if (block < 0 || static_cast<std::uint64_t>(block) >= num_blocks) {
        if (threadIdx.x == 0) flag_error(error_word, kErrBadBlock);
        return;
    }
    const std::size_t slot = token % block_tokens;
    const std::size_t words = row_bytes / sizeof(Word);
    for (std::size_t i = threadIdx.x; i < kv_heads * words; i += blockDim.x) {
        const std::size_t head = i / words;
        const std::size_t w = i % words;
        const std::size_t src =
            ((static_cast<std::size_t>(block) * kv_heads + head) * block_tokens + slot) * row_bytes;
        const std::size_t dst = (token * kv_heads + head) * row_bytes;
        reinterpret_cast<Word*>(keys_out + dst)[w] =
            reinterpret_cast<const Word*>(key_arena + src)[w];
        reinterpret_cast<Word*>(values_out + dst)[w] =
            reinterpret_cast<const Word*>(value_arena + src)[w];
    }
}

template <typename PoolT>
void launch_append(InferlabCudaKvPool& pool, const void* key_rows, const void* value_rows,
                   std::uint32_t row_dtype, const std::int32_t* row_sequences,
                   const std::int32_t* positions, std::uint64_t rows, const std::int32_t* tables,
                   std::uint32_t max_blocks, cudaStream_t stream) {
    auto* karena = static_cast<PoolT*>(pool.key_arena);
    auto* varena = static_cast<PoolT*>(pool.value_arena);
    const dim3 grid(static_cast<unsigned>(rows));
    if (row_dtype == kFp32) {
        kv_append_kernel<PoolT, float><<<grid, kAppendThreads, 0, stream>>>(
            karena, varena, static_cast<const float*>(key_rows),
            static_cast<const float*>(value_rows), row_sequences, positions, tables, max_blocks,
            pool.num_blocks, pool.kv_heads, pool.block_tokens, pool.head_dim, pool.error_word);
    } else {
        kv_append_kernel<PoolT, PoolT><<<grid, kAppendThreads, 0, stream>>>(
            karena, varena, static_cast<const PoolT*>(key_rows),
            static_cast<const PoolT*>(value_rows), row_sequences, positions, tables, max_blocks,
            pool.num_blocks, pool.kv_heads, pool.block_tokens, pool.head_dim, pool.error_word);
    }
}

}  // namespace
}  // namespace ilb

namespace ilb {

void launch_kv_append(InferlabCudaKvPool& pool, const void* key_rows, const void* value_rows,
                      std::uint32_t row_dtype, const std::int32_t* row_sequences,
                      const std::int32_t* positions, std::uint64_t rows,
                      const std::int32_t* block_tables, std::uint32_t max_blocks,
                      cudaStream_t stream) {
    if (pool.dtype == kFp32) {
        launch_append<float>(pool, key_rows, value_rows, row_dtype, row_sequences, positions, rows,
                             block_tables, max_blocks, stream);
    } else if (pool.dtype == kF16) {
        launch_append<__half>(pool, key_rows, value_rows, row_dtype, row_sequences, positions,
                              rows, block_tables, max_blocks, stream);
    } else {
        launch_append<__nv_bfloat16>(pool, key_rows, value_rows, row_dtype, row_sequences,
                                     positions, rows, block_tables, max_blocks, stream);
    }
    cuda_check(cudaGetLastError(), "kv_append launch");
}

}  // namespace ilb

extern "C" int inferlab_cuda_pool_create(std::int32_t device, std::uint32_t dtype,
                                         std::uint64_t num_blocks, std::uint32_t block_tokens,
                                         std::uint32_t kv_heads, std::uint32_t head_dim,
                                         InferlabCudaKvPool** pool, char* error,
                                         std::size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        using namespace ilb;
        if (pool == nullptr) throw std::runtime_error("paged KV pool output pointer is null");
        *pool = nullptr;
        if (dtype > 2) throw std::runtime_error("paged KV dtype must be 0 (FP32), 1 (FP16), or 2 (BF16)");
        if (num_blocks == 0 || block_tokens == 0 || kv_heads == 0 || head_dim == 0) {
            throw std::runtime_error("paged KV cache dimensions must be positive");
        }
        if (num_blocks > 0x7FFFFFFFull) {
            throw std::runtime_error("paged KV num_blocks must fit a 32-bit block id");
        }
        int count = 0;
        cuda_check(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
        if (device < 0 || device >= count) throw std::runtime_error("CUDA device index out of range");
        DeviceGuard guard(device);
        auto owned = std::make_unique<InferlabCudaKvPool>();
        owned->device = device;
        owned->dtype = dtype;
        owned->element_bytes = dtype == kFp32 ? 4 : 2;
        owned->block_tokens = block_tokens;
        owned->kv_heads = kv_heads;
        owned->head_dim = head_dim;
        owned->num_blocks = num_blocks;
        const char* overflow = "paged KV pool size overflows";
        owned->block_bytes = checked_mul(
            checked_mul(checked_mul(block_tokens, kv_heads, overflow), head_dim, overflow),
            owned->element_bytes, overflow);
        owned->arena_bytes = checked_mul(owned->block_bytes, num_blocks, overflow);
        cuda_check(cudaMalloc(&owned->key_arena, owned->arena_bytes), "cudaMalloc key arena");
        const cudaError_t second = cudaMalloc(&owned->value_arena, owned->arena_bytes);
        if (second != cudaSuccess) {
            cudaFree(owned->key_arena);
            cuda_check(second, "cudaMalloc value arena");
        }
        cuda_check(cudaMalloc(&owned->error_word, ilb::kPoolWordBytes), "cudaMalloc error word");
        cuda_check(cudaMallocHost(&owned->error_host, 16), "cudaMallocHost");
        cuda_check(cudaMemset(owned->key_arena, 0, owned->arena_bytes), "cudaMemset");
        cuda_check(cudaMemset(owned->value_arena, 0, owned->arena_bytes), "cudaMemset");
        cuda_check(cudaMemset(owned->error_word, 0, ilb::kPoolWordBytes), "cudaMemset");
        cuda_check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
        *pool = owned.release();
    });
}

extern "C" void inferlab_cuda_pool_destroy(InferlabCudaKvPool* pool) {
    if (pool == nullptr) return;
    {
        int previous = 0;
        cudaGetDevice(&previous);
        cudaSetDevice(pool->device);
        cudaDeviceSynchronize();
        cudaFree(pool->key_arena);
        cudaFree(pool->value_arena);
        cudaFree(pool->error_word);
        cudaFreeHost(pool->error_host);
        if (pool->step_host != nullptr) cudaFreeHost(pool->step_host);
        if (pool->step_device != nullptr) cudaFree(pool->step_device);
        cudaSetDevice(previous);
    }
    delete pool;
}

extern "C" int inferlab_cuda_pool_info(const InferlabCudaKvPool* pool, InferlabCudaPoolInfo* info,
                                       char* error, std::size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        const auto& p = ilb::checked_pool(pool);
        if (info == nullptr) throw std::runtime_error("paged KV info pointer is null");
        info->device = p.device;
        info->dtype = p.dtype;
        info->block_tokens = p.block_tokens;
        info->kv_heads = p.kv_heads;
        info->head_dim = p.head_dim;
        info->element_bytes = p.element_bytes;
        info->num_blocks = p.num_blocks;
        info->block_bytes = p.block_bytes;
        info->arena_bytes = p.arena_bytes;
        info->key_arena = p.key_arena;
        info->value_arena = p.value_arena;
    });
}

extern "C" int inferlab_cuda_pool_synchronize(InferlabCudaKvPool* pool, void* stream,
                                              std::uint32_t timeout_ms, char* error,
                                              std::size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        using namespace ilb;
        auto& p = checked_pool(pool);
        DeviceGuard guard(p.device);
        std::lock_guard<std::mutex> lock(p.mutex);
        auto s = static_cast<cudaStream_t>(stream);
        cuda_check(cudaMemcpyAsync(p.error_host, p.error_word, sizeof(std::uint32_t),
                                   cudaMemcpyDeviceToHost, s),
                   "cudaMemcpyAsync error word");
        wait_stream(s, timeout_ms);
        const std::uint32_t bits = *p.error_host;
        if (bits != 0) {
            cuda_check(cudaMemsetAsync(p.error_word, 0, sizeof(std::uint32_t), s), "cudaMemsetAsync");
            wait_stream(s, timeout_ms);
            throw std::runtime_error(describe_error_bits(bits));
        }
    });
}

extern "C" int inferlab_cuda_kv_append(InferlabCudaKvPool* pool, const void* key_rows,
                                       const void* value_rows, std::uint32_t row_dtype,
                                       const std::int32_t* row_sequences,
                                       const std::int32_t* positions, std::uint64_t rows,
                                       const std::int32_t* block_tables,
                                       std::uint32_t max_blocks_per_seq, void* stream, char* error,
                                       std::size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        using namespace ilb;
        auto& p = checked_pool(pool);
        if (rows == 0) return;
        if (key_rows == nullptr || value_rows == nullptr || row_sequences == nullptr ||
            positions == nullptr || block_tables == nullptr) {
            throw std::runtime_error("paged KV append pointer is null");
        }
        if (row_dtype != kFp32 && row_dtype != p.dtype) {
            throw std::runtime_error("paged KV row dtype must be FP32 or the pool dtype");
        }
        if (max_blocks_per_seq == 0) throw std::runtime_error("paged KV block table is empty");
        if (rows > 0x7FFFFFFFull) throw std::runtime_error("paged KV append row count is too large");
        DeviceGuard guard(p.device);
        auto s = static_cast<cudaStream_t>(stream);
        if (p.dtype == kFp32) {
            launch_append<float>(p, key_rows, value_rows, row_dtype, row_sequences, positions, rows,
                                 block_tables, max_blocks_per_seq, s);
        } else if (p.dtype == kF16) {
            launch_append<__half>(p, key_rows, value_rows, row_dtype, row_sequences, positions,
                                  rows, block_tables, max_blocks_per_seq, s);
        } else {
            launch_append<__nv_bfloat16>(p, key_rows, value_rows, row_dtype, row_sequences,
                                         positions, rows, block_tables, max_blocks_per_seq, s);
        }
        cuda_check(cudaGetLastError(), "kv_append launch");
    });
}

extern "C" int inferlab_cuda_kv_gather(InferlabCudaKvPool* pool, const std::int32_t* block_table,
                                       std::uint64_t tokens, void* keys_out, void* values_out,
                                       void* stream, char* error, std::size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        using namespace ilb;
        auto& p = checked_pool(pool);
        if (tokens == 0) return;
        if (block_table == nullptr || keys_out == nullptr || values_out == nullptr) {
            throw std::runtime_error("paged KV gather pointer is null");
        }
        if (tokens > 0x7FFFFFFFull) throw std::runtime_error("paged KV gather is too long");
        DeviceGuard guard(p.device);
        auto s = static_cast<cudaStream_t>(stream);
        const std::size_t row_bytes = static_cast<std::size_t>(p.head_dim) * p.element_bytes;
        const auto* ka = static_cast<const unsigned char*>(p.key_arena);
        const auto* va = static_cast<const unsigned char*>(p.value_arena);
        auto* ko = static_cast<unsigned char*>(keys_out);
        auto* vo = static_cast<unsigned char*>(values_out);
        const bool aligned16 = row_bytes % 16 == 0 &&
                               reinterpret_cast<std::uintptr_t>(keys_out) % 16 == 0 &&
                               reinterpret_cast<std::uintptr_t>(values_out) % 16 == 0;
        const dim3 grid(static_cast<unsigned>(tokens));
        if (aligned16) {
            kv_gather_kernel<uint4><<<grid, 128, 0, s>>>(ka, va, block_table, p.num_blocks,
                                                         p.kv_heads, p.block_tokens, row_bytes, ko,
                                                         vo, p.error_word);
        } else {
            kv_gather_kernel<std::uint16_t><<<grid, 128, 0, s>>>(
                ka, va, block_table, p.num_blocks, p.kv_heads, p.block_tokens, row_bytes, ko, vo,
                p.error_word);
        }
        cuda_check(cudaGetLastError(), "kv_gather launch");
    });
}
