// pool.cuh - the HBM-resident paged KV pool shared by the append, gather,
// decode and prefill kernels.
#pragma once

#include "common.cuh"

#include <atomic>
#include <mutex>

struct InferlabCudaKvPool {
    int device = 0;
    std::uint32_t dtype = 0;
    std::uint32_t element_bytes = 4;
    std::uint32_t block_tokens = 16;
    std::uint32_t kv_heads = 1;
    std::uint32_t head_dim = 1;
    std::uint64_t num_blocks = 0;
    std::uint64_t block_bytes = 0;  // one block, all kv-heads, one arena
    std::uint64_t arena_bytes = 0;
    void* key_arena = nullptr;
    void* value_arena = nullptr;
    std::uint32_t* error_word = nullptr;       // device: error word, then work-queue counters
    std::uint32_t* error_host = nullptr;       // pinned mirror
    std::mutex mutex;                          // guards error_host / error readback
    // Grow-only staging of the host-buffer step entry (decode_step.cu).
    std::mutex step_mutex;
    unsigned char* step_host = nullptr;        // pinned
    unsigned char* step_device = nullptr;
    std::size_t step_capacity = 0;
    // Persistent prefill launches take their work-queue counter pair
    // (next item, CTAs finished) round-robin from kSchedulerSlots pairs that
    // follow the error word; each launch returns its pair to zero on exit.
    std::atomic<std::uint32_t> scheduler_next{0};
    // Decode split length in 16-token blocks (0: the planner chooses);
    // inferlab_cuda_pool_set_decode_split sets it.
    std::uint32_t decode_blocks_per_split = 0;
};

namespace ilb {

constexpr std::uint32_t kSchedulerSlots = 64;
// Device words behind pool.error_word: the error word (16 bytes), then the
// work-queue counter pairs.
constexpr std::size_t kPoolWordBytes = 16 + kSchedulerSlots * 2 * sizeof(std::uint32_t);

inline InferlabCudaKvPool& checked_pool(InferlabCudaKvPool* pool) {
    if (pool == nullptr) throw std::runtime_error("paged KV pool pointer is null");
    return *pool;
}

inline const InferlabCudaKvPool& checked_pool(const InferlabCudaKvPool* pool) {
    if (pool == nullptr) throw std::runtime_error("paged KV pool pointer is null");
    return *pool;
}

// Bytes of one kv-head's block tile in one arena.
inline std::size_t head_tile_bytes(const InferlabCudaKvPool& pool) {
    return static_cast<std::size_t>(pool.block_tokens) * pool.head_dim * pool.element_bytes;
}

}  // namespace ilb
