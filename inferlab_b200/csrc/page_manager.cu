// page_manager.cu - block ownership for the device KV pool, kept on the host.
//
// The device pool (kv_pool.cu) is a flat arena of blocks; which sequence owns
// which block is host policy. This file provides that policy with the
// semantics of the reference's PagedKvPool (worker/cpp/inferlab_runtime.cpp:
// 649-1032), metadata only:
//   * blocks are handed out from a free list, the most recently freed first
//     (the list starts as page_count - 1, ..., 0, so the first block is 0);
//   * every block has a reference count; a block returns to the free list when
//     the count reaches zero (release, :958-971);
//   * published prefixes (token sequence -> leading blocks) hold a reference on
//     their blocks; a lookup takes the longest published prefix of a token
//     sequence (:679-708) and retains its blocks for the caller;
//   * when no block is free, the least recently used prefix is evicted
//     (:993-1008), repeatedly, before the allocation fails with
//     "paged KV cache capacity exhausted" (:973-991);
//   * appending a token to a sequence whose tail block is shared copies the
//     block first (copy on write, :710-767); the copy itself is a device
//     operation (inferlab_cuda_pages_copy), the manager only says which;
//   * statistics follow PagedKvPool::stats (:877-911) with the device pool's
//     row and block sizes.
// One mutex serialises all calls on a manager.
#include "common.cuh"
#include "pool.cuh"

#include "../../include/inferlab_attention.h"

#include <algorithm>
#include <map>
#include <memory>
#include <mutex>
#include <vector>

struct InferlabCudaPageManager {
    struct Block {
        std::uint64_t used = 0;        // token rows written
        std::uint64_t references = 0;  // sequences and prefixes holding it
        bool live = false;
    };
    struct Prefix {
        std::vector<std::int32_t> blocks;
        std::uint64_t stamp = 0;  // last use, for eviction
    };

    std::uint64_t block_tokens = 0;
    std::uint64_t row_bytes = 0;  // one token row, K and V, all kv-heads
    std::uint64_t prefix_capacity = 0;
    std::vector<Block> blocks;
    std::vector<std::int32_t> free_list;  // back = next to hand out
    std::map<std::vector<std::uint32_t>, Prefix> prefixes;
    std::uint64_t clock = 0;
    std::uint64_t prefix_hits = 0;
    std::uint64_t prefix_misses = 0;
    std::uint64_t prefix_tokens_reused = 0;
    std::uint64_t copies = 0;
    std::uint64_t evictions = 0;
    std::uint64_t allocation_failures = 0;
    std::mutex mutex;

    Block& live_block(std::int32_t id) {
        if (id < 0 || static_cast<std::uint64_t>(id) >= blocks.size() || !blocks[id].live) {
            throw std::runtime_error("paged KV block table contains an invalid page");
        }
        return blocks[id];
    }

    void retain(std::int32_t id) { ++live_block(id).references; }

    void release(std::int32_t id) {
        Block& b = live_block(id);
        if (b.references == 0) throw std::runtime_error("paged KV page reference count underflow");
        if (--b.references == 0) {
            b = Block{};
            free_list.push_back(id);
        }
    }

    void evict_oldest() {
        if (prefixes.empty()) return;
        auto oldest = prefixes.begin();
        for (auto it = prefixes.begin(); it != prefixes.end(); ++it) {
            if (it->second.stamp < oldest->second.stamp) oldest = it;
        }
        for (const std::int32_t id : oldest->second.blocks) release(id);
        prefixes.erase(oldest);
        ++evictions;
    }

    std::int32_t allocate() {
        while (free_list.empty() && !prefixes.empty()) evict_oldest();
        if (free_list.empty()) {
            ++allocation_failures;
            throw std::runtime_error("paged KV cache capacity exhausted");
        }
        const std::int32_t id = free_list.back();
        free_list.pop_back();
        Block& b = blocks[id];
        if (b.live || b.references != 0) throw std::runtime_error("paged KV free list contains a live page");
        b.live = true;
        b.used = 0;
        b.references = 1;
        return id;
    }
};

namespace {

InferlabCudaPageManager& checked(InferlabCudaPageManager* m) {
    if (m == nullptr) throw std::runtime_error("page manager is null");
    return *m;
}

}  // namespace

extern "C" int inferlab_cuda_pages_create(uint64_t page_count, uint32_t block_tokens,
                                          uint64_t row_bytes, uint64_t prefix_capacity,
                                          InferlabCudaPageManager** manager, char* error,
                                          size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        if (manager == nullptr) throw std::runtime_error("page manager output is null");
        *manager = nullptr;
        // PagedKvPool's constructor check (:661-663).
        if (page_count == 0 || block_tokens == 0 || row_bytes == 0) {
            throw std::runtime_error("paged KV cache dimensions must be positive");
        }
        if (page_count > 0x7FFFFFFFull) throw std::runtime_error("page manager holds at most 2^31 - 1 blocks");
        auto m = std::make_unique<InferlabCudaPageManager>();
        m->block_tokens = block_tokens;
        m->row_bytes = row_bytes;
        m->prefix_capacity = prefix_capacity;
        m->blocks.resize(page_count);
        m->free_list.reserve(page_count);
        for (std::uint64_t i = page_count; i-- > 0;) m->free_list.push_back(static_cast<std::int32_t>(i));
        *manager = m.release();
    });
}

extern "C" void inferlab_cuda_pages_destroy(InferlabCudaPageManager* manager) { delete manager; }

extern "C" int inferlab_cuda_pages_prepare_append(InferlabCudaPageManager* manager, int32_t* table,
                                                  uint32_t table_capacity, uint32_t* table_length,
                                                  uint64_t cached_tokens, int32_t* copy_from,
                                                  int32_t* copy_to, char* error,
                                                  size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        auto& m = checked(manager);
        if (table == nullptr || table_length == nullptr || copy_from == nullptr || copy_to == nullptr) {
            throw std::runtime_error("page manager argument is null");
        }
        std::lock_guard<std::mutex> lock(m.mutex);
        *copy_from = -1;
        *copy_to = -1;
        const std::uint64_t slot = cached_tokens % m.block_tokens;
        std::uint32_t length = *table_length;
        if (length != (cached_tokens + m.block_tokens - 1) / m.block_tokens) {
            throw std::runtime_error("paged KV block table length is inconsistent");
        }
        std::int32_t id;
        if (slot == 0) {
            if (length >= table_capacity) throw std::runtime_error("paged KV block table is full");
            id = m.allocate();
            table[length++] = id;
        } else {
            if (length == 0) throw std::runtime_error("paged KV block table is empty for a tail row");
            id = table[length - 1];
            InferlabCudaPageManager::Block* tail = &m.live_block(id);
            if (tail->used != slot) throw std::runtime_error("paged KV tail occupancy is inconsistent");
            // A shared tail is copied before it is written; make room by
            // evicting prefixes first rather than failing the copy.
            while (m.free_list.empty() && !m.prefixes.empty() && tail->references > 1) {
                m.evict_oldest();
                tail = &m.live_block(id);
            }
            if (tail->references > 1) {
                const std::int32_t fresh = m.allocate();
                m.blocks[fresh].used = slot;
                table[length - 1] = fresh;
                m.release(id);
                *copy_from = id;
                *copy_to = fresh;
                ++m.copies;
                id = fresh;
            }
        }
        auto& b = m.live_block(id);
        if (b.references != 1 || b.used != slot) {
            throw std::runtime_error("paged KV append target is not privately writable");
        }
        b.used = slot + 1;
        *table_length = length;
    });
}

extern "C" int inferlab_cuda_pages_release(InferlabCudaPageManager* manager, const int32_t* table,
                                           uint32_t length, char* error, size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        auto& m = checked(manager);
        if (table == nullptr && length != 0) throw std::runtime_error("page manager argument is null");
        std::lock_guard<std::mutex> lock(m.mutex);
        for (std::uint32_t i = 0; i < length; ++i) m.release(table[i]);
    });
}

extern "C" int inferlab_cuda_pages_publish_prefix(InferlabCudaPageManager* manager,
                                                  const uint32_t* tokens, uint64_t token_count,
                                                  const int32_t* table, uint32_t length,
                                                  uint64_t cached_tokens, char* error,
                                                  size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        auto& m = checked(manager);
        if (m.prefix_capacity == 0 || token_count == 0) return;
        if (tokens == nullptr || table == nullptr) throw std::runtime_error("page manager argument is null");
        std::lock_guard<std::mutex> lock(m.mutex);
        if (token_count > cached_tokens) throw std::runtime_error("cannot publish an incomplete paged KV prefix");
        const std::uint64_t need = (token_count + m.block_tokens - 1) / m.block_tokens;
        if (length < need) throw std::runtime_error("paged KV prefix block table is incomplete");
        std::vector<std::uint32_t> key(tokens, tokens + token_count);
        std::vector<std::int32_t> held(table, table + need);
        auto found = m.prefixes.find(key);
        if (found != m.prefixes.end()) {
            for (const std::int32_t id : held) m.retain(id);
            for (const std::int32_t id : found->second.blocks) m.release(id);
            found->second.blocks = std::move(held);
            found->second.stamp = ++m.clock;
            return;
        }
        while (m.prefixes.size() >= m.prefix_capacity) m.evict_oldest();
        for (const std::int32_t id : held) m.retain(id);
        m.prefixes.emplace(std::move(key), InferlabCudaPageManager::Prefix{std::move(held), ++m.clock});
    });
}

extern "C" int inferlab_cuda_pages_acquire_prefix(InferlabCudaPageManager* manager,
                                                  const uint32_t* tokens, uint64_t token_count,
                                                  int32_t* table, uint32_t table_capacity,
                                                  uint32_t* table_length, uint64_t* prefix_tokens,
                                                  char* error, size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        auto& m = checked(manager);
        if ((tokens == nullptr && token_count != 0) || table == nullptr || table_length == nullptr ||
            prefix_tokens == nullptr) {
            throw std::runtime_error("page manager argument is null");
        }
        std::lock_guard<std::mutex> lock(m.mutex);
        *table_length = 0;
        *prefix_tokens = 0;
        // Longest published prefix of `tokens`.
        const InferlabCudaPageManager::Prefix* best = nullptr;
        std::uint64_t best_len = 0;
        for (auto& entry : m.prefixes) {
            const auto& key = entry.first;
            if (key.size() > token_count || (best != nullptr && key.size() <= best_len)) continue;
            if (std::equal(key.begin(), key.end(), tokens)) {
                best = &entry.second;
                best_len = key.size();
            }
        }
        if (best == nullptr) {
            ++m.prefix_misses;
            return;
        }
        if (best->blocks.size() > table_capacity) throw std::runtime_error("paged KV block table is full");
        for (const std::int32_t id : best->blocks) m.retain(id);
        const_cast<InferlabCudaPageManager::Prefix*>(best)->stamp = ++m.clock;
        ++m.prefix_hits;
        m.prefix_tokens_reused += best_len;
        std::copy(best->blocks.begin(), best->blocks.end(), table);
        *table_length = static_cast<std::uint32_t>(best->blocks.size());
        *prefix_tokens = best_len;
    });
}

extern "C" int inferlab_cuda_pages_shared(InferlabCudaPageManager* manager, const int32_t* table,
                                          uint32_t length, uint64_t* shared, char* error,
                                          size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        auto& m = checked(manager);
        if ((table == nullptr && length != 0) || shared == nullptr) {
            throw std::runtime_error("page manager argument is null");
        }
        std::lock_guard<std::mutex> lock(m.mutex);
        std::uint64_t n = 0;
        for (std::uint32_t i = 0; i < length; ++i) n += m.live_block(table[i]).references > 1 ? 1 : 0;
        *shared = n;
    });
}

extern "C" int inferlab_cuda_pages_stats(InferlabCudaPageManager* manager,
                                         InferlabPagedCacheStats* stats, char* error,
                                         size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        auto& m = checked(manager);
        if (stats == nullptr) throw std::runtime_error("page manager argument is null");
        std::lock_guard<std::mutex> lock(m.mutex);
        InferlabPagedCacheStats r{};
        r.page_tokens = m.block_tokens;
        r.page_count = m.blocks.size();
        r.prefix_capacity = m.prefix_capacity;
        r.page_bytes = m.block_tokens * m.row_bytes;
        r.capacity_bytes = r.page_bytes * r.page_count;
        for (const auto& b : m.blocks) {
            if (!b.live) continue;
            ++r.allocated_pages;
            r.used_token_slots += b.used;
            r.live_references += b.references;
            r.maximum_refcount = std::max(r.maximum_refcount, b.references);
            if (b.references > 1) ++r.shared_pages;
            r.physical_used_bytes += b.used * m.row_bytes;
            r.logical_referenced_bytes += b.used * m.row_bytes * b.references;
        }
        r.free_pages = r.page_count - r.allocated_pages;
        r.allocated_token_slots = r.allocated_pages * m.block_tokens;
        r.internal_fragmentation_bytes = (r.allocated_token_slots - r.used_token_slots) * m.row_bytes;
        r.bytes_saved_by_sharing = r.logical_referenced_bytes - r.physical_used_bytes;
        r.prefix_entries = m.prefixes.size();
        r.prefix_hits = m.prefix_hits;
        r.prefix_misses = m.prefix_misses;
        r.prefix_tokens_reused = m.prefix_tokens_reused;
        r.copy_on_write_copies = m.copies;
        r.evictions = m.evictions;
        r.allocation_failures = m.allocation_failures;
        *stats = r;
    });
}

extern "C" int inferlab_cuda_pages_copy(InferlabCudaKvPool* pool, const int32_t* from,
                                        const int32_t* to, uint32_t count, void* stream,
                                        char* error, size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        using namespace ilb;
        auto& p = checked_pool(pool);
        if (count == 0) return;
        if (from == nullptr || to == nullptr) throw std::runtime_error("page manager argument is null");
        DeviceGuard guard(p.device);
        auto s = static_cast<cudaStream_t>(stream);
        const std::size_t block_bytes =
            static_cast<std::size_t>(p.kv_heads) * p.block_tokens * p.head_dim * p.element_bytes;
        for (std::uint32_t i = 0; i < count; ++i) {
            if (from[i] < 0 || to[i] < 0 || static_cast<std::uint64_t>(from[i]) >= p.num_blocks ||
                static_cast<std::uint64_t>(to[i]) >= p.num_blocks) {
                throw std::runtime_error("paged KV block table contains an invalid page");
            }
            // A block of one arena, all kv-heads, is one contiguous run.
            for (unsigned char* arena : {static_cast<unsigned char*>(p.key_arena),
                                         static_cast<unsigned char*>(p.value_arena)}) {
                cuda_check(cudaMemcpyAsync(arena + static_cast<std::size_t>(to[i]) * block_bytes,
                                           arena + static_cast<std::size_t>(from[i]) * block_bytes,
                                           block_bytes, cudaMemcpyDeviceToDevice, s),
                           "cudaMemcpyAsync block copy");
            }
        }
    });
}
