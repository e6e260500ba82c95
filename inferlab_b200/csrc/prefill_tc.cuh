// prefill_tc.cuh - causal / chunked prefill on the sm_100a tensor cores.
//
// Work item: (segment, q-head, 256-query block) = two 128-query tiles A and B
// that share every K/V tile. Persistent grid, one CTA per SM: items are
// numbered longest causal block first and taken from a global counter, so
// the CTAs that finish early take the short items at the end. A CTA starts
// the next item's Q and K/V loads and its first S MMAs while the softmax
// warps finish the current one. The keys a query may see follow
// legal_sources (kernels/attention_cpu.cpp:113-123): query i of a segment
// that starts at position P sees keys [0, P + i].
//
// Roles (384 threads):
//   warps 0-3 / 4-7  softmax for tile A / B: thread t owns query row t. Per
//              128-key tile it reads its S row from TMEM once (tcgen05.ld
//              32x32b.x128), masks, takes the row max, computes fp16
//              probabilities and writes them back into TMEM over the first 64
//              columns of S (tcgen05.st), where the PV MMA reads them as its A
//              operand. O stays in TMEM, accumulated by the MMA; it is rescaled
//              (load, multiply, store in TMEM) only when a row's running max
//              grows by more than 2^8, so probabilities relative to the kept
//              max stay <= 256 (exact in fp16's range) and the result is the
//              same online-softmax recurrence (kernels/attention_cpu.cpp:364-386).
//              Before P_t(j) the tile's warps also check that V(j) and, when
//              the tile continues, K(j + 1) are resident, so the issuer needs
//              no other wait than P. At the end a full tile's O / l
//              leaves through the tile's 16 KB staging box by tensor stores;
//              a ragged last tile stores its rows directly.
//   warp 8     takes the work items (counter -> shared-memory ring), loads
//              both Q tiles by TMA (3-D map over [tokens][q_heads][128]), then
//              the K tiles: per 128-key tile the eight 16-token blocks the
//              table names, gathered with 16-byte cp.async into the 128-byte
//              swizzled layout, block ids read one tile ahead.
//   warp 9     MMA issuer (one thread): S_t = Q_t K^T (M=N=128, K=128,
//              f16/bf16, fp32 in TMEM) and O_t += P_t V (P from TMEM, V an
//              MN-major shared-memory operand). MMAs of one thread run in
//              issue order, so S_t(j + 1) follows PV_t(j) without a wait; the
//              order PV_A, S_A, PV_B, S_B lets one tile's softmax run while the
//              tensor core works on the other tile.
//   warp 10    the V tiles, gathered like K.
//   warp 11    (bf16 pools) widens each V tile from bf16 to fp16 in shared
//              memory before its PV, so P keeps fp16's 11-bit significand.
// TMEM (512 columns): tile t uses [256t, 256t + 128) for S / P and
// [256t + 128, 256t + 256) for O.
// Every mbarrier wait is bounded; a wait that gives up records
// kErrWaitTimeout, and the CTA drains its own copies and MMAs (bounded) and
// frees its TMEM before returning. Warp-collective TMEM instructions are only
// ever reached by whole warps.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "pool.cuh"
#include "tc_common.cuh"

#include <algorithm>
#include <cmath>
#include <mutex>

namespace ilb {
namespace tc {

constexpr int kBM = 128;                 // rows of one Q tile
constexpr int kQBlock = 2 * kBM;         // queries per CTA (tiles A and B)
constexpr int kBN = 128;                 // keys per K/V tile
constexpr int kD = 128;
constexpr int kBlockTokens = 16;
constexpr int kThreads = 384;  // 8 softmax warps, K and V producers, MMA issuer, V widening
constexpr int kHalf = 16384;             // one 64-column half of a 128 x 128 16-bit tile
constexpr int kTile = 2 * kHalf;         // 32 KB
constexpr int kQ0 = 0;                   // Q tiles A, B
constexpr int kK0 = 2 * kTile;           // two K stages
constexpr int kV0 = kK0 + 2 * kTile;     // two V stages
constexpr int kOut0 = kV0 + 2 * kTile;   // output staging: one 128 x 32 fp32 box per tile
constexpr int kBars = kOut0 + 2 * kHalf; // 224 KB
constexpr int kRing = 4;                 // work-item slots between the scheduler and the roles
constexpr int kNumBars = 27;
constexpr int kMisc = kBars + kNumBars * 8;  // TMEM address, abort flag, work-item slots
constexpr int kSmemBytes = kMisc + 64;
constexpr int kSmemAlloc = kSmemBytes + 1024;  // slack to align the base to 1024 B
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O when the max grows by > 2^8

enum Bar : int {
    kBarQ = 0,         // the work item's Q tiles landed
    kBarQFree = 1,     // the work item's last S MMA completed (Q may be reloaded)
    kBarK = 2,         // +stage
    kBarV = 4,         // +stage
    kBarKFree = 6,     // +stage
    kBarVFree = 8,     // +stage
    kBarS = 10,        // +tile
    kBarP = 12,        // +tile, 4 arrivals (one per softmax warp)
    kBarO = 14,        // +tile
    kBarVReady = 16,   // +stage (bf16 widening)
    kBarDone = 18,
    kBarItem = 19,     // +slot: work-item index written
    kBarItemFree = 23, // +slot: every consuming warp has read it
};

struct Params {
    const unsigned char* key_arena;    // [block][kv_head][slot][128], 16-bit elements
    const unsigned char* value_arena;
    std::uint32_t kv_heads;
    const std::int32_t* tables;
    std::uint32_t max_blocks;
    const std::int32_t* starts;
    const std::int32_t* counts;
    const std::int32_t* offsets;
    std::uint32_t num_segments;
    std::uint32_t q_heads;
    std::uint32_t group;
    std::uint32_t q_blocks;
    std::uint64_t num_blocks;
    long long total_queries;
    float scale_log2;
    float* out;
    std::uint32_t* error_word;
    std::uint32_t num_items;   // num_segments * q_heads * q_blocks
    std::uint32_t* scheduler;  // [0] next work item - gridDim.x, [1] CTAs finished
};

// One work item: 256 queries (tiles A and B) of one (segment, q-head).
struct Item {
    int start, count, offset, q_lo;
    int rows0, rows1;      // rows of tiles A and B inside the segment
    int ntiles0, ntiles1;  // K/V tiles each needs
    int n_total, nblk_total;
    std::uint32_t head, kv_head;
    const std::int32_t* table;
};

// Work item `idx` in longest-first order: all (segment, head) pairs of the
// last query block first, then the block before it, ... False when the block
// lies past the segment's queries, or the segment is malformed (recorded when
// `flag`).
__device__ __forceinline__ bool load_item(const Params& p, std::uint32_t idx, Item& w, bool flag) {
    const std::uint32_t pairs = p.num_segments * p.q_heads;
    const std::uint32_t qblk = p.q_blocks - 1 - idx / pairs;
    const std::uint32_t seg = (idx % pairs) / p.q_heads;
    w.head = (idx % pairs) % p.q_heads;
    w.count = p.counts[seg];
    w.q_lo = static_cast<int>(qblk) * kQBlock;
    if (w.q_lo >= w.count) return false;
    w.start = p.starts[seg];
    w.offset = p.offsets[seg];
    if (w.start < 0 || w.count < 1 || w.offset < 0 ||
        static_cast<long long>(w.offset) + w.count > p.total_queries ||
        static_cast<long long>(w.start) + w.count > static_cast<long long>(p.max_blocks) * kBlockTokens) {
        if (flag) flag_error(p.error_word, kErrSegment);
        return false;
    }
    // Tile B holds the later queries, so ntiles1 >= ntiles0 unless it is empty.
    w.rows0 = min(kBM, w.count - w.q_lo);
    w.rows1 = max(0, min(kBM, w.count - (w.q_lo + kBM)));
    w.ntiles0 = (w.start + w.q_lo + w.rows0 + kBN - 1) / kBN;
    w.ntiles1 = w.rows1 > 0 ? (w.start + w.q_lo + kBM + w.rows1 + kBN - 1) / kBN : 0;
    w.n_total = max(w.ntiles0, w.ntiles1);
    w.nblk_total = (w.start + w.count + kBlockTokens - 1) / kBlockTokens;
    w.kv_head = w.head / p.group;
    w.table = p.tables + static_cast<std::size_t>(seg) * p.max_blocks;
    return true;
}

template <bool kBf16>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap q_map,
                      const __grid_constant__ CUtensorMap out_map, const Params p) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<std::uintptr_t>(smem_raw) + 1023) & ~static_cast<std::uintptr_t>(1023));
    auto* bars = reinterpret_cast<std::uint64_t*>(smem + kBars);
    auto* tmem_slot = reinterpret_cast<std::uint32_t*>(smem + kMisc);
    int* abort = reinterpret_cast<int*>(smem + kMisc + 16);
    auto* items = reinterpret_cast<volatile std::uint32_t*>(smem + kMisc + 32);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int b = 0; b < kNumBars; ++b) {
            std::uint32_t arrivals = 1;
            if (b == kBarP || b == kBarP + 1) arrivals = 4;  // the tile's four softmax warps
            // Every warp that reads a work-item slot: 8 softmax warps, the
            // issuer, the V producer and (bf16) the V widening warp.
            if (b >= kBarItemFree && b < kBarItemFree + kRing) arrivals = kBf16 ? 11 : 10;
            mbar_init(&bars[b], arrivals);
        }
        *abort = 0;
        fence_barrier_init();
    }
    if (warp == 9) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const std::uint32_t tmem = *tmem_slot;
    const Waiter wait{abort, p.error_word};

    // Work items are handed out through a ring of kRing slots in shared
    // memory: the K producer takes the CTA's next item (its own block index
    // first, then a global counter, so the longest items go first and the CTAs
    // that finish early take the rest), writes it to slot r % kRing and
    // arrives on kBarItem; every other role reads the slot in the same order
    // and arrives on kBarItemFree. Every role keeps running counts (items,
    // K/V tiles, S steps per tile) across items, so barrier phases continue
    // and the producers and the issuer start the next item while the softmax
    // warps finish the current one. A slot index >= num_items ends the CTA.

    if (warp == 8 || warp == 10) {
        // ------------------------------------------------------------ K / V producers
        // Warp 8 gathers K tiles (and loads the Q tiles), warp 10 V tiles,
        // 16 bytes a lane per cp.async (one 2 KB TMA box per block and half
        // costs the TMA unit ~90 cycles; the LSU path keeps up with the tensor
        // core). Lane-chunk map of a 128-key tile: chunk = lane + 32 i
        // (i < 64) is bytes [16 (chunk & 15), +16) of key row chunk >> 4, i.e.
        // row 2i + lane / 16 of block i / 8; it lands in 64-column half
        // (chunk >> 3) & 1 at row * 128 + 16 ((chunk & 7) ^ (row & 7)) - the
        // 128-byte swizzle the MMA descriptors name. A tile is announced on
        // its full barrier once the warp's copies have landed (wait_group,
        // proxy fence, one arrival); before the warp blocks on anything it
        // announces what it has copied, so no role waits on a tile that is
        // only held back by this warp.
        const bool is_k = warp == 8;
        const unsigned char* arena_base = (is_k ? p.key_arena : p.value_arena) +
                                          static_cast<std::size_t>((lane >> 4) * 256 + (lane & 15) * 16);
        const std::size_t block_bytes = static_cast<std::size_t>(p.kv_heads) * (kBlockTokens * kD * 2);
        const std::uint32_t stage0 = smem_u32(smem + (is_k ? kK0 : kV0));
        const int full_bar = is_k ? kBarK : kBarV;
        const int free_bar = is_k ? kBarKFree : kBarVFree;
        const int half = (lane >> 3) & 1;
        const int c = lane & 7;
        int pending = -1;  // tile (running count) whose copies are in flight, not yet announced
        auto announce = [&](int g) {
            fence_proxy_async_shared();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[full_bar + (g & 1)]);
        };
        // Bounded wait that first announces the pending tile if it would block.
        auto wait_flush = [&](std::uint64_t* bar, std::uint32_t parity) {
            if (warp_ok(mbar_test_wait(bar, parity))) return true;
            if (pending >= 0) {
                cp_async_wait_group<0>();
                announce(pending);
                pending = -1;
            }
            return warp_ok(wait(bar, parity));
        };
        std::uint32_t g = 0;  // K/V tiles so far
        std::uint32_t it = 0; // items processed so far
        bool ok = true;
        for (int r = 0; ok; ++r) {
            const int slot = r % kRing;
            std::uint32_t idx = 0;
            if (is_k) {
                if (r >= kRing && !(ok = wait_flush(&bars[kBarItemFree + slot], ((r / kRing) - 1) & 1))) break;
                if (lane == 0) {
                    idx = r == 0 ? blockIdx.x : gridDim.x + atomicAdd(p.scheduler, 1u);
                    items[slot] = idx;
                    mbar_arrive(&bars[kBarItem + slot]);
                }
                idx = __shfl_sync(0xffffffffu, idx, 0);
            } else {
                if (!(ok = wait_flush(&bars[kBarItem + slot], (r / kRing) & 1))) break;
                idx = items[slot];
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars[kBarItemFree + slot]);
            }
            if (idx >= p.num_items) break;
            Item w;
            if (!load_item(p, idx, w, false)) continue;
            if (is_k) {
                // Both Q tiles, once the previous item's S MMAs have read theirs.
                if (it > 0 && !(ok = wait_flush(&bars[kBarQFree], (it - 1) & 1))) break;
                if (lane == 0) {
                    mbar_arrive_expect_tx(&bars[kBarQ], 2 * kTile);
#pragma unroll
                    for (int t = 0; t < 2; ++t) {
                        tma_load_3d(smem + kQ0 + t * kTile, &q_map, 0, static_cast<int>(w.head),
                                    w.offset + w.q_lo + t * kBM, &bars[kBarQ]);
                        tma_load_3d(smem + kQ0 + t * kTile + kHalf, &q_map, 64, static_cast<int>(w.head),
                                    w.offset + w.q_lo + t * kBM, &bars[kBarQ]);
                    }
                }
            }
            ++it;
            const unsigned char* arena =
                arena_base + static_cast<std::size_t>(w.kv_head) * (kBlockTokens * kD * 2);
            auto read_id = [&](int j) {
                const int logical = j * 8 + (lane & 7);
                return w.table[logical < w.nblk_total ? logical : 0];
            };
            std::int32_t next_id = read_id(0);
            for (int j = 0; j < w.n_total; ++j, ++g) {
                const int st = g & 1;
                std::int32_t id = next_id;
                if (id < 0 || static_cast<std::uint64_t>(id) >= p.num_blocks) {
                    if (lane < 8) flag_error(p.error_word, kErrBadBlock);
                    id = 0;
                }
                if (j + 1 < w.n_total) next_id = read_id(j + 1);
                if (g >= 2 && !(ok = wait_flush(&bars[free_bar + st], ((g >> 1) - 1) & 1))) break;
                const std::uint32_t dst = stage0 + static_cast<std::uint32_t>(st * kTile + half * kHalf);
#pragma unroll
                for (int b = 0; b < 8; ++b) {
                    const unsigned char* src =
                        arena + static_cast<std::size_t>(__shfl_sync(0xffffffffu, id, b)) * block_bytes;
#pragma unroll
                    for (int rr = 0; rr < 8; ++rr) {
                        const int row = b * 16 + rr * 2 + (lane >> 4);
                        cp_async16(dst + static_cast<std::uint32_t>(row * 128 + ((c ^ (row & 7)) << 4)),
                                   src + rr * 512);
                    }
                }
                cp_async_commit();
                if (pending >= 0) {
                    cp_async_wait_group<1>();
                    announce(pending);
                }
                pending = static_cast<int>(g);
            }
        }
        cp_async_wait_group<0>();
        if (pending >= 0) announce(pending);
    } else if (warp == 9) {
        // ------------------------------------------------------------ MMA issuer
        // tcgen05.mma operations from one thread run in issue order, so
        // S_t(j + 1) may be issued right behind PV_t(j): it overwrites the S/P
        // columns only after PV_t(j) has read P_t(j). Issue order per K/V
        // tile j: PV_A(j), S_A(j + 1), PV_B(j), S_B(j + 1) - tile A's softmax
        // runs while the tensor core works on tile B and the other way round.
        // The next item's S_t(0) follows the last PV_t of the current one in
        // the same way, and its PV_t(0) (accumulate off) waits for P_t(0),
        // which the softmax warps give only after they have read O_t out.
        //
        // Every mbarrier wait in this thread stalls the tensor pipe (measured:
        // 70-300 cycles of idle tensor core per wait, even on a completed
        // phase), so inside an item the issuer waits on P alone. The softmax
        // warps of tile t arrive on P_t(j) only after V(j) (widened, for bf16)
        // and, when the tile continues, K(j + 1) are resident. Descriptors are
        // built once; the K steps add constants to them.
        if (lane == 0) {
            constexpr std::uint32_t in_type = kBf16 ? 1u : 0u;
            const std::uint32_t idesc_s = idesc_f16(in_type, in_type, 0);
            const std::uint32_t idesc_pv = idesc_f16(0, 0, 1);  // P and V as fp16, V MN-major
            // Scalars, not arrays indexed at run time (those would live in local memory).
            const std::uint64_t q_desc0 = sw128_desc(smem_u32(smem + kQ0), 16, 1024);
            const std::uint64_t q_desc1 = sw128_desc(smem_u32(smem + kQ0 + kTile), 16, 1024);
            const std::uint64_t k_desc0 = sw128_desc(smem_u32(smem + kK0), 16, 1024);
            const std::uint64_t k_desc1 = sw128_desc(smem_u32(smem + kK0 + kTile), 16, 1024);
            const std::uint64_t v_desc0 = sw128_desc(smem_u32(smem + kV0), kHalf, 1024);
            const std::uint64_t v_desc1 = sw128_desc(smem_u32(smem + kV0 + kTile), kHalf, 1024);
            // S_t = Q_t K(g)^T: 8 K steps of 16; step k starts (k & 3) * 32 B
            // into the (k >> 2)-th 64-column half (descriptor address unit 16 B).
            auto issue_s = [&](int t, std::uint32_t g) {
                const std::uint64_t a = t ? q_desc1 : q_desc0;
                const std::uint64_t b = (g & 1) ? k_desc1 : k_desc0;
                const std::uint32_t d = tmem + static_cast<std::uint32_t>(t * 256);
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const std::uint64_t off = static_cast<std::uint64_t>(((k >> 2) * kHalf + (k & 3) * 32) >> 4);
                    mma_f16(d, a + off, b + off, idesc_s, k > 0 ? 1u : 0u);
                }
                mma_commit(&bars[kBarS + t]);
            };
            std::uint32_t g = 0, it = 0;
            std::uint32_t np0 = 0, np1 = 0;  // P phases consumed per tile
            bool ok = true;
            for (int r = 0; ok; ++r) {
                const int slot = r % kRing;
                if (!(ok = wait(&bars[kBarItem + slot], (r / kRing) & 1))) break;
                const std::uint32_t idx = items[slot];
                mbar_arrive(&bars[kBarItemFree + slot]);
                if (idx >= p.num_items) break;
                Item w;
                if (!load_item(p, idx, w, false)) continue;
                if (!(ok = wait(&bars[kBarQ], it & 1) && wait(&bars[kBarK + (g & 1)], (g >> 1) & 1))) break;
                ++it;
                tc_fence_after();
                issue_s(0, g);
                if (w.ntiles1 > 0) issue_s(1, g);
                mma_commit(&bars[kBarKFree + (g & 1)]);
                if (w.n_total == 1) mma_commit(&bars[kBarQFree]);
                for (int j = 0; ok && j < w.n_total; ++j) {
                    const std::uint32_t gj = g + static_cast<std::uint32_t>(j);
                    const std::uint64_t vb = (gj & 1) ? v_desc1 : v_desc0;
                    for (int t = 0; t < 2; ++t) {
                        const int nt = t ? w.ntiles1 : w.ntiles0;
                        if (j >= nt) continue;
                        if (!(ok = wait(&bars[kBarP + t], (t ? np1 : np0) & 1))) break;
                        if (t) ++np1; else ++np0;
                        tc_fence_after();
                        const std::uint32_t s_tmem = tmem + static_cast<std::uint32_t>(t * 256);
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            // P columns [8k, 8k + 8) hold keys [16k, 16k + 16) as f16 pairs;
                            // V rows [16k, 16k + 16) start 2048 B further per step.
                            mma_f16_tmem_a(s_tmem + 128, s_tmem + k * 8,
                                           vb + static_cast<std::uint64_t>((k * 2048) >> 4), idesc_pv,
                                           (j > 0 || k > 0) ? 1u : 0u);
                        }
                        mma_commit(&bars[kBarO + t]);
                        // A commit tracks every earlier MMA of this thread, so V(j)
                        // is released right after the last PV that reads it, before
                        // the next S is queued behind it.
                        if (t == 1 || j >= w.ntiles1) mma_commit(&bars[kBarVFree + (gj & 1)]);
                        if (j + 1 < nt) issue_s(t, gj + 1);
                    }
                    if (!ok) break;
                    if (j + 1 < w.n_total) {
                        mma_commit(&bars[kBarKFree + ((gj + 1) & 1)]);
                        if (j + 2 == w.n_total) mma_commit(&bars[kBarQFree]);  // the item's last S
                    }
                }
                g += static_cast<std::uint32_t>(w.n_total);
            }
            // All MMAs issued by this thread complete before TMEM is released.
            mma_commit(&bars[kBarDone]);
            mbar_wait_bounded(&bars[kBarDone], 0, p.error_word);
        }
    } else if (warp == 11) {
        // ------------------------------------------------------------ V widening (bf16)
        if constexpr (kBf16) {
            std::uint32_t g = 0;
            bool ok = true;
            for (int r = 0; ok; ++r) {
                const int slot = r % kRing;
                if (!(ok = warp_ok(wait(&bars[kBarItem + slot], (r / kRing) & 1)))) break;
                const std::uint32_t idx = items[slot];
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars[kBarItemFree + slot]);
                if (idx >= p.num_items) break;
                Item w;
                if (!load_item(p, idx, w, false)) continue;
                for (int j = 0; j < w.n_total; ++j, ++g) {
                    const int st = g & 1;
                    if (!(ok = warp_ok(wait(&bars[kBarV + st], (g >> 1) & 1)))) break;
                    uint4* v = reinterpret_cast<uint4*>(smem + kV0 + st * kTile);
                    for (int i = lane; i < kTile / 16; i += 32) {
                        uint4 x = v[i];
                        std::uint32_t* u = reinterpret_cast<std::uint32_t*>(&x);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float lo = __uint_as_float(u[e] << 16);
                            const float hi = __uint_as_float(u[e] & 0xFFFF0000u);
                            const __half2 h = __floats2half2_rn(lo, hi);
                            u[e] = *reinterpret_cast<const std::uint32_t*>(&h);
                        }
                        v[i] = x;
                    }
                    fence_proxy_async_shared();
                    // One arrival per warp: 32 arrivals on one mbarrier word
                    // serialise and delay the phase by about a thousand cycles.
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&bars[kBarVReady + st]);
                }
            }
        }
    } else {
        // ------------------------------------------------------------ softmax (tiles A, B)
        const int t = warp >> 2;
        const int row = threadIdx.x & 127;  // TMEM lane = row of the tile
        const std::uint32_t lane_addr = tmem + (static_cast<std::uint32_t>((warp & 3) * 32) << 16) +
                                        static_cast<std::uint32_t>(t * 256);
        unsigned char* stage = smem + kOut0 + t * kHalf;
        std::uint32_t g = 0;   // K/V tiles so far
        std::uint32_t ns = 0;  // S / P / O phases of this tile so far
        bool ok = true;
        for (int r = 0; ok; ++r) {
            const int slot = r % kRing;
            if (!(ok = warp_ok(wait(&bars[kBarItem + slot], (r / kRing) & 1)))) break;
            const std::uint32_t idx = items[slot];
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[kBarItemFree + slot]);
            if (idx >= p.num_items) break;
            Item w;
            if (!load_item(p, idx, w, threadIdx.x == 0)) continue;
            const int n = t ? w.ntiles1 : w.ntiles0;
            const int rows = t ? w.rows1 : w.rows0;
            const int tile_lo = w.start + w.q_lo + t * kBM;  // first query position of the tile
            const int qpos = tile_lo + row;                  // this row's position in its sequence
            float m = -INFINITY;  // kept max (log2 units)
            float l = 0.0f;
            for (int j = 0; ok && j < n; ++j) {
                const std::uint32_t gj = g + static_cast<std::uint32_t>(j);
                const std::uint32_t sj = ns + static_cast<std::uint32_t>(j);
                if (!(ok = warp_ok(wait(&bars[kBarS + t], sj & 1)))) break;
                tc_fence_after();
                std::uint32_t s[128];
                tmem_load128(lane_addr, s);
                const int key0 = j * kBN;
                // Tiles on the causal diagonal: masked scores become -inf, which
                // the exponent below turns into p = 0. The branch is uniform per
                // warp group (it depends on the tile, not the row).
                if (key0 + kBN - 1 > tile_lo) {
#pragma unroll
                    for (int i = 0; i < 128; ++i) {
                        if (key0 + i > qpos) s[i] = __float_as_uint(-INFINITY);
                    }
                }
                // Row max with the three-input max (two new scores per
                // instruction), four independent chains.
                float mx4[4] = {__uint_as_float(s[0]), __uint_as_float(s[1]), __uint_as_float(s[2]),
                                __uint_as_float(s[3])};
#pragma unroll
                for (int i = 4; i < 128; i += 2) {
                    mx4[(i >> 1) & 3] = fmax3(mx4[(i >> 1) & 3], __uint_as_float(s[i]), __uint_as_float(s[i + 1]));
                }
                const float mx = fmax3(mx4[0], mx4[1], fmaxf(mx4[2], mx4[3]));
                const float m_seen = fmaxf(m, mx * p.scale_log2);
                if (j == 0) {
                    m = m_seen;
                } else {
                    const bool grow = m_seen > m + kRescaleThreshold;
                    if (__any_sync(0xffffffffu, grow)) {
                        // O_t must be complete before it is rescaled in place.
                        if (!(ok = warp_ok(wait(&bars[kBarO + t], (sj - 1) & 1)))) break;
                        tc_fence_after();
                        const float alpha = grow ? exp2f(m - m_seen) : 1.0f;
#pragma unroll
                        for (int cc = 0; cc < 4; ++cc) {
                            float o[32];
                            tmem_load32(lane_addr + 128 + cc * 32, o);
                            std::uint32_t x[32];
#pragma unroll
                            for (int i = 0; i < 32; ++i) x[i] = __float_as_uint(o[i] * alpha);
                            tmem_store32(lane_addr + 128 + cc * 32, x);
                        }
                        tmem_store_wait();
                        if (grow) {
                            l *= alpha;
                            m = m_seen;
                        }
                    }
                }
                // P = 2^(s * scale - m) in fp16, written over the first 64 columns
                // of S. Pairs of scores go through one packed f32x2 FMA, then an
                // exponent: three pairs in four on the MUFU unit, the fourth as a
                // polynomial on the FMA pipe (relative error 1.5e-4, under the
                // fp16 rounding of P), so both pipes share the work. The row sum
                // is kept in fp32 (four pair sums).
                const std::uint64_t scale2 = pack_f32x2(p.scale_log2, p.scale_log2);
                const std::uint64_t neg_m2 = pack_f32x2(-m, -m);
                std::uint64_t sum2[4] = {0, 0, 0, 0};
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    std::uint32_t packed[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const int i = cc * 32 + e * 2;
                        const std::uint64_t x = ffma_f32x2(pack_u32x2(s[i], s[i + 1]), scale2, neg_m2);
                        float p0, p1;
                        if ((e & 3) == 3) {
                            const std::uint64_t e2 = ex2_poly_f32x2(low_f32(x), high_f32(x));
                            p0 = low_f32(e2);
                            p1 = high_f32(e2);
                        } else {
                            p0 = ex2_ftz(low_f32(x));
                            p1 = ex2_ftz(high_f32(x));
                        }
                        sum2[e & 3] = fadd_f32x2(sum2[e & 3], pack_f32x2(p0, p1));
                        const __half2 h = __floats2half2_rn(p0, p1);
                        packed[e] = *reinterpret_cast<const std::uint32_t*>(&h);
                    }
                    tmem_store16(lane_addr + cc * 16, packed);
                }
                tmem_store_wait();
                const std::uint64_t s01 = fadd_f32x2(sum2[0], sum2[1]);
                const std::uint64_t s23 = fadd_f32x2(sum2[2], sum2[3]);
                const std::uint64_t s0123 = fadd_f32x2(s01, s23);
                l += low_f32(s0123) + high_f32(s0123);
                // PV_t(j) reads V(j) and S_t(j + 1) reads K(j + 1): both must be
                // resident before P_t(j) releases the issuer (which waits on P
                // only). Checked last, so that copies still in flight overlap
                // this step's softmax.
                if (kBf16) {
                    if (!(ok = warp_ok(wait(&bars[kBarVReady + (gj & 1)], (gj >> 1) & 1)))) break;
                } else {
                    if (!(ok = warp_ok(wait(&bars[kBarV + (gj & 1)], (gj >> 1) & 1)))) break;
                }
                if (j + 1 < n && !(ok = warp_ok(wait(&bars[kBarK + ((gj + 1) & 1)], ((gj + 1) >> 1) & 1)))) break;
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars[kBarP + t]);  // one arrival per warp
            }
            g += static_cast<std::uint32_t>(w.n_total);
            if (!ok || n == 0) continue;
            ns += static_cast<std::uint32_t>(n);
            ok = warp_ok(wait(&bars[kBarO + t], (ns - 1) & 1));
            // The tile's four warps agree (named barrier) before any of them
            // takes part in the shared staging below.
            ok = named_barrier_and(1 + t, kBM, ok);
            if (!ok) break;
            tc_fence_after();
            const float inv = 1.0f / l;
            if (rows == kBM) {
                // Full tile: O / l through the tile's staging box and tensor
                // stores, 32 columns at a time: a 128-row x 32-float box,
                // 128-byte swizzled (row r's 16-byte chunk c at r * 128 +
                // 16 (c ^ (r & 7))), so the staging writes are free of bank
                // conflicts and the global writes are whole lines. Before a
                // box is rewritten, the store that read it last (this item's
                // previous box or the previous item's last) has read it.
                const int q_row = w.offset + w.q_lo + t * kBM;
#pragma unroll 1
                for (int cb = 0; cb < 4; ++cb) {
                    float o[32];
                    tmem_load32(lane_addr + 128 + cb * 32, o);
                    if (row == 0) bulk_wait_group_read0();
                    named_barrier_sync(1 + t, kBM);
                    unsigned char* box = stage + row * 128;
#pragma unroll
                    for (int cch = 0; cch < 8; ++cch) {
                        *reinterpret_cast<float4*>(box + ((cch ^ (row & 7)) << 4)) =
                            make_float4(o[4 * cch] * inv, o[4 * cch + 1] * inv, o[4 * cch + 2] * inv,
                                        o[4 * cch + 3] * inv);
                    }
                    fence_proxy_async_shared();
                    named_barrier_sync(1 + t, kBM);
                    if (row == 0) {
                        tma_store_3d(&out_map, stage, cb * 32, static_cast<int>(w.head), q_row);
                        bulk_commit_group();
                    }
                }
            } else {
                // Ragged last tile of a segment: rows past its end belong
                // to the next segment, so only rows inside it store.
                const bool store = row < rows;
                float* out = p.out + (static_cast<std::size_t>(w.offset + w.q_lo + t * kBM + (store ? row : 0)) *
                                          p.q_heads + w.head) * kD;
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    float o[32];
                    tmem_load32(lane_addr + 128 + cc * 32, o);
                    if (store) {
#pragma unroll
                        for (int i = 0; i < 32; i += 4) {
                            *reinterpret_cast<float4*>(out + cc * 32 + i) =
                                make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv);
                        }
                    }
                }
            }
            if (row < rows && !(isfinite(l) && l > 0.0f)) flag_error(p.error_word, kErrNormalizer);
        }
        // Output stores out of the staging box complete before the CTA ends.
        if (row == 0) bulk_wait_group0();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
    // The last CTA to finish returns the launch's work-queue counters to
    // zero for the next launch that takes this pair; every CTA has taken its
    // last item by now.
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(p.scheduler + 1, 1u) == gridDim.x - 1) {
            atomicExch(p.scheduler, 0u);
            atomicExch(p.scheduler + 1, 0u);
        }
    }
}

// Rounds fp32 queries to the pool type for the tensor-core path.
template <typename T>
__global__ void convert_queries_kernel(const float* in, T* out, std::size_t n) {
    for (std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<std::size_t>(gridDim.x) * blockDim.x) {
        out[i] = Storage<T>::from_float(in[i]);
    }
}

}  // namespace tc

inline bool tc_prefill_supported(const InferlabCudaKvPool& pool, std::uint32_t q_heads) {
    return (pool.dtype == kF16 || pool.dtype == kBf16) && pool.head_dim == tc::kD &&
           pool.block_tokens == tc::kBlockTokens && q_heads % pool.kv_heads == 0;
}

inline void run_tc_prefill(InferlabCudaKvPool& pool, const void* queries, std::uint32_t query_dtype,
                           const std::int32_t* tables, std::uint32_t max_blocks,
                           const std::int32_t* starts, const std::int32_t* counts,
                           const std::int32_t* offsets, std::uint32_t num_segments,
                           std::uint32_t q_heads, std::uint32_t max_query_count,
                           long long total_queries, float* out, cudaStream_t stream) {
    using namespace tc;
    const bool bf16 = pool.dtype == kBf16;
    const std::size_t q_elems = static_cast<std::size_t>(total_queries) * q_heads * kD;
    void* q16 = const_cast<void*>(queries);
    void* temp = nullptr;
    if (query_dtype == kFp32) {
        cuda_check(cudaMallocAsync(&temp, q_elems * 2, stream), "cudaMallocAsync");
        const unsigned grid = static_cast<unsigned>(std::min<std::size_t>((q_elems + 255) / 256, 4096));
        if (bf16) {
            convert_queries_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
                static_cast<const float*>(queries), static_cast<__nv_bfloat16*>(temp), q_elems);
        } else {
            convert_queries_kernel<__half><<<grid, 256, 0, stream>>>(
                static_cast<const float*>(queries), static_cast<__half*>(temp), q_elems);
        }
        cuda_check(cudaGetLastError(), "query conversion launch");
        q16 = temp;
    }
    struct TempGuard {
        void* ptr;
        cudaStream_t stream;
        ~TempGuard() {
            if (ptr != nullptr) cudaFreeAsync(ptr, stream);
        }
    } guard{temp, stream};
    if (reinterpret_cast<std::uintptr_t>(q16) % 16 != 0) {
        throw std::runtime_error("paged prefill queries must be 16-byte aligned");
    }
    const CUtensorMapDataType type =
        bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const cuuint64_t q_dims[3] = {kD, q_heads, static_cast<cuuint64_t>(total_queries)};
    const cuuint64_t q_strides[2] = {kD * 2, static_cast<cuuint64_t>(q_heads) * kD * 2};
    const cuuint32_t q_box[3] = {64, 1, kBM};  // one 128-query tile per box
    const CUtensorMap q_map = make_map(q16, type, 3, q_dims, q_strides, q_box);
    if (reinterpret_cast<std::uintptr_t>(out) % 16 != 0) {
        throw std::runtime_error("paged prefill output must be 16-byte aligned");
    }
    const cuuint64_t o_dims[3] = {kD, q_heads, static_cast<cuuint64_t>(total_queries)};
    const cuuint64_t o_strides[2] = {kD * 4, static_cast<cuuint64_t>(q_heads) * kD * 4};
    const cuuint32_t o_box[3] = {32, 1, kBM};  // 128 rows x 32 floats (128 B)
    const CUtensorMap out_map = make_map(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, o_dims, o_strides, o_box);

    Params params{};
    params.key_arena = static_cast<const unsigned char*>(pool.key_arena);
    params.value_arena = static_cast<const unsigned char*>(pool.value_arena);
    params.kv_heads = pool.kv_heads;
    params.tables = tables;
    params.max_blocks = max_blocks;
    params.starts = starts;
    params.counts = counts;
    params.offsets = offsets;
    params.num_segments = num_segments;
    params.q_heads = q_heads;
    params.group = q_heads / pool.kv_heads;
    params.q_blocks = (max_query_count + kQBlock - 1) / kQBlock;
    params.num_blocks = pool.num_blocks;
    params.total_queries = total_queries;
    params.scale_log2 = (1.0f / std::sqrt(static_cast<float>(kD))) * kLog2e;
    params.out = out;
    params.error_word = pool.error_word;
    const std::uint64_t num_items = static_cast<std::uint64_t>(num_segments) * q_heads * params.q_blocks;
    if (num_items > 0x7FFFFFFFull) throw std::runtime_error("paged prefill grid is too large");
    if (num_items == 0) return;
    params.num_items = static_cast<std::uint32_t>(num_items);
    const std::uint32_t slot = pool.scheduler_next.fetch_add(1) % kSchedulerSlots;
    params.scheduler = pool.error_word + 4 + 2 * slot;
    // Persistent grid: one CTA per SM (the shared-memory and TMEM footprint
    // allow one), never more CTAs than work items.
    int sms = 0;
    cuda_check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, pool.device),
               "cudaDeviceGetAttribute");
    const unsigned grid = static_cast<unsigned>(std::min<std::uint64_t>(num_items, static_cast<std::uint64_t>(std::max(sms, 1))));
    auto kernel = bf16 ? prefill_tc_kernel<true> : prefill_tc_kernel<false>;
    cuda_check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemAlloc),
               "cudaFuncSetAttribute");
    kernel<<<grid, kThreads, kSmemAlloc, stream>>>(q_map, out_map, params);
    cuda_check(cudaGetLastError(), "tensor-core prefill launch");
}

}  // namespace ilb
