// paged_decode.cu - memory-bound paged decode attention for sm_100a.
//
// The decode branch of the reference (worker/cpp/inferlab_runtime.cpp:
// 2373-2393) gathers every page of a sequence into contiguous fp32
// (PagedKvPool::materialize, :769-803) and then runs the scalar
// attention_forward(q, K, V, 1, T, H, d, T - 1) (:1458-1470,
// kernels/attention_cpu.cpp:306-401). Here one launch covers the whole batch
// and reads the pool in place:
//
//  * grid: one CTA per (sequence, kv-head, split); a split is up to
//    blocks_per_split consecutive 16-token blocks of the context.
//  * each warp streams its own blocks (block w, w + W, ...) through a
//    STAGES-deep ring of shared-memory tiles. Lane 0 issues one bulk async
//    copy (cp.async.bulk, the TMA engine, no multicast) per tile: the K and V
//    tiles of one block for one kv-head are each a contiguous
//    16 x head_dim run in the arena, completion tracked by an mbarrier.
//  * lanes split as (token slot, 16-byte chunk group): kG lanes share one
//    token row, each holding kDpl dims of every q-head of the GQA group in
//    registers; dot products reduce with kG-wide xor shuffles; every token
//    slot keeps its own online-softmax state (m, l, acc) in the log2 domain,
//    its kept max moving only when exceeded by more than 2^8 (the
//    accumulators are rescaled only then).
//  * at the end the slot states merge by shuffles, the warps by shared
//    memory, and - when the context was split - the CTAs by a fused
//    log-sum-exp combine: every CTA writes (m, l, acc) to the workspace, and
//    the last CTA of its (sequence, kv-head) to arrive merges all splits and
//    writes the output.
//
// K/V bytes are read from HBM exactly once per (sequence, kv-head).
#include "common.cuh"
#include "generic_attention.cuh"
#include "internal.cuh"
#include "lse_merge.cuh"
#include "pool.cuh"

#include "../../include/inferlab_attention.h"

#include <algorithm>
#include <cmath>
#include <map>
#include <mutex>

namespace ilb {
namespace {

constexpr int kDecodeBlockTokens = 16;
constexpr int kDecodeWarps = 4;
constexpr int kDecodeStages = 2;
constexpr int kMaxBlocksPerSplit = 1024;
// Splits per context are capped so that the last CTA's merge stays short
// (at 64 splits it reads 64 x (head_dim + 2) floats per q-head).
constexpr std::uint32_t kMaxSplits = 64;

constexpr int ilog2(int x) { return x <= 1 ? 0 : 1 + ilog2(x / 2); }
// Lazy rescale (log2 units): a running max moves only when a block's max
// exceeds it by more than 2^8, so probabilities relative to the kept max stay
// <= 256 (no fp32 overflow) and the accumulators are rescaled only then - the
// same online-softmax recurrence (kernels/attention_cpu.cpp:364-386).
constexpr float kDecodeRescale = 8.0f;

template <typename KvT, int D, int GROUP>
struct DecodeShape {
    static constexpr int kElem = sizeof(KvT);
    static constexpr int kEpc = 16 / kElem;              // elements per 16-byte chunk
    static constexpr int kChunks = D * kElem / 16;       // chunks per token row
    static constexpr int kChA = kChunks / 8 > 0 ? kChunks / 8 : 1;
    static constexpr int kChB = 64 / (GROUP * kEpc) > 0 ? 64 / (GROUP * kEpc) : 1;
    static constexpr int kCh = kChA < kChB ? kChA : kChB;  // chunks per lane
    static constexpr int kG = kChunks / kCh;             // lanes per token row
    static constexpr int kTS = 32 / kG;                  // token slots per warp
    static constexpr int kR = kDecodeBlockTokens / kTS;  // tokens per slot per block
    static constexpr int kDpl = kCh * kEpc;              // dims per lane
    static constexpr int kTileBytes = kDecodeBlockTokens * D * kElem;
    // A token row's kG lanes split the heads of the group (kG / GROUP lanes
    // per head) for the softmax instead of all running every head.
    static constexpr bool kSplitHeads = GROUP >= 2 && kG >= GROUP && kG % GROUP == 0;
    static_assert(kChunks * 16 == D * kElem, "head_dim must fill 16-byte chunks");
    static_assert(kG >= 1 && kG <= 32 && 32 % kG == 0, "lane split");
    static_assert(kDecodeBlockTokens % kTS == 0, "token slots");
};

struct DecodeParams {
    const unsigned char* key_arena;
    const unsigned char* value_arena;
    std::uint64_t num_blocks;
    std::uint32_t kv_heads;
    const float* queries;
    std::uint32_t q_heads;
    const std::int32_t* tables;
    std::uint32_t max_blocks;
    const std::int32_t* context_lens;
    std::uint32_t max_context;
    std::uint32_t blocks_per_split;
    std::uint32_t max_splits;
    float scale_log2;
    int emit_partials;  // 0: normalised out; 1: (m, l, o) rows
    float* out;
    float* part_m;
    float* part_l;
    float* part_o;
    float* ws_o;             // [seq][q_head][split][D]
    float* ws_ml;            // [seq][q_head][split][2]
    std::uint32_t* ws_count; // [seq][kv_head]
    std::uint32_t* error_word;
    // Split-sequence decode with the peer exchange fused (kExchange kernels
    // only): the CTA that finishes a (sequence, kv-head) stores its rows'
    // (m, l, o) as step-tagged words into every rank's receive buffer, waits
    // for those rows from all ranks and merges them into xout.
    std::uint64_t* xwords[8];
    float* xout;
    std::uint64_t xrows;  // rows of the exchanged block: num_seqs * q_heads
    std::uint32_t xworld;
    std::uint32_t xrank;
    std::uint32_t xstep;
};

// Shared-memory layout of one CTA.
template <typename KvT, int D, int GROUP>
struct DecodeSmem {
    using S = DecodeShape<KvT, D, GROUP>;
    static constexpr std::size_t kTiles = 0;
    static constexpr std::size_t kTilesBytes =
        static_cast<std::size_t>(kDecodeWarps) * kDecodeStages * 2 * S::kTileBytes;
    static constexpr std::size_t kBars = kTilesBytes;
    static constexpr std::size_t kIds = kBars + kDecodeWarps * kDecodeStages * 8;
    static constexpr std::size_t kFlag = kIds + kMaxBlocksPerSplit * 4;
    static constexpr std::size_t kBytes = kFlag + 16;
    // Each warp's end-of-stream state (acc per q-head of the group, then
    // (m, l) per q-head) goes into the start of its own tile ring, which its
    // copies no longer use by then: no separate reduction area, so the
    // 16-bit GQA kernels fit three CTAs per SM.
    static constexpr std::size_t kWarpRegion = static_cast<std::size_t>(kDecodeStages) * 2 * S::kTileBytes;
    static constexpr std::size_t kRedMlOff = static_cast<std::size_t>(GROUP) * D * 4;
    static_assert(kRedMlOff + GROUP * 8 <= kWarpRegion, "warp state must fit its tile ring");
    static_assert(GROUP * kMaxSplits * 4 <= kTilesBytes, "split weights must fit the tile area");
};

__device__ __forceinline__ float safe_max(float m) { return m == -INFINITY ? 0.0f : m; }

// Packed fp32 pairs (one f32x2 instruction for two lanes of work, each lane
// rounded as a scalar fma.rn / mul.rn would be; no flush to zero).
__device__ __forceinline__ std::uint64_t fma2(std::uint64_t a, std::uint64_t b, std::uint64_t c) {
    std::uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ std::uint64_t mul2(std::uint64_t a, std::uint64_t b) {
    std::uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// A 16-byte chunk of storage elements as fp32 pairs (element 2i low, 2i + 1 high).
__device__ __forceinline__ void widen16_pairs(const uint4& raw, std::uint64_t* out, float) {
    out[0] = pack_u32x2(raw.x, raw.y);
    out[1] = pack_u32x2(raw.z, raw.w);
}
__device__ __forceinline__ void widen16_pairs(const uint4& raw, std::uint64_t* out, __half) {
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        out[i] = pack_f32x2(f.x, f.y);
    }
}
__device__ __forceinline__ void widen16_pairs(const uint4& raw, std::uint64_t* out, __nv_bfloat16) {
    // bf16 -> fp32 is a 16-bit shift of the bit pattern.
    const std::uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) out[i] = pack_u32x2(w[i] << 16, w[i] & 0xFFFF0000u);
}

// Fused split-sequence exchange: word index of element (row, dim) in the
// packed [m | l | o] block, and the step-tagged store of one element into
// slot `xrank` of every rank's receive buffer (plain peer stores through
// NVSwitch, no multicast; an aligned 8-byte store is single-copy atomic, so a
// receiver that sees the step also sees the value).
template <int D>
__device__ __forceinline__ void push_word(const DecodeParams& p, std::uint64_t index, float value) {
    const std::uint64_t block = p.xrows * (D + 2);
    const std::uint64_t word = (static_cast<std::uint64_t>(p.xstep) << 32) | __float_as_uint(value);
    const std::uint64_t at = (static_cast<std::uint64_t>(p.xstep & 1u) * p.xworld + p.xrank) * block + index;
    for (std::uint32_t r = 0; r < p.xworld; ++r) p.xwords[r][at] = word;
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ std::uint64_t load_word(const std::uint64_t* w) {
    std::uint64_t v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(w) : "memory");
    return v;
}

// The CTA that finished rows [row0, row0 + GROUP) has pushed them; it now
// receives those rows of every rank's block (bounded: 2 s of the global
// timer, a timeout records kErrWaitTimeout), stages them in `stage` (shared
// memory, world x GROUP x (D + 2) floats) and merges them in rank order into
// xout with the same per-row code as the standalone combine.
template <int D, int GROUP>
__device__ void receive_and_merge(const DecodeParams& p, std::size_t row0, float* stage) {
    const std::uint64_t block = p.xrows * (D + 2);
    const std::uint64_t tag = static_cast<std::uint64_t>(p.xstep) << 32;
    const std::uint64_t* own = p.xwords[p.xrank] + static_cast<std::uint64_t>(p.xstep & 1u) * p.xworld * block;
    float* sm_m = stage;
    float* sm_l = stage + p.xworld * GROUP;
    float* sm_o = stage + 2 * p.xworld * GROUP;
    constexpr std::uint32_t kPerSrc = GROUP * (D + 2);
    const std::uint32_t total = p.xworld * kPerSrc;
    const unsigned long long deadline = global_ns() + 2000000000ull;
    bool ok = true;
    constexpr int kBatch = 8;
    for (std::uint32_t base = threadIdx.x; ok && base < total; base += kBatch * blockDim.x) {
        const std::uint64_t* w[kBatch];
        float* slot[kBatch];
        std::uint64_t v[kBatch];
        bool need[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const std::uint32_t j = base + u * blockDim.x;
            need[u] = j < total;
            w[u] = own;
            slot[u] = sm_m;
            if (!need[u]) continue;
            const std::uint32_t src = j / kPerSrc;
            const std::uint32_t i = j % kPerSrc;
            std::uint64_t e;
            if (i < GROUP) {
                e = row0 + i;
                slot[u] = sm_m + src * GROUP + i;
            } else if (i < 2 * GROUP) {
                e = p.xrows + row0 + (i - GROUP);
                slot[u] = sm_l + src * GROUP + (i - GROUP);
            } else {
                const std::uint32_t k = i - 2 * GROUP;
                e = 2 * p.xrows + row0 * D + k;
                slot[u] = sm_o + src * (GROUP * D) + k;
            }
            w[u] = own + src * block + e;
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) v[u] = need[u] ? load_word(w[u]) : 0;
        for (;;) {
            bool waiting = false;
#pragma unroll
            for (int u = 0; u < kBatch; ++u) {
                if (!need[u]) continue;
                if ((v[u] & 0xFFFFFFFF00000000ull) == tag) {
                    *slot[u] = __uint_as_float(static_cast<std::uint32_t>(v[u]));
                    need[u] = false;
                } else {
                    waiting = true;
                }
            }
            if (!waiting) break;
            if (global_ns() > deadline) {
                ok = false;
                break;
            }
            __nanosleep(64);
#pragma unroll
            for (int u = 0; u < kBatch; ++u) {
                if (need[u]) v[u] = load_word(w[u]);
            }
        }
    }
    if (!ok) flag_error(p.error_word, kErrWaitTimeout);
    if (!__syncthreads_and(ok)) return;
    for (int h = threadIdx.x / 32; h < GROUP; h += blockDim.x / 32) {
        lse_merge_row(sm_m, sm_l, sm_o, p.xworld, h, D, GROUP, GROUP, GROUP * D, p.xout + row0 * D,
                      threadIdx.x & 31);
    }
}

template <typename KvT, int D, int GROUP, bool kExchange = false>
// Three CTAs per SM for groups of up to four q-heads (the fp32 pairs of q and
// the accumulators fit ~168 registers); GQA-8 keeps the compiler's choice.
// kExchange: the split-sequence variant, whose CTAs that finish a (sequence,
// kv-head) exchange its rows with the other ranks and merge them.
__global__ void __launch_bounds__(kDecodeWarps * 32, GROUP >= 8 ? 1 : 3)
    paged_decode_kernel(const DecodeParams p) {
    using S = DecodeShape<KvT, D, GROUP>;
    using L = DecodeSmem<KvT, D, GROUP>;
    extern __shared__ __align__(128) unsigned char smem[];
    auto* bars = reinterpret_cast<std::uint64_t*>(smem + L::kBars);
    auto* ids = reinterpret_cast<std::int32_t*>(smem + L::kIds);
    auto red_acc = [&](int w, int h) {
        return reinterpret_cast<float*>(smem + w * L::kWarpRegion + static_cast<std::size_t>(h) * D * 4);
    };
    auto red_ml = [&](int w, int h) {
        return reinterpret_cast<float*>(smem + w * L::kWarpRegion + L::kRedMlOff + h * 8);
    };
    auto* flag = reinterpret_cast<int*>(smem + L::kFlag);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const std::uint32_t split = blockIdx.x % p.max_splits;
    const std::uint32_t pair = blockIdx.x / p.max_splits;
    const std::uint32_t kv_head = pair % p.kv_heads;
    const std::uint32_t seq = pair / p.kv_heads;
    const std::size_t row0 = static_cast<std::size_t>(seq) * p.q_heads + kv_head * GROUP;

    const int ctx = p.context_lens[seq];
    const int max_ctx = static_cast<int>(min(p.max_context, p.max_blocks * kDecodeBlockTokens));
    if (ctx < 1 || ctx > max_ctx) {
        if (split == 0) {
            if (threadIdx.x == 0) flag_error(p.error_word, kErrContext);
            for (int i = threadIdx.x; i < GROUP * D; i += blockDim.x) {
                if (p.emit_partials) {
                    p.part_o[row0 * D + i] = 0.0f;
                    if (i % D == 0) {
                        p.part_m[row0 + i / D] = -INFINITY;
                        p.part_l[row0 + i / D] = 0.0f;
                    }
                } else {
                    p.out[row0 * D + i] = 0.0f;
                }
            }
        }
        return;
    }
    const int nblk = (ctx + kDecodeBlockTokens - 1) / kDecodeBlockTokens;
    const int bps = static_cast<int>(p.blocks_per_split);
    const int nsplit = (nblk + bps - 1) / bps;
    if (static_cast<int>(split) >= nsplit) return;
    const int b0 = static_cast<int>(split) * bps;
    const int nb = min(nblk - b0, bps);

    // This warp's blocks: local index warp, warp + W, ...
    const int my_count = warp < nb ? (nb - warp + kDecodeWarps - 1) / kDecodeWarps : 0;
    unsigned char* tiles = smem + static_cast<std::size_t>(warp) * kDecodeStages * 2 * S::kTileBytes;
    std::uint64_t* my_bars = bars + warp * kDecodeStages;
    const std::size_t head_offset = static_cast<std::size_t>(kv_head) * S::kTileBytes;
    const std::size_t block_stride = static_cast<std::size_t>(p.kv_heads) * S::kTileBytes;
    // Physical block of the split's local block i (an id outside the pool is
    // reported and replaced by block 0, never dereferenced).
    auto block_id = [&](int i) {
        std::int32_t id = p.tables[static_cast<std::size_t>(seq) * p.max_blocks + b0 + i];
        if (id < 0 || static_cast<std::uint64_t>(id) >= p.num_blocks) {
            flag_error(p.error_word, kErrBadBlock);
            id = 0;
        }
        return id;
    };
    auto issue_block = [&](int j, std::int32_t id) {
        const int stage = j % kDecodeStages;
        const std::size_t src = static_cast<std::size_t>(id) * block_stride + head_offset;
        unsigned char* dst = tiles + static_cast<std::size_t>(stage) * 2 * S::kTileBytes;
        mbar_arrive_expect_tx(&my_bars[stage], 2 * S::kTileBytes);
        bulk_copy_g2s(dst, p.key_arena + src, S::kTileBytes, &my_bars[stage]);
        bulk_copy_g2s(dst + S::kTileBytes, p.value_arena + src, S::kTileBytes, &my_bars[stage]);
    };
    // Each warp starts its first copies at once: lane 0 initialises the
    // warp's own barriers and reads those blocks' ids itself, before the CTA
    // has read the rest of the split's table and the queries.
    if (lane == 0) {
        for (int st = 0; st < kDecodeStages; ++st) mbar_init(&my_bars[st], 1);
        fence_barrier_init();
        std::int32_t first[kDecodeStages];
        const int n_first = min(my_count, kDecodeStages);
#pragma unroll
        for (int j = 0; j < kDecodeStages; ++j) first[j] = j < n_first ? block_id(warp + j * kDecodeWarps) : 0;
#pragma unroll
        for (int j = 0; j < kDecodeStages; ++j) {
            if (j < n_first) issue_block(j, first[j]);
        }
    }
    for (int i = threadIdx.x; i < nb; i += blockDim.x) ids[i] = block_id(i);
    if (threadIdx.x == 0) *flag = 0;
    __syncthreads();

    // Queries of the GQA group, rounded to the pool type (the reference rounds
    // Q in its Fp16/Bf16 modes, kernels/attention_cpu.cpp:456-457).
    const int ts = lane / S::kG;
    const int cg = lane % S::kG;
    // q and the accumulators are held as fp32 pairs (dims 2i, 2i + 1), so the
    // dot products and the P x V update take one f32x2 FMA per two dims: the
    // kernel is bound by instruction issue, not by the fp32 pipe.
    // With the head-split softmax, slot i of a lane's q holds head
    // i ^ own_head, so that every reduce-scatter round below keeps the lower
    // half of the slots (no per-lane selects).
    std::uint64_t q2[GROUP][S::kDpl / 2];
    const int own_head = S::kSplitHeads ? cg / (S::kG / GROUP) : 0;
    bool q_bad = false;
#pragma unroll
    for (int h = 0; h < GROUP; ++h) {
        const float* qrow = p.queries + (row0 + (h ^ own_head)) * D;
#pragma unroll
        for (int c = 0; c < S::kCh; ++c) {
            const int base = (cg + S::kG * c) * S::kEpc;
#pragma unroll
            for (int e = 0; e < S::kEpc; e += 4) {
                const float4 v = *reinterpret_cast<const float4*>(qrow + base + e);
                q_bad |= !(isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w));
                const int i = (c * S::kEpc + e) / 2;
                q2[h][i] = pack_f32x2(round_storage(v.x, Storage<KvT>::kType),
                                      round_storage(v.y, Storage<KvT>::kType));
                q2[h][i + 1] = pack_f32x2(round_storage(v.z, Storage<KvT>::kType),
                                          round_storage(v.w, Storage<KvT>::kType));
            }
        }
    }
    if (q_bad) flag_error(p.error_word, kErrNonFinite);

    auto issue = [&](int j) { issue_block(j, ids[warp + j * kDecodeWarps]); };

    float m[GROUP];
    float l[GROUP];
    float m_own = -INFINITY;  // head-split softmax: this lane's own head
    float l_own = 0.0f;
    const int slot_base = lane - cg;  // first lane of this token row
    std::uint64_t acc2[GROUP][S::kDpl / 2];
#pragma unroll
    for (int h = 0; h < GROUP; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.0f;
#pragma unroll
        for (int e = 0; e < S::kDpl / 2; ++e) acc2[h][e] = 0;
    }

    int consumed = 0;
    for (int j = 0; j < my_count; ++j) {
        const int stage = j % kDecodeStages;
        // Warp-uniform outcome: the shuffles below need every lane.
        if (!__all_sync(0xffffffffu,
                        mbar_wait_bounded(&my_bars[stage], (j / kDecodeStages) & 1, p.error_word))) {
            *flag = 1;
            break;
        }
        consumed = j + 1;
        const unsigned char* ktile = tiles + static_cast<std::size_t>(stage) * 2 * S::kTileBytes;
        const unsigned char* vtile = ktile + S::kTileBytes;
        const int first_token = (b0 + warp + j * kDecodeWarps) * kDecodeBlockTokens;
        const int valid = min(kDecodeBlockTokens, ctx - first_token);

        float s[GROUP][S::kR];
#pragma unroll
        for (int r = 0; r < S::kR; ++r) {
            const int trow = ts + S::kTS * r;
            std::uint64_t part2[GROUP];
#pragma unroll
            for (int h = 0; h < GROUP; ++h) part2[h] = 0;
#pragma unroll
            for (int c = 0; c < S::kCh; ++c) {
                const uint4 raw = *reinterpret_cast<const uint4*>(
                    ktile + (static_cast<std::size_t>(trow) * S::kChunks + cg + S::kG * c) * 16);
                std::uint64_t k2[S::kEpc / 2];
                widen16_pairs(raw, k2, KvT{});
#pragma unroll
                for (int h = 0; h < GROUP; ++h) {
#pragma unroll
                    for (int e = 0; e < S::kEpc / 2; ++e) {
                        part2[h] = fma2(q2[h][c * S::kEpc / 2 + e], k2[e], part2[h]);
                    }
                }
            }
#pragma unroll
            for (int h = 0; h < GROUP; ++h) s[h][r] = low_f32(part2[h]) + high_f32(part2[h]);
        }
        if constexpr (S::kSplitHeads) {
            // Reduce-scatter over the heads: each round halves the heads a
            // lane holds, keeping the half with its own head (cg / kLph), then
            // the kLph lanes of that head sum its scores. Slot i holds head
            // i ^ own_head, so the kept half is always slots [0, n / 2) and the
            // partner lane (own_head differing in the round's bit) sends the
            // same heads from its slots [n / 2, n). s[0] then holds this
            // lane's own head.
            constexpr int kLph = S::kG / GROUP;
#pragma unroll
            for (int k = 0; k < ilog2(GROUP); ++k) {
                const int n = GROUP >> k;
                const int off = S::kG >> (k + 1);
#pragma unroll
                for (int i = 0; i < n / 2; ++i) {
#pragma unroll
                    for (int r = 0; r < S::kR; ++r) {
                        s[i][r] += __shfl_xor_sync(0xffffffffu, s[i + n / 2][r], off);
                    }
                }
            }
#pragma unroll
            for (int off = kLph / 2; off >= 1; off >>= 1) {
#pragma unroll
                for (int r = 0; r < S::kR; ++r) s[0][r] += __shfl_xor_sync(0xffffffffu, s[0][r], off);
            }
            float mx = -INFINITY;
#pragma unroll
            for (int r = 0; r < S::kR; ++r) {
                s[0][r] = (ts + S::kTS * r) < valid ? s[0][r] * p.scale_log2 : -INFINITY;
                mx = fmaxf(mx, s[0][r]);
            }
            const float m_new = fmaxf(m_own, mx);
            const bool grow = m_new > m_own + kDecodeRescale;
            float alpha_own = 1.0f;
            if (grow) {
                alpha_own = exp2f(m_own - m_new);
                m_own = m_new;
            }
            const float base = safe_max(m_own);
            float sum = 0.0f;
#pragma unroll
            for (int r = 0; r < S::kR; ++r) {
                s[0][r] = exp2f(s[0][r] - base);
                sum += s[0][r];
            }
            l_own = l_own * alpha_own + sum;
            // Every head's probabilities (and, when some head's max moved, its
            // rescale factor) from its lanes.
            if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
                for (int h = 0; h < GROUP; ++h) {
                    const float alpha = __shfl_sync(0xffffffffu, alpha_own, slot_base + h * kLph);
                    const std::uint64_t alpha2 = pack_f32x2(alpha, alpha);
#pragma unroll
                    for (int e = 0; e < S::kDpl / 2; ++e) acc2[h][e] = mul2(acc2[h][e], alpha2);
                }
            }
            float p_all[GROUP][S::kR];
#pragma unroll
            for (int h = 0; h < GROUP; ++h) {
                const int src = slot_base + h * kLph;
#pragma unroll
                for (int r = 0; r < S::kR; ++r) p_all[h][r] = __shfl_sync(0xffffffffu, s[0][r], src);
            }
#pragma unroll
            for (int h = 0; h < GROUP; ++h) {
#pragma unroll
                for (int r = 0; r < S::kR; ++r) s[h][r] = p_all[h][r];
            }
        } else {
    #pragma unroll
            for (int off = 1; off < S::kG; off <<= 1) {
    #pragma unroll
                for (int h = 0; h < GROUP; ++h) {
    #pragma unroll
                    for (int r = 0; r < S::kR; ++r) s[h][r] += __shfl_xor_sync(0xffffffffu, s[h][r], off);
                }
            }
    #pragma unroll
            for (int h = 0; h < GROUP; ++h) {
                float mx = -INFINITY;
    #pragma unroll
                for (int r = 0; r < S::kR; ++r) {
                    s[h][r] = (ts + S::kTS * r) < valid ? s[h][r] * p.scale_log2 : -INFINITY;
                    mx = fmaxf(mx, s[h][r]);
                }
                const float m_new = fmaxf(m[h], mx);
                const bool grow = m_new > m[h] + kDecodeRescale;
                float alpha = 1.0f;
                if (grow) {
                    alpha = exp2f(m[h] - m_new);
                    m[h] = m_new;
                }
                const float base = safe_max(m[h]);
                float sum = 0.0f;
    #pragma unroll
                for (int r = 0; r < S::kR; ++r) {
                    s[h][r] = exp2f(s[h][r] - base);
                    sum += s[h][r];
                }
                l[h] = l[h] * alpha + sum;
                if (__any_sync(0xffffffffu, grow)) {
                    const std::uint64_t alpha2 = pack_f32x2(alpha, alpha);
    #pragma unroll
                    for (int e = 0; e < S::kDpl / 2; ++e) acc2[h][e] = mul2(acc2[h][e], alpha2);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < S::kR; ++r) {
            const int trow = ts + S::kTS * r;
            if (trow >= valid) continue;
            std::uint64_t p2[GROUP];
#pragma unroll
            for (int h = 0; h < GROUP; ++h) p2[h] = pack_f32x2(s[h][r], s[h][r]);
#pragma unroll
            for (int c = 0; c < S::kCh; ++c) {
                const uint4 raw = *reinterpret_cast<const uint4*>(
                    vtile + (static_cast<std::size_t>(trow) * S::kChunks + cg + S::kG * c) * 16);
                std::uint64_t v2[S::kEpc / 2];
                widen16_pairs(raw, v2, KvT{});
#pragma unroll
                for (int h = 0; h < GROUP; ++h) {
                    const std::uint64_t s2 = p2[h];
#pragma unroll
                    for (int e = 0; e < S::kEpc / 2; ++e) {
                        acc2[h][c * S::kEpc / 2 + e] = fma2(s2, v2[e], acc2[h][c * S::kEpc / 2 + e]);
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0 && j + kDecodeStages < my_count) issue(j + kDecodeStages);
    }
    if constexpr (S::kSplitHeads) {
#pragma unroll
        for (int h = 0; h < GROUP; ++h) {
            const int src = slot_base + h * (S::kG / GROUP);
            m[h] = __shfl_sync(0xffffffffu, m_own, src);
            l[h] = __shfl_sync(0xffffffffu, l_own, src);
        }
    }
    if (*flag) {
        // A wait gave up: drain this warp's copies still in flight (bounded)
        // before the CTA's shared memory can be released.
        for (int j = consumed; j < min(my_count, consumed + kDecodeStages); ++j) {
            mbar_wait_bounded(&my_bars[j % kDecodeStages], (j / kDecodeStages) & 1, p.error_word);
        }
    }

    // Merge the token-slot states inside the warp (butterfly over slot bits).
#pragma unroll
    for (int off = S::kG; off < 32; off <<= 1) {
#pragma unroll
        for (int h = 0; h < GROUP; ++h) {
            const float mo = __shfl_xor_sync(0xffffffffu, m[h], off);
            const float lo = __shfl_xor_sync(0xffffffffu, l[h], off);
            const float mn = fmaxf(m[h], mo);
            const float base = safe_max(mn);
            const float a = exp2f(m[h] - base);
            const float b = exp2f(mo - base);
            l[h] = l[h] * a + lo * b;
#pragma unroll
            for (int e = 0; e < S::kDpl / 2; ++e) {
                const float x0 = low_f32(acc2[h][e]);
                const float x1 = high_f32(acc2[h][e]);
                const float o0 = __shfl_xor_sync(0xffffffffu, x0, off);
                const float o1 = __shfl_xor_sync(0xffffffffu, x1, off);
                acc2[h][e] = pack_f32x2(x0 * a + o0 * b, x1 * a + o1 * b);
            }
            m[h] = mn;
        }
    }
    if (ts == 0) {
#pragma unroll
        for (int h = 0; h < GROUP; ++h) {
            float* dst = red_acc(warp, h);
#pragma unroll
            for (int c = 0; c < S::kCh; ++c) {
#pragma unroll
                for (int e = 0; e < S::kEpc / 2; ++e) {
                    const std::uint64_t x = acc2[h][c * S::kEpc / 2 + e];
                    dst[(cg + S::kG * c) * S::kEpc + 2 * e] = low_f32(x);
                    dst[(cg + S::kG * c) * S::kEpc + 2 * e + 1] = high_f32(x);
                }
            }
            if (cg == 0) {
                red_ml(warp, h)[0] = m[h];
                red_ml(warp, h)[1] = l[h];
            }
        }
    }
    __syncthreads();
    if (*flag) return;

    // Merge the warps; write the output or this split's partial.
    const bool single = nsplit == 1;
    for (int i = threadIdx.x; i < GROUP * D; i += blockDim.x) {
        const int h = i / D;
        const int dim = i % D;
        float mw = -INFINITY;
#pragma unroll
        for (int w = 0; w < kDecodeWarps; ++w) mw = fmaxf(mw, red_ml(w, h)[0]);
        const float base = safe_max(mw);
        float lsum = 0.0f;
        float a = 0.0f;
#pragma unroll
        for (int w = 0; w < kDecodeWarps; ++w) {
            const float f = exp2f(red_ml(w, h)[0] - base);
            lsum += red_ml(w, h)[1] * f;
            a += red_acc(w, h)[dim] * f;
        }
        const std::size_t row = row0 + h;
        if (single) {
            if constexpr (kExchange) {
                push_word<D>(p, 2 * p.xrows + row * D + dim, a);
                if (dim == 0) {
                    push_word<D>(p, row, mw * kLn2);
                    push_word<D>(p, p.xrows + row, lsum);
                }
            } else if (p.emit_partials) {
                p.part_o[row * D + dim] = a;
                if (dim == 0) {
                    p.part_m[row] = mw * kLn2;
                    p.part_l[row] = lsum;
                }
            } else {
                if (dim == 0 && !(isfinite(lsum) && lsum > 0.0f)) flag_error(p.error_word, kErrNormalizer);
                p.out[row * D + dim] = a / lsum;
            }
        } else {
            const std::size_t slot = row * p.max_splits + split;
            p.ws_o[slot * D + dim] = a;
            if (dim == 0) {
                p.ws_ml[slot * 2] = mw;
                p.ws_ml[slot * 2 + 1] = lsum;
            }
        }
    }
    if (single) {
        if constexpr (kExchange) {
            __syncthreads();  // the tile area is free: it stages the received rows
            receive_and_merge<D, GROUP>(p, row0, reinterpret_cast<float*>(smem));
        }
        return;
    }

    // Fused split combine: the last CTA of this (sequence, kv-head) merges.
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const std::uint32_t previous = atomicAdd(&p.ws_count[pair], 1u);
        *flag = previous == static_cast<std::uint32_t>(nsplit - 1) ? 2 : 0;
    }
    __syncthreads();
    if (*flag != 2) return;
    __threadfence();
    // Split weights, once per q-head (one warp per head), into the tile area,
    // which no copy uses any more: w[h][sp] = 2^(m_sp - M_h), and per head
    // (M_h, L_h = sum_sp l_sp w[h][sp]) into warp 0's (m, l) slots.
    float* w = reinterpret_cast<float*>(smem);
    for (int h = warp; h < GROUP; h += kDecodeWarps) {
        const float* ml = p.ws_ml + (row0 + h) * p.max_splits * 2;
        float mw = -INFINITY;
        for (int sp = lane; sp < nsplit; sp += 32) mw = fmaxf(mw, __ldcg(ml + sp * 2));
        mw = warp_max(mw);
        const float base = safe_max(mw);
        float lsum = 0.0f;
        for (int sp = lane; sp < nsplit; sp += 32) {
            const float f = exp2f(__ldcg(ml + sp * 2) - base);
            w[h * nsplit + sp] = f;
            lsum += __ldcg(ml + sp * 2 + 1) * f;
        }
        lsum = warp_sum(lsum);
        if (lane == 0) {
            red_ml(0, h)[0] = mw;
            red_ml(0, h)[1] = lsum;
        }
    }
    __syncthreads();
    // Each thread merges four consecutive dims (one float4 per split), eight
    // splits in flight at a time, so the L2 reads of the partials overlap.
    for (int i4 = threadIdx.x; i4 < GROUP * D / 4; i4 += blockDim.x) {
        const int h = (i4 * 4) / D;
        const int dim = (i4 * 4) % D;
        const std::size_t row = row0 + h;
        const float4* o = reinterpret_cast<const float4*>(p.ws_o + row * p.max_splits * D + dim);
        const float* wh = w + h * nsplit;
        float4 a = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        int sp = 0;
        for (; sp + 8 <= nsplit; sp += 8) {
            float4 x[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) x[u] = __ldcg(o + static_cast<std::size_t>(sp + u) * (D / 4));
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const float f = wh[sp + u];
                a.x = fmaf(x[u].x, f, a.x);
                a.y = fmaf(x[u].y, f, a.y);
                a.z = fmaf(x[u].z, f, a.z);
                a.w = fmaf(x[u].w, f, a.w);
            }
        }
        for (; sp < nsplit; ++sp) {
            const float4 x = __ldcg(o + static_cast<std::size_t>(sp) * (D / 4));
            const float f = wh[sp];
            a.x = fmaf(x.x, f, a.x);
            a.y = fmaf(x.y, f, a.y);
            a.z = fmaf(x.z, f, a.z);
            a.w = fmaf(x.w, f, a.w);
        }
        const float mw = red_ml(0, h)[0];
        const float lsum = red_ml(0, h)[1];
        if constexpr (kExchange) {
            push_word<D>(p, 2 * p.xrows + row * D + dim, a.x);
            push_word<D>(p, 2 * p.xrows + row * D + dim + 1, a.y);
            push_word<D>(p, 2 * p.xrows + row * D + dim + 2, a.z);
            push_word<D>(p, 2 * p.xrows + row * D + dim + 3, a.w);
            if (dim == 0) {
                push_word<D>(p, row, mw * kLn2);
                push_word<D>(p, p.xrows + row, lsum);
            }
        } else if (p.emit_partials) {
            *reinterpret_cast<float4*>(p.part_o + row * D + dim) = a;
            if (dim == 0) {
                p.part_m[row] = mw * kLn2;
                p.part_l[row] = lsum;
            }
        } else {
            if (dim == 0 && !(isfinite(lsum) && lsum > 0.0f)) flag_error(p.error_word, kErrNormalizer);
            *reinterpret_cast<float4*>(p.out + row * D + dim) =
                make_float4(a.x / lsum, a.y / lsum, a.z / lsum, a.w / lsum);
        }
    }
    if (threadIdx.x == 0) p.ws_count[pair] = 0;
    if constexpr (kExchange) {
        __syncthreads();  // the split weights in the tile area are dead
        receive_and_merge<D, GROUP>(p, row0, reinterpret_cast<float*>(smem));
    }
}

// K4: log-sum-exp merge of partials in part order; one warp per row.
// Part i of the merge reads m at part_m + i * stride_m, l at part_l +
// i * stride_l and o at part_o + i * stride_o: dense [parts][rows] arrays, or
// one packed [m | l | o] block per part as an all-gather delivers it.
__global__ void lse_combine_kernel(const float* part_m, const float* part_l, const float* part_o,
                                   std::uint32_t parts, std::uint64_t rows, std::uint32_t head_dim,
                                   std::uint64_t stride_m, std::uint64_t stride_l,
                                   std::uint64_t stride_o, float* out) {
    const std::uint64_t row = static_cast<std::uint64_t>(blockIdx.x) * (blockDim.x / 32) +
                              threadIdx.x / 32;
    if (row >= rows) return;
    lse_merge_row(part_m, part_l, part_o, parts, row, head_dim, stride_m, stride_l, stride_o, out,
                  threadIdx.x & 31);
}

struct DecodePlan {
    std::uint32_t blocks_per_split;
    std::uint32_t max_splits;
};

DecodePlan plan_decode(std::uint32_t num_seqs, std::uint32_t kv_heads,
                       std::uint32_t max_context_len, std::uint32_t fixed_blocks_per_split) {
    const std::uint32_t max_blocks =
        (max_context_len + kDecodeBlockTokens - 1) / kDecodeBlockTokens;
    std::uint32_t bps = fixed_blocks_per_split;
    if (bps == 0) {
        // Aim for about 2048 CTAs (4.6 waves of three CTAs per SM across 148
        // SMs) if every context were max_context_len long, with at least 8
        // blocks per split. Measured on 64 x U[64, 2048] fp32 (32 blocks per
        // split best: 16 blocks 4% and 22-26 blocks 3% slower) and on the
        // Zipf-skewed 32 x [32, 8192] bf16 GQA batch (64 blocks per split
        // 98.4 us; 57 blocks 106.4, 74 blocks 104.4, 86 blocks 114.6).
        const std::uint64_t pairs = static_cast<std::uint64_t>(num_seqs) * kv_heads;
        const std::uint64_t target = 2048;
        std::uint64_t splits = (target + pairs - 1) / pairs;
        splits = std::max<std::uint64_t>(1, std::min<std::uint64_t>(splits, max_blocks));
        bps = static_cast<std::uint32_t>((max_blocks + splits - 1) / splits);
        bps = std::max<std::uint32_t>(bps, 8);
    }
    // Splits of at most 256 blocks (4096 tokens) keep CTAs short enough to
    // balance; only contexts beyond kMaxSplits * 256 blocks get longer ones.
    bps = std::min<std::uint32_t>(std::max<std::uint32_t>(bps, 1), 256);
    // The fused merge keeps one weight per (q-head, split) in the tile area:
    // at most kMaxSplits splits per context.
    bps = std::max<std::uint32_t>(bps, (max_blocks + kMaxSplits - 1) / kMaxSplits);
    if (bps > kMaxBlocksPerSplit) {
        throw std::runtime_error(
            "paged decode context is longer than the kernel supports (1048576 tokens)");
    }
    const std::uint32_t max_splits = std::max<std::uint32_t>(1, (max_blocks + bps - 1) / bps);
    return DecodePlan{bps, max_splits};
}

std::size_t workspace_bytes_for(std::uint32_t num_seqs, std::uint32_t q_heads,
                                std::uint32_t kv_heads, std::uint32_t head_dim,
                                const DecodePlan& plan) {
    const std::size_t counters = (static_cast<std::size_t>(num_seqs) * kv_heads * 4 + 255) & ~std::size_t(255);
    const std::size_t slots = static_cast<std::size_t>(num_seqs) * q_heads * plan.max_splits;
    const std::size_t ml = (slots * 2 * 4 + 255) & ~std::size_t(255);
    return counters + ml + slots * head_dim * 4;
}

using DecodeKernel = void (*)(const DecodeParams);

template <typename KvT, int D, bool kExchange = false>
DecodeKernel pick_group(std::uint32_t group) {
    switch (group) {
        case 1: return paged_decode_kernel<KvT, D, 1, kExchange>;
        case 2: return paged_decode_kernel<KvT, D, 2, kExchange>;
        case 4: return paged_decode_kernel<KvT, D, 4, kExchange>;
        case 8: return paged_decode_kernel<KvT, D, 8, kExchange>;
        default: return nullptr;
    }
}

template <typename KvT, int D>
std::size_t smem_for_group(std::uint32_t group) {
    switch (group) {
        case 1: return DecodeSmem<KvT, D, 1>::kBytes;
        case 2: return DecodeSmem<KvT, D, 2>::kBytes;
        case 4: return DecodeSmem<KvT, D, 4>::kBytes;
        case 8: return DecodeSmem<KvT, D, 8>::kBytes;
        default: return 0;
    }
}

template <typename KvT, bool kExchange = false>
DecodeKernel pick_kernel(std::uint32_t head_dim, std::uint32_t group, std::size_t& smem) {
    if (head_dim == 64) {
        smem = smem_for_group<KvT, 64>(group);
        return pick_group<KvT, 64, kExchange>(group);
    }
    if (head_dim == 128) {
        smem = smem_for_group<KvT, 128>(group);
        return pick_group<KvT, 128, kExchange>(group);
    }
    return nullptr;
}

// The fast kernel covers block_tokens 16, head_dim 64/128 and GQA groups of
// 1/2/4/8; other pool geometries use the generic CUDA-core kernel.
// `exchange` picks the split-sequence variant with the peer exchange fused.
DecodeKernel select_decode(const InferlabCudaKvPool& pool, std::uint32_t group, std::size_t& smem,
                           bool exchange = false) {
    if (pool.block_tokens != kDecodeBlockTokens) return nullptr;
    if (pool.dtype == kFp32) {
        return exchange ? pick_kernel<float, true>(pool.head_dim, group, smem)
                        : pick_kernel<float>(pool.head_dim, group, smem);
    }
    if (pool.dtype == kF16) {
        return exchange ? pick_kernel<__half, true>(pool.head_dim, group, smem)
                        : pick_kernel<__half>(pool.head_dim, group, smem);
    }
    return exchange ? pick_kernel<__nv_bfloat16, true>(pool.head_dim, group, smem)
                    : pick_kernel<__nv_bfloat16>(pool.head_dim, group, smem);
}

// CTAs of `kernel` resident per SM times the SMs of `device` (cached per
// kernel and device; 0 when unknown).
std::uint32_t resident_slots(DecodeKernel kernel, std::size_t smem, int device) {
    static std::mutex mutex;
    static std::map<std::pair<const void*, int>, std::uint32_t> cache;
    std::lock_guard<std::mutex> lock(mutex);
    const auto key = std::make_pair(reinterpret_cast<const void*>(kernel), device);
    const auto found = cache.find(key);
    if (found != cache.end()) return found->second;
    int per_sm = 0, sms = 0;
    std::uint32_t slots = 0;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) == cudaSuccess &&
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kDecodeWarps * 32, smem) ==
            cudaSuccess &&
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) == cudaSuccess) {
        slots = static_cast<std::uint32_t>(per_sm * sms);
    } else {
        cudaGetLastError();
    }
    cache.emplace(key, slots);
    return slots;
}

// The split plan of a batch on this pool. One sequence (the split long
// sequence, or a batch of one) is cut into as many equal splits as fill one
// wave of resident CTAs exactly: a wave and a sliver (e.g. 64 splits x 8
// kv-heads = 512 CTAs on 444 slots) would take two CTA durations.
DecodePlan full_plan(const InferlabCudaKvPool& p, std::uint32_t num_seqs, std::uint32_t q_heads,
                     std::uint32_t max_context_len) {
    DecodePlan plan = plan_decode(num_seqs, p.kv_heads, max_context_len, p.decode_blocks_per_split);
    if (num_seqs != 1 || p.decode_blocks_per_split != 0 || q_heads % p.kv_heads != 0) return plan;
    std::size_t smem = 0;
    DecodeKernel kernel = select_decode(p, q_heads / p.kv_heads, smem);
    if (kernel == nullptr) return plan;
    const std::uint32_t slots = resident_slots(kernel, smem, p.device);
    if (slots == 0 || plan.max_splits * p.kv_heads <= slots) return plan;
    const std::uint32_t max_blocks =
        (max_context_len + kDecodeBlockTokens - 1) / kDecodeBlockTokens;
    const std::uint32_t splits = std::min<std::uint32_t>(kMaxSplits, slots / p.kv_heads);
    if (splits == 0) return plan;
    const std::uint32_t bps = (max_blocks + splits - 1) / splits;
    if (bps > static_cast<std::uint32_t>(kMaxBlocksPerSplit)) return plan;
    return DecodePlan{bps, (max_blocks + bps - 1) / bps};
}

void validate_decode(const InferlabCudaKvPool& p, const float* queries,
                     const std::int32_t* block_tables, std::uint32_t max_blocks,
                     const std::int32_t* context_lens, std::uint32_t num_seqs,
                     std::uint32_t q_heads, std::uint32_t max_context_len) {
    if (queries == nullptr || block_tables == nullptr || context_lens == nullptr) {
        throw std::runtime_error("paged decode pointer is null");
    }
    if (q_heads == 0 || q_heads % p.kv_heads != 0) {
        throw std::runtime_error("paged decode q_heads must be a positive multiple of kv_heads");
    }
    if (max_blocks == 0 || max_context_len == 0) {
        throw std::runtime_error("paged decode block table and context bound must be positive");
    }
    if (num_seqs > 0x7FFFFFFFu / std::max<std::uint32_t>(1, p.kv_heads)) {
        throw std::runtime_error("paged decode batch is too large");
    }
}

void run_decode(InferlabCudaKvPool& p, const float* queries, const std::int32_t* block_tables,
                std::uint32_t max_blocks, const std::int32_t* context_lens, std::uint32_t num_seqs,
                std::uint32_t q_heads, std::uint32_t max_context_len, float* out, float* part_m,
                float* part_l, float* part_o, void* workspace, std::size_t workspace_bytes,
                cudaStream_t stream, const ExchangeView* xview = nullptr) {
    const std::uint32_t group = q_heads / p.kv_heads;
    std::size_t smem = 0;
    DecodeKernel kernel = select_decode(p, group, smem, xview != nullptr);
    if (kernel == nullptr) {
        // Generic CUDA-core path (any head_dim / block size / group).
        if (xview != nullptr) {
            throw std::runtime_error(
                "paged decode exchange needs block_tokens 16, head_dim 64 or 128 and a GQA group of 1, 2, 4 or 8");
        }
        if (part_m != nullptr) {
            throw std::runtime_error(
                "paged decode partials need block_tokens 16, head_dim 64 or 128 and a GQA group of 1, 2, 4 or 8");
        }
        if (p.head_dim > kGenericMaxHeadDim) {
            throw std::runtime_error("attention head_dimension exceeds the CUDA kernel limit of 4096");
        }
        GenericParams g{};
        g.queries = queries;
        g.query_precision = p.dtype;
        g.out = out;
        g.query_rows = num_seqs;
        g.q_heads = q_heads;
        g.kv_heads = p.kv_heads;
        g.head_dim = p.head_dim;
        g.scale = 1.0f / std::sqrt(static_cast<float>(p.head_dim));
        g.error_word = p.error_word;
        g.check_normalizer = 1;
        SegmentMap seg{};
        seg.mode = 1;
        seg.context_lens = context_lens;
        seg.max_kv = std::min<long long>(max_context_len,
                                         static_cast<long long>(max_blocks) * p.block_tokens);
        const std::size_t gsmem = generic_smem_bytes(p.head_dim);
        const unsigned grid = static_cast<unsigned>(
            (static_cast<std::size_t>(num_seqs) * q_heads + kGenericWarps - 1) / kGenericWarps);
        auto launch = [&](auto kv) {
            auto* fn = generic_attention_kernel<decltype(kv)>;
            cuda_check(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(gsmem)),
                       "cudaFuncSetAttribute");
            fn<<<grid, kGenericWarps * 32, gsmem, stream>>>(g, kv, seg);
        };
        if (p.dtype == kFp32) {
            launch(PagedKv<float>{static_cast<const float*>(p.key_arena),
                                  static_cast<const float*>(p.value_arena), block_tables,
                                  max_blocks, p.block_tokens, p.kv_heads, p.head_dim,
                                  p.num_blocks, p.error_word});
        } else if (p.dtype == kF16) {
            launch(PagedKv<__half>{static_cast<const __half*>(p.key_arena),
                                   static_cast<const __half*>(p.value_arena), block_tables,
                                   max_blocks, p.block_tokens, p.kv_heads, p.head_dim,
                                   p.num_blocks, p.error_word});
        } else {
            launch(PagedKv<__nv_bfloat16>{static_cast<const __nv_bfloat16*>(p.key_arena),
                                          static_cast<const __nv_bfloat16*>(p.value_arena),
                                          block_tables, max_blocks, p.block_tokens, p.kv_heads,
                                          p.head_dim, p.num_blocks, p.error_word});
        }
        cuda_check(cudaGetLastError(), "generic decode launch");
        return;
    }
    if (reinterpret_cast<std::uintptr_t>(queries) % 16 != 0) {
        throw std::runtime_error("paged decode queries must be 16-byte aligned");
    }
    const DecodePlan plan = full_plan(p, num_seqs, q_heads, max_context_len);
    const std::size_t need = workspace_bytes_for(num_seqs, q_heads, p.kv_heads, p.head_dim, plan);
    if (plan.max_splits > 1 && (workspace == nullptr || workspace_bytes < need)) {
        throw std::runtime_error("paged decode workspace is too small");
    }
    DecodeParams d{};
    d.key_arena = static_cast<const unsigned char*>(p.key_arena);
    d.value_arena = static_cast<const unsigned char*>(p.value_arena);
    d.num_blocks = p.num_blocks;
    d.kv_heads = p.kv_heads;
    d.queries = queries;
    d.q_heads = q_heads;
    d.tables = block_tables;
    d.max_blocks = max_blocks;
    d.context_lens = context_lens;
    d.max_context = max_context_len;
    d.blocks_per_split = plan.blocks_per_split;
    d.max_splits = plan.max_splits;
    d.scale_log2 = (1.0f / std::sqrt(static_cast<float>(p.head_dim))) * kLog2e;
    d.emit_partials = part_m != nullptr ? 1 : 0;
    d.out = out;
    d.part_m = part_m;
    d.part_l = part_l;
    d.part_o = part_o;
    if (workspace != nullptr) {
        auto* base = static_cast<unsigned char*>(workspace);
        const std::size_t counters =
            (static_cast<std::size_t>(num_seqs) * p.kv_heads * 4 + 255) & ~std::size_t(255);
        const std::size_t slots = static_cast<std::size_t>(num_seqs) * q_heads * plan.max_splits;
        const std::size_t ml = (slots * 2 * 4 + 255) & ~std::size_t(255);
        d.ws_count = reinterpret_cast<std::uint32_t*>(base);
        d.ws_ml = reinterpret_cast<float*>(base + counters);
        d.ws_o = reinterpret_cast<float*>(base + counters + ml);
    }
    d.error_word = p.error_word;
    if (xview != nullptr) {
        for (std::uint32_t r = 0; r < xview->world; ++r) d.xwords[r] = xview->words[r];
        d.xout = out;
        d.xrows = xview->rows;
        d.xworld = xview->world;
        d.xrank = xview->rank;
        d.xstep = xview->step;
    }
    cuda_check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem)),
               "cudaFuncSetAttribute");
    const std::uint64_t grid = static_cast<std::uint64_t>(num_seqs) * p.kv_heads * plan.max_splits;
    if (grid > 0x7FFFFFFFull) throw std::runtime_error("paged decode grid is too large");
    kernel<<<static_cast<unsigned>(grid), kDecodeWarps * 32, smem, stream>>>(d);
    cuda_check(cudaGetLastError(), "paged decode launch");
}

}  // namespace
}  // namespace ilb

// Shared launch path for decode entry points in other files (internal.cuh).
namespace ilb {

std::size_t decode_workspace_bytes(const InferlabCudaKvPool& pool, std::uint32_t num_seqs,
                                   std::uint32_t q_heads, std::uint32_t max_context_len) {
    const auto plan = full_plan(pool, num_seqs, q_heads, max_context_len);
    return workspace_bytes_for(num_seqs, q_heads, pool.kv_heads, pool.head_dim, plan);
}

std::size_t decode_scratch_bytes(const InferlabCudaKvPool& pool, std::uint32_t num_seqs,
                                 std::uint32_t q_heads, std::uint32_t max_context_len) {
    std::size_t smem = 0;
    if (select_decode(pool, q_heads / pool.kv_heads, smem) == nullptr) return 0;
    const auto plan = full_plan(pool, num_seqs, q_heads, max_context_len);
    if (plan.max_splits <= 1) return 0;
    return workspace_bytes_for(num_seqs, q_heads, pool.kv_heads, pool.head_dim, plan);
}

std::size_t decode_counter_bytes(const InferlabCudaKvPool& pool, std::uint32_t num_seqs) {
    return (static_cast<std::size_t>(num_seqs) * pool.kv_heads * 4 + 255) & ~std::size_t(255);
}

void check_decode_arguments(const InferlabCudaKvPool& pool, const float* queries,
                            const std::int32_t* block_tables, std::uint32_t max_blocks,
                            const std::int32_t* context_lens, std::uint32_t num_seqs,
                            std::uint32_t q_heads, std::uint32_t max_context_len) {
    validate_decode(pool, queries, block_tables, max_blocks, context_lens, num_seqs, q_heads,
                    max_context_len);
}

void launch_paged_decode(InferlabCudaKvPool& pool, const float* queries,
                         const std::int32_t* block_tables, std::uint32_t max_blocks,
                         const std::int32_t* context_lens, std::uint32_t num_seqs,
                         std::uint32_t q_heads, std::uint32_t max_context_len, float* out,
                         void* workspace, std::size_t workspace_bytes, cudaStream_t stream) {
    run_decode(pool, queries, block_tables, max_blocks, context_lens, num_seqs, q_heads,
               max_context_len, out, nullptr, nullptr, nullptr, workspace, workspace_bytes, stream);
}

}  // namespace ilb

extern "C" int inferlab_cuda_paged_decode_exchange(InferlabCudaKvPool* pool, const float* queries,
                                                   const std::int32_t* block_tables, std::uint32_t max_blocks,
                                                   const std::int32_t* context_lens, std::uint32_t num_seqs,
                                                   std::uint32_t q_heads, std::uint32_t max_context_len,
                                                   void* workspace, std::size_t workspace_bytes,
                                                   InferlabCudaPeerExchange* exchange, float* out, void* stream,
                                                   char* error, std::size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        auto& p = ilb::checked_pool(pool);
        ilb::validate_decode(p, queries, block_tables, max_blocks, context_lens, num_seqs, q_heads,
                             max_context_len);
        if (out == nullptr) throw std::runtime_error("paged decode pointer is null");
        if (num_seqs == 0) return;
        ilb::DeviceGuard guard(p.device);
        std::size_t smem = 0;
        ilb::DecodeKernel kernel = ilb::select_decode(p, q_heads / p.kv_heads, smem, true);
        if (kernel == nullptr) {
            throw std::runtime_error(
                "paged decode exchange needs block_tokens 16, head_dim 64 or 128 and a GQA group of 1, 2, 4 or 8");
        }
        // The CTAs that finish a (sequence, kv-head) wait for the other ranks'
        // matching CTAs; they must never fill the GPU, or a rank could hold
        // every slot waiting while the CTAs its peers wait for are unscheduled.
        const std::uint32_t slots = ilb::resident_slots(kernel, smem, p.device);
        if (slots == 0 || static_cast<std::uint64_t>(num_seqs) * p.kv_heads * 2 > slots) {
            throw std::runtime_error("paged decode exchange batch is too large for one launch");
        }
        // Every check that can reject the call runs before the step is taken:
        // a rank whose call failed after taking it would wait one step ahead
        // of its peers from then on.
        if (reinterpret_cast<std::uintptr_t>(queries) % 16 != 0) {
            throw std::runtime_error("paged decode queries must be 16-byte aligned");
        }
        const ilb::DecodePlan plan = ilb::full_plan(p, num_seqs, q_heads, max_context_len);
        const std::size_t need =
            ilb::workspace_bytes_for(num_seqs, q_heads, p.kv_heads, p.head_dim, plan);
        if (plan.max_splits > 1 && (workspace == nullptr || workspace_bytes < need)) {
            throw std::runtime_error("paged decode workspace is too small");
        }
        const ilb::ExchangeView view = ilb::exchange_take_step(
            exchange, p.device, static_cast<std::uint64_t>(num_seqs) * q_heads, p.head_dim);
        ilb::run_decode(p, queries, block_tables, max_blocks, context_lens, num_seqs, q_heads,
                        max_context_len, out, nullptr, nullptr, nullptr, workspace, workspace_bytes,
                        static_cast<cudaStream_t>(stream), &view);
    });
}

extern "C" std::size_t inferlab_cuda_paged_decode_workspace_size(const InferlabCudaKvPool* pool,
                                                                 std::uint32_t num_seqs,
                                                                 std::uint32_t q_heads,
                                                                 std::uint32_t max_context_len) {
    if (pool == nullptr || num_seqs == 0 || q_heads == 0 || max_context_len == 0) return 0;
    try {
        const auto plan = ilb::full_plan(*pool, num_seqs, q_heads, max_context_len);
        return ilb::workspace_bytes_for(num_seqs, q_heads, pool->kv_heads, pool->head_dim, plan);
    } catch (...) {
        return 0;  // the decode call itself reports why
    }
}

extern "C" int inferlab_cuda_pool_set_decode_split(InferlabCudaKvPool* pool,
                                                   std::uint32_t blocks_per_split, char* error,
                                                   std::size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        auto& p = ilb::checked_pool(pool);
        if (blocks_per_split > static_cast<std::uint32_t>(ilb::kMaxBlocksPerSplit)) {
            throw std::runtime_error("paged decode split length must be at most 1024 blocks");
        }
        p.decode_blocks_per_split = blocks_per_split;
    });
}

extern "C" int inferlab_cuda_paged_decode_workspace_init(void* workspace,
                                                         std::size_t workspace_bytes,
                                                         void* stream, char* error,
                                                         std::size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        if (workspace == nullptr || workspace_bytes == 0) return;
        ilb::cuda_check(cudaMemsetAsync(workspace, 0, workspace_bytes,
                                        static_cast<cudaStream_t>(stream)),
                        "cudaMemsetAsync workspace");
    });
}

extern "C" int inferlab_cuda_paged_decode(InferlabCudaKvPool* pool, const float* queries,
                                          const std::int32_t* block_tables,
                                          std::uint32_t max_blocks_per_seq,
                                          const std::int32_t* context_lens, std::uint32_t num_seqs,
                                          std::uint32_t q_heads, std::uint32_t max_context_len,
                                          float* out, void* workspace, std::size_t workspace_bytes,
                                          void* stream, char* error, std::size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        using namespace ilb;
        auto& p = checked_pool(pool);
        if (num_seqs == 0) return;
        validate_decode(p, queries, block_tables, max_blocks_per_seq, context_lens, num_seqs,
                        q_heads, max_context_len);
        if (out == nullptr) throw std::runtime_error("paged decode output pointer is null");
        DeviceGuard guard(p.device);
        run_decode(p, queries, block_tables, max_blocks_per_seq, context_lens, num_seqs, q_heads,
                   max_context_len, out, nullptr, nullptr, nullptr, workspace, workspace_bytes,
                   static_cast<cudaStream_t>(stream));
    });
}

extern "C" int inferlab_cuda_paged_decode_partials(
    InferlabCudaKvPool* pool, const float* queries, const std::int32_t* block_tables,
    std::uint32_t max_blocks_per_seq, const std::int32_t* context_lens, std::uint32_t num_seqs,
    std::uint32_t q_heads, std::uint32_t max_context_len, float* part_m, float* part_l,
    float* part_o, void* workspace, std::size_t workspace_bytes, void* stream, char* error,
    std::size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        using namespace ilb;
        auto& p = checked_pool(pool);
        if (num_seqs == 0) return;
        validate_decode(p, queries, block_tables, max_blocks_per_seq, context_lens, num_seqs,
                        q_heads, max_context_len);
        if (part_m == nullptr || part_l == nullptr || part_o == nullptr) {
            throw std::runtime_error("paged decode partial output pointer is null");
        }
        DeviceGuard guard(p.device);
        run_decode(p, queries, block_tables, max_blocks_per_seq, context_lens, num_seqs, q_heads,
                   max_context_len, nullptr, part_m, part_l, part_o, workspace, workspace_bytes,
                   static_cast<cudaStream_t>(stream));
    });
}

namespace {

void launch_lse_combine(const float* part_m, const float* part_l, const float* part_o,
                        std::uint32_t parts, std::uint64_t rows, std::uint32_t head_dim,
                        std::uint64_t stride_m, std::uint64_t stride_l, std::uint64_t stride_o,
                        float* out, void* stream) {
    if (parts == 0 || head_dim == 0) {
        throw std::runtime_error("lse combine parts and head_dim must be positive");
    }
    const std::uint64_t blocks = (rows + 3) / 4;
    if (blocks > 0x7FFFFFFFull) throw std::runtime_error("lse combine is too large");
    ilb::lse_combine_kernel<<<static_cast<unsigned>(blocks), 128, 0, static_cast<cudaStream_t>(stream)>>>(
        part_m, part_l, part_o, parts, rows, head_dim, stride_m, stride_l, stride_o, out);
    ilb::cuda_check(cudaGetLastError(), "lse combine launch");
}

}  // namespace

extern "C" int inferlab_cuda_lse_combine(const float* part_m, const float* part_l,
                                         const float* part_o, std::uint32_t parts,
                                         std::uint64_t rows, std::uint32_t head_dim, float* out,
                                         void* stream, char* error, std::size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        if (rows == 0) return;
        if (part_m == nullptr || part_l == nullptr || part_o == nullptr || out == nullptr) {
            throw std::runtime_error("lse combine pointer is null");
        }
        launch_lse_combine(part_m, part_l, part_o, parts, rows, head_dim, rows, rows,
                           rows * head_dim, out, stream);
    });
}

extern "C" int inferlab_cuda_lse_combine_packed(const float* packed, std::uint32_t parts,
                                                std::uint64_t rows, std::uint32_t head_dim,
                                                float* out, void* stream, char* error,
                                                std::size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        if (rows == 0) return;
        if (packed == nullptr || out == nullptr) throw std::runtime_error("lse combine pointer is null");
        const std::uint64_t part = rows * (static_cast<std::uint64_t>(head_dim) + 2);
        launch_lse_combine(packed, packed + rows, packed + 2 * rows, parts, rows, head_dim, part,
                           part, part, out, stream);
    });
}
