// prefill_tc.cuh - causal / chunked prefill on the sm_100a tensor cores.
//
// Work item: one CTA per (segment, q-head, 128-query tile). The keys a query
// may see follow legal_sources (kernels/attention_cpu.cpp:113-123): query i of
// a segment starting at position P sees keys [0, P + i].
//
// Roles (192 threads):
//   warps 0-3  softmax: thread t owns query row t. S rows come out of TMEM with
//              tcgen05.ld (32x32b: one lane per row, no shuffles), the running
//              max / sum are per thread, P is written to shared memory as
//              fp16 in the 128-byte-swizzled K-major layout the MMA reads, and
//              O lives in 128 fp32 registers per thread.
//   warp 4     TMA producer: Q tile once (3-D map over [tokens][q_heads][128]),
//              then per 128-key tile eight 16-token blocks of K and of V, each
//              a box of the 4-D map over the arena [block][kv_head][slot][128]
//              at the block id the table names (no multicast).
//   warp 5     MMA issuer: S = Q K^T (M=N=128, K=128, f16/bf16 in, fp32 out)
//              into one of two TMEM buffers, so S(j+1) runs while softmax(j)
//              works; PV(j) = P_j V_j (V as an MN-major operand) into a third
//              TMEM buffer, which softmax(j+1) folds into O after rescaling:
//              O <- (O + PV(j)) * alpha(j+1), the online-softmax recurrence of
//              kernels/attention_cpu.cpp:364-386 in the log2 domain.
// Every mbarrier wait is bounded; a wait that gives up records
// kErrWaitTimeout, the CTA drains its own copies and MMAs (bounded) and frees
// its TMEM before returning.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "pool.cuh"

#include <algorithm>
#include <cmath>
#include <mutex>

namespace ilb {
namespace tc {

constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kD = 128;
constexpr int kBlockTokens = 16;
constexpr int kThreads = 192;
constexpr int kHalf = 16384;             // one 64-column half of a 128 x 128 16-bit tile
constexpr int kTile = 2 * kHalf;         // 32 KB
constexpr int kQ = 0;
constexpr int kK0 = kQ + kTile;          // two K stages
constexpr int kV0 = kK0 + 2 * kTile;     // two V stages
constexpr int kP = kV0 + 2 * kTile;
constexpr int kBars = kP + kTile;        // 192 KB
constexpr int kNumBars = 16;
constexpr int kSmemBytes = kBars + kNumBars * 8 + 64;
constexpr int kSmemAlloc = kSmemBytes + 1024;  // slack to align the base to 1024 B
constexpr uint32_t kTmemCols = 512;      // S0 [0,128) S1 [128,256) PV [256,384)

enum Bar : int {
    kBarQ = 0,
    kBarK = 1,      // +stage
    kBarV = 3,      // +stage
    kBarS = 5,      // +buffer
    kBarSFree = 7,  // +buffer, 128 arrivals
    kBarP = 9,      // 128 arrivals
    kBarPV = 10,
    kBarKFree = 11, // +stage
    kBarVFree = 13, // +stage
    kBarDone = 15,
};

struct Params {
    const std::int32_t* tables;
    std::uint32_t max_blocks;
    const std::int32_t* starts;
    const std::int32_t* counts;
    const std::int32_t* offsets;
    std::uint32_t num_segments;
    std::uint32_t q_heads;
    std::uint32_t group;
    std::uint32_t q_tiles;
    std::uint64_t num_blocks;
    long long total_queries;
    float scale_log2;
    float* out;
    std::uint32_t* error_word;
};

// ---- tcgen05 / TMA wrappers ----------------------------------------------
__device__ __forceinline__ void tmem_alloc(std::uint32_t* dst, std::uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst)),
                 "r"(cols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(std::uint32_t taddr, std::uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void mma_f16(std::uint32_t d_tmem, std::uint64_t a_desc,
                                        std::uint64_t b_desc, std::uint32_t idesc,
                                        std::uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void mma_commit(std::uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, std::uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<std::uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, int c3, std::uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<std::uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
        "r"(smem_u32(bar))
        : "memory");
}

// 32 consecutive TMEM columns of this thread's lane (32x32b shape).
__device__ __forceinline__ void tmem_load32(std::uint32_t taddr, float* out) {
    std::uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
    // The wait names every destination register, so no use of them can be
    // scheduled before the load has landed.
    asm volatile(
        "tcgen05.wait::ld.sync.aligned;"
        : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
          "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]),
          "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]),
          "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]),
          "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]),
          "+r"(r[31])
        :
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) out[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor (sm_100 layout): start, leading and stride
// byte offsets in 16-byte units, version 1, 128-byte swizzle.
__device__ __forceinline__ std::uint64_t sw128_desc(std::uint32_t saddr, std::uint32_t lbo,
                                                    std::uint32_t sbo) {
    return static_cast<std::uint64_t>((saddr >> 4) & 0x3FFFu) |
           (static_cast<std::uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
           (static_cast<std::uint64_t>((sbo >> 4) & 0x3FFFu) << 32) |
           (static_cast<std::uint64_t>(1) << 46) | (static_cast<std::uint64_t>(2) << 61);
}

// Instruction descriptor for kind::f16 with fp32 accumulation, M = N = 128.
__host__ __device__ constexpr std::uint32_t idesc_f16(std::uint32_t a_type, std::uint32_t b_type,
                                                      std::uint32_t b_mn_major) {
    return (1u << 4) | (a_type << 7) | (b_type << 10) | (b_mn_major << 16) | ((128u >> 3) << 17) |
           ((128u >> 4) << 24);
}

// Warp-uniform outcome, so that no lane reaches a warp-collective TMEM load
// (tcgen05.ld .sync.aligned) without the others.
__device__ __forceinline__ bool warp_ok(bool ok) { return __all_sync(0xffffffffu, ok); }

struct Waiter {
    int* abort;
    std::uint32_t* error_word;
    // Bounded wait that fails fast once any role of the CTA has given up.
    __device__ __forceinline__ bool operator()(std::uint64_t* bar, std::uint32_t parity) const {
        if (*reinterpret_cast<volatile int*>(abort)) return false;
        if (mbar_wait_bounded(bar, parity, error_word, 1000000000ull)) return true;
        *reinterpret_cast<volatile int*>(abort) = 1;
        return false;
    }
};

template <bool kBf16>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap q_map,
                      const __grid_constant__ CUtensorMap k_map,
                      const __grid_constant__ CUtensorMap v_map, const Params p) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<std::uintptr_t>(smem_raw) + 1023) & ~static_cast<std::uintptr_t>(1023));
    auto* bars = reinterpret_cast<std::uint64_t*>(smem + kBars);
    auto* tmem_slot = reinterpret_cast<std::uint32_t*>(smem + kBars + kNumBars * 8);
    int* abort = reinterpret_cast<int*>(smem + kBars + kNumBars * 8 + 16);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // Work item, heaviest (last) query tiles first.
    const std::uint32_t tile = p.q_tiles - 1 - blockIdx.x % p.q_tiles;
    const std::uint32_t head = (blockIdx.x / p.q_tiles) % p.q_heads;
    const std::uint32_t seg = blockIdx.x / (p.q_tiles * p.q_heads);
    const int count = p.counts[seg];
    const int q_lo = static_cast<int>(tile) * kBM;
    if (q_lo >= count) return;
    const int start = p.starts[seg];
    const int offset = p.offsets[seg];
    const int total = start + count;
    if (start < 0 || count < 1 || offset < 0 ||
        static_cast<long long>(offset) + count > p.total_queries ||
        static_cast<long long>(start) + count > static_cast<long long>(p.max_blocks) * kBlockTokens) {
        if (threadIdx.x == 0) flag_error(p.error_word, kErrSegment);
        return;
    }
    const int rows = min(kBM, count - q_lo);
    const int kv_end = start + q_lo + rows;  // keys [0, kv_end) are visible to this tile
    const int n_tiles = (kv_end + kBN - 1) / kBN;
    const int nblk_total = (total + kBlockTokens - 1) / kBlockTokens;
    const std::uint32_t kv_head = head / p.group;
    const std::int32_t* table = p.tables + static_cast<std::size_t>(seg) * p.max_blocks;

    if (threadIdx.x == 0) {
        for (int b = 0; b < kNumBars; ++b) {
            mbar_init(&bars[b], (b == kBarSFree || b == kBarSFree + 1 || b == kBarP) ? 128 : 1);
        }
        *abort = 0;
        fence_barrier_init();
    }
    if (warp == 5) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const std::uint32_t tmem = *tmem_slot;
    const Waiter wait{abort, p.error_word};

    if (warp == 4) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            mbar_arrive_expect_tx(&bars[kBarQ], kTile);
            tma_load_3d(smem + kQ, &q_map, 0, static_cast<int>(head), offset + q_lo, &bars[kBarQ]);
            tma_load_3d(smem + kQ + kHalf, &q_map, 64, static_cast<int>(head), offset + q_lo,
                        &bars[kBarQ]);
            int issued = 0;
            for (int j = 0; j < n_tiles; ++j) {
                const int st = j & 1;
                if (j >= 2 && !wait(&bars[kBarKFree + st], ((j >> 1) - 1) & 1)) break;
                std::int32_t ids[8];
#pragma unroll
                for (int b = 0; b < 8; ++b) {
                    const int logical = j * 8 + b;
                    std::int32_t id = table[logical < nblk_total ? logical : 0];
                    if (id < 0 || static_cast<std::uint64_t>(id) >= p.num_blocks) {
                        flag_error(p.error_word, kErrBadBlock);
                        id = 0;
                    }
                    ids[b] = id;
                }
                unsigned char* kdst = smem + kK0 + st * kTile;
                mbar_arrive_expect_tx(&bars[kBarK + st], kTile);
#pragma unroll
                for (int b = 0; b < 8; ++b) {
                    tma_load_4d(kdst + b * 2048, &k_map, 0, 0, static_cast<int>(kv_head), ids[b],
                                &bars[kBarK + st]);
                    tma_load_4d(kdst + kHalf + b * 2048, &k_map, 64, 0, static_cast<int>(kv_head),
                                ids[b], &bars[kBarK + st]);
                }
                if (j >= 2 && !wait(&bars[kBarVFree + st], ((j >> 1) - 1) & 1)) {
                    issued = j * 2 + 1;
                    break;
                }
                unsigned char* vdst = smem + kV0 + st * kTile;
                mbar_arrive_expect_tx(&bars[kBarV + st], kTile);
#pragma unroll
                for (int b = 0; b < 8; ++b) {
                    tma_load_4d(vdst + b * 2048, &v_map, 0, 0, static_cast<int>(kv_head), ids[b],
                                &bars[kBarV + st]);
                    tma_load_4d(vdst + kHalf + b * 2048, &v_map, 64, 0, static_cast<int>(kv_head),
                                ids[b], &bars[kBarV + st]);
                }
                issued = j * 2 + 2;
            }
            // Drain: the last copy issued into each barrier must land before exit.
            mbar_wait_bounded(&bars[kBarQ], 0, p.error_word);
            for (int c = issued - 1; c >= 0 && c >= issued - 4; --c) {
                const int j = c >> 1;
                const int bar = (c & 1) ? kBarV + (j & 1) : kBarK + (j & 1);
                mbar_wait_bounded(&bars[bar], (j >> 1) & 1, p.error_word);
            }
        }
    } else if (warp == 5) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr std::uint32_t a_type = kBf16 ? 1u : 0u;
            const std::uint32_t idesc_s = idesc_f16(a_type, a_type, 0);
            const std::uint32_t idesc_pv = idesc_f16(0, 0, 1);  // P and V as fp16
            const std::uint32_t q_base = smem_u32(smem + kQ);
            bool ok = wait(&bars[kBarQ], 0);
            auto issue_s = [&](int j) {
                const int st = j & 1;
                const std::uint32_t k_base = smem_u32(smem + kK0 + st * kTile);
                const std::uint32_t d = tmem + static_cast<std::uint32_t>(st * 128);
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const std::uint32_t off = (k >> 2) * kHalf + (k & 3) * 32;
                    mma_f16(d, sw128_desc(q_base + off, 16, 1024), sw128_desc(k_base + off, 16, 1024),
                            idesc_s, k > 0 ? 1u : 0u);
                }
                mma_commit(&bars[kBarS + st]);
                mma_commit(&bars[kBarKFree + st]);
            };
            if (ok && (ok = wait(&bars[kBarK], 0))) {
                tc_fence_after();
                issue_s(0);
            }
            for (int j = 0; ok && j < n_tiles; ++j) {
                if (j + 1 < n_tiles) {
                    const int st1 = (j + 1) & 1;
                    if (!(ok = wait(&bars[kBarK + st1], ((j + 1) >> 1) & 1))) break;
                    if (j >= 1 && !(ok = wait(&bars[kBarSFree + st1], ((j - 1) >> 1) & 1))) break;
                    tc_fence_after();
                    issue_s(j + 1);
                }
                if (!(ok = wait(&bars[kBarP], j & 1))) break;
                if (!(ok = wait(&bars[kBarV + (j & 1)], (j >> 1) & 1))) break;
                tc_fence_after();
                const std::uint32_t p_base = smem_u32(smem + kP);
                const std::uint32_t v_base = smem_u32(smem + kV0 + (j & 1) * kTile);
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const std::uint32_t a_off = (k >> 2) * kHalf + (k & 3) * 32;
                    mma_f16(tmem + 256, sw128_desc(p_base + a_off, 16, 1024),
                            sw128_desc(v_base + k * 2048, kHalf, 1024), idesc_pv, k > 0 ? 1u : 0u);
                }
                mma_commit(&bars[kBarPV]);
                mma_commit(&bars[kBarVFree + (j & 1)]);
            }
            // All MMAs issued by this thread complete before TMEM is released.
            mma_commit(&bars[kBarDone]);
            mbar_wait_bounded(&bars[kBarDone], 0, p.error_word);
        }
    } else {
        // ------------------------------------------------------------ softmax
        const int row = threadIdx.x;  // 0..127, TMEM lane = row
        const std::uint32_t lane_addr = tmem + (static_cast<std::uint32_t>(warp * 32) << 16);
        const int qpos = start + q_lo + row;  // this row's position in its sequence
        float o[kD];
#pragma unroll
        for (int i = 0; i < kD; ++i) o[i] = 0.0f;
        float m = -INFINITY;
        float l = 0.0f;
        bool ok = true;
        for (int j = 0; j < n_tiles; ++j) {
            const int st = j & 1;
            if (!(ok = warp_ok(wait(&bars[kBarS + st], (j >> 1) & 1)))) break;
            tc_fence_after();
            const int key0 = j * kBN;
            const bool full = key0 + kBN - 1 <= start + q_lo;  // no masking anywhere in the tile
            const std::uint32_t s_addr = lane_addr + static_cast<std::uint32_t>(st * 128);
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                float s[32];
                tmem_load32(s_addr + c * 32, s);
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const bool valid = full || (key0 + c * 32 + i <= qpos);
                    mx = fmaxf(mx, valid ? s[i] : -INFINITY);
                }
            }
            const float m_new = fmaxf(m, mx * p.scale_log2);
            const float base = m_new == -INFINITY ? 0.0f : m_new;
            const float alpha = exp2f(m - base);
            if (j > 0) {
                if (!(ok = warp_ok(wait(&bars[kBarPV], (j - 1) & 1)))) break;
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float pv[32];
                    tmem_load32(lane_addr + 256 + c * 32, pv);
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[c * 32 + i] = (o[c * 32 + i] + pv[i]) * alpha;
                }
            }
            if constexpr (kBf16) {
                // V arrived as bf16; PV runs with fp16 operands (P needs fp16's
                // 11-bit significand), so widen V in place: same 16-bit layout.
                if (!(ok = warp_ok(wait(&bars[kBarV + st], (j >> 1) & 1)))) break;
                uint4* v = reinterpret_cast<uint4*>(smem + kV0 + st * kTile);
                for (int i = row; i < kTile / 16; i += 128) {
                    uint4 w = v[i];
                    std::uint32_t* u = reinterpret_cast<std::uint32_t*>(&w);
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const float lo = __uint_as_float(u[t] << 16);
                        const float hi = __uint_as_float(u[t] & 0xFFFF0000u);
                        const __half2 h = __floats2half2_rn(lo, hi);
                        u[t] = *reinterpret_cast<const std::uint32_t*>(&h);
                    }
                    v[i] = w;
                }
            }
            float sum = 0.0f;
            unsigned char* prow = smem + kP + row * 128;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                float s[32];
                tmem_load32(s_addr + c * 32, s);
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    std::uint32_t packed[4];
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const int i = g * 8 + t * 2;
                        const bool v0 = full || (key0 + c * 32 + i <= qpos);
                        const bool v1 = full || (key0 + c * 32 + i + 1 <= qpos);
                        const float p0 = v0 ? exp2f(s[i] * p.scale_log2 - base) : 0.0f;
                        const float p1 = v1 ? exp2f(s[i + 1] * p.scale_log2 - base) : 0.0f;
                        const __half2 h = __floats2half2_rn(p0, p1);
                        const float2 back = __half22float2(h);
                        sum += back.x + back.y;  // normalise by what the MMA multiplies
                        packed[t] = *reinterpret_cast<const std::uint32_t*>(&h);
                    }
                    // key chunk (c * 4 + g) of 8 keys: half (chunk / 8), 16-byte slot (chunk % 8)
                    const int chunk = c * 4 + g;
                    unsigned char* dst = prow + (chunk >> 3) * kHalf +
                                         (((chunk & 7) ^ (row & 7)) << 4);
                    *reinterpret_cast<uint4*>(dst) =
                        make_uint4(packed[0], packed[1], packed[2], packed[3]);
                }
            }
            l = l * alpha + sum;
            m = m_new;
            fence_proxy_async_shared();
            tc_fence_before();
            mbar_arrive(&bars[kBarSFree + st]);
            mbar_arrive(&bars[kBarP]);
        }
        if (ok && warp_ok(wait(&bars[kBarPV], (n_tiles - 1) & 1))) {
            tc_fence_after();
            const float inv = 1.0f / l;
            // Every lane takes part in the TMEM loads (warp-collective); only
            // rows inside the segment store.
            const bool store = row < rows;
            float* out = p.out + (static_cast<std::size_t>(offset + q_lo + (store ? row : 0)) *
                                      p.q_heads + head) * kD;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                float pv[32];
                tmem_load32(lane_addr + 256 + c * 32, pv);
                if (store) {
#pragma unroll
                    for (int i = 0; i < 32; i += 4) {
                        float4 w;
                        w.x = (o[c * 32 + i] + pv[i]) * inv;
                        w.y = (o[c * 32 + i + 1] + pv[i + 1]) * inv;
                        w.z = (o[c * 32 + i + 2] + pv[i + 2]) * inv;
                        w.w = (o[c * 32 + i + 3] + pv[i + 3]) * inv;
                        *reinterpret_cast<float4*>(out + c * 32 + i) = w;
                    }
                }
            }
            if (store && !(isfinite(l) && l > 0.0f)) flag_error(p.error_word, kErrNormalizer);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
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

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                 const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                 const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiled encode_fn() {
    static std::once_flag once;
    static EncodeTiled fn = nullptr;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult status{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &status) ==
                cudaSuccess &&
            status == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<EncodeTiled>(ptr);
        }
    });
    if (fn == nullptr) throw std::runtime_error("cuTensorMapEncodeTiled is unavailable");
    return fn;
}

inline CUtensorMap make_map(void* base, CUtensorMapDataType type, int rank, const cuuint64_t* dims,
                            const cuuint64_t* strides, const cuuint32_t* box) {
    CUtensorMap map;
    const cuuint32_t element_strides[4] = {1, 1, 1, 1};
    const CUresult status =
        encode_fn()(&map, type, static_cast<cuuint32_t>(rank), base, dims, strides, box,
                    element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (status != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed");
    return map;
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
    const cuuint32_t q_box[3] = {64, 1, kBM};
    const CUtensorMap q_map = make_map(q16, type, 3, q_dims, q_strides, q_box);
    const cuuint64_t kv_dims[4] = {kD, kBlockTokens, pool.kv_heads, pool.num_blocks};
    const cuuint64_t kv_strides[3] = {kD * 2, kBlockTokens * kD * 2,
                                      static_cast<cuuint64_t>(pool.kv_heads) * kBlockTokens * kD * 2};
    const cuuint32_t kv_box[4] = {64, kBlockTokens, 1, 1};
    const CUtensorMap k_map = make_map(pool.key_arena, type, 4, kv_dims, kv_strides, kv_box);
    const CUtensorMap v_map = make_map(pool.value_arena, type, 4, kv_dims, kv_strides, kv_box);

    Params params{};
    params.tables = tables;
    params.max_blocks = max_blocks;
    params.starts = starts;
    params.counts = counts;
    params.offsets = offsets;
    params.num_segments = num_segments;
    params.q_heads = q_heads;
    params.group = q_heads / pool.kv_heads;
    params.q_tiles = (max_query_count + kBM - 1) / kBM;
    params.num_blocks = pool.num_blocks;
    params.total_queries = total_queries;
    params.scale_log2 = (1.0f / std::sqrt(static_cast<float>(kD))) * kLog2e;
    params.out = out;
    params.error_word = pool.error_word;
    const std::uint64_t grid = static_cast<std::uint64_t>(num_segments) * q_heads * params.q_tiles;
    if (grid > 0x7FFFFFFFull) throw std::runtime_error("paged prefill grid is too large");
    auto kernel = bf16 ? prefill_tc_kernel<true> : prefill_tc_kernel<false>;
    cuda_check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemAlloc),
               "cudaFuncSetAttribute");
    kernel<<<static_cast<unsigned>(grid), kThreads, kSmemAlloc, stream>>>(q_map, k_map, v_map,
                                                                          params);
    cuda_check(cudaGetLastError(), "tensor-core prefill launch");
}

}  // namespace ilb
