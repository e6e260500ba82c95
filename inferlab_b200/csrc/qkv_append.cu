// qkv_append.cu - the Q/K/V projection beside attention on the sm_100a tensor
// cores, with the new K and V rows written straight into the paged pool.
//
// The reference projects the normalised hidden states with three fp32
// `linear` calls (worker/cpp/inferlab_runtime.cpp:1318-1325; linear at
// :1266-1285: output[row][out] = sum_in input[row][in] * weight(out, in)) and
// then appends each token's K/V row to its pages one call at a time
// (PagedKvPool::append, :713-767). Here one persistent kernel computes
// Y = X W^T for the stacked weight W = [W_q; W_k; W_v] ([N][D] with N =
// (q_heads + 2 kv_heads) head_dim, rows = output features) from f16 / bf16
// operands with fp32 accumulation in TMEM, and its epilogue writes
//   * Q columns to q_out [T][q_heads][head_dim],
//   * K / V columns of token t to (table[seq[t]][pos[t] / block_tokens],
//     pos[t] % block_tokens) of the pool's key / value arena,
// all in the pool's 16-bit type (round to nearest even).
//
// Tiles: 128 tokens x 256 features, K in steps of 64 (one 128-byte swizzled
// TMA box per operand and stage, 4 stages = 192 KB of shared memory). Roles
// (192 threads): warp 0 issues the TMA loads, warp 1 allocates TMEM and one
// thread issues tcgen05.mma (M=128, N=256, K=16, four per stage), warps 2-5
// move finished accumulators out of TMEM (thread = token row). The two
// accumulator buffers (2 x 256 TMEM columns) let the epilogue of one tile
// run under the MMAs of the next. Every mbarrier wait is bounded (the CTA
// records kErrWaitTimeout, drains its MMAs and frees TMEM).
#include "common.cuh"
#include "internal.cuh"
#include "pool.cuh"
#include "tc_common.cuh"

#include "../../include/inferlab_attention.h"

#include <algorithm>
#include <type_traits>

namespace ilb {
namespace qkv {

using namespace ilb::tc;

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kStages = 4;
constexpr int kThreads = 192;
constexpr int kAStage = kBM * kBK * 2;  // 16 KB
constexpr int kBStage = kBN * kBK * 2;  // 32 KB
constexpr int kStageBytes = kAStage + kBStage;
constexpr int kBars = kStages * kStageBytes;  // 192 KB
enum Bar : int {
    kBarFull = 0,                      // +stage: both boxes landed
    kBarEmpty = kStages,               // +stage: the stage's MMAs completed
    kBarAccFull = 2 * kStages,         // +buffer: the tile's accumulator is complete
    kBarAccEmpty = 2 * kStages + 2,    // +buffer: the epilogue has read it (4 warps)
    kBarDone = 2 * kStages + 4,
    kNumBars = 2 * kStages + 5,
};
constexpr int kSmemBytes = kBars + kNumBars * 8 + 32;
constexpr int kSmemAlloc = kSmemBytes + 1024;  // slack to align the base to 1024 B
constexpr std::uint32_t kTmemCols = 512;

struct Params {
    std::uint32_t tokens;
    std::uint32_t features;  // N
    std::uint32_t k_stages;  // ceil(D / 64)
    std::uint32_t m_tiles;
    std::uint32_t n_tiles;
    std::uint32_t q_heads;
    std::uint32_t kv_heads;
    std::uint32_t head_dim;
    std::uint32_t block_tokens;
    std::uint32_t num_seqs;
    std::uint32_t max_blocks;
    std::uint64_t num_blocks;
    const std::int32_t* row_sequences;
    const std::int32_t* positions;
    const std::int32_t* tables;
    unsigned char* q_out;
    unsigned char* key_arena;
    unsigned char* value_arena;
    const float* residual;  // output projection: [T][N] fp32 added to the product, or null
    float* out;             // output projection: [T][N] fp32
    std::uint32_t* error_word;
};

// Epilogue modes of the shared GEMM kernel.
constexpr int kModeQkvAppend = 0;  // Q rows out, K/V rows into the pool (pool type)
constexpr int kModeOutput = 1;     // fp32 rows out, plus an optional fp32 residual

template <typename T>
__device__ __forceinline__ std::uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ std::uint32_t pack2<__half>(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const std::uint32_t*>(&h);
}
template <>
__device__ __forceinline__ std::uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const std::uint32_t*>(&h);
}

template <typename T, int kMode>
__global__ void __launch_bounds__(kThreads, 1)
    qkv_append_kernel(const __grid_constant__ CUtensorMap x_map,
                      const __grid_constant__ CUtensorMap w_map, const Params p) {
    constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<std::uintptr_t>(smem_raw) + 1023) & ~static_cast<std::uintptr_t>(1023));
    auto* bars = reinterpret_cast<std::uint64_t*>(smem + kBars);
    auto* tmem_slot = reinterpret_cast<std::uint32_t*>(smem + kBars + kNumBars * 8);
    int* abort = reinterpret_cast<int*>(smem + kBars + kNumBars * 8 + 16);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int b = 0; b < kNumBars; ++b) {
            mbar_init(&bars[b], (b == kBarAccEmpty || b == kBarAccEmpty + 1) ? 4u : 1u);
        }
        *abort = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const std::uint32_t tmem = *tmem_slot;
    const Waiter wait{abort, p.error_word};
    const std::uint32_t total = p.m_tiles * p.n_tiles;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        // Tiles in order m fastest: the CTAs working at the same time share
        // one 256-row slice of W, which stays in L2.
        if (lane == 0) {
            std::uint32_t it = 0;
            bool ok = true;
            for (std::uint32_t tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
                const int m = static_cast<int>(tile % p.m_tiles);
                const int n = static_cast<int>(tile / p.m_tiles);
                for (std::uint32_t ks = 0; ks < p.k_stages; ++ks, ++it) {
                    const std::uint32_t s = it % kStages;
                    if (it >= kStages && !(ok = wait(&bars[kBarEmpty + s], ((it / kStages) - 1) & 1))) break;
                    unsigned char* stage = smem + s * kStageBytes;
                    mbar_arrive_expect_tx(&bars[kBarFull + s], kStageBytes);
                    tma_load_2d(stage, &x_map, static_cast<int>(ks) * kBK, m * kBM, &bars[kBarFull + s]);
                    tma_load_2d(stage + kAStage, &w_map, static_cast<int>(ks) * kBK, n * kBN,
                                &bars[kBarFull + s]);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr std::uint32_t type = kBf16 ? 1u : 0u;
            const std::uint32_t idesc = idesc_f16(type, type, 0, kBN);
            std::uint32_t it = 0, lt = 0;
            bool ok = true;
            for (std::uint32_t tile = blockIdx.x; ok && tile < total; tile += gridDim.x, ++lt) {
                const std::uint32_t b = lt & 1;
                if (lt >= 2 && !(ok = wait(&bars[kBarAccEmpty + b], ((lt >> 1) - 1) & 1))) break;
                tc_fence_after();
                const std::uint32_t d = tmem + b * kBN;
                for (std::uint32_t ks = 0; ks < p.k_stages; ++ks, ++it) {
                    const std::uint32_t s = it % kStages;
                    if (!(ok = wait(&bars[kBarFull + s], (it / kStages) & 1))) break;
                    tc_fence_after();
                    const std::uint64_t a_desc = sw128_desc(smem_u32(smem + s * kStageBytes), 16, 1024);
                    const std::uint64_t b_desc =
                        sw128_desc(smem_u32(smem + s * kStageBytes + kAStage), 16, 1024);
#pragma unroll
                    for (int k = 0; k < kBK / 16; ++k) {
                        // K step k starts 32 B further into every 128-byte row.
                        const std::uint64_t off = static_cast<std::uint64_t>((k * 32) >> 4);
                        mma_f16(d, a_desc + off, b_desc + off, idesc, (ks > 0 || k > 0) ? 1u : 0u);
                    }
                    mma_commit(&bars[kBarEmpty + s]);
                }
                if (!ok) break;
                mma_commit(&bars[kBarAccFull + b]);
            }
            // All MMAs issued by this thread complete before TMEM is released.
            mma_commit(&bars[kBarDone]);
            mbar_wait_bounded(&bars[kBarDone], 0, p.error_word);
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int group = warp & 3;  // TMEM lanes 32 group .. 32 group + 31
        const int row = group * 32 + lane;
        const std::uint32_t lane_addr = tmem + (static_cast<std::uint32_t>(group * 32) << 16);
        const std::uint32_t q_cols = p.q_heads * p.head_dim;
        std::uint32_t lt = 0;
        for (std::uint32_t tile = blockIdx.x; tile < total; tile += gridDim.x, ++lt) {
            const std::uint32_t b = lt & 1;
            if (!warp_ok(wait(&bars[kBarAccFull + b], (lt >> 1) & 1))) break;
            tc_fence_after();
            const std::uint32_t m = tile % p.m_tiles;
            const std::uint32_t n = tile / p.m_tiles;
            const std::uint32_t token = m * kBM + static_cast<std::uint32_t>(row);
            bool live = token < p.tokens;
            // Where this token's K/V rows go, when the tile holds K/V columns.
            std::size_t kv_row = 0;  // (block * kv_heads) * block_tokens + slot, in rows
            if (kMode == kModeQkvAppend && live && n * kBN + kBN > q_cols) {
                const std::int32_t seq = p.row_sequences[token];
                const std::int32_t pos = p.positions[token];
                if (seq < 0 || static_cast<std::uint32_t>(seq) >= p.num_seqs || pos < 0 ||
                    static_cast<std::uint32_t>(pos) / p.block_tokens >= p.max_blocks) {
                    flag_error(p.error_word, kErrPosition);
                    live = false;
                } else {
                    const std::int32_t block =
                        p.tables[static_cast<std::size_t>(seq) * p.max_blocks +
                                 static_cast<std::uint32_t>(pos) / p.block_tokens];
                    if (block < 0 || static_cast<std::uint64_t>(block) >= p.num_blocks) {
                        flag_error(p.error_word, kErrBadBlock);
                        live = false;
                    } else {
                        kv_row = static_cast<std::size_t>(block) * p.kv_heads * p.block_tokens +
                                 static_cast<std::uint32_t>(pos) % p.block_tokens;
                    }
                }
            }
            bool bad = false;
#pragma unroll 1
            for (int c = 0; c < kBN / 32; ++c) {
                const std::uint32_t f0 = n * kBN + static_cast<std::uint32_t>(c) * 32;
                if (f0 >= p.features) break;  // uniform: the tile's last columns lie past N
                float v[32];
                tmem_load32(lane_addr + b * kBN + static_cast<std::uint32_t>(c) * 32, v);
                if (token >= p.tokens) continue;
                if constexpr (kMode == kModeOutput) {
                    // out = product (+ residual), fp32, 32 consecutive columns.
                    const std::size_t at = static_cast<std::size_t>(token) * p.features + f0;
                    float4* o4 = reinterpret_cast<float4*>(p.out + at);
                    const float4* r4 = reinterpret_cast<const float4*>(p.residual + at);
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        float4 r = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                        if (p.residual != nullptr) r = r4[q];
                        o4[q] = make_float4(v[4 * q] + r.x, v[4 * q + 1] + r.y, v[4 * q + 2] + r.z,
                                            v[4 * q + 3] + r.w);
                    }
                    continue;
                }
                if (!live && f0 >= q_cols) continue;
                // head_dim is a multiple of 32, so the 32 columns are one head's.
                const std::uint32_t head = f0 / p.head_dim;
                const std::uint32_t dim0 = f0 % p.head_dim;
                unsigned char* dst;
                if (head < p.q_heads) {
                    dst = p.q_out + ((static_cast<std::size_t>(token) * p.q_heads + head) * p.head_dim + dim0) * 2;
                } else {
                    const std::uint32_t kv = head - p.q_heads;
                    const bool is_v = kv >= p.kv_heads;
                    const std::uint32_t kh = is_v ? kv - p.kv_heads : kv;
#pragma unroll
                    for (int i = 0; i < 32; ++i) bad |= !isfinite(v[i]);
                    dst = (is_v ? p.value_arena : p.key_arena) +
                          ((kv_row + static_cast<std::size_t>(kh) * p.block_tokens) * p.head_dim + dim0) * 2;
                }
                uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    d4[q] = make_uint4(pack2<T>(v[8 * q], v[8 * q + 1]), pack2<T>(v[8 * q + 2], v[8 * q + 3]),
                                       pack2<T>(v[8 * q + 4], v[8 * q + 5]), pack2<T>(v[8 * q + 6], v[8 * q + 7]));
                }
            }
            // The reference's prepare() rejects non-finite K/V
            // (kernels/attention_cpu.cpp:131-134); here the step reports it.
            if (bad) flag_error(p.error_word, kErrNonFinite);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[kBarAccEmpty + b]);  // one arrival per warp
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace qkv
}  // namespace ilb

extern "C" int inferlab_cuda_qkv_project_append(
    InferlabCudaKvPool* pool, const void* hidden, const void* weights, std::uint32_t tokens,
    std::uint32_t model_dim, std::uint32_t q_heads, const std::int32_t* row_sequences,
    const std::int32_t* positions, const std::int32_t* block_tables, std::uint32_t num_seqs,
    std::uint32_t max_blocks_per_seq, void* q_out, void* stream, char* error,
    std::size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        using namespace ilb;
        using namespace ilb::qkv;
        auto& p = checked_pool(pool);
        if (tokens == 0) return;
        if (hidden == nullptr || weights == nullptr || row_sequences == nullptr ||
            positions == nullptr || block_tables == nullptr || q_out == nullptr) {
            throw std::runtime_error("projection pointer is null");
        }
        if (p.dtype != kF16 && p.dtype != kBf16) {
            throw std::runtime_error("projection needs an F16 or BF16 pool");
        }
        if (p.head_dim % 32 != 0) throw std::runtime_error("projection head_dim must be a multiple of 32");
        if (q_heads == 0 || q_heads % p.kv_heads != 0) {
            throw std::runtime_error("paged decode q_heads must be a positive multiple of kv_heads");
        }
        if (model_dim == 0 || model_dim % 8 != 0) {
            throw std::runtime_error("projection model_dim must be a positive multiple of 8");
        }
        if (num_seqs == 0 || max_blocks_per_seq == 0) throw std::runtime_error("paged KV block table is empty");
        for (const void* ptr : {hidden, weights, static_cast<const void*>(q_out)}) {
            if (reinterpret_cast<std::uintptr_t>(ptr) % 16 != 0) {
                throw std::runtime_error("projection buffers must be 16-byte aligned");
            }
        }
        const std::uint64_t features =
            static_cast<std::uint64_t>(q_heads + 2 * p.kv_heads) * p.head_dim;
        if (features > 0x7FFFFFFFull || tokens > 0x7FFFFFFFu) {
            throw std::runtime_error("projection is too large");
        }
        DeviceGuard guard(p.device);
        auto s = static_cast<cudaStream_t>(stream);
        const CUtensorMapDataType type =
            p.dtype == kBf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
        const cuuint64_t x_dims[2] = {model_dim, tokens};
        const cuuint64_t x_strides[1] = {static_cast<cuuint64_t>(model_dim) * 2};
        const cuuint32_t x_box[2] = {kBK, kBM};
        const CUtensorMap x_map = make_map(const_cast<void*>(hidden), type, 2, x_dims, x_strides, x_box);
        const cuuint64_t w_dims[2] = {model_dim, features};
        const cuuint32_t w_box[2] = {kBK, kBN};
        const CUtensorMap w_map = make_map(const_cast<void*>(weights), type, 2, w_dims, x_strides, w_box);

        Params prm{};
        prm.tokens = tokens;
        prm.features = static_cast<std::uint32_t>(features);
        prm.k_stages = (model_dim + kBK - 1) / kBK;
        prm.m_tiles = (tokens + kBM - 1) / kBM;
        prm.n_tiles = static_cast<std::uint32_t>((features + kBN - 1) / kBN);
        prm.q_heads = q_heads;
        prm.kv_heads = p.kv_heads;
        prm.head_dim = p.head_dim;
        prm.block_tokens = p.block_tokens;
        prm.num_seqs = num_seqs;
        prm.max_blocks = max_blocks_per_seq;
        prm.num_blocks = p.num_blocks;
        prm.row_sequences = row_sequences;
        prm.positions = positions;
        prm.tables = block_tables;
        prm.q_out = static_cast<unsigned char*>(q_out);
        prm.key_arena = static_cast<unsigned char*>(p.key_arena);
        prm.value_arena = static_cast<unsigned char*>(p.value_arena);
        prm.error_word = p.error_word;
        const std::uint64_t total = static_cast<std::uint64_t>(prm.m_tiles) * prm.n_tiles;
        if (total > 0x7FFFFFFFull) throw std::runtime_error("projection is too large");
        int sms = 0;
        cuda_check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, p.device),
                   "cudaDeviceGetAttribute");
        const unsigned grid = static_cast<unsigned>(std::min<std::uint64_t>(total, static_cast<std::uint64_t>(std::max(sms, 1))));
        auto kernel = p.dtype == kBf16 ? qkv_append_kernel<__nv_bfloat16, kModeQkvAppend>
                                       : qkv_append_kernel<__half, kModeQkvAppend>;
        cuda_check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemAlloc),
                   "cudaFuncSetAttribute");
        kernel<<<grid, kThreads, kSmemAlloc, s>>>(x_map, w_map, prm);
        cuda_check(cudaGetLastError(), "projection launch");
    });
}

namespace ilb {
namespace qkv {
namespace {

// fp32 -> pool type (round to nearest even), for attention outputs handed to
// the output projection in fp32: eight elements per thread and step (two
// 16-byte loads, one 16-byte store; n is a multiple of 8 since in_dim is).
template <typename T>
__global__ void round_rows_kernel(const float* in, T* out, std::size_t n) {
    const auto* in4 = reinterpret_cast<const float4*>(in);
    auto* out4 = reinterpret_cast<uint4*>(out);
    for (std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n / 8;
         i += static_cast<std::size_t>(gridDim.x) * blockDim.x) {
        const float4 a = in4[2 * i];
        const float4 b = in4[2 * i + 1];
        out4[i] = make_uint4(pack2<T>(a.x, a.y), pack2<T>(a.z, a.w), pack2<T>(b.x, b.y),
                             pack2<T>(b.z, b.w));
    }
}

}  // namespace
}  // namespace qkv
}  // namespace ilb

extern "C" int inferlab_cuda_output_project(InferlabCudaKvPool* pool, const void* attention,
                                            std::uint32_t attention_dtype, const void* weights,
                                            const float* residual, std::uint32_t tokens,
                                            std::uint32_t in_dim, std::uint32_t out_dim, float* out,
                                            void* stream, char* error, std::size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        using namespace ilb;
        using namespace ilb::qkv;
        auto& p = checked_pool(pool);
        if (tokens == 0) return;
        if (attention == nullptr || weights == nullptr || out == nullptr) {
            throw std::runtime_error("projection pointer is null");
        }
        if (p.dtype != kF16 && p.dtype != kBf16) {
            throw std::runtime_error("projection needs an F16 or BF16 pool");
        }
        if (attention_dtype != kFp32 && attention_dtype != p.dtype) {
            throw std::runtime_error("projection input dtype must be FP32 or the pool dtype");
        }
        if (in_dim == 0 || in_dim % 8 != 0) {
            throw std::runtime_error("projection model_dim must be a positive multiple of 8");
        }
        if (out_dim == 0 || out_dim % 32 != 0) {
            throw std::runtime_error("projection output width must be a positive multiple of 32");
        }
        if (tokens > 0x7FFFFFFFu) throw std::runtime_error("projection is too large");
        for (const void* ptr : {attention, weights, static_cast<const void*>(out),
                                static_cast<const void*>(residual)}) {
            if (reinterpret_cast<std::uintptr_t>(ptr) % 16 != 0) {
                throw std::runtime_error("projection buffers must be 16-byte aligned");
            }
        }
        DeviceGuard guard(p.device);
        auto s = static_cast<cudaStream_t>(stream);
        const bool bf16 = p.dtype == kBf16;
        const void* a16 = attention;
        void* temp = nullptr;
        if (attention_dtype == kFp32) {
            const std::size_t n = static_cast<std::size_t>(tokens) * in_dim;
            cuda_check(cudaMallocAsync(&temp, n * 2, s), "cudaMallocAsync");
            const unsigned grid = static_cast<unsigned>(std::min<std::size_t>((n / 8 + 255) / 256, 148 * 16));
            if (bf16) {
                round_rows_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
                    static_cast<const float*>(attention), static_cast<__nv_bfloat16*>(temp), n);
            } else {
                round_rows_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const float*>(attention),
                                                               static_cast<__half*>(temp), n);
            }
            cuda_check(cudaGetLastError(), "projection input rounding launch");
            a16 = temp;
        }
        struct TempGuard {
            void* ptr;
            cudaStream_t stream;
            ~TempGuard() {
                if (ptr != nullptr) cudaFreeAsync(ptr, stream);
            }
        } guard_temp{temp, s};
        const CUtensorMapDataType type =
            bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
        const cuuint64_t x_dims[2] = {in_dim, tokens};
        const cuuint64_t x_strides[1] = {static_cast<cuuint64_t>(in_dim) * 2};
        const cuuint32_t x_box[2] = {kBK, kBM};
        const CUtensorMap x_map = make_map(const_cast<void*>(a16), type, 2, x_dims, x_strides, x_box);
        const cuuint64_t w_dims[2] = {in_dim, out_dim};
        const cuuint32_t w_box[2] = {kBK, kBN};
        const CUtensorMap w_map = make_map(const_cast<void*>(weights), type, 2, w_dims, x_strides, w_box);
        Params prm{};
        prm.tokens = tokens;
        prm.features = out_dim;
        prm.k_stages = (in_dim + kBK - 1) / kBK;
        prm.m_tiles = (tokens + kBM - 1) / kBM;
        prm.n_tiles = (out_dim + kBN - 1) / kBN;
        prm.residual = residual;
        prm.out = out;
        prm.error_word = p.error_word;
        const std::uint64_t total = static_cast<std::uint64_t>(prm.m_tiles) * prm.n_tiles;
        if (total > 0x7FFFFFFFull) throw std::runtime_error("projection is too large");
        int sms = 0;
        cuda_check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, p.device),
                   "cudaDeviceGetAttribute");
        const unsigned grid = static_cast<unsigned>(std::min<std::uint64_t>(total, static_cast<std::uint64_t>(std::max(sms, 1))));
        auto kernel = bf16 ? qkv_append_kernel<__nv_bfloat16, kModeOutput>
                           : qkv_append_kernel<__half, kModeOutput>;
        cuda_check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemAlloc),
                   "cudaFuncSetAttribute");
        kernel<<<grid, kThreads, kSmemAlloc, s>>>(x_map, w_map, prm);
        cuda_check(cudaGetLastError(), "projection launch");
    });
}
