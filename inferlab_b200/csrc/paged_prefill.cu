// paged_prefill.cu - causal and chunked prefill over the paged pool.
//
// The reference's full-sequence call is attention_forward(q, k, v, T, T, H, d,
// 0, cfg) from Model::forward_all (worker/cpp/inferlab_runtime.cpp:1327-1339);
// chunked prefill is the same call with query_start_position > 0
// (kernels/attention_cpu.cpp:113-123, :443-447). Segments here carry their
// own start, count and block table row, so one launch covers a continuous
// batch of prompt chunks.
//
// f16/bf16 pools with head_dim 128 and 16-token blocks run the tcgen05
// tensor-core kernel (prefill_tc.cuh); every other pool runs the fp32
// CUDA-core kernel (generic_attention.cuh), which the 1e-5 fp32 tolerance
// requires for fp32 pools.
#include "common.cuh"
#include "generic_attention.cuh"
#include "pool.cuh"
#include "prefill_tc.cuh"

#include "../../include/inferlab_attention.h"

#include <cmath>

namespace ilb {
namespace {

void run_generic_prefill(InferlabCudaKvPool& p, const float* queries,
                         const std::int32_t* block_tables, std::uint32_t max_blocks,
                         const std::int32_t* starts, const std::int32_t* counts,
                         const std::int32_t* offsets, std::uint32_t num_segments,
                         std::uint32_t q_heads, long long total_queries, float* out,
                         cudaStream_t stream) {
    if (p.head_dim > kGenericMaxHeadDim) {
        throw std::runtime_error("attention head_dimension exceeds the CUDA kernel limit of 4096");
    }
    GenericParams g{};
    g.queries = queries;
    g.query_precision = p.dtype;
    g.out = out;
    g.query_rows = total_queries;
    g.q_heads = q_heads;
    g.kv_heads = p.kv_heads;
    g.head_dim = p.head_dim;
    g.scale = 1.0f / std::sqrt(static_cast<float>(p.head_dim));
    g.error_word = p.error_word;
    g.check_normalizer = 1;
    SegmentMap seg{};
    seg.mode = 2;
    seg.starts = starts;
    seg.counts = counts;
    seg.offsets = offsets;
    seg.num_segments = static_cast<int>(num_segments);
    seg.max_kv = static_cast<long long>(max_blocks) * p.block_tokens;
    const std::size_t gsmem = generic_smem_bytes(p.head_dim);
    const std::size_t rows = static_cast<std::size_t>(total_queries) * q_heads;
    if ((rows + kGenericWarps - 1) / kGenericWarps > 0x7FFFFFFFull) {
        throw std::runtime_error("paged prefill grid is too large");
    }
    const unsigned grid = static_cast<unsigned>((rows + kGenericWarps - 1) / kGenericWarps);
    auto launch = [&](auto kv) {
        auto* fn = generic_attention_kernel<decltype(kv)>;
        cuda_check(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(gsmem)),
                   "cudaFuncSetAttribute");
        fn<<<grid, kGenericWarps * 32, gsmem, stream>>>(g, kv, seg);
    };
    if (p.dtype == kFp32) {
        launch(PagedKv<float>{static_cast<const float*>(p.key_arena),
                              static_cast<const float*>(p.value_arena), block_tables, max_blocks,
                              p.block_tokens, p.kv_heads, p.head_dim, p.num_blocks, p.error_word});
    } else if (p.dtype == kF16) {
        launch(PagedKv<__half>{static_cast<const __half*>(p.key_arena),
                               static_cast<const __half*>(p.value_arena), block_tables, max_blocks,
                               p.block_tokens, p.kv_heads, p.head_dim, p.num_blocks, p.error_word});
    } else {
        launch(PagedKv<__nv_bfloat16>{static_cast<const __nv_bfloat16*>(p.key_arena),
                                      static_cast<const __nv_bfloat16*>(p.value_arena),
                                      block_tables, max_blocks, p.block_tokens, p.kv_heads,
                                      p.head_dim, p.num_blocks, p.error_word});
    }
    cuda_check(cudaGetLastError(), "generic prefill launch");
}

}  // namespace
}  // namespace ilb

extern "C" int inferlab_cuda_paged_prefill(InferlabCudaKvPool* pool, const void* queries,
                                           std::uint32_t query_dtype,
                                           const std::int32_t* block_tables,
                                           std::uint32_t max_blocks_per_seq,
                                           const std::int32_t* query_starts,
                                           const std::int32_t* query_counts,
                                           const std::int32_t* query_offsets,
                                           std::uint32_t num_segments, std::uint32_t q_heads,
                                           std::uint32_t max_query_count,
                                           std::uint64_t total_queries, float* out,
                                           void* stream, char* error,
                                           std::size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        using namespace ilb;
        auto& p = checked_pool(pool);
        if (num_segments == 0 || total_queries == 0) return;
        if (queries == nullptr || block_tables == nullptr || query_starts == nullptr ||
            query_counts == nullptr || query_offsets == nullptr || out == nullptr) {
            throw std::runtime_error("paged prefill pointer is null");
        }
        if (q_heads == 0 || q_heads % p.kv_heads != 0) {
            throw std::runtime_error("paged prefill q_heads must be a positive multiple of kv_heads");
        }
        if (max_blocks_per_seq == 0 || max_query_count == 0) {
            throw std::runtime_error("paged prefill block table and query bound must be positive");
        }
        if (total_queries > 0x7FFFFFFFull) throw std::runtime_error("paged prefill batch is too large");
        if (query_dtype != kFp32 && query_dtype != p.dtype) {
            throw std::runtime_error("paged prefill query dtype must be FP32 or the pool dtype");
        }
        DeviceGuard guard(p.device);
        auto s = static_cast<cudaStream_t>(stream);
        if (tc_prefill_supported(p, q_heads)) {
            run_tc_prefill(p, queries, query_dtype, block_tables, max_blocks_per_seq, query_starts,
                           query_counts, query_offsets, num_segments, q_heads, max_query_count,
                           static_cast<long long>(total_queries), out, s);
            return;
        }
        if (query_dtype != kFp32) {
            throw std::runtime_error("paged prefill on this pool geometry takes FP32 queries");
        }
        run_generic_prefill(p, static_cast<const float*>(queries), block_tables,
                            max_blocks_per_seq, query_starts, query_counts, query_offsets,
                            num_segments, q_heads, static_cast<long long>(total_queries), out, s);
    });
}
