// internal.cuh - launch paths shared between the library's .cu files (not
// part of the C ABI).
#pragma once

#include "pool.cuh"

struct InferlabCudaPeerExchange;

namespace ilb {

// Bytes of decode workspace a batch of this shape needs, and how many of its
// leading bytes are the split counters that must be zero before a launch.
std::size_t decode_workspace_bytes(const InferlabCudaKvPool& pool, std::uint32_t num_seqs,
                                   std::uint32_t q_heads, std::uint32_t max_context_len);
std::size_t decode_counter_bytes(const InferlabCudaKvPool& pool, std::uint32_t num_seqs);
// Bytes of that workspace the launch actually touches: 0 when no context is
// split (one split per sequence) or the shape takes the generic kernel, which
// keeps no partials; otherwise decode_workspace_bytes.
std::size_t decode_scratch_bytes(const InferlabCudaKvPool& pool, std::uint32_t num_seqs,
                                 std::uint32_t q_heads, std::uint32_t max_context_len);

// Argument checks of inferlab_cuda_paged_decode (throws std::runtime_error).
void check_decode_arguments(const InferlabCudaKvPool& pool, const float* queries,
                            const std::int32_t* block_tables, std::uint32_t max_blocks,
                            const std::int32_t* context_lens, std::uint32_t num_seqs,
                            std::uint32_t q_heads, std::uint32_t max_context_len);

// Launches the decode kernel with the given workspace; the pool's device must
// be current.
void launch_paged_decode(InferlabCudaKvPool& pool, const float* queries,
                         const std::int32_t* block_tables, std::uint32_t max_blocks,
                         const std::int32_t* context_lens, std::uint32_t num_seqs,
                         std::uint32_t q_heads, std::uint32_t max_context_len, float* out,
                         void* workspace, std::size_t workspace_bytes, cudaStream_t stream);

// The buffers of a peer exchange (peer_exchange.cu) for one call: every
// rank's receive words, this rank, the exchanged block's rows and head_dim,
// and the call's step number (taken by exchange_take_step).
struct ExchangeView {
    std::uint64_t* words[8];
    std::uint32_t world;
    std::uint32_t rank;
    std::uint32_t step;
    std::uint64_t rows;
    std::uint32_t head_dim;
    int device;
};

// Takes the next step of `exchange` (serialised per exchange) and describes
// its buffers; throws, without taking a step, on a null exchange or one made
// for another device, row count or head_dim.
ExchangeView exchange_take_step(InferlabCudaPeerExchange* exchange, int device, std::uint64_t rows,
                                std::uint32_t head_dim);

// Launches kv_append (see inferlab_cuda_kv_append); the pool's device must be
// current.
void launch_kv_append(InferlabCudaKvPool& pool, const void* key_rows, const void* value_rows,
                      std::uint32_t row_dtype, const std::int32_t* row_sequences,
                      const std::int32_t* positions, std::uint64_t rows,
                      const std::int32_t* block_tables, std::uint32_t max_blocks,
                      cudaStream_t stream);

}  // namespace ilb
