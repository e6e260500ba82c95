// prefill_tc.cuh - tcgen05 tensor-core causal prefill (f16/bf16 pools).
#pragma once

#include "common.cuh"
#include "pool.cuh"

namespace ilb {

inline bool tc_prefill_supported(const InferlabCudaKvPool&, std::uint32_t) { return false; }

inline void run_tc_prefill(InferlabCudaKvPool&, const void*, std::uint32_t, const std::int32_t*,
                           std::uint32_t, const std::int32_t*, const std::int32_t*,
                           const std::int32_t*, std::uint32_t, std::uint32_t, std::uint32_t,
                           long long, float*, cudaStream_t) {
    throw std::runtime_error("tensor-core prefill is not available");
}

}  // namespace ilb
