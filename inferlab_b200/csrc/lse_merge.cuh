// lse_merge.cuh - the log-sum-exp merge of split-KV partials, one warp per
// row, shared by the standalone combine (inferlab_cuda_lse_combine*) and the
// peer exchange, so both produce the same bits for the same partials.
//
// Part i of a row holds m (the running max, natural-log units), l (the sum of
// exp(s - m)) and o (the unnormalised sum of exp(s - m) v) of a contiguous
// key range; parts with l = 0 saw no key. The parts merge in index order
// (deterministic, independent of arrival order): the output row is
// sum_i exp(m_i - M) o_i / sum_i exp(m_i - M) l_i with M the largest m_i of
// the non-empty parts - the online-softmax recurrence of
// kernels/attention_cpu.cpp:364-386 applied to whole ranges.
#pragma once

#include "common.cuh"

namespace ilb {

// Part i of the row: m at part_m[i * stride_m + row], l at
// part_l[i * stride_l + row], o at part_o[i * stride_o + row * head_dim].
__device__ __forceinline__ void lse_merge_row(const float* part_m, const float* part_l,
                                              const float* part_o, std::uint32_t parts,
                                              std::uint64_t row, std::uint32_t head_dim,
                                              std::uint64_t stride_m, std::uint64_t stride_l,
                                              std::uint64_t stride_o, float* out, int lane) {
    float mw = -INFINITY;
    for (std::uint32_t i = 0; i < parts; ++i) {
        if (part_l[i * stride_l + row] > 0.0f) mw = fmaxf(mw, part_m[i * stride_m + row]);
    }
    float lsum = 0.0f;
    for (std::uint32_t i = 0; i < parts; ++i) {
        const float li = part_l[i * stride_l + row];
        if (li > 0.0f) lsum += li * expf(part_m[i * stride_m + row] - mw);
    }
    for (std::uint32_t dim = lane; dim < head_dim; dim += 32) {
        float a = 0.0f;
        for (std::uint32_t i = 0; i < parts; ++i) {
            if (part_l[i * stride_l + row] > 0.0f) {
                a += part_o[i * stride_o + row * head_dim + dim] * expf(part_m[i * stride_m + row] - mw);
            }
        }
        out[row * head_dim + dim] = a / lsum;
    }
}

}  // namespace ilb
