// Test infrastructure: exposes the reference runtime's internal fp32 `linear`
// (worker/cpp/inferlab_runtime.cpp:1266-1285) and its LinearWeight (:493-600,
// Fp32 mode) through a C entry, so that the projection oracle can be checked
// against the reference's own code. The reference source is compiled in place
// (this file includes it; nothing is copied); see the Makefile's ref target.
#include "inferlab_runtime.cpp"

extern "C" int oracle_ref_linear(const float* input, std::size_t rows, std::size_t input_columns,
                                 const float* weight, std::size_t output_columns, float* output) {
    try {
        const std::vector<float> in(input, input + rows * input_columns);
        const LinearWeight w = LinearWeight::from_fp32(
            std::vector<float>(weight, weight + output_columns * input_columns), output_columns,
            input_columns, QuantizationMode::Fp32);
        const std::vector<float> out = linear(in, rows, input_columns, w, output_columns);
        std::copy(out.begin(), out.end(), output);
        return 0;
    } catch (...) {
        return -1;
    }
}
