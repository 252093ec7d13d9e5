// Compiles the reference's source/q4rdna_cpu_experiment.cpp where it lies and
// exports its fp16 converters (:39-100) and its Q4_K block dequantiser
// dequantize_q4_k (:112-135) through a C ABI.  Test infrastructure only: these
// are the functions the oracle's fp16 and Q4_K code restates.
#define main q4ref_cpuexp_main
#include "q4rdna_cpu_experiment.cpp"
#undef main

extern "C" {
float q4ref_exp_fp16_to_float(uint16_t v) { return fp16_to_float(v); }
uint16_t q4ref_exp_float_to_fp16(float v) { return float_to_fp16(v); }
// nblocks consecutive 144-byte blocks -> nblocks * 256 floats.
void q4ref_exp_dequant_q4k(const uint8_t *blocks, uint64_t nblocks, float *out) {
    std::array<uint8_t, Q4_K_BLOCK_BYTES> blk{};
    std::array<float, QK_K> w{};
    for (uint64_t i = 0; i < nblocks; ++i) {
        std::memcpy(blk.data(), blocks + i * Q4_K_BLOCK_BYTES, Q4_K_BLOCK_BYTES);
        dequantize_q4_k(blk, w);
        std::memcpy(out + i * QK_K, w.data(), sizeof(float) * QK_K);
    }
}
}
