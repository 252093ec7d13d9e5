// Compiles the reference's source/q4rdna_cpu_experiment.cpp where it lies and
// exports its fp16 converters (:39-100) through a C ABI.  Test infrastructure
// only: these are the converters the oracle's fp16 code restates.
#define main q4ref_cpuexp_main
#include "q4rdna_cpu_experiment.cpp"
#undef main

extern "C" {
float q4ref_exp_fp16_to_float(uint16_t v) { return fp16_to_float(v); }
uint16_t q4ref_exp_float_to_fp16(float v) { return float_to_fp16(v); }
}
