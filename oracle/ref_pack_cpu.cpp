// Compiles the reference's source/q4rdna_sidecar_pack.cpp where it lies and
// exports its scale search (select_scale, :140-179), quantize_value (:126-129)
// and fp16 converters (:73-124) through a C ABI.  Test infrastructure only.
#define main q4ref_pack_main
#include "q4rdna_sidecar_pack.cpp"
#undef main

extern "C" {
uint16_t q4ref_pack_select_scale(const float *v64) { return select_scale(v64); }
int q4ref_pack_quantize_value(float v, float s) { return quantize_value(v, s); }
float q4ref_pack_fp16_to_float(uint16_t v) { return fp16_to_float(v); }
uint16_t q4ref_pack_float_to_fp16(float v) { return float_to_fp16(v); }
}
