// Compiles the reference's source/q4rdna_gemv_bench.hip, unmodified and where
// it lies, as host C++ (HIP headers replaced by oracle/ref_shim) and exports its
// CPU GEMV reference (reference_q4_rdna, q4rdna_gemv_bench.hip:189-211) and
// half_to_float (:163-187) through a C ABI.  Test infrastructure only: it pins
// the oracle restatement against the reference's own code.
#include <cstring>
#define main q4ref_bench_main
#include "q4rdna_gemv_bench.hip"
#undef main

extern "C" {
// The reference function is fixed at ROWS x COLUMNS = 12288 x 4096.
int q4ref_bench_rows() { return ROWS; }
int q4ref_bench_columns() { return COLUMNS; }
float q4ref_bench_half_to_float(uint16_t v) { return half_to_float(v); }
int q4ref_bench_gemv(const uint8_t *tiles, uint64_t nbytes, const float *x, float *y) {
    if (nbytes != uint64_t(ROWS) * COLUMNS / GROUP * 34) return -1;
    std::vector<uint8_t> w(tiles, tiles + nbytes);
    std::vector<float> a(x, x + COLUMNS);
    std::vector<float> out = reference_q4_rdna(w, a);
    std::memcpy(y, out.data(), sizeof(float) * out.size());
    return 0;
}
}

// Prepared form for timing: the tile vector is built once, so a timed call is
// exactly one reference_q4_rdna call (plus the 16 KB activation vector it takes).
extern "C" {
void *q4ref_bench_prepare(const uint8_t *tiles, uint64_t nbytes) {
    if (nbytes != uint64_t(ROWS) * COLUMNS / GROUP * 34) return nullptr;
    return new std::vector<uint8_t>(tiles, tiles + nbytes);
}
int q4ref_bench_run(void *prepared, const float *x, float *y) {
    if (prepared == nullptr) return -1;
    const std::vector<float> a(x, x + COLUMNS);
    const std::vector<float> out = reference_q4_rdna(*static_cast<std::vector<uint8_t> *>(prepared), a);
    std::memcpy(y, out.data(), sizeof(float) * out.size());
    return 0;
}
void q4ref_bench_release(void *prepared) { delete static_cast<std::vector<uint8_t> *>(prepared); }
}
