// Sidecar packer on the GPU: bf16 weights -> Q4_RDNA tiles, byte for byte what
// the reference packer writes (source/q4rdna_sidecar_pack.cpp:126-179 for the
// per-group scale search, :262-279 for the tile layout; the Python packer,
// source/pack_q4rdna_sidecar.py:44-73, writes the same bytes).
//
// Per group of 64 weights (one row, 64 consecutive columns):
//   * start scales: for factor in {1, .9, .8, .7, .6}, the positive-range start
//     max(pmax / 7, nmax / 8) and the negative-range start -max(pmax / 8,
//     nmax / 7), each times the factor, rounded to fp16;
//   * up to 12 least-squares refinements per start: q = clamp(rint(v / s),
//     -8, 7), error = sum (s q - v)^2, s' = fp16(sum v q / sum q q), stopping
//     when s' repeats or sum q q is 0; the scale with the smallest error wins
//     (the first one on ties);
//   * codes q = clamp(rint(v / s), -8, 7) with the chosen fp16 scale s.
// Every f32 operation is the reference's, in its order, without contraction
// (__fmul_rn / __fadd_rn / __fsub_rn / __fdiv_rn), and every sum runs over
// i = 0..63 in order, so the result is bit-identical.
//
// The one shortcut: rint(v / s) is needed for 64 elements per refinement.
// t = v * (1 / s) differs from the correctly rounded quotient by less than
// 2^-17 for |t| < 2^30, so when t is at least 2^-16 away from every
// half-integer both round to the same integer.  Only the elements near a
// rounding boundary (and the overflow, NaN and infinity cases, whose int
// conversion the reference leaves to the x86 conversion: INT_MIN, hence -8)
// take the exact IEEE division.
//
// Layout: one warp per tile; lane r packs row 32 * row_tile + r of the tile's
// 64 columns, so the scale (2 bytes at 2r) and each code byte (64 + 32 i + r)
// of the 32 lanes are consecutive and the stores coalesce.

#include <cuda_runtime.h>

#include <atomic>
#include <climits>
#include <cstdint>

#include "q4rdna.h"
#include "q4rdna_tile.h"

namespace q4 {
extern std::atomic<uint64_t> g_launches;  // q4rdna_gemv.cu: kernels launched by the library
}

namespace q4pack {

// fp16 -> f32 as the reference packer decodes it (q4rdna_sidecar_pack.cpp:71-92):
// exact for normal values, but a subnormal m * 2^-24 comes out as m * 2^-25
// (its exponent is one short).  The packer evaluates and quantises with this
// value, so the GPU packer must too.
__device__ __forceinline__ float h2f(uint32_t h) {
    const uint32_t sign = (h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    if (e == 0) {
        if (m == 0) return __uint_as_float(sign);
        const int sh = __clz(m) - 21;  // shifts that bring m's top bit to bit 10
        m = (m << sh) & 0x3ffu;
        e = (uint32_t)(127 - 15 - sh);
        return __uint_as_float(sign | (e << 23) | (m << 13));
    }
    if (e == 31) return __uint_as_float(sign | 0x7f800000u | (m << 13));
    return __uint_as_float(sign | ((e + 127 - 15) << 23) | (m << 13));
}

// f32 -> fp16, round to nearest even; above the fp16 range (and for NaN) the
// result is infinity, below half the smallest subnormal it is zero: the
// reference packer's conversion.
__device__ __forceinline__ uint32_t f2h(float v) {
    const uint32_t b = __float_as_uint(v);
    const uint32_t sign = (b >> 16) & 0x8000u;
    const uint32_t man = b & 0x7fffffu;
    const int e = (int)((b >> 23) & 0xffu) - 127 + 15;
    if (e <= 0) {
        if (e < -10) return sign;
        const uint32_t norm = man | 0x800000u;
        const int sh = 14 - e;
        uint32_t r = norm >> sh;
        const uint32_t rem = norm & ((1u << sh) - 1u), half = 1u << (sh - 1);
        if (rem > half || (rem == half && (r & 1u))) ++r;
        return sign | r;
    }
    if (e >= 31) return sign | 0x7c00u;
    uint32_t r = man >> 13;
    const uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) {
        ++r;
        if (r == 0x400u) return e + 1 >= 31 ? (sign | 0x7c00u) : (sign | ((uint32_t)(e + 1) << 10));
    }
    return sign | ((uint32_t)e << 10) | r;
}

// clamp((int) nearbyint(v / s), -8, 7) with the x86 conversion of an
// out-of-range or NaN quotient (INT_MIN).
__device__ __forceinline__ int quant_exact(float v, float s) {
    const float r = rintf(__fdiv_rn(v, s));
    const int q = (r >= -2147483648.0f && r < 2147483648.0f) ? (int)r : INT_MIN;
    return q < -8 ? -8 : (q > 7 ? 7 : q);
}

// Same result; inv = 1 / s (rounded), s != 0.  For |t| < 9 the estimate t and
// the rounded quotient differ by less than 2^-18, so a margin of 2^-16 to the
// nearest half-integer decides; for 9 <= |t| < 2^30 the clamp decides.
__device__ __forceinline__ int quant_fast(float v, float s, float inv) {
    const float t = v * inv;
    const float n = rintf(t);
    // distance to the nearest half-integer boundary: 0.5 - |t - rint(t)|
    const float d = 0.5f - fabsf(t - n);
    if (fabsf(t) < 1073741824.0f && d >= 1.52587890625e-05f) {  // 2^30, 2^-16
        const int q = (int)n;
        return q < -8 ? -8 : (q > 7 ? 7 : q);
    }
    return quant_exact(v, s);
}

// Error, numerator and denominator of one refinement at scale s (s != 0 and
// finite: the fast path needs a finite reciprocal).
__device__ __forceinline__ void refine_sums(const float (&v)[Q4_GROUP], float s, float &err, float &num, float &den) {
    const float inv = 1.0f / s;
    const bool fast = isfinite(inv) && inv != 0.0f;
    float e = 0.0f, n = 0.0f, dn = 0.0f;
#pragma unroll
    for (int i = 0; i < Q4_GROUP; ++i) {
        const int q = fast ? quant_fast(v[i], s, inv) : quant_exact(v[i], s);
        const float qf = (float)q;
        const float dlt = __fsub_rn(__fmul_rn(s, qf), v[i]);
        e = __fadd_rn(e, __fmul_rn(dlt, dlt));
        n = __fadd_rn(n, __fmul_rn(v[i], qf));
        dn = __fadd_rn(dn, (float)(q * q));
    }
    err = e;
    num = n;
    den = dn;
}

__device__ __forceinline__ uint32_t select_scale(const float (&v)[Q4_GROUP]) {
    float pmax = 0.0f, nmax = 0.0f;
#pragma unroll
    for (int i = 0; i < Q4_GROUP; ++i) {
        pmax = pmax < v[i] ? v[i] : pmax;  // std::max(pmax, v[i])
        nmax = nmax < -v[i] ? -v[i] : nmax;
    }
    if (pmax == 0.0f && nmax == 0.0f) return 0;
    const float a = __fdiv_rn(pmax, 7.0f), b = __fdiv_rn(nmax, 8.0f);
    const float c = __fdiv_rn(pmax, 8.0f), d = __fdiv_rn(nmax, 7.0f);
    const float pos = a < b ? b : a;
    const float neg = -(c < d ? d : c);
    const float factors[5] = {1.0f, 0.9f, 0.8f, 0.7f, 0.6f};
    uint32_t best_bits = 0;
    float best_err = __int_as_float(0x7f800000);
    for (int f = 0; f < 5; ++f) {
        for (int sg = 0; sg < 2; ++sg) {
            uint32_t bits = f2h(__fmul_rn(sg == 0 ? pos : neg, factors[f]));
            for (int it = 0; it < 12; ++it) {
                const float s = h2f(bits);
                float err, num, den;
                if (s == 0.0f) {
                    // every q is 0: error = sum v^2 in order, den = 0
                    err = 0.0f;
#pragma unroll
                    for (int i = 0; i < Q4_GROUP; ++i) {
                        const float dlt = -v[i];
                        err = __fadd_rn(err, __fmul_rn(dlt, dlt));
                    }
                    num = 0.0f;
                    den = 0.0f;
                } else {
                    refine_sums(v, s, err, num, den);
                }
                if (err < best_err) {
                    best_err = err;
                    best_bits = bits;
                }
                if (den == 0.0f) break;
                const uint32_t next = f2h(__fdiv_rn(num, den));
                if (next == bits) break;
                bits = next;
            }
        }
    }
    return best_bits;
}

__global__ void __launch_bounds__(128) q4_pack_bf16_kernel(const uint16_t *__restrict__ bf16,
                                                          uint8_t *__restrict__ tiles, int N, int K) {
    const int lane = threadIdx.x & 31;
    const long long tile = (long long)blockIdx.x * 4 + (threadIdx.x >> 5);
    const int G = K / Q4_GROUP;
    const long long ntiles = (long long)(N / Q4_TILE_ROWS) * G;
    if (tile >= ntiles) return;
    const long long row_tile = tile / G;
    const int cg = (int)(tile % G);
    const long long row = row_tile * Q4_TILE_ROWS + lane;
    const uint4 *src = reinterpret_cast<const uint4 *>(bf16 + row * K + (long long)cg * Q4_GROUP);
    float v[Q4_GROUP];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint4 w = __ldg(src + j);
        const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            v[8 * j + 2 * k] = __uint_as_float(u[k] << 16);
            v[8 * j + 2 * k + 1] = __uint_as_float(u[k] & 0xffff0000u);
        }
    }
    const uint32_t sb = select_scale(v);
    const float s = h2f(sb);
    uint8_t *t = tiles + tile * Q4_TILE_BYTES;
    reinterpret_cast<uint16_t *>(t)[lane] = (uint16_t)sb;
#pragma unroll
    for (int i = 0; i < Q4_GROUP / 2; ++i) {
        const int lo = s == 0.0f ? 0 : quant_exact(v[2 * i], s);
        const int hi = s == 0.0f ? 0 : quant_exact(v[2 * i + 1], s);
        t[Q4_SCALE_BYTES + i * Q4_TILE_ROWS + lane] = (uint8_t)((lo & 15) | ((hi & 15) << 4));
    }
}

}  // namespace q4pack

extern "C" q4rdna_status q4rdna_pack_bf16(const uint16_t *bf16, uint8_t *tiles, int N, int K,
                                          q4rdna_stream_t stream) {
    if (bf16 == nullptr || tiles == nullptr || N <= 0 || K <= 0) return Q4RDNA_ERR_INVALID_ARGUMENT;
    if (N % Q4_TILE_ROWS != 0 || K % Q4_GROUP != 0) return Q4RDNA_ERR_SHAPE;
    if ((reinterpret_cast<uintptr_t>(bf16) & 15) != 0 || (reinterpret_cast<uintptr_t>(tiles) & 1) != 0)
        return Q4RDNA_ERR_ALIGNMENT;
    const long long ntiles = (long long)(N / Q4_TILE_ROWS) * (K / Q4_GROUP);
    const long long blocks = (ntiles + 3) / 4;
    if (blocks > INT_MAX) return Q4RDNA_ERR_TOO_LARGE;
    q4pack::q4_pack_bf16_kernel<<<(unsigned)blocks, 128, 0, (cudaStream_t)stream>>>(bf16, tiles, N, K);
    if (cudaGetLastError() != cudaSuccess) return Q4RDNA_ERR_CUDA;
    q4::g_launches.fetch_add(1, std::memory_order_relaxed);
    return Q4RDNA_OK;
}
