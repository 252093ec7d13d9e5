/*
 * CPU oracle for the Q4_RDNA group-64 GEMV.  TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the CPU arithmetic of the reference project
 * (davidchen-rocm/RDNA-gfx1201-v0.1).  Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / --impl reference legs may load it, and only as the
 * checker or as the timed CPU baseline.  The product (the CUDA library) never
 * links it and never falls back to it.
 *
 * Each function names the reference lines it follows.  Layout rule
 * (source/q4rdna.cu:20-24, source/q4rdna_sidecar_pack.cpp:268-278):
 *   a tile is 32 rows x 64 columns in 1088 bytes;
 *   bytes [0,64) are 32 little-endian fp16 scales, one per row lane;
 *   byte 64 + 32*i + r holds row r, columns 2i (low nibble) and 2i+1 (high
 *   nibble), both two's-complement int4;
 *   tile index = row_tile * groups + group.
 *
 * Scale decoding: every GEMV/dequant function takes `ieee`.  ieee = 0 uses the
 * reference CPU decoder restated below (q4o_fp16_to_f32, bit-exact with the
 * reference's CPU GEMV, including its halving of fp16 subnormals); ieee = 1
 * uses IEEE binary16 decoding, which is what the reference's GPU kernel
 * computes with __half2float and what the CUDA path is checked against.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define Q4O_GROUP 64
#define Q4O_TILE_ROWS 32
#define Q4O_TILE_BYTES 1088

static float bits_f32(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static uint32_t f32_bits(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }

/* Exact fp16 -> f32, subnormals and inf/nan included.
 * Follows source/q4rdna_cpu_experiment.cpp:39-60 (the bench's copy at
 * source/q4rdna_gemv_bench.hip:163-187 is the same minus the exp==31 branch). */
float q4o_fp16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    if (e == 0) {
        if (m == 0) return bits_f32(sign);
        int sh = 0;
        while ((m & 0x400u) == 0) { m <<= 1; ++sh; }
        m &= 0x3ffu;
        e = (uint32_t)(127 - 15 - sh);
    } else if (e == 31) {
        e = 255;
    } else {
        e += 127 - 15;
    }
    return bits_f32(sign | (e << 23) | (m << 13));
}

/* IEEE-754 binary16 -> f32 (what the reference GPU kernel's __half2float
 * does, source/q4rdna.cu:370).  The reference CPU decoder above differs only on
 * subnormals: it normalises them with exponent 127-15-shift where IEEE needs
 * 127-14-shift, so every subnormal decodes to half its value (0x0001 gives
 * 2^-25 instead of 2^-24).  The same expression is in all three CPU copies
 * (q4rdna_cpu_experiment.cpp:53, q4rdna_sidecar_pack.cpp:87,
 * q4rdna_gemv_bench.hip:179). */
float q4o_fp16_to_f32_ieee(uint16_t h) {
    const uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    if (e == 0 && m != 0) {
        const float v = (float)m * 5.9604644775390625e-08f; /* m * 2^-24, exact */
        return (h & 0x8000u) ? -v : v;
    }
    return q4o_fp16_to_f32(h);
}

/* f32 -> fp16, round to nearest even, with the reference's subnormal and
 * overflow handling.  Follows source/q4rdna_cpu_experiment.cpp:62-100
 * (identical to source/q4rdna_sidecar_pack.cpp:96-124). */
uint16_t q4o_f32_to_fp16(float v) {
    uint32_t b = f32_bits(v);
    uint16_t sign = (uint16_t)((b >> 16) & 0x8000u);
    uint32_t man = b & 0x7fffffu;
    int e = (int)((b >> 23) & 0xffu) - 127 + 15;
    if (e <= 0) {
        if (e < -10) return sign;
        uint32_t norm = man | 0x800000u;
        int sh = 14 - e;
        uint32_t r = norm >> sh;
        uint32_t rem = norm & ((1u << sh) - 1u);
        uint32_t half = 1u << (sh - 1);
        if (rem > half || (rem == half && (r & 1u))) ++r;
        return (uint16_t)(sign | r);
    }
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    uint32_t r = man >> 13;
    uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) {
        ++r;
        if (r == 0x400u) {
            if (e + 1 >= 31) return (uint16_t)(sign | 0x7c00u);
            return (uint16_t)(sign | (uint16_t)((e + 1) << 10));
        }
    }
    return (uint16_t)(sign | (uint16_t)(e << 10) | (uint16_t)r);
}

/* Signed nibbles, source/q4rdna.cu:181-187 and q4rdna_gemv_bench.hip:202-203. */
static inline int nib_lo(uint8_t b) { return (int)(int8_t)(uint8_t)(b << 4) >> 4; }
static inline int nib_hi(uint8_t b) { return (int)(int8_t)b >> 4; }

static inline const uint8_t *tile_at(const uint8_t *tiles, int64_t row_tile, int64_t groups, int64_t g) {
    return tiles + (uint64_t)(row_tile * groups + g) * Q4O_TILE_BYTES;
}

/* ieee = 0: the reference CPU decoder (bit-exact with the reference's CPU GEMV);
 * ieee = 1: IEEE decode, the reference GPU kernel's semantics. */
static inline float tile_scale(const uint8_t *t, int lane, int ieee) {
    uint16_t s; memcpy(&s, t + 2 * lane, 2);
    return ieee ? q4o_fp16_to_f32_ieee(s) : q4o_fp16_to_f32(s);
}

/* Dequantise to a dense row-major f32 matrix W[N][K].  fp16 scale x int in
 * [-8,7] is exact in f32, so this is the bit-exact dequant
 * (q4rdna_cpu_experiment.cpp:266-272 computes stored_scale * float(q)). */
void q4o_dequant(const uint8_t *tiles, int64_t N, int64_t K, float *W, int ieee) {
    const int64_t groups = K / Q4O_GROUP;
    for (int64_t row = 0; row < N; ++row) {
        const int64_t rt = row / Q4O_TILE_ROWS; const int lane = (int)(row % Q4O_TILE_ROWS);
        for (int64_t g = 0; g < groups; ++g) {
            const uint8_t *t = tile_at(tiles, rt, groups, g);
            const float s = tile_scale(t, lane, ieee);
            for (int i = 0; i < Q4O_GROUP / 2; ++i) {
                const uint8_t p = t[64 + i * Q4O_TILE_ROWS + lane];
                W[row * K + g * Q4O_GROUP + 2 * i] = s * (float)nib_lo(p);
                W[row * K + g * Q4O_GROUP + 2 * i + 1] = s * (float)nib_hi(p);
            }
        }
    }
}

/* One row of the reference CPU GEMV, fp32, order exactly as
 * source/q4rdna_gemv_bench.hip:189-211: groups ascending, i ascending,
 * sum = fma(scale*low, x[2i], sum); sum = fma(scale*high, x[2i+1], sum). */
static float row_f32(const uint8_t *tiles, int64_t row, int64_t groups, const float *x, int ieee) {
    const int64_t rt = row / Q4O_TILE_ROWS; const int lane = (int)(row % Q4O_TILE_ROWS);
    float sum = 0.0f;
    for (int64_t g = 0; g < groups; ++g) {
        const uint8_t *t = tile_at(tiles, rt, groups, g);
        const float s = tile_scale(t, lane, ieee);
        const float *xg = x + g * Q4O_GROUP;
        for (int i = 0; i < Q4O_GROUP / 2; ++i) {
            const uint8_t p = t[64 + i * Q4O_TILE_ROWS + lane];
            sum = fmaf(s * (float)nib_lo(p), xg[2 * i], sum);
            sum = fmaf(s * (float)nib_hi(p), xg[2 * i + 1], sum);
        }
    }
    return sum;
}

/* y[b][n] = sum_k W[n][k] x[b][k], B activation columns stored as x[b*K + k].
 * Row-parallel over `threads` OpenMP threads (threads <= 1: serial, as the
 * reference bench runs it). */
void q4o_gemv_f32(const uint8_t *tiles, const float *x, float *y,
                  int64_t N, int64_t K, int64_t B, int threads, int ieee) {
    const int64_t groups = K / Q4O_GROUP;
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1) if (threads > 1)
    for (int64_t row = 0; row < N; ++row)
        for (int64_t b = 0; b < B; ++b)
            y[b * N + row] = row_f32(tiles, row, groups, x + b * K, ieee);
}

/* fp64-accumulated y and the per-row magnitude sum |W[n][k] x[k]| used by the
 * normwise tolerance.  Not in the reference; it is the accuracy yardstick. */
void q4o_gemv_f64(const uint8_t *tiles, const float *x, double *y, double *absdot,
                  int64_t N, int64_t K, int64_t B, int threads, int ieee) {
    const int64_t groups = K / Q4O_GROUP;
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1) if (threads > 1)
    for (int64_t row = 0; row < N; ++row) {
        const int64_t rt = row / Q4O_TILE_ROWS; const int lane = (int)(row % Q4O_TILE_ROWS);
        for (int64_t b = 0; b < B; ++b) {
            const float *xb = x + b * K;
            double sum = 0.0, mag = 0.0;
            for (int64_t g = 0; g < groups; ++g) {
                const uint8_t *t = tile_at(tiles, rt, groups, g);
                const double s = (double)tile_scale(t, lane, ieee);
                for (int i = 0; i < Q4O_GROUP / 2; ++i) {
                    const uint8_t p = t[64 + i * Q4O_TILE_ROWS + lane];
                    const double a = s * nib_lo(p) * (double)xb[g * Q4O_GROUP + 2 * i];
                    const double c = s * nib_hi(p) * (double)xb[g * Q4O_GROUP + 2 * i + 1];
                    sum += a + c; mag += fabs(a) + fabs(c);
                }
            }
            y[b * N + row] = sum;
            if (absdot) absdot[b * N + row] = mag;
        }
    }
}

/* Fused epilogues of the reference operator surface:
 *   mul_mat_add  (source/q4rdna.cu:747-767, kernel line 393): y = W.x + add
 *   mul_mat_glu  (source/q4rdna.cu:769-793, kernel line 394): y = (W_up.x) * silu(W_gate.x)
 * SiLU itself lives in ggml (ggml_cuda_op_silu_single, not vendored); the
 * published ggml definition is x / (1 + exp(-x)), restated here in f32.
 * No reference test pins these epilogues. */
float q4o_silu(float v) { return v / (1.0f + expf(-v)); }

void q4o_gemv_add_f32(const uint8_t *tiles, const float *x, const float *add, float *y,
                      int64_t N, int64_t K, int64_t B, int threads, int ieee) {
    q4o_gemv_f32(tiles, x, y, N, K, B, threads, ieee);
    for (int64_t i = 0; i < N * B; ++i) y[i] += add[i];
}

void q4o_gemv_swiglu_f32(const uint8_t *up, const uint8_t *gate, const float *x, float *y,
                         float *scratch_gate, int64_t N, int64_t K, int64_t B, int threads, int ieee) {
    q4o_gemv_f32(up, x, y, N, K, B, threads, ieee);
    q4o_gemv_f32(gate, x, scratch_gate, N, K, B, threads, ieee);
    for (int64_t i = 0; i < N * B; ++i) y[i] *= q4o_silu(scratch_gate[i]);
}

/* ---- packer (format writer), restated from source/q4rdna_sidecar_pack.cpp ---- */

static float bf16_f32(uint16_t v) { return bits_f32((uint32_t)v << 16); }

/* q4rdna_sidecar_pack.cpp:126-129: clamp(nearbyint(v/s), -8, 7), 0 when s == 0.
 * nearbyintf under the default FE_TONEAREST mode (the packer sets it, :221). */
static int quant_value(float v, float s) {
    if (s == 0.0f) return 0;
    int q = (int)nearbyintf(v / s);
    return q < -8 ? -8 : (q > 7 ? 7 : q);
}

static float scale_error(const float *in, float s) {
    float err = 0.0f;
    for (int i = 0; i < Q4O_GROUP; ++i) {
        const float d = s * (float)quant_value(in[i], s) - in[i];
        err += d * d;
    }
    return err;
}

/* 5-factor x {positive, negative} range start, 12 fp16-aware least-squares
 * refinements, best squared error wins (first one on ties).
 * q4rdna_sidecar_pack.cpp:140-179, same f32 arithmetic and order. */
uint16_t q4o_select_scale(const float *in) {
    float pmax = 0.0f, nmax = 0.0f;
    for (int i = 0; i < Q4O_GROUP; ++i) {
        if (in[i] > pmax) pmax = in[i];
        if (-in[i] > nmax) nmax = -in[i];
    }
    if (pmax == 0.0f && nmax == 0.0f) return 0;
    const float pos = fmaxf(pmax / 7.0f, nmax / 8.0f);
    const float neg = -fmaxf(pmax / 8.0f, nmax / 7.0f);
    static const float factors[5] = {1.0f, 0.9f, 0.8f, 0.7f, 0.6f};
    uint16_t best_bits = 0;
    float best_err = INFINITY;
    for (int f = 0; f < 5; ++f) {
        for (int sgn = 0; sgn < 2; ++sgn) {
            const float init = (sgn == 0 ? pos : neg) * factors[f];
            uint16_t bits = q4o_f32_to_fp16(init);
            for (int it = 0; it < 12; ++it) {
                const float s = q4o_fp16_to_f32(bits);
                const float err = scale_error(in, s);
                if (err < best_err) { best_err = err; best_bits = bits; }
                float num = 0.0f, den = 0.0f;
                for (int i = 0; i < Q4O_GROUP; ++i) {
                    const int q = quant_value(in[i], s);
                    num += in[i] * (float)q;
                    den += (float)(q * q);
                }
                if (den == 0.0f) break;
                const uint16_t next = q4o_f32_to_fp16(num / den);
                if (next == bits) break;
                bits = next;
            }
        }
    }
    return best_bits;
}

/* Pack a row-major bf16 matrix [N][K] into tiles (q4rdna_sidecar_pack.cpp:262-279). */
void q4o_pack_bf16(const uint16_t *bf16, int64_t N, int64_t K, uint8_t *tiles, int threads) {
    const int64_t gpr = K / Q4O_GROUP;
    const int64_t ngroups = N * gpr;
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1) if (threads > 1)
    for (int64_t grp = 0; grp < ngroups; ++grp) {
        float v[Q4O_GROUP];
        for (int i = 0; i < Q4O_GROUP; ++i) v[i] = bf16_f32(bf16[grp * Q4O_GROUP + i]);
        const uint16_t sb = q4o_select_scale(v);
        const float s = q4o_fp16_to_f32(sb);
        const int64_t row = grp / gpr, cg = grp % gpr;
        const int64_t tile = (row / Q4O_TILE_ROWS) * gpr + cg;
        const int64_t lane = row % Q4O_TILE_ROWS;
        uint8_t *t = tiles + tile * Q4O_TILE_BYTES;
        memcpy(t + lane * 2, &sb, 2);
        for (int i = 0; i < Q4O_GROUP / 2; ++i) {
            const int lo = quant_value(v[2 * i], s), hi = quant_value(v[2 * i + 1], s);
            t[64 + i * Q4O_TILE_ROWS + lane] = (uint8_t)((lo & 15) | ((hi & 15) << 4));
        }
    }
}

/* ---- Q4_K: the tensors the reference leaves on llama.cpp's stock path ----
 * The qkv-fallback scope (source/q4rdna.cu:685-691) keeps the Q/K/V
 * projections in ggml's block_q4_K format, and the reference bench times a
 * Q4_K GEMV beside its own (q4rdna_gemv_bench.hip:93-135).  A block holds 256
 * weights of one row in 144 bytes (q4rdna_cpu_experiment.cpp:17,
 * q4rdna_gemv_bench.hip:25-26):
 *   bytes 0-1   fp16 d, bytes 2-3 fp16 dmin;
 *   bytes 4-15  eight 6-bit scales and eight 6-bit mins (q4k_scale_min);
 *   bytes 16-143 quants: byte 16 + 32c + i holds weight 64c + i in its low
 *               nibble and weight 64c + 32 + i in its high nibble (unsigned).
 * weight = (d * scale_j) * q - dmin * min_j for sub-block j = k / 32.
 * A row is K / 256 consecutive blocks; rows are consecutive. */
#define Q4O_QK 256
#define Q4O_QK_BYTES 144

/* q4rdna_cpu_experiment.cpp:102-110 (get_scale_min; the bench's copy is the same). */
static void q4k_scale_min(int j, const uint8_t *s, int *sc, int *mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

static inline float q4k_half(const uint8_t *p, int ieee) {
    uint16_t h; memcpy(&h, p, 2);
    return ieee ? q4o_fp16_to_f32_ieee(h) : q4o_fp16_to_f32(h);
}

/* Dense W[N][K] from Q4_K rows, q4rdna_cpu_experiment.cpp:112-135: per
 * chunk c, weight 64c + i = d*scale0*float(q & 15) - dmin*min0 and weight
 * 64c + 32 + i = d*scale1*float(q >> 4) - dmin*min1, evaluated left to right
 * in f32 (d*scale*q is exact, so the subtraction is the only rounding). */
void q4o_q4k_dequant(const uint8_t *blocks, int64_t N, int64_t K, float *W, int ieee) {
    const int64_t nb = K / Q4O_QK;
    for (int64_t row = 0; row < N; ++row)
        for (int64_t b = 0; b < nb; ++b) {
            const uint8_t *blk = blocks + (uint64_t)(row * nb + b) * Q4O_QK_BYTES;
            const float d = q4k_half(blk, ieee), dmin = q4k_half(blk + 2, ieee);
            float *w = W + row * K + b * Q4O_QK;
            for (int c = 0; c < 4; ++c) {
                int s0, m0, s1, m1;
                q4k_scale_min(2 * c, blk + 4, &s0, &m0);
                q4k_scale_min(2 * c + 1, blk + 4, &s1, &m1);
                for (int i = 0; i < 32; ++i) {
                    const uint8_t p = blk[16 + 32 * c + i];
                    w[64 * c + i] = d * (float)s0 * (float)(p & 15) - dmin * (float)m0;
                    w[64 * c + 32 + i] = d * (float)s1 * (float)(p >> 4) - dmin * (float)m1;
                }
            }
        }
}

/* One row of the reference's Q4_K GEMV in its f32 order
 * (q4rdna_gemv_bench.hip:93-135, one lane per row): blocks ascending, chunks
 * ascending, i ascending; ds = d*scale, dm = dmin*min per sub-block;
 * sum = fmaf(ds0*q_lo - dm0, x[64c+i], sum); sum = fmaf(ds1*q_hi - dm1,
 * x[64c+32+i], sum).  ds*q is exact, so contracting ds*q - dm into one fma
 * (as a GPU compiler may) gives the same weight. */
static float q4k_row_f32(const uint8_t *row_blocks, int64_t nb, const float *x, int ieee) {
    float sum = 0.0f;
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t *blk = row_blocks + (uint64_t)b * Q4O_QK_BYTES;
        const float d = q4k_half(blk, ieee), dmin = q4k_half(blk + 2, ieee);
        const float *xb = x + b * Q4O_QK;
        for (int c = 0; c < 4; ++c) {
            int s0, m0, s1, m1;
            q4k_scale_min(2 * c, blk + 4, &s0, &m0);
            q4k_scale_min(2 * c + 1, blk + 4, &s1, &m1);
            const float ds0 = d * (float)s0, dm0 = dmin * (float)m0;
            const float ds1 = d * (float)s1, dm1 = dmin * (float)m1;
            for (int i = 0; i < 32; ++i) {
                const uint8_t p = blk[16 + 32 * c + i];
                const float w0 = ds0 * (float)(p & 15) - dm0;
                const float w1 = ds1 * (float)(p >> 4) - dm1;
                sum = fmaf(w0, xb[64 * c + i], sum);
                sum = fmaf(w1, xb[64 * c + 32 + i], sum);
            }
        }
    }
    return sum;
}

/* y[b][n] in the reference Q4_K kernel's order, B columns x[b*K + k]. */
void q4o_q4k_gemv_f32(const uint8_t *blocks, const float *x, float *y,
                      int64_t N, int64_t K, int64_t B, int threads, int ieee) {
    const int64_t nb = K / Q4O_QK;
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1) if (threads > 1)
    for (int64_t row = 0; row < N; ++row)
        for (int64_t b = 0; b < B; ++b)
            y[b * N + row] = q4k_row_f32(blocks + (uint64_t)row * nb * Q4O_QK_BYTES, nb, x + b * K, ieee);
}

/* fp64-accumulated y over the dequantised weights (q4o_q4k_dequant's values)
 * and the per-row sum |W x|: the accuracy yardstick, as q4o_gemv_f64. */
void q4o_q4k_gemv_f64(const uint8_t *blocks, const float *x, double *y, double *absdot,
                      int64_t N, int64_t K, int64_t B, int threads, int ieee) {
    const int64_t nb = K / Q4O_QK;
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1) if (threads > 1)
    for (int64_t row = 0; row < N; ++row) {
        float w[Q4O_QK];
        for (int64_t b = 0; b < B; ++b) {
            y[b * N + row] = 0.0;
            if (absdot) absdot[b * N + row] = 0.0;
        }
        for (int64_t k0 = 0; k0 < nb; ++k0) {
            q4o_q4k_dequant(blocks + (uint64_t)(row * nb + k0) * Q4O_QK_BYTES, 1, Q4O_QK, w, ieee);
            for (int64_t b = 0; b < B; ++b) {
                const float *xb = x + b * K + k0 * Q4O_QK;
                double sum = 0.0, mag = 0.0;
                for (int i = 0; i < Q4O_QK; ++i) {
                    const double a = (double)w[i] * (double)xb[i];
                    sum += a; mag += fabs(a);
                }
                y[b * N + row] += sum;
                if (absdot) absdot[b * N + row] += mag;
            }
        }
    }
}
