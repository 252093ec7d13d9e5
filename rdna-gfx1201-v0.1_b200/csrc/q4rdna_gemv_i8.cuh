// int8 tensor-core group math for B = 1..2 (included into q4rdna_gemv.cu
// inside namespace q4; the kernel built on it is q4rdna_gemv_cta.cuh).  A warp
// streams the four 32-row tiles of a 128-row block, one group (64 columns) per
// step, with 128-bit loads through a register pipeline.
//
//   * codes: a nibble in the HIGH half of a byte is exactly 16 * code as an s8,
//     so a 32-bit code word (4 rows x 2 columns) becomes two A registers with
//     hi = w & 0xF0F0F0F0 and lo = (w << 4) & 0xF0F0F0F0: 3 integer ops per 8
//     weights, no conversion and no offset to undo;
//   * activation: per group, x is scaled by a power of two so its largest
//     magnitude lies in [2^29, 2^30) and rounded to an integer X, so every
//     element keeps an absolute error <= 2^-30 of the group's largest |x|.  X is
//     written in four balanced base-256 digits, X = d3 2^24 + d2 2^16 + d1 2^8
//     + d0 with every d in [-128, 127]: the digit word is
//     (X + 0x808080) ^ 0x808080 read as four s8 bytes (bytes 0..2 are the
//     biased digits d + 128 with the XOR undoing the bias; byte 3 absorbs the
//     carries);
//   * mma.sync m16n8k32 s8 x s8 -> s32 sums the products of one group exactly
//     per digit; the epilogue combines the digit sums in f32 and applies
//     scale * 2^e / 16 once per (row, group), as the reference applies its
//     scale (q4rdna.cu:370-371).
//
// Fragment mapping (m16n8k32, A row-major, B col-major).  Lane (grp, c) loads,
// for k-step m, 16 bytes of tile t = grp >> 1 at 64 + 128m + 32c + 16h
// (h = grp & 1): words q0..q3 = rows 16h + 4j + {0..3} of column pair
// i = 4m + c.  Row set r (r = 0, 1) uses q[2r] for MMA row grp and q[2r+1] for
// MMA row grp + 8: A k-slots 4c + j hold the low-nibble column 2i of row
// (16h + 8r + j [+4]), k-slots 16 + 4c + j the high-nibble column 2i + 1.  The
// four rows of a register are separated by the B operand: for "MMA a" column
// n = 2 * slot + q carries digit d1 (q = 0) or d0 (q = 1) of X placed in byte
// `slot` of the B register; for "MMA b" column 2 * slot + bb carries d2 of batch
// column bb, and for BB = 1 (where bb = 1 is free) d3 of column 0 instead; at
// BB = 2 "MMA c" carries d3 the way "MMA b" carries d2.  So lane (grp, c) ends
// up holding, without any shuffle, all four digit sums of rows
// 16h + c + {0, 4, 8, 12} of tile t.
// Accumulation order: exact int32 inside a group per digit; the digit sums
// recombined as ((S0 + 256 S1) + 2^16 S2) + 2^24 S3 (three f32 roundings);
// groups of a split in ascending order as sum = fma(scale / 16, v * 2^e, sum);
// splits in ascending order in f32 (finish_rows).

// One group of the activation, ready for the B operand.
template <int BB>
struct __align__(16) I8X {
    uint32_t xq[BB][Q4_GROUP];  // per k: the four balanced digits of X (one s8 each)
    float up[BB];               // 2^e: undoes the group's power-of-two scaling
    float ss[BB];               // fused RMSNorm: the group's sum of h^2
};

// Activation scaling shared by both int8 kernels.  E = biased exponent of the
// group's largest |x| = m, clamped to >= 30 so that both 2^(156 - E) and
// 2^(E - 156) are normal f32 numbers: m * 2^(156 - E) lies in [2^29, 2^30), so
// |X| <= 2^30 after rounding.  Groups whose largest |x| is below 2^-97 lose
// bits to the clamp.
__device__ __forceinline__ uint32_t act_exponent(float m) { return max((__float_as_uint(m) >> 23) & 0xffu, 30u); }
__device__ __forceinline__ float act_scale(uint32_t e) { return __uint_as_float((283u - e) << 23); }   // 2^(156 - E)
__device__ __forceinline__ float act_unscale(uint32_t e) { return __uint_as_float((e - 29u) << 23); }  // 2^(E - 156)
// X (|X| <= 2^30) -> its four balanced base-256 digits as s8 bytes.
__device__ __forceinline__ uint32_t act_digits(int X) { return ((uint32_t)X + 0x00808080u) ^ 0x00808080u; }

// NORM kernels: v is the raw RMSNorm input h and gv the norm weight of the same
// columns (1 for the launch's tasks without a norm); the group is prepared as
// h * g and its sum of h^2 goes to *ss.  Branch-free either way, so that the
// compiler can interleave it with the previous group's MMAs.
template <bool NORM>
__device__ __forceinline__ void prep_group_i8(float2 v, float2 gv, bool norm, uint32_t *xq_row, float *up,
                                              float *ss, int lane) {
    (void)norm;
    float m;
    if (NORM) {
        // the sum of h^2 and the max of |h * g| share the shuffle rounds
        float q = fmaf(v.x, v.x, v.y * v.y);
        v.x *= gv.x;
        v.y *= gv.y;
        m = fmaxf(fabsf(v.x), fabsf(v.y));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            q += __shfl_xor_sync(0xffffffffu, q, o);
        }
        if (lane == 0) *ss = q;
    } else {
        m = warp_max(fmaxf(fabsf(v.x), fabsf(v.y)));
    }
    const uint32_t e = act_exponent(m);
    const bool nz = m > 0.0f;
    const float f = nz ? act_scale(e) : 1.0f;
    const float u = nz ? act_unscale(e) : 1.0f;
    uint2 w;
    w.x = act_digits(__float2int_rn(v.x * f));
    w.y = act_digits(__float2int_rn(v.y * f));
    reinterpret_cast<uint2 *>(xq_row)[lane] = w;
    if (lane == 0) *up = u;
}

// An int32 sum S with |S| < 2^22 accumulated on top of kMagicI reads, as f32
// bits, 1.5 * 2^23 + S exactly: the int -> float conversion becomes one
// subtraction (or one fma with a scaled bias) on the full-rate pipe.  A digit
// sum of one group is at most 64 * 128 * 128 = 2^20 in magnitude.
constexpr int kMagicI = 0x4B400000;
constexpr float kMagicF = 12582912.0f;  // 1.5 * 2^23

__device__ __forceinline__ void imma16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Number of "MMA a" (d1, d0 of one batch column) and of high-digit MMAs: at
// BB = 1 one MMA carries d2 and d3; at BB = 2 "MMA b" carries d2 and "MMA c"
// d3 of the batch pair.
template <int BB>
struct I8Shape {
    static constexpr int NA = BB;
    static constexpr int NH = BB == 1 ? 1 : 2;
};

// B-operand selectors of this lane (fixed per kernel): byte `slot` of the
// register takes byte `src` of the per-k digit word; all other bytes are zero.
struct I8Sel {
    uint32_t a;      // MMA a: digit 1 or 0
    uint32_t b2;     // high MMAs: digit 2 in byte `slot`
    uint32_t b3;     // high MMAs: digit 3 in byte `slot`
    int bcol_odd;    // high MMAs: this lane's column is odd (bb = 1)
};

__device__ __forceinline__ uint32_t sel_one(int slot, int src) {
    return (0x4444u & ~(0xFu << (4 * slot))) | ((uint32_t)src << (4 * slot));
}
// Code and scale words of one (tensor, group) step for this lane.
struct StepBufI8 {
    uint4 q[8];     // k-step m: 16 code bytes
    uint32_t s[4];  // fp16 scale bits of rows 16h + c + 4q (low 16 bits)
};

__device__ __forceinline__ uint32_t ld_stream2(const uint8_t *p) {
    unsigned short v;
    asm("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

// Lane's address pieces inside a tile: codes at +64 + 32c + 16h (+128 m),
// scales at +32h + 2c (+8 q).
__device__ __forceinline__ void load_step_i8(StepBufI8 &b, const uint8_t *tile, int c, int h) {
    const uint8_t *qp = tile + Q4_SCALE_BYTES + 32 * c + 16 * h;
#pragma unroll
    for (int m = 0; m < 8; ++m) b.q[m] = ld_stream16(qp + 128 * m);
    const uint8_t *sp = tile + 32 * h + 2 * c;
#pragma unroll
    for (int q = 0; q < 4; ++q) b.s[q] = ld_stream2(sp + 8 * q);
}

// Where a step's code and scale words come from: the register pipeline (slot m
// of the buffer is refilled from the following step's tile as soon as it is
// consumed, so one step of loads is always in flight and the loop has no
// branches).
struct RegSource {
    StepBufI8 &buf;
    const uint8_t *nq, *ns;  // following step: code and scale addresses of this lane
    __device__ __forceinline__ RegSource(StepBufI8 &b, const uint8_t *next, int c, int h)
        : buf(b), nq(next + Q4_SCALE_BYTES + 32 * c + 16 * h), ns(next + 32 * h + 2 * c) {}
    __device__ __forceinline__ void scales(uint32_t (&sw)[4]) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            sw[q] = buf.s[q];
            buf.s[q] = ld_stream2(ns + 8 * q);
        }
    }
    __device__ __forceinline__ uint4 codes(int m) {
        const uint4 cur = buf.q[m];
        buf.q[m] = ld_stream16(nq + 128 * m);
        return cur;
    }
};

// One group of one tensor: 32 (BB = 1) int8 MMAs per warp, exact int32 digit
// sums, then the per-(row, group) scale in f32.
template <int BB, class Src>
__device__ __forceinline__ void mma_step_i8(Src &src, const I8X<BB> &sm, float (&acc)[4][BB], int lane,
                                            const I8Sel &sel) {
    constexpr int NA = I8Shape<BB>::NA, NH = I8Shape<BB>::NH;
    int D[2][NA + NH][4];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int k = 0; k < NA + NH; ++k)
#pragma unroll
            for (int e = 0; e < 4; ++e) D[r][k][e] = kMagicI;  // read back as f32 with one add
    uint32_t sw[4];
    src.scales(sw);
    const int c4 = lane & 3;
    const bool odd = sel.bcol_odd != 0;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        const uint4 cur = src.codes(m);
        uint32_t ba0[NA], ba1[NA], bh0[NH], bh1[NH];
        uint2 W[BB];
#pragma unroll
        for (int b = 0; b < BB; ++b) W[b] = *reinterpret_cast<const uint2 *>(&sm.xq[b][8 * m + 2 * c4]);
#pragma unroll
        for (int b = 0; b < NA; ++b) {
            ba0[b] = __byte_perm(W[b].x, 0u, sel.a);
            ba1[b] = __byte_perm(W[b].y, 0u, sel.a);
        }
        if (BB == 1) {
            // even columns: d2, odd columns: d3, both of batch column 0
            const uint32_t s = odd ? sel.b3 : sel.b2;
            bh0[0] = __byte_perm(W[0].x, 0u, s);
            bh1[0] = __byte_perm(W[0].y, 0u, s);
        } else {
            // even columns: batch 0, odd columns: batch 1; MMA b d2, MMA c d3
            const uint2 w = W[BB > 1 && odd ? 1 : 0];
#pragma unroll
            for (int p = 0; p < NH; ++p) {
                const uint32_t s = p == 0 ? sel.b2 : sel.b3;
                bh0[p] = __byte_perm(w.x, 0u, s);
                bh1[p] = __byte_perm(w.y, 0u, s);
            }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const uint32_t wa = r == 0 ? cur.x : cur.z;  // rows 16h + 8r + {0..3}: MMA row grp
            const uint32_t wb = r == 0 ? cur.y : cur.w;  // rows 16h + 8r + 4 + {0..3}: MMA row grp + 8
            const uint32_t a0 = (wa << 4) & 0xF0F0F0F0u;  // 16 * low-nibble code (column 2i)
            const uint32_t a1 = (wb << 4) & 0xF0F0F0F0u;
            const uint32_t a2 = wa & 0xF0F0F0F0u;         // 16 * high-nibble code (column 2i + 1)
            const uint32_t a3 = wb & 0xF0F0F0F0u;
#pragma unroll
            for (int b = 0; b < NA; ++b) imma16832(D[r][b], a0, a1, a2, a3, ba0[b], ba1[b]);
#pragma unroll
            for (int p = 0; p < NH; ++p) imma16832(D[r][NA + p], a0, a1, a2, a3, bh0[p], bh1[p]);
        }
    }
    // rows 16h + c + 4q, q = 2r + half: digit sums S1 = Da[2*half], S0 = Da[2*half+1];
    // BB = 1: S2 = Dh[2*half], S3 = Dh[2*half+1]; BB = 2: S2 = Db[2*half + b], S3 = Dc[2*half + b]
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int r = q >> 1, hf = q & 1;
        const float sc = __half2float(__ushort_as_half((unsigned short)sw[q])) * 0.0625f;
#pragma unroll
        for (int b = 0; b < BB; ++b) {
            const int d2 = BB == 1 ? D[r][NA][2 * hf] : D[r][NA][2 * hf + b];
            const int d3 = BB == 1 ? D[r][NA][2 * hf + 1] : D[r][NA + 1][2 * hf + b];
            // digit sums over kMagicI (|S| <= 2^20): S1 * 2^8, S2 * 2^16 and
            // S3 * 2^24 come out of the fmas exactly; v rounds once per add
            const float s0 = __int_as_float(D[r][b][2 * hf + 1]) - kMagicF;
            const float lo = fmaf(__int_as_float(D[r][b][2 * hf]), 256.0f, -256.0f * kMagicF) + s0;
            const float mid = fmaf(__int_as_float(d2), 65536.0f, -65536.0f * kMagicF) + lo;
            const float v = fmaf(__int_as_float(d3), 16777216.0f, -16777216.0f * kMagicF) + mid;
            // v * 2^e is exact (a power of two, in range), so this is one rounding
            acc[q][b] = fmaf(sc, v * sm.up[b], acc[q][b]);
        }
    }
}
