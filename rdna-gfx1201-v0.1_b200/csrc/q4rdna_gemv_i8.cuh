// int8 tensor-core GEMV for B = 1..2 (included into q4rdna_gemv.cu inside
// namespace q4).  A warp work item is one 128-row block (four 32-row tiles) x
// one K-range of Gs groups; the warp streams its tiles with 128-bit loads
// through a register pipeline.
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

// Branch-free, so that the compiler can interleave it with the previous
// group's MMAs (see run_item_i8).
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

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

// Where a step's code and scale words come from.  RegSource: the register
// pipeline (slot m of the buffer is refilled from the following step's tile as
// soon as it is consumed, so one step of loads is always in flight and the loop
// has no branches).  SmemSource: a staged tile in shared memory.
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

struct SmemSource {
    const uint8_t *q, *s;
    __device__ __forceinline__ SmemSource(const uint8_t *tile, int c, int h)
        : q(tile + Q4_SCALE_BYTES + 32 * c + 16 * h), s(tile + 32 * h + 2 * c) {}
    __device__ __forceinline__ void scales(uint32_t (&sw)[4]) {
#pragma unroll
        for (int k = 0; k < 4; ++k) sw[k] = *reinterpret_cast<const unsigned short *>(s + 8 * k);
    }
    __device__ __forceinline__ uint4 codes(int m) { return *reinterpret_cast<const uint4 *>(q + 128 * m); }
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

// Epilogue of one item in the int8 layout: lane rows tile_row*32 + 16h + c + 4q.
// iss: fused RMSNorm (NORM kernels), the item's sum of h^2 per batch column.
template <int BB, bool DUAL, bool NORM>
__device__ __forceinline__ void finish_rows_i8(const Task &T, int rb, int s, int B, float (&acc)[2][4][BB],
                                               const float (&iss)[BB], int lane, bool valid, int tile_row, int h,
                                               int c) {
    const int row0 = tile_row * Q4_TILE_ROWS + 16 * h + c;
    if (T.S == 1) {
        if (valid) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
#pragma unroll
                for (int b = 0; b < BB; ++b) {
                    if (b >= B) continue;
                    const size_t idx = (size_t)b * T.N + row0 + 4 * q;
                    float v = acc[0][q][b], gate = acc[DUAL ? 1 : 0][q][b];
                    if (NORM && T.gn != nullptr) {
                        const float r = norm_scale(T, iss[b]);  // the compiler hoists it out of q
                        v *= r;
                        gate *= r;
                    }
                    put_y(T, idx, finish(v, gate, T.op, T.add, idx));
                }
        }
        return;
    }
    constexpr int planes = DUAL ? 2 : 1;
    if (NORM && T.gn != nullptr && lane == 0) {
#pragma unroll
        for (int b = 0; b < BB; ++b)
            if (b < B) __stcg(&T.nss[((size_t)rb * T.S + s) * B + b], iss[b]);
    }
    if (valid) {
#pragma unroll
        for (int pl = 0; pl < planes; ++pl)
#pragma unroll
            for (int q = 0; q < 4; ++q)
#pragma unroll
                for (int b = 0; b < BB; ++b) {
                    if (b >= B) continue;
                    __stcg(&T.part[(((size_t)s * planes + pl) * B + b) * T.N + row0 + 4 * q], acc[pl][q][b]);
                }
    }
    __threadfence();
    __syncwarp();
    unsigned prev = 0;
    if (lane == 0) prev = atomicAdd(&T.ticket[rb], 1u);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev != (unsigned)(T.S - 1)) return;
    reduce_splits<DUAL, NORM>(T, rb, B, lane);
}

// This lane's tile of step 0 of an item, and the item's first group.  Rows past
// N read the block's first row tile instead (always present), so every load is
// in bounds and unconditional; those rows are never stored.
__device__ __forceinline__ const uint8_t *item_tile0(const Task &T, int local, int lane, int *g0_out) {
    const int rb = local / T.S, sp = local % T.S;
    const int g0 = sp * T.Gs;
    const int t = lane >> 3;
    int tile_row = rb * Q4_BLOCK_TILES + t;
    if (tile_row >= (T.N >> 5)) tile_row = rb * Q4_BLOCK_TILES;
    if (g0_out) *g0_out = g0;
    return T.w + ((size_t)tile_row * T.G + g0) * Q4_TILE_BYTES;
}

// Flat cursor over the warp's activation groups (its items in order, each with
// its groups): the raw f32 of the group it points at is fetched two groups
// ahead of the group being multiplied.
struct XCursor {
    long long it;      // item (>= total: past the warp's last group)
    int g, ng, g0, K;  // group within the item, the item's groups, first group, columns
    const float *x;
    const float *gn;   // fused RMSNorm weight, or null
};

__device__ __forceinline__ void xc_load(const Launch &L, XCursor &c) {
    if (c.it >= L.total_items) return;
    const Task &T = find_task(L, c.it);
    const int local = (int)(c.it - T.item_begin);
    c.g0 = (local % T.S) * T.Gs;
    c.ng = min(T.Gs, T.G - c.g0);
    c.g = 0;
    c.K = T.K;
    c.x = T.x;
    c.gn = T.gn;
}

__device__ __forceinline__ void xc_advance(const Launch &L, XCursor &c, long long nw) {
    if (c.it >= L.total_items) return;
    if (++c.g >= c.ng) {
        c.it += nw;
        xc_load(L, c);
    }
}

template <int BB, bool NORM>
__device__ __forceinline__ void xc_fetch(const Launch &L, const XCursor &c, int lane, float2 (&xv)[BB], float2 &gv,
                                         bool &norm) {
    if (c.it >= L.total_items) return;
#pragma unroll
    for (int b = 0; b < BB; ++b)
        if (b < L.B)
            xv[b] = __ldg(reinterpret_cast<const float2 *>(c.x + (size_t)b * c.K + (size_t)(c.g0 + c.g) * Q4_GROUP) +
                          lane);
    if (NORM) {
        // a predicated load, not a branch: tasks without a norm take g = 1
        norm = c.gn != nullptr;
        const float2 *gp = reinterpret_cast<const float2 *>((norm ? c.gn : c.x) + (size_t)(c.g0 + c.g) * Q4_GROUP) + lane;
        const float2 g = __ldg(gp);
        gv = norm ? g : make_float2(1.0f, 1.0f);
    }
}

// Per-warp state carried from item to item.
template <int BB>
struct I8Pipe {
    StepBufI8 buf;   // code and scale words of the next step (register pipeline)
    float2 xv[BB];   // raw x of the next group to prepare
    float2 gv;       // fused RMSNorm: the norm weight of that group's columns
    bool norm;       // that group belongs to a fused-RMSNorm task
    XCursor xc;      // the group whose raw x is in xv
    int par;         // activation buffer holding the group being multiplied
};

// Prepare the raw x in P.xv (the cursor's group) into activation buffer xs;
// past the warp's last group it writes a spare buffer that is never read.
template <int BB, bool NORM>
__device__ __forceinline__ void prep_ahead(I8Pipe<BB> &P, I8X<BB> &xs, int lane) {
#pragma unroll
    for (int b = 0; b < BB; ++b) prep_group_i8<NORM>(P.xv[b], P.gv, P.norm, xs.xq[b], &xs.up[b], &xs.ss[b], lane);
}

template <int BB, bool DUAL, bool NORM>
__device__ __forceinline__ void run_item_i8(const Launch &L, const Task &T, int local, I8X<BB> (&xs)[2], int lane,
                                            const I8Sel &sel, I8Pipe<BB> &P, const Task *nT, int nlocal,
                                            long long nw) {
    const int rb = local / T.S, s = local % T.S;
    const int g0 = s * T.Gs, ng = min(T.Gs, T.G - g0);
    const int grp = lane >> 2, c = lane & 3, t = grp >> 1, h = grp & 1;
    const int tile_row = rb * Q4_BLOCK_TILES + t;
    const bool valid = tile_row < (T.N >> 5);
    const uint8_t *base0 = item_tile0(T, local, lane, nullptr);
    const uint8_t *base1 = DUAL ? T.w2 + (base0 - T.w) : base0;
    const uint8_t *after = nT ? item_tile0(*nT, nlocal, lane, nullptr)
                              : (DUAL ? base1 : base0) + (size_t)(ng - 1) * Q4_TILE_BYTES;
    const int nsteps = ng * (DUAL ? 2 : 1);
    (void)g0;

    float acc[2][4][BB];
#pragma unroll
    for (int pl = 0; pl < 2; ++pl)
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int b = 0; b < BB; ++b) acc[pl][q][b] = 0.0f;
    float iss[BB];
#pragma unroll
    for (int b = 0; b < BB; ++b) iss[b] = 0.0f;

    for (int st = 0; st < nsteps; ++st) {
        const int tt = DUAL ? (st & 1) : 0;
        const uint8_t *next;
        if (st + 1 < nsteps) {
            const int tn = DUAL ? ((st + 1) & 1) : 0, gn = DUAL ? ((st + 1) >> 1) : st + 1;
            next = (tn ? base1 : base0) + (size_t)gn * Q4_TILE_BYTES;
        } else {
            next = after;
        }
        RegSource src(P.buf, next, c, h);
        I8X<BB> &cur = xs[P.par];
        if (tt == 0) {
            mma_step_i8<BB>(src, cur, acc[0], lane, sel);
            if (NORM) {
#pragma unroll
                for (int b = 0; b < BB; ++b) iss[b] += cur.ss[b];  // groups in ascending order
            }
            // The next group's activation goes into the other buffer while the
            // MMAs above drain: no branch in between, so the compiler can
            // interleave the two independent chains.
            prep_ahead<BB, NORM>(P, xs[P.par ^ 1], lane);
        } else {
            mma_step_i8<BB>(src, cur, acc[1], lane, sel);
        }
        if (!DUAL || tt == 1) {
            // end of the group: the prepared buffer becomes current for everyone,
            // and no lane still reads the old one when it is rewritten next
            __syncwarp();
            P.par ^= 1;
            xc_advance(L, P.xc, nw);
            xc_fetch<BB, NORM>(L, P.xc, lane, P.xv, P.gv, P.norm);
        }
    }
    if (DUAL)
        finish_rows_i8<BB, true, NORM>(T, rb, s, L.B, acc, iss, lane, valid, tile_row, h, c);
    else
        finish_rows_i8<BB, false, NORM>(T, rb, s, L.B, acc, iss, lane, valid, tile_row, h, c);
}

// HAS_DUAL = false: the launch holds no SwiGLU task, so the SwiGLU path (and its
// registers) is compiled out.
// NORM = false: the launch holds no fused-RMSNorm task, so that path is compiled out.
template <int BB, bool HAS_DUAL, bool NORM>
__global__ void __launch_bounds__(kThreads, BB <= 2 ? 2 : 1) q4_gemv_i8_kernel(const __grid_constant__ Launch L) {
    __shared__ I8X<BB> xsm[kWarps][2];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long nw = (long long)gridDim.x * kWarps;
    long long it = (long long)blockIdx.x * kWarps + warp;
    if (it >= L.total_items) return;
    I8Sel sel;
    {
        const int n = lane >> 2;  // this lane's B column
        sel.a = sel_one(n >> 1, (n & 1) ? 0 : 1);
        sel.b2 = sel_one(n >> 1, 2);
        sel.b3 = sel_one(n >> 1, 3);
        sel.bcol_odd = n & 1;
    }
    const int c = lane & 3, h = (lane >> 2) & 1;
    I8X<BB>(&xs)[2] = xsm[warp];
    I8Pipe<BB> P;
    P.par = 0;
    {
        const Task &T = find_task(L, it);
        load_step_i8(P.buf, item_tile0(T, (int)(it - T.item_begin), lane, nullptr), c, h);
    }
#pragma unroll
    for (int b = 0; b < BB; ++b) P.xv[b] = make_float2(0.0f, 0.0f);
    P.gv = make_float2(0.0f, 0.0f);
    P.norm = false;
    // the warp's first group into buffer 0, the second group's raw x in flight
    P.xc.it = it;
    xc_load(L, P.xc);
    xc_fetch<BB, NORM>(L, P.xc, lane, P.xv, P.gv, P.norm);
    prep_ahead<BB, NORM>(P, xs[0], lane);
    xc_advance(L, P.xc, nw);
    xc_fetch<BB, NORM>(L, P.xc, lane, P.xv, P.gv, P.norm);
    __syncwarp();
    for (; it < L.total_items; it += nw) {
        const Task &T = find_task(L, it);
        const long long nit = it + nw;
        const Task *nT = nit < L.total_items ? &find_task(L, nit) : nullptr;
        const int nlocal = nT ? (int)(nit - nT->item_begin) : 0;
        if (HAS_DUAL && T.op == Q4RDNA_OP_SWIGLU)
            run_item_i8<BB, true, NORM>(L, T, (int)(it - T.item_begin), xs, lane, sel, P, nT, nlocal, nw);
        else
            run_item_i8<BB, false, NORM>(L, T, (int)(it - T.item_begin), xs, lane, sel, P, nT, nlocal, nw);
    }
}
