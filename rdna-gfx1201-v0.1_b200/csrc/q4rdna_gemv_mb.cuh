// Small-batch tile path, B = 3..16 activation columns (included into
// q4rdna_gemv.cu inside namespace q4, after q4rdna_gemv_i8.cuh).
//
// At B >= 3 the work is a dense contraction: every weight meets B activations.
// The batch-1 kernel's fragment mapping spends most of each MMA on zeros (it
// keeps rows in the K slots so that lanes need no transposition), which is
// right for B <= 2 and wasteful above it.  This kernel uses the full
// m16n8k32 fragment instead:
//
//   * one CTA (4 warps) owns one work item: 128 rows (4 row tiles) x a split of
//     the groups; warp w owns row tile 4 rb + w;
//   * lane (g, c) loads, per group, the 8 code words (row quad g = rows
//     4g..4g+3) x (column pair P = 16 ks + 4 j + c, j = 0..3, ks = 0..1), each
//     at tile + 64 + 32 P + 4 g: every warp load covers one full 128-byte line;
//   * a 4x4 byte transpose (8 prmt) turns the 4 words of a k-step into 4 row
//     words (row 4g + r, pairs P_0..P_3); hi = w & 0xF0F0F0F0 and
//     lo = (w << 4) & 0xF0F0F0F0 are exactly 16 * code as s8;
//   * MMA row g <-> tile row 4g + 2 rs, MMA row g + 8 <-> 4g + 2 rs + 1
//     (row set rs = 0, 1); k-slot 4c + j <-> column 2 P_j, k-slot 16 + 4c + j
//     <-> column 2 P_j + 1;
//   * the activation of one group, scaled by 2^(156 - E) (E = biased exponent
//     of the group's largest |x|, per batch column, as in the batch-1 kernel)
//     and rounded to an integer X with |X| <= 2^30, is used as its four
//     balanced base-256 digits (act_digits: X = d3 2^24 + d2 2^16 + d1 2^8 +
//     d0, every digit an s8).  The n-tiles are digit-major: n-tile
//     t = limb * NBB + bb holds digit `limb` of batch columns 8 bb .. 8 bb + 7.
//     The whole CTA prepares the B fragments of a chunk of groups once, in
//     shared memory, for its four warps;
//   * per group the int32 digit sums are exact (accumulated over a float bias,
//     so that reading them as f32 costs one add: kMagicI); the epilogue
//     combines them as ((S0 + 2^8 S1) + 2^16 S2) + 2^24 S3, rounding once per
//     add, and accumulates fma(scale / 16, v * 2^e, acc) in f32, groups in
//     ascending order; splits are added in ascending order (mb_finish).
//
// Pipeline: the code words of chunk q + 1 are loaded into a slot's registers
// as soon as that slot of chunk q is consumed, the activations of chunk q + 1
// are prefetched into L1 while chunk q computes, and the CTA meets once per
// chunk (double-buffered fragments).

template <int BP>
struct MbShape {
    static constexpr int NBB = BP / 8;          // batch blocks of 8 columns
    static constexpr int NT = 4 * NBB;          // n-tiles (digit-major)
    static constexpr int SLOTS = 4;             // tile slots per chunk (groups x planes)
    static constexpr int GPP = 128 / (8 * BP);  // groups prepared per pass of 128 threads
    static constexpr int PASSES = 4 / GPP;
};
constexpr int kMbThreads = 128;
constexpr int kMbWarps = 4;

template <int BP>
struct __align__(16) MbSmem {
    uint2 b[2][4][MbShape<BP>::NT][2][32];  // [buffer][group][n-tile][k-step][lane]: b0, b1
    float up[2][4][BP];                     // 2^e per (group, batch column)
    float ss[2][4][BP];                     // fused RMSNorm: sum of h^2 per (group, batch column)
    float nr[BP];                           // fused RMSNorm: scale per batch column (split reduction)
    unsigned last;                          // split ticket of this CTA's item
};

// Rows 4g..4g+3 of pairs P_0..P_3 (words w0..w3) -> row words r0..r3.
__device__ __forceinline__ void transpose4(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, uint32_t &r0,
                                           uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    const uint32_t t0 = __byte_perm(w0, w1, 0x5140), t1 = __byte_perm(w0, w1, 0x7362);
    const uint32_t t2 = __byte_perm(w2, w3, 0x5140), t3 = __byte_perm(w2, w3, 0x7362);
    r0 = __byte_perm(t0, t2, 0x5410);
    r1 = __byte_perm(t0, t2, 0x7632);
    r2 = __byte_perm(t1, t3, 0x5410);
    r3 = __byte_perm(t1, t3, 0x7632);
}

__device__ __forceinline__ uint32_t s8_hi(uint32_t w) { return w & 0xF0F0F0F0u; }
__device__ __forceinline__ uint32_t s8_lo(uint32_t w) { return (w << 4) & 0xF0F0F0F0u; }

// D (+)= A (s8) * B (s8); Z: the accumulator starts at kMagicI
// (q4rdna_gemv_i8.cuh) instead of D.
template <bool Z>
__device__ __forceinline__ void imma_mb(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    if (Z)
        asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%10,%10,%10,%10};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(kMagicI));
    else
        asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Code words and scales of one tile for this lane.
struct MbTileRegs {
    uint32_t w[8];  // [ks * 4 + j]: row quad g, pair 16 ks + 4 j + c
    uint2 sc;       // fp16 scales of rows 4g .. 4g + 3
};

__device__ __forceinline__ void mb_load_tile(MbTileRegs &r, const uint8_t *tile, int g, int c) {
    const uint8_t *q = tile + Q4_SCALE_BYTES + 4 * g + 32 * c;
#pragma unroll
    for (int ks = 0; ks < 2; ++ks)
#pragma unroll
        for (int j = 0; j < 4; ++j) r.w[ks * 4 + j] = ld_stream4(q + 32 * (16 * ks + 4 * j));
    uint2 s;
    asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(s.x), "=r"(s.y) : "l"(tile + 8 * g));
    r.sc = s;
}

// Byte `limb` of each of four words -> one B register (byte j from word j).
__device__ __forceinline__ uint32_t gather_byte(uint32_t p0, uint32_t p1, uint32_t p2, uint32_t p3, int limb) {
    const uint32_t s = (uint32_t)limb;
    const uint32_t sel01 = s | ((s + 4) << 4);  // bytes: p0.limb, p1.limb
    const uint32_t u01 = __byte_perm(p0, p1, sel01), u23 = __byte_perm(p2, p3, sel01);
    return __byte_perm(u01, u23, 0x5410);
}

// Position of the CTA's work: item `it` (>= total: none) and its chunk at `base`.
struct MbCursor {
    long long it;
    const Task *T;
    int rb, s, gbeg, ng, base, ncg;
    bool dual;
};

template <bool HAS_DUAL>
__device__ __forceinline__ void mb_item(const Launch &L, MbCursor &c, long long it) {
    c.it = it;
    if (it >= L.total_items) return;
    const Task &T = find_task(L, it);
    c.T = &T;
    const int local = (int)(it - T.item_begin);
    c.rb = local / T.S;
    c.s = local % T.S;
    c.gbeg = c.s * T.Gs;
    c.ng = min(T.Gs, T.G - c.gbeg);
    c.dual = HAS_DUAL && T.op == Q4RDNA_OP_SWIGLU;
    c.base = 0;
    c.ncg = min(c.dual ? 2 : 4, c.ng);
}

// Next chunk: the item's next 4 groups (2 for SwiGLU), else the CTA's next item.
template <bool HAS_DUAL>
__device__ __forceinline__ void mb_advance(const Launch &L, MbCursor &c, long long stride) {
    const int cg = c.dual ? 2 : 4;
    if (c.base + cg < c.ng) {
        c.base += cg;
        c.ncg = min(cg, c.ng - c.base);
    } else {
        mb_item<HAS_DUAL>(L, c, c.it + stride);
    }
}

__device__ __forceinline__ bool mb_last_chunk(const MbCursor &c) { return c.base + (c.dual ? 2 : 4) >= c.ng; }
__device__ __forceinline__ int mb_nslot(const MbCursor &c) { return c.dual ? 2 * c.ncg : c.ncg; }

// This warp's tile of slot sl of chunk c.  Rows past N read the block's first
// row tile (always present) so every load stays in bounds; they are never stored.
__device__ __forceinline__ const uint8_t *mb_tile_addr(const MbCursor &c, int sl, int warp) {
    const Task &T = *c.T;
    const int tile_row = c.rb * Q4_BLOCK_TILES + warp;
    const int trow = tile_row < (T.N >> 5) ? tile_row : c.rb * Q4_BLOCK_TILES;
    const int gi = c.dual ? (sl >> 1) : sl;
    const uint8_t *w = (c.dual && (sl & 1)) ? T.w2 : T.w;
    return w + ((size_t)trow * T.G + c.gbeg + c.base + gi) * Q4_TILE_BYTES;
}

// Activation columns this thread prepares in pass `pass` of chunk c: thread
// (group gi, batch b, k-step ks, pair lane cc) owns columns
// 32 ks + 8 j + 2 cc + {0, 1}, j = 0..3 (one 128-byte line) of batch column b.
template <int BP>
__device__ __forceinline__ const float *mb_xline(const MbCursor &c, int B, int pass, int tid, bool &live) {
    using S = MbShape<BP>;
    constexpr int PER = 8 * BP;  // threads per group
    const int gi = pass * S::GPP + tid / PER;
    const int r = tid % PER;
    const int b = r >> 3, ks = (r >> 2) & 1, cc = r & 3;
    live = gi < c.ncg && b < B;
    const Task &T = *c.T;
    return T.x + (size_t)(live ? b : 0) * T.K + (size_t)(c.gbeg + c.base + (live ? gi : 0)) * Q4_GROUP + 32 * ks +
           2 * cc;
}

template <int BP>
__device__ __forceinline__ void mb_prefetch_x(const MbCursor &c, int B, int tid) {
#pragma unroll
    for (int pass = 0; pass < MbShape<BP>::PASSES; ++pass) {
        bool live;
        const float *xp = mb_xline<BP>(c, B, pass, tid, live);
        if (live) asm volatile("prefetch.global.L1 [%0];" ::"l"(xp));
    }
}

// The CTA prepares the B fragments of chunk c into buffer `par`.
template <int BP, bool NORM>
__device__ __forceinline__ void mb_prep(MbSmem<BP> &sm, int par, const MbCursor &c, int B, int tid) {
    using S = MbShape<BP>;
    constexpr int PER = 8 * BP;
#pragma unroll
    for (int pass = 0; pass < S::PASSES; ++pass) {
        const int gi = pass * S::GPP + tid / PER;
        const int r = tid % PER;
        const int b = r >> 3, ks = (r >> 2) & 1, cc = r & 3;
        bool live;
        const float *xp = mb_xline<BP>(c, B, pass, tid, live);
        float2 v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
            v[j] = live ? __ldg(reinterpret_cast<const float2 *>(xp + 8 * j)) : make_float2(0.0f, 0.0f);
        float ssq = 0.0f;
        if (NORM) {
            // fused RMSNorm: v is the raw input h; the group is prepared as h * g
            // (g = 1 for the launch's tasks without a norm: predicated, no branch)
            const float *gn = c.T->gn;
            const bool nrm = gn != nullptr;
            const float *gp = (nrm ? gn : c.T->x) + (xp - (c.T->x + (size_t)(live ? b : 0) * c.T->K));
            float q = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                q = fmaf(v[j].x, v[j].x, q);
                q = fmaf(v[j].y, v[j].y, q);
                const float2 gl = __ldg(reinterpret_cast<const float2 *>(gp + 8 * j));
                const float2 g = nrm ? gl : make_float2(1.0f, 1.0f);
                v[j].x *= g.x;
                v[j].y *= g.y;
            }
            ssq = q;
        }
        float m = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) m = fmaxf(m, fmaxf(fabsf(v[j].x), fabsf(v[j].y)));
        // the 8 threads of (gi, b) are lanes 8k .. 8k + 7 of one warp; with NORM
        // the sum of h^2 shares the shuffle rounds
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (NORM) ssq += __shfl_xor_sync(0xffffffffu, ssq, o);
        }
        if (NORM && gi < c.ncg && (r & 7) == 0) sm.ss[par][gi][b] = ssq;
        const uint32_t e = act_exponent(m);  // as prep_group_i8
        const bool nz = m > 0.0f;
        const float f = nz ? act_scale(e) : 1.0f;
        const float u = nz ? act_unscale(e) : 1.0f;
        uint32_t p0[4], p1[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            p0[j] = act_digits(__float2int_rn(v[j].x * f));
            p1[j] = act_digits(__float2int_rn(v[j].y * f));
        }
        if (gi < c.ncg) {
            const int lane = (b & 7) * 4 + cc, bb = b >> 3;
#pragma unroll
            for (int limb = 0; limb < 4; ++limb) {
                uint2 w;
                w.x = gather_byte(p0[0], p0[1], p0[2], p0[3], limb);
                w.y = gather_byte(p1[0], p1[1], p1[2], p1[3], limb);
                sm.b[par][gi][limb * S::NBB + bb][ks][lane] = w;
            }
            if ((r & 7) == 0) sm.up[par][gi][b] = u;
        }
    }
}

// One tile (one group of one tensor) for this warp: 4 NT MMAs, then the
// per-(row, group) scale into acc[4 rows][NBB][2 columns].
template <int BP>
__device__ __forceinline__ void mb_tile(const MbTileRegs &r, const MbSmem<BP> &sm, int par, int gi, int lane,
                                        float (&acc)[4][BP / 8][2]) {
    using S = MbShape<BP>;
    int D[2][S::NT][4];
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
        uint32_t R[4];
        transpose4(r.w[4 * ks], r.w[4 * ks + 1], r.w[4 * ks + 2], r.w[4 * ks + 3], R[0], R[1], R[2], R[3]);
        uint32_t A[2][4];
#pragma unroll
        for (int rs = 0; rs < 2; ++rs) {
            A[rs][0] = s8_lo(R[2 * rs]);
            A[rs][1] = s8_lo(R[2 * rs + 1]);
            A[rs][2] = s8_hi(R[2 * rs]);
            A[rs][3] = s8_hi(R[2 * rs + 1]);
        }
#pragma unroll
        for (int t = 0; t < S::NT; ++t) {
            const uint2 bf = sm.b[par][gi][t][ks][lane];
#pragma unroll
            for (int rs = 0; rs < 2; ++rs) {
                if (ks == 0) imma_mb<true>(D[rs][t], A[rs][0], A[rs][1], A[rs][2], A[rs][3], bf.x, bf.y);
                else imma_mb<false>(D[rs][t], A[rs][0], A[rs][1], A[rs][2], A[rs][3], bf.x, bf.y);
            }
        }
    }
    const int c = lane & 3;
    float s[4];
    s[0] = __half2float(__ushort_as_half((unsigned short)(r.sc.x & 0xffffu))) * 0.0625f;
    s[1] = __half2float(__ushort_as_half((unsigned short)(r.sc.x >> 16))) * 0.0625f;
    s[2] = __half2float(__ushort_as_half((unsigned short)(r.sc.y & 0xffffu))) * 0.0625f;
    s[3] = __half2float(__ushort_as_half((unsigned short)(r.sc.y >> 16))) * 0.0625f;
#pragma unroll
    for (int bb = 0; bb < S::NBB; ++bb) {
        const float2 uq = *reinterpret_cast<const float2 *>(&sm.up[par][gi][8 * bb + 2 * c]);
#pragma unroll
        for (int rs = 0; rs < 2; ++rs)
#pragma unroll
            for (int e = 0; e < 2; ++e)
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const int k = 2 * e + q;
                    // digit sums S0..S3 (|S| <= 2^20) over kMagicI; S1 * 2^8,
                    // S2 * 2^16 and S3 * 2^24 come out of the fmas exactly, so v is
                    // ((S0 + 2^8 S1) + 2^16 S2) + 2^24 S3 with three roundings
                    const float s0 = __int_as_float(D[rs][bb][k]) - kMagicF;
                    const float lo = fmaf(__int_as_float(D[rs][S::NBB + bb][k]), 256.0f, -256.0f * kMagicF) + s0;
                    const float mid =
                        fmaf(__int_as_float(D[rs][2 * S::NBB + bb][k]), 65536.0f, -65536.0f * kMagicF) + lo;
                    const float v =
                        fmaf(__int_as_float(D[rs][3 * S::NBB + bb][k]), 16777216.0f, -16777216.0f * kMagicF) + mid;
                    acc[2 * rs + e][bb][q] = fmaf(s[2 * rs + e], v * (q ? uq.y : uq.x), acc[2 * rs + e][bb][q]);
                }
    }
}

// Item epilogue: store (S == 1), or write this warp's split partials and, in the
// CTA that arrives last at row block rb, add the splits in ascending order.
// iss: fused RMSNorm (NORM kernels), the item's sum of h^2 per (batch block,
// column) of this lane.
// Sm: the kernel's shared block (members `last` and `nr[BP]`).
template <int BP, bool HAS_DUAL, bool NORM, class Sm>
__device__ __forceinline__ void mb_finish(const Task &T, int rb, int s, int B, float (&acc)[HAS_DUAL ? 2 : 1][4][BP / 8][2],
                                          const float (&iss)[BP / 8][2], bool dual, bool valid, int tile_row,
                                          int lane, int tid, Sm &sm) {
    using S = MbShape<BP>;
    const int g = lane >> 2, c = lane & 3;
    const int row0 = tile_row * Q4_TILE_ROWS + 4 * g;
    const bool norm = NORM && T.gn != nullptr;
    if (T.S == 1) {
        if (valid) {
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int bb = 0; bb < S::NBB; ++bb)
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const int b = 8 * bb + 2 * c + q;
                        if (b >= B) continue;
                        const size_t idx = (size_t)b * T.N + row0 + r;
                        float v = acc[0][r][bb][q];
                        float gate = HAS_DUAL ? acc[HAS_DUAL ? 1 : 0][r][bb][q] : 0.0f;
                        if (NORM && norm) {
                            const float nr = norm_scale(T, iss[bb][q]);
                            v *= nr;
                            gate *= nr;
                        }
                        put_y(T, idx, finish(v, dual ? gate : 0.0f, T.op, T.add, idx));
                    }
        }
        return;
    }
    const int planes = dual ? 2 : 1;
    if (NORM && norm && tid < 4) {  // warp 0, lanes g = 0: every batch column once
#pragma unroll
        for (int bb = 0; bb < S::NBB; ++bb)
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int b = 8 * bb + 2 * c + q;
                if (b < B) __stcg(&T.nss[((size_t)rb * T.S + s) * B + b], iss[bb][q]);
            }
    }
    if (valid) {
#pragma unroll
        for (int pl = 0; pl < (HAS_DUAL ? 2 : 1); ++pl) {
            if (pl >= planes) break;
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int bb = 0; bb < S::NBB; ++bb)
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const int b = 8 * bb + 2 * c + q;
                        if (b >= B) continue;
                        __stcg(&T.part[(((size_t)s * planes + pl) * B + b) * T.N + row0 + r], acc[pl][r][bb][q]);
                    }
        }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) sm.last = atomicAdd(&T.ticket[rb], 1u) == (unsigned)(T.S - 1) ? 1u : 0u;
    __syncthreads();
    if (sm.last == 0) return;
    __threadfence();
    if (NORM && norm) {  // every column's scale once, then shared
        if (tid < B) sm.nr[tid] = norm_scale(T, split_sumsq(T, rb, tid, B));
        __syncthreads();
    }
    const int row = rb * Q4_BLOCK_ROWS + tid;  // 128 threads, 128 rows
    if (row < T.N) {
        const size_t split_stride = (size_t)planes * B * T.N;
        for (int b = 0; b < B; ++b) {
            const float *p0 = T.part + (size_t)b * T.N + row;
            float s0 = 0.0f, s1 = 0.0f;
            for (int sp = 0; sp < T.S; ++sp) {
                s0 += __ldcg(p0 + sp * split_stride);
                if (dual) s1 += __ldcg(p0 + sp * split_stride + (size_t)B * T.N);
            }
            if (NORM && norm) {
                s0 *= sm.nr[b];
                s1 *= sm.nr[b];
            }
            const size_t idx = (size_t)b * T.N + row;
            put_y(T, idx, finish(s0, s1, T.op, T.add, idx));
        }
    }
    if (tid == 0) atomicExch(&T.ticket[rb], 0u);
}

// Persistent: CTA-level work items (it = blockIdx.x, += gridDim.x), walked as a
// flat sequence of chunks of 4 tile slots (4 groups, or 2 groups x {up, gate}
// for SwiGLU).  Per chunk: each warp runs its row tile through the chunk's slots
// and refills every slot with the next chunk's tile as soon as it is consumed;
// then the CTA prepares the next chunk's activation fragments (prefetched into
// L1 one chunk earlier) into the other buffer and meets once.
// NORM = false: the launch holds no fused-RMSNorm task, so that path is compiled out.
template <int BP, bool HAS_DUAL, bool NORM>
__global__ void __launch_bounds__(kMbThreads, BP <= 8 ? 4 : 3) q4_gemv_mb_kernel(const __grid_constant__ Launch L) {
    using S = MbShape<BP>;
    __shared__ MbSmem<BP> sm;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, c = lane & 3;
    const long long stride = gridDim.x;
    MbCursor cur;
    mb_item<HAS_DUAL>(L, cur, blockIdx.x);
    if (cur.it >= L.total_items) return;  // uniform across the CTA
    MbTileRegs tr[S::SLOTS];
    {
        const int ns = mb_nslot(cur);
#pragma unroll
        for (int sl = 0; sl < S::SLOTS; ++sl)
            if (sl < ns) mb_load_tile(tr[sl], mb_tile_addr(cur, sl, warp), g, c);
    }
    mb_prep<BP, NORM>(sm, 0, cur, L.B, tid);
    __syncthreads();
    MbCursor nxt = cur;
    mb_advance<HAS_DUAL>(L, nxt, stride);
    if (nxt.it < L.total_items) mb_prefetch_x<BP>(nxt, L.B, tid);
    int par = 0;

    float acc[HAS_DUAL ? 2 : 1][4][S::NBB][2];
    float iss[S::NBB][2];
#pragma unroll
    for (int pl = 0; pl < (HAS_DUAL ? 2 : 1); ++pl)
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int bb = 0; bb < S::NBB; ++bb) acc[pl][r][bb][0] = acc[pl][r][bb][1] = 0.0f;
#pragma unroll
    for (int bb = 0; bb < S::NBB; ++bb) iss[bb][0] = iss[bb][1] = 0.0f;

    while (true) {
        const bool more = nxt.it < L.total_items;
        const int ns = mb_nslot(cur), nns = more ? mb_nslot(nxt) : 0;
#pragma unroll
        for (int sl = 0; sl < S::SLOTS; ++sl) {
            if (sl < ns) {
                const int gi = cur.dual ? (sl >> 1) : sl;
                if (HAS_DUAL && cur.dual && (sl & 1)) {
                    mb_tile<BP>(tr[sl], sm, par, gi, lane, acc[HAS_DUAL ? 1 : 0]);
                } else {
                    mb_tile<BP>(tr[sl], sm, par, gi, lane, acc[0]);
                    if (NORM) {  // fused RMSNorm: groups in ascending order
#pragma unroll
                        for (int bb = 0; bb < S::NBB; ++bb) {
                            iss[bb][0] += sm.ss[par][gi][8 * bb + 2 * c];
                            iss[bb][1] += sm.ss[par][gi][8 * bb + 2 * c + 1];
                        }
                    }
                }
            }
            if (sl < nns) mb_load_tile(tr[sl], mb_tile_addr(nxt, sl, warp), g, c);
        }
        if (mb_last_chunk(cur)) {
            const int tile_row = cur.rb * Q4_BLOCK_TILES + warp;
            const bool valid = tile_row < (cur.T->N >> 5);
            mb_finish<BP, HAS_DUAL, NORM>(*cur.T, cur.rb, cur.s, L.B, acc, iss, cur.dual, valid, tile_row, lane, tid, sm);
#pragma unroll
            for (int pl = 0; pl < (HAS_DUAL ? 2 : 1); ++pl)
#pragma unroll
                for (int r = 0; r < 4; ++r)
#pragma unroll
                    for (int bb = 0; bb < S::NBB; ++bb) acc[pl][r][bb][0] = acc[pl][r][bb][1] = 0.0f;
#pragma unroll
            for (int bb = 0; bb < S::NBB; ++bb) iss[bb][0] = iss[bb][1] = 0.0f;
        }
        if (!more) break;
        mb_prep<BP, NORM>(sm, par ^ 1, nxt, L.B, tid);
        __syncthreads();
        par ^= 1;
        cur = nxt;
        mb_advance<HAS_DUAL>(L, nxt, stride);
        if (nxt.it < L.total_items) mb_prefetch_x<BP>(nxt, L.B, tid);
    }
}
