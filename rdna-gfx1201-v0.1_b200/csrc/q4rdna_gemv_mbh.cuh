// Small-batch tile path on the f16 tensor cores (included into q4rdna_gemv.cu
// inside namespace q4, after q4rdna_gemv_mb.cuh, whose work items, cursor, tile
// addressing and epilogue it shares).  The default for B = 3..16;
// Q4RDNA_TILE=i8 selects the int8 tile path of q4rdna_gemv_mb.cuh.
//
// Why f16 here: the int8 formulation needs three byte MMAs per product and an
// epilogue that recombines the three int32 sums for every (row, batch column,
// group), which dominates at B = 16.  In f16 the codes are exact, and x splits
// into two fp16 halves, x = hi + lo (hi = fp16(x), lo = fp16(x - hi): 22
// significant bits), that share the same A registers.  One f32 accumulator per
// (row, column) then holds sum_k code (hi + lo) for the group, and the
// epilogue is one multiply and one multiply-add.
//
//   * one CTA (4 warps) per work item: 128 rows x a split of the groups; warp w
//     owns row tile 4 rb + w (the int8 tile path's items);
//   * mma.sync m16n8k16 f16 x f16 -> f32.  MMA row g <-> tile row 4g + 2 rs,
//     row g + 8 <-> 4g + 2 rs + 1 (row set rs = 0, 1).  For k-step kk (16
//     columns = pairs 8 kk .. 8 kk + 7) lane (g, c) holds pairs 8 kk + c
//     (k-slots 2c, 2c+1) and 8 kk + c + 4 (k-slots 8 + 2c, 9 + 2c).  One A
//     register is one tile byte (row, pair) = f16x2 (code 2i, code 2i+1), so a
//     lane needs no transposition: its two 32-bit words per k-step (rows
//     4g..4g+3 of the two pairs) give the A registers of both row sets;
//   * byte -> f16x2 in 3 instructions: prmt spreads the byte to bytes 0 and 2,
//     lop3 masks the two nibbles into 1024 + n (low) and 1024 + 16 n (high)
//     with n = code + 8, and one hfma2 maps both to the signed code, exactly;
//   * the activation of a group is scaled per batch column by a power of two
//     so that its largest |x| lies in [2^14, 2^15) (exact), split into hi/lo,
//     and written by the CTA as B fragments into shared memory; the MMAs of
//     the hi and the lo halves chain into the same accumulator;
//   * epilogue per (row, group): acc = fma(scale, D * 2^-e, acc).  The
//     products code * hi and code * lo are exact in f32 (4 + 11 bits); D
//     accumulates them in f32 in the tensor core's order.

template <int BP>
struct MbhShape {
    static constexpr int NBB = BP / 8;            // n-tiles: batch blocks of 8 columns
    static constexpr int PER = 16 * BP;           // prep threads per group: (b, kk, c)
    static constexpr int PASSES = 4 * PER / 128;  // passes of 128 threads per 4-group chunk
};

template <int BP>
struct __align__(16) MbhSmem {
    // [buffer][group][k-step][limb hi/lo][batch block][lane]: b0, b1 (f16x2 each)
    uint2 b[2][4][4][2][MbhShape<BP>::NBB][32];
    float u[2][4][BP];   // 2^-e per (group, batch column)
    float ss[2][4][BP];  // fused RMSNorm: sum of h^2 per (group, batch column)
    float nr[BP];        // fused RMSNorm: scale per batch column (split reduction)
    unsigned last;       // split ticket of this CTA's item
};

// Tile byte j of w (row 4g + j of one column pair) -> f16x2 (low code, high code).
__device__ __forceinline__ uint32_t byte_to_h2(uint32_t w, int j) {
    const uint32_t sel = (uint32_t)j | (4u << 4) | ((uint32_t)j << 8) | (4u << 12);  // [w.j, 0, w.j, 0]
    const uint32_t t = __byte_perm(w, 0u, sel);
    uint32_t r;
    // (t & 0x00F0000F) ^ 0x64806408: 1024 + (lo ^ 8) | (1024 + 16 (hi ^ 8)) << 16
    asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(r) : "r"(t), "r"(0x00F0000Fu), "r"(0x64806408u));
    // (1024 + n) * 1 - 1032 and (1024 + 16 n) / 16 - 72: the signed code, exactly
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(r), "r"(0x2C003C00u), "r"(0xD480E408u));
    return r;
}

template <bool Z>
__device__ __forceinline__ void hmma_mb(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    if (Z)
        asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%10,%10,%10,%10};"
            : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
    else
        asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Code words of one tile for this lane: w[2 kk + half] = rows 4g..4g+3 of pair
// 8 kk + c + 4 half; sc = fp16 scales of rows 4g..4g+3.
__device__ __forceinline__ void mbh_load_tile(MbTileRegs &r, const uint8_t *tile, int g, int c) {
    const uint8_t *q = tile + Q4_SCALE_BYTES + 4 * g + 32 * c;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) r.w[2 * kk + hf] = ld_stream4(q + 32 * (8 * kk + 4 * hf));
    uint2 s;
    asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(s.x), "=r"(s.y) : "l"(tile + 8 * g));
    r.sc = s;
}

__device__ __forceinline__ uint32_t pack_h2(__half lo, __half hi) {
    return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

// Columns 16 kk + 2c + {0, 1} and 16 kk + 2c + 8 + {0, 1} of batch column b of
// group gi (pass `pass` of thread tid), and whether the thread holds live data.
template <int BP>
__device__ __forceinline__ const float *mbh_xcols(const MbCursor &c, int B, int pass, int tid, int &gi, int &b,
                                                  int &kk, int &cc, bool &live) {
    using S = MbhShape<BP>;
    const int idx = pass * 128 + tid;  // over the chunk's 4 groups x PER threads
    gi = idx / S::PER;
    const int r = idx % S::PER;
    b = r >> 4;
    kk = (r >> 2) & 3;
    cc = r & 3;
    live = gi < c.ncg && b < B;
    const Task &T = *c.T;
    return T.x + (size_t)(live ? b : 0) * T.K + (size_t)(c.gbeg + c.base + (live ? gi : 0)) * Q4_GROUP + 16 * kk +
           2 * cc;
}

template <int BP>
__device__ __forceinline__ void mbh_prefetch_x(const MbCursor &c, int B, int tid) {
#pragma unroll
    for (int pass = 0; pass < MbhShape<BP>::PASSES; ++pass) {
        int gi, b, kk, cc;
        bool live;
        const float *xp = mbh_xcols<BP>(c, B, pass, tid, gi, b, kk, cc, live);
        if (live && (kk & 1) == 0 && cc == 0) asm volatile("prefetch.global.L1 [%0];" ::"l"(xp));
    }
}

// The CTA prepares the hi/lo B fragments of chunk c into buffer `par`.  The 16
// threads of one (group, batch column) are 16 consecutive lanes of one warp.
template <int BP, bool NORM>
__device__ __forceinline__ void mbh_prep(MbhSmem<BP> &sm, int par, const MbCursor &c, int B, int tid) {
    using S = MbhShape<BP>;
#pragma unroll
    for (int pass = 0; pass < S::PASSES; ++pass) {
        int gi, b, kk, cc;
        bool live;
        const float *xp = mbh_xcols<BP>(c, B, pass, tid, gi, b, kk, cc, live);
        float2 v0 = live ? __ldg(reinterpret_cast<const float2 *>(xp)) : make_float2(0.0f, 0.0f);
        float2 v1 = live ? __ldg(reinterpret_cast<const float2 *>(xp + 8)) : make_float2(0.0f, 0.0f);
        float ssq = 0.0f;
        if (NORM) {
            // fused RMSNorm: v is the raw input h; prepared as h * g (g = 1 for
            // the launch's tasks without a norm: predicated, no branch)
            const float *gn = c.T->gn;
            const bool nrm = gn != nullptr;
            const float *gp = (nrm ? gn : c.T->x) + (xp - (c.T->x + (size_t)(live ? b : 0) * c.T->K));
            ssq = fmaf(v0.x, v0.x, fmaf(v0.y, v0.y, fmaf(v1.x, v1.x, v1.y * v1.y)));
            const float2 g0 = __ldg(reinterpret_cast<const float2 *>(gp));
            const float2 g1 = __ldg(reinterpret_cast<const float2 *>(gp + 8));
            v0.x *= nrm ? g0.x : 1.0f;
            v0.y *= nrm ? g0.y : 1.0f;
            v1.x *= nrm ? g1.x : 1.0f;
            v1.y *= nrm ? g1.y : 1.0f;
        }
        float m = fmaxf(fmaxf(fabsf(v0.x), fabsf(v0.y)), fmaxf(fabsf(v1.x), fabsf(v1.y)));
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) {
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (NORM) ssq += __shfl_xor_sync(0xffffffffu, ssq, o);
        }
        // max * f in [2^14, 2^15): f = 2^(141 - E), E = biased exponent of the max
        // (E >= 15 keeps f and 1 / f normal; groups below 2^-112 lose bits)
        const uint32_t e = max((__float_as_uint(m) >> 23) & 0xffu, 15u);
        const bool nz = m > 0.0f;
        const float f = nz ? __uint_as_float((268u - e) << 23) : 1.0f;
        const float u = nz ? __uint_as_float((e - 14u) << 23) : 1.0f;
        const float s0 = v0.x * f, s1 = v0.y * f, s8 = v1.x * f, s9 = v1.y * f;
        const __half h0 = __float2half_rn(s0), h1 = __float2half_rn(s1);
        const __half h8 = __float2half_rn(s8), h9 = __float2half_rn(s9);
        const __half l0 = __float2half_rn(s0 - __half2float(h0)), l1 = __float2half_rn(s1 - __half2float(h1));
        const __half l8 = __float2half_rn(s8 - __half2float(h8)), l9 = __float2half_rn(s9 - __half2float(h9));
        if (gi < c.ncg) {
            const int lane = (b & 7) * 4 + cc, bb = b >> 3;
            sm.b[par][gi][kk][0][bb][lane] = make_uint2(pack_h2(h0, h1), pack_h2(h8, h9));
            sm.b[par][gi][kk][1][bb][lane] = make_uint2(pack_h2(l0, l1), pack_h2(l8, l9));
            if (kk == 0 && cc == 0) {
                sm.u[par][gi][b] = u;
                if (NORM) sm.ss[par][gi][b] = ssq;
            }
        }
    }
}

// One tile (one group of one tensor) for this warp: 4 k-steps x {hi, lo} f16
// MMAs per (row set, batch block), chained into one f32 accumulator, then
// acc[2 rs + e][bb][q] = fma(scale, D * 2^-e, acc) per (row, column).
template <int BP>
__device__ __forceinline__ void mbh_tile(const MbTileRegs &r, const MbhSmem<BP> &sm, int par, int gi, int lane,
                                         float (&acc)[4][BP / 8][2]) {
    using S = MbhShape<BP>;
    float D[2][S::NBB][4];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
        const uint32_t w0 = r.w[2 * kk], w1 = r.w[2 * kk + 1];
        uint32_t A[2][4];
#pragma unroll
        for (int rs = 0; rs < 2; ++rs) {
            A[rs][0] = byte_to_h2(w0, 2 * rs);      // MMA row g, pair 8 kk + c
            A[rs][1] = byte_to_h2(w0, 2 * rs + 1);  // MMA row g + 8
            A[rs][2] = byte_to_h2(w1, 2 * rs);      // MMA row g, pair 8 kk + c + 4
            A[rs][3] = byte_to_h2(w1, 2 * rs + 1);
        }
#pragma unroll
        for (int limb = 0; limb < 2; ++limb)
#pragma unroll
            for (int bb = 0; bb < S::NBB; ++bb) {
                const uint2 bf = sm.b[par][gi][kk][limb][bb][lane];
#pragma unroll
                for (int rs = 0; rs < 2; ++rs) {
                    if (kk == 0 && limb == 0)
                        hmma_mb<true>(D[rs][bb], A[rs][0], A[rs][1], A[rs][2], A[rs][3], bf.x, bf.y);
                    else
                        hmma_mb<false>(D[rs][bb], A[rs][0], A[rs][1], A[rs][2], A[rs][3], bf.x, bf.y);
                }
            }
    }
    const int c = lane & 3;
    float s[4];
    s[0] = __half2float(__ushort_as_half((unsigned short)(r.sc.x & 0xffffu)));
    s[1] = __half2float(__ushort_as_half((unsigned short)(r.sc.x >> 16)));
    s[2] = __half2float(__ushort_as_half((unsigned short)(r.sc.y & 0xffffu)));
    s[3] = __half2float(__ushort_as_half((unsigned short)(r.sc.y >> 16)));
#pragma unroll
    for (int bb = 0; bb < S::NBB; ++bb) {
        const float2 uq = *reinterpret_cast<const float2 *>(&sm.u[par][gi][8 * bb + 2 * c]);
#pragma unroll
        for (int rs = 0; rs < 2; ++rs)
#pragma unroll
            for (int e = 0; e < 2; ++e)
#pragma unroll
                for (int q = 0; q < 2; ++q)
                    acc[2 * rs + e][bb][q] =
                        fmaf(s[2 * rs + e], D[rs][bb][2 * e + q] * (q ? uq.y : uq.x), acc[2 * rs + e][bb][q]);
    }
}

// Persistent: CTA-level work items walked as chunks of 4 tile slots, as in
// q4_gemv_mb_kernel; each slot is refilled with the next chunk's tile as soon
// as it is consumed, and the CTA prepares the next chunk's fragments into the
// other buffer and meets once per chunk.
template <int BP, bool HAS_DUAL, bool NORM>
__global__ void __launch_bounds__(kMbThreads, BP <= 8 ? 4 : 3) q4_gemv_mbh_kernel(const __grid_constant__ Launch L) {
    using S = MbhShape<BP>;
    __shared__ MbhSmem<BP> sm;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, c = lane & 3;
    const long long stride = gridDim.x;
    MbCursor cur;
    mb_item<HAS_DUAL>(L, cur, blockIdx.x);
    if (cur.it >= L.total_items) return;  // uniform across the CTA
    MbTileRegs tr[4];
    {
        const int ns = mb_nslot(cur);
#pragma unroll
        for (int sl = 0; sl < 4; ++sl)
            if (sl < ns) mbh_load_tile(tr[sl], mb_tile_addr(cur, sl, warp), g, c);
    }
    mbh_prep<BP, NORM>(sm, 0, cur, L.B, tid);
    __syncthreads();
    MbCursor nxt = cur;
    mb_advance<HAS_DUAL>(L, nxt, stride);
    if (nxt.it < L.total_items) mbh_prefetch_x<BP>(nxt, L.B, tid);
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
        for (int sl = 0; sl < 4; ++sl) {
            if (sl < ns) {
                const int gi = cur.dual ? (sl >> 1) : sl;
                if (HAS_DUAL && cur.dual && (sl & 1)) {
                    mbh_tile<BP>(tr[sl], sm, par, gi, lane, acc[HAS_DUAL ? 1 : 0]);
                } else {
                    mbh_tile<BP>(tr[sl], sm, par, gi, lane, acc[0]);
                    if (NORM) {  // fused RMSNorm: groups in ascending order
#pragma unroll
                        for (int bb = 0; bb < S::NBB; ++bb) {
                            iss[bb][0] += sm.ss[par][gi][8 * bb + 2 * c];
                            iss[bb][1] += sm.ss[par][gi][8 * bb + 2 * c + 1];
                        }
                    }
                }
            }
            if (sl < nns) mbh_load_tile(tr[sl], mb_tile_addr(nxt, sl, warp), g, c);
        }
        if (mb_last_chunk(cur)) {
            const int tile_row = cur.rb * Q4_BLOCK_TILES + warp;
            const bool valid = tile_row < (cur.T->N >> 5);
            mb_finish<BP, HAS_DUAL, NORM>(*cur.T, cur.rb, cur.s, L.B, acc, iss, cur.dual, valid, tile_row, lane, tid,
                                          sm);
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
        mbh_prep<BP, NORM>(sm, par ^ 1, nxt, L.B, tid);
        __syncthreads();
        par ^= 1;
        cur = nxt;
        mb_advance<HAS_DUAL>(L, nxt, stride);
        if (nxt.it < L.total_items) mbh_prefetch_x<BP>(nxt, L.B, tid);
    }
}
