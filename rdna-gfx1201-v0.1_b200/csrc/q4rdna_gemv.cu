// Q4_RDNA group-64 GEMV for B200 (sm_100a).
//
// One warp work item = one 128-row block (four 32-row tiles) x one K-range of
// `Gs` groups, for one tensor (two for the fused SwiGLU).  The warp streams its
// tiles straight from HBM with 128-bit loads, unpacks the int4 codes to fp16 in
// registers and lets the tensor cores (mma.sync m16n8k16, f32 accumulate) do
// the dot products against the activation, which is carried as an exact
// fp16 hi + lo pair per element.  The fp16 group scale is applied once per
// (row, group) in f32, as the reference does (source/q4rdna.cu:370-371).
// Split-K partial sums go to a workspace; the last warp to finish a row block
// (arrival ticket) adds them in split order and applies the add / SwiGLU
// epilogue, so results are deterministic.
//
// Why tensor cores at batch 1: at 6.5 TB/s the stream is ~12e12 weights/s,
// which leaves ~3 issue slots per weight on the CUDA cores.  Unpack + convert +
// FFMA per weight does not fit; here the per-weight cost is ~1.1 integer/half
// instructions plus 1/8 of an MMA issue.
//
// Register-fragment mapping (m16n8k16, A row-major, B col-major):
//   lane L: grp = L>>2 (0..7), c = L&3; tile t = grp>>1, half h = grp&1.
//   For MMA step m (0..7) the lane's 16-byte load is tile t, code bytes
//   64 + 128m + 32c + 16h: rows 16h..16h+15 of column pair i = 4m + c.
//   Its j-th 32-bit word (j = 0..3) holds rows rho = 16h + 4j + {0,1,2,3} and
//   feeds MMA j.  Nibbles are expanded with the fp16 magic-number trick:
//     P0 = (b0.lo, b2.lo), P1 = (b0.hi, b2.hi), P2 = (b1.lo, b3.lo), P3 = (b1.hi, b3.hi)
//   and used as A registers a0a1 = P0, a2a3 = P2, a4a5 = P1, a6a7 = P3.  So MMA
//   row grp carries weight rows rho+0 (even k-slots) and rho+2 (odd k-slots),
//   MMA row grp+8 carries rho+1 / rho+3.  The B operand separates the two
//   slots into different columns: column n = 4*bb + role, role 0/1 = slot 0
//   (x_hi / x_lo), role 2/3 = slot 1 (x_hi / x_lo), bb = batch within the
//   MMA's batch pair.  D column pairs (2c, 2c+1) therefore hold hi and lo for
//   rows rho + 2(c&1) (+1 for the grp+8 half) of batch 2*nb + (c>>1).
// Accumulation order of an output: inside a group the tensor core sums exact
// products (int4 x fp16) in f32; groups of one split are added in ascending
// order, each as sum = fma(scale * 2^e, hi + lo, sum); splits are then added
// in ascending split order in f32.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <vector>

#include "q4rdna.h"
#include "q4rdna_q4k.h"
#include "q4rdna_tile.h"

namespace q4 {

constexpr int kWarps = 8;             // warps per CTA
constexpr int kThreads = kWarps * 32;

constexpr int kMaxMirrors = 8;  // GPUs of one box

struct Task {
    const uint8_t *w;   // primary tiles (W, or W_up for SwiGLU)
    const uint8_t *w2;  // W_gate for SwiGLU, else null
    const float *x;     // [B][K]
    const float *add;   // [B][N] for OP_ADD, else null
    float *y;           // [B][N]
    float *part;        // [S][planes][B][N] split partials (S > 1)
    unsigned *ticket;   // [RB] arrival counters (S > 1)
    int N, K, G, RB, S, Gs, op;
    int nmirror;        // tensor-parallel gather: copies of y in every rank's gathered buffer
    long long item_begin;
    const float *gn;    // fused RMSNorm: the norm weight [K] (x is then the raw input h), else null
    float eps;          // fused RMSNorm: y = W (h * g) / sqrt(mean(h^2) + eps)
    int pad2;
    float *nss;         // fused RMSNorm with S > 1: sums of h^2 per [RB][S][B]
    float *mirror[kMaxMirrors];  // [B][N] each, on this GPU or a peer (plain P2P stores)
};

struct Launch {
    const Task *table;  // device array of ntasks tasks, or null: use `one`
    Task one;
    int ntasks;
    int B;
    long long total_items;
};

// ---------------------------------------------------------------- device helpers

__device__ __forceinline__ uint4 ld_stream16(const uint8_t *p) {
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t ld_stream4(const uint8_t *p) {
    uint32_t v;
    asm("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// (1024 + (n ^ 8)) - 1032 = signed code, exact in fp16.
__device__ __forceinline__ uint32_t unbias_lo(uint32_t p) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(p), "r"(0x64086408u));
    return r;
}
// (1024 + 16 (n ^ 8)) / 16 - 72 = signed code, exact in fp16.
__device__ __forceinline__ uint32_t unbias_hi(uint32_t p) {
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(p), "r"(0x2C002C00u), "r"(0xD480D480u));
    return r;
}

// One 32-bit code word (4 rows x 1 column pair) -> the four A registers.
__device__ __forceinline__ void word_to_a(uint32_t w, uint32_t &a0, uint32_t &a1, uint32_t &a2,
                                          uint32_t &a3) {
    const uint32_t w8 = w >> 8;
    a0 = unbias_lo((w & 0x000F000Fu) ^ 0x64086408u);   // (b0.lo, b2.lo)
    a1 = unbias_lo((w8 & 0x000F000Fu) ^ 0x64086408u);  // (b1.lo, b3.lo)
    a2 = unbias_hi((w & 0x00F000F0u) ^ 0x64806480u);   // (b0.hi, b2.hi)
    a3 = unbias_hi((w8 & 0x00F000F0u) ^ 0x64806480u);  // (b1.hi, b3.hi)
}

__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Per-warp shared scratch: one group of the activation as (x_hi | x_lo << 16)
// per element for each batch column of the pass, and the power of two that
// undoes the group's normalisation.
template <int NB>
struct __align__(16) WarpSmem {
    uint32_t xq[2 * NB][Q4_GROUP];
    float up[2 * NB];
};

// Normalise one 64-element group of x by a power of two so that its largest
// magnitude lands in [2^14, 2^15) (exact), then split every element into
// x_hi = fp16(x) and x_lo = fp16(x - x_hi); x_hi + x_lo keeps ~22 significant
// bits and the fp16 range can no longer overflow or underflow the group.
__device__ __forceinline__ void prep_group(float2 v, uint32_t *xq_row, float *up, int lane) {
    const float m = warp_max(fmaxf(fabsf(v.x), fabsf(v.y)));
    float f = 1.0f, u = 1.0f;
    if (m > 0.0f) {
        const uint32_t e = max((__float_as_uint(m) >> 23) & 0xffu, 15u);
        f = __uint_as_float((268u - e) << 23);  // 2^(141 - e)
        u = __uint_as_float((e - 14u) << 23);   // 2^(e - 141)
    }
    const float s0 = v.x * f, s1 = v.y * f;
    const __half2 hi = __floats2half2_rn(s0, s1);
    const float2 hf = __half22float2(hi);
    const __half2 lo = __floats2half2_rn(s0 - hf.x, s1 - hf.y);
    const uint32_t hb = *reinterpret_cast<const uint32_t *>(&hi);
    const uint32_t lb = *reinterpret_cast<const uint32_t *>(&lo);
    uint2 q;
    q.x = __byte_perm(hb, lb, 0x5410);  // element 2*lane:   hi | lo << 16
    q.y = __byte_perm(hb, lb, 0x7632);  // element 2*lane+1
    reinterpret_cast<uint2 *>(xq_row)[lane] = q;
    if (lane == 0) *up = u;
}

// Code words and scale words of one (tensor, group) step for this lane.
struct StepBuf {
    uint4 q[8];     // MMA step m: 16 code bytes
    uint32_t s[4];  // fp16 scale pair of the lane's two rows for MMA j
};

__device__ __forceinline__ void load_step(StepBuf &b, const uint8_t *tile, bool valid, int c, int h) {
    if (valid) {
        const uint8_t *qp = tile + Q4_SCALE_BYTES + 32 * c + 16 * h;
#pragma unroll
        for (int m = 0; m < 8; ++m) b.q[m] = ld_stream16(qp + 128 * m);
        const uint8_t *sp = tile + 32 * h + 4 * (c & 1);
#pragma unroll
        for (int j = 0; j < 4; ++j) b.s[j] = ld_stream4(sp + 8 * j);
    } else {
#pragma unroll
        for (int m = 0; m < 8; ++m) b.q[m] = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int j = 0; j < 4; ++j) b.s[j] = 0u;
    }
}

__device__ __forceinline__ uint32_t word_of(const uint4 &v, int j) {
    return j == 0 ? v.x : (j == 1 ? v.y : (j == 2 ? v.z : v.w));
}

// One group of one tensor: 32 MMAs per warp (4 row slices x 8 k-steps x NB
// batch pairs), then the per-(row, group) scale in f32.  While slot m of `buf`
// is consumed it is refilled with slot m of the next step (`next`, when
// non-null), so one step of loads stays in flight with one buffer of registers.
template <int NB>
__device__ __forceinline__ void compute_step(StepBuf &buf, const uint8_t *next, bool valid, int c, int h,
                                             const WarpSmem<NB> &sm, float (&acc)[4][NB][2], int lane,
                                             const uint32_t (&sel)[NB], const int (&xrow)[NB],
                                             const int (&urow)[NB]) {
    float D[4][NB][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int nb = 0; nb < NB; ++nb)
#pragma unroll
            for (int r = 0; r < 4; ++r) D[j][nb][r] = 0.0f;
    uint32_t sw[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) sw[j] = buf.s[j];
    const bool refill = next != nullptr && valid;
    const uint8_t *nq = next + Q4_SCALE_BYTES + 32 * c + 16 * h;
    if (refill) {
        const uint8_t *sp = next + 32 * h + 4 * (c & 1);
#pragma unroll
        for (int j = 0; j < 4; ++j) buf.s[j] = ld_stream4(sp + 8 * j);
    }
    const int c4 = lane & 3;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        const uint4 cur = buf.q[m];
        if (refill) buf.q[m] = ld_stream16(nq + 128 * m);
        uint32_t b0[NB], b1[NB];
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
            const uint2 p = *reinterpret_cast<const uint2 *>(&sm.xq[xrow[nb]][8 * m + 2 * c4]);
            b0[nb] = __byte_perm(p.x, 0u, sel[nb]);
            b1[nb] = __byte_perm(p.y, 0u, sel[nb]);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t a0, a1, a2, a3;
            word_to_a(word_of(cur, j), a0, a1, a2, a3);
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) mma16816(D[j][nb], a0, a1, a2, a3, b0[nb], b1[nb]);
        }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float2 sc = __half22float2(*reinterpret_cast<const __half2 *>(&sw[j]));
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
            const float u = sm.up[urow[nb]];
            acc[j][nb][0] = fmaf(sc.x * u, D[j][nb][0] + D[j][nb][1], acc[j][nb][0]);
            acc[j][nb][1] = fmaf(sc.y * u, D[j][nb][2] + D[j][nb][3], acc[j][nb][1]);
        }
    }
}

// Final store of one output: y, and its copies in the ranks' gathered buffers
// when the launch gathers over peers (the fused all-gather).
__device__ __forceinline__ void put_y(const Task &T, size_t idx, float v) {
    T.y[idx] = v;
    for (int p = 0; p < T.nmirror; ++p) T.mirror[p][idx] = v;
}

__device__ __forceinline__ float finish(float v, float gate, int op, const float *add, size_t idx) {
    if (op == Q4RDNA_OP_ADD) v += add[idx];
    if (op == Q4RDNA_OP_SWIGLU) v *= silu(gate);
    return v;
}

// Fused RMSNorm: the output scale 1 / sqrt(mean(h^2) + eps) from the sum of h^2
// over all K columns (ggml_rms_norm's definition).
__device__ __forceinline__ float norm_scale(const Task &T, float sumsq) {
    return 1.0f / sqrtf(sumsq / (float)T.K + T.eps);
}

// Fused RMSNorm, S > 1: the sum of h^2 of batch column b over the row block's
// splits, in ascending split order.
__device__ __forceinline__ float split_sumsq(const Task &T, int rb, int b, int B) {
    float s = 0.0f;
    for (int sp = 0; sp < T.S; ++sp) s += __ldcg(&T.nss[((size_t)rb * T.S + sp) * B + b]);
    return s;
}

// Last warp to arrive at row block rb: add the split partials in ascending
// split order, apply the epilogue, store y, and leave the ticket at zero.
template <bool DUAL, bool NORM = false>
__device__ __forceinline__ void reduce_splits(const Task &T, int rb, int B, int lane) {
    constexpr int planes = DUAL ? 2 : 1;
    __threadfence();
    // fused RMSNorm: lane b computes batch column b's scale once (B <= 16)
    float nr_lane = 1.0f;
    if (NORM && T.gn != nullptr && lane < B) nr_lane = norm_scale(T, split_sumsq(T, rb, lane, B));
    for (int q4r = 0; q4r < Q4_BLOCK_TILES; ++q4r) {
        const int row = rb * Q4_BLOCK_ROWS + 32 * q4r + lane;
        if (row >= T.N) break;
        for (int b = 0; b < B; ++b) {
            float s0 = 0.0f, s1 = 0.0f;
            const float *p0 = T.part + (size_t)b * T.N + row;
            const size_t split_stride = (size_t)planes * B * T.N;
#pragma unroll 8
            for (int sp = 0; sp < T.S; ++sp) {
                s0 += __ldcg(p0 + sp * split_stride);
                if (DUAL) s1 += __ldcg(p0 + sp * split_stride + (size_t)B * T.N);
            }
            if (NORM && T.gn != nullptr) {
                const float r = __shfl_sync(0xffffffffu, nr_lane, b);
                s0 *= r;
                s1 *= r;
            }
            const size_t idx = (size_t)b * T.N + row;
            put_y(T, idx, finish(s0, s1, T.op, T.add, idx));
        }
    }
    if (lane == 0) atomicExch(&T.ticket[rb], 0u);
}

// Epilogue of one work item: store (S == 1), or write the split partials and,
// in the last warp to arrive at the row block, add the splits in ascending
// order and apply the add / SwiGLU epilogue.
template <int NB, bool DUAL>
__device__ __forceinline__ void finish_item(const Task &T, int rb, int s, int B,
                                            float (&acc)[DUAL ? 2 : 1][4][NB][2], int lane, bool valid,
                                            int tile_row, int h, int c) {
    // Rows of this lane: tile t, rows 16h + 4j + 2(c&1) + e; batch 2nb + (c>>1).
    const int row0 = tile_row * Q4_TILE_ROWS + 16 * h + 2 * (c & 1);
    if (T.S == 1) {
        if (valid) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int nb = 0; nb < NB; ++nb) {
                    const int b = 2 * nb + (c >> 1);
                    if (b >= B) continue;
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const size_t idx = (size_t)b * T.N + row0 + 4 * j + e;
                        put_y(T, idx, finish(acc[0][j][nb][e], acc[DUAL ? 1 : 0][j][nb][e], T.op, T.add, idx));
                    }
                }
        }
        return;
    }

    constexpr int planes = DUAL ? 2 : 1;
    if (valid) {
#pragma unroll
        for (int q = 0; q < planes; ++q)
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int nb = 0; nb < NB; ++nb) {
                    const int b = 2 * nb + (c >> 1);
                    if (b >= B) continue;
#pragma unroll
                    for (int e = 0; e < 2; ++e)
                        __stcg(&T.part[(((size_t)s * planes + q) * B + b) * T.N + row0 + 4 * j + e], acc[q][j][nb][e]);
                }
    }
    __threadfence();
    __syncwarp();
    unsigned prev = 0;
    if (lane == 0) prev = atomicAdd(&T.ticket[rb], 1u);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev != (unsigned)(T.S - 1)) return;

    reduce_splits<DUAL>(T, rb, B, lane);
}

// One work item: row block rb, split s of task T; NB batch pairs (B <= 2*NB).
template <int NB, bool DUAL>
__device__ __forceinline__ void run_item(const Task &T, long long local, int B, WarpSmem<NB> &sm, int lane) {
    const int rb = (int)(local / T.S), s = (int)(local % T.S);
    const int g0 = s * T.Gs, ng = min(T.Gs, T.G - g0);
    const int grp = lane >> 2, c = lane & 3, t = grp >> 1, h = grp & 1;
    const int tile_row = rb * Q4_BLOCK_TILES + t;
    const bool valid = tile_row < (T.N >> 5);
    const size_t tile0 = ((size_t)tile_row * T.G + g0) * Q4_TILE_BYTES;
    const uint8_t *base0 = T.w + (valid ? tile0 : 0);
    const uint8_t *base1 = DUAL ? T.w2 + (valid ? tile0 : 0) : nullptr;

    // B operand selectors: lane's column is n = lane>>2 -> batch 2nb + (lane>>4), role (lane>>2)&3.
    uint32_t sel[NB];
    int xrow[NB], urow[NB];
    {
        const int role = (lane >> 2) & 3;
        const uint32_t role_sel = role == 0 ? 0x4410u : role == 1 ? 0x4432u : role == 2 ? 0x1044u : 0x3244u;
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
            const int bx = 2 * nb + (lane >> 4);
            sel[nb] = bx < B ? role_sel : 0x4444u;
            xrow[nb] = min(bx, B - 1);
            urow[nb] = min(2 * nb + (c >> 1), B - 1);
        }
    }

    float acc[DUAL ? 2 : 1][4][NB][2];
#pragma unroll
    for (int q = 0; q < (DUAL ? 2 : 1); ++q)
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) acc[q][j][nb][0] = acc[q][j][nb][1] = 0.0f;

    // Activation of the first group; later groups are fetched one group ahead.
    float2 xv[2 * NB];
#pragma unroll
    for (int b = 0; b < 2 * NB; ++b)
        xv[b] = b < B ? __ldg(reinterpret_cast<const float2 *>(T.x + (size_t)b * T.K + (size_t)g0 * Q4_GROUP) + lane)
                      : make_float2(0.0f, 0.0f);

    const int nsteps = ng * (DUAL ? 2 : 1);
    auto step_tile = [&](int st) -> const uint8_t * {
        const int tt = DUAL ? (st & 1) : 0, gl = DUAL ? (st >> 1) : st;
        return (tt ? base1 : base0) + (size_t)gl * Q4_TILE_BYTES;
    };
    StepBuf buf;
    load_step(buf, step_tile(0), valid, c, h);
    for (int st = 0; st < nsteps; ++st) {
        const int tt = DUAL ? (st & 1) : 0, gl = DUAL ? (st >> 1) : st;
        if (tt == 0) {
            __syncwarp();
#pragma unroll
            for (int b = 0; b < 2 * NB; ++b)
                if (b < B) prep_group(xv[b], sm.xq[b], &sm.up[b], lane);
            if (gl + 1 < ng) {
#pragma unroll
                for (int b = 0; b < 2 * NB; ++b)
                    if (b < B)
                        xv[b] = __ldg(reinterpret_cast<const float2 *>(T.x + (size_t)b * T.K +
                                                                       (size_t)(g0 + gl + 1) * Q4_GROUP) + lane);
            }
            __syncwarp();
        }
        const uint8_t *next = st + 1 < nsteps ? step_tile(st + 1) : nullptr;
        if (DUAL && tt == 1)
            compute_step<NB>(buf, next, valid, c, h, sm, acc[DUAL ? 1 : 0], lane, sel, xrow, urow);
        else
            compute_step<NB>(buf, next, valid, c, h, sm, acc[0], lane, sel, xrow, urow);
    }

    finish_item<NB, DUAL>(T, rb, s, B, acc, lane, valid, tile_row, h, c);
}

__device__ __forceinline__ const Task &find_task(const Launch &L, long long item) {
    if (L.table == nullptr) return L.one;
    int lo = 0, hi = L.ntasks - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (L.table[mid].item_begin <= item) lo = mid; else hi = mid - 1;
    }
    return L.table[lo];
}

// Persistent over work items: warp w of the grid takes items w, w + nwarps, ...
template <int NB>
__global__ void __launch_bounds__(kThreads, NB == 1 ? 2 : 1) q4_gemv_kernel(const __grid_constant__ Launch L) {
    __shared__ WarpSmem<NB> smem[kWarps];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long nw = (long long)gridDim.x * kWarps;
    for (long long it = (long long)blockIdx.x * kWarps + warp; it < L.total_items; it += nw) {
        const Task &T = find_task(L, it);
        if (T.op == Q4RDNA_OP_SWIGLU)
            run_item<NB, true>(T, it - T.item_begin, L.B, smem[warp], lane);
        else
            run_item<NB, false>(T, it - T.item_begin, L.B, smem[warp], lane);
    }
}

// Debug dequantisation: one thread per (row, group) writes 64 exact values.
__global__ void q4_dequant_kernel(const uint8_t *tiles, float *W, int N, int K) {
    const long long G = K / Q4_GROUP;
    const long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (id >= (long long)N * G) return;
    const long long row = id / G, g = id % G;
    const uint8_t *t = tiles + ((row / Q4_TILE_ROWS) * G + g) * Q4_TILE_BYTES;
    const int lane = (int)(row % Q4_TILE_ROWS);
    const float s = __half2float(*reinterpret_cast<const __half *>(t + 2 * lane));
    float *o = W + row * K + g * Q4_GROUP;
    for (int i = 0; i < Q4_GROUP / 2; ++i) {
        const uint8_t p = t[Q4_SCALE_BYTES + i * Q4_TILE_ROWS + lane];
        o[2 * i] = s * (float)((int)(int8_t)(uint8_t)(p << 4) >> 4);
        o[2 * i + 1] = s * (float)((int)(int8_t)p >> 4);
    }
}

#include "q4rdna_gemv_tma.cuh"
#include "q4rdna_gemv_i8.cuh"
#include "q4rdna_gemv_i8_tma.cuh"
#include "q4rdna_gemv_mb.cuh"
#include "q4rdna_gemv_mbh.cuh"

// ------------------------------------------------------------------ host side

constexpr int kMaxDevices = 64;
constexpr int kMaxPassBatch = 4;  // batch columns the batch-1 kernels can take (BB <= 4)
std::atomic<uint64_t> g_launches{0};

// Kernel variants: the int8 tensor-core kernel with register loads (default,
// fastest measured), the same math fed by a TMA ring, or the fp16 tensor-core
// kernel.  Q4RDNA_KERNEL=i8|i8tma|ldg selects one for A/B measurements.
enum Variant { kI8 = 0, kI8Tma, kLdg, kVariants };
constexpr int kDefaultVariant = kI8;

int variant() {
    static const int v = [] {
        const char *e = std::getenv("Q4RDNA_KERNEL");
        if (e == nullptr || *e == '\0') return kDefaultVariant;
        const char *names[kVariants] = {"i8", "i8tma", "ldg"};
        for (int i = 0; i < kVariants; ++i)
            if (std::strcmp(e, names[i]) == 0) return i;
        return kDefaultVariant;
    }();
    return v;
}

struct KernelCfg {
    const void *fn;
    int threads, smem, warps;
};

// Batch class of a launch: 0 -> 1 column, 1 -> 2, 2 -> 3..4, 3 -> 5..8, 4 -> 9..16.
constexpr int kBatchClasses = 5;
int batch_class(int pb) { return pb <= 1 ? 0 : pb == 2 ? 1 : pb <= 4 ? 2 : pb <= 8 ? 3 : 4; }
int class_batch(int bc) { return bc == 0 ? 1 : bc == 1 ? 2 : bc == 2 ? 4 : bc == 3 ? 8 : 16; }

// Tile path for B >= tile_min_batch(): one work item per CTA.  The int8
// kernel (q4rdna_gemv_mb.cuh) by default; Q4RDNA_TILE=f16 selects the f16 one
// (q4rdna_gemv_mbh.cuh), kept for A/B measurements: on the Qwen3-8B step it
// took 1695 / 1729 / 3441 us at B = 4 / 8 / 16 against 1249 / 1281 / 2373 us
// for the int8 kernel (long-scoreboard bound at 142 registers, 3 CTAs/SM).
bool tile_i8() {
    static const bool v = [] {
        const char *e = std::getenv("Q4RDNA_TILE");
        return e == nullptr || std::strcmp(e, "f16") != 0;
    }();
    return v;
}

template <bool NORM>
KernelCfg mb_cfg_n(int pb, bool dual) {
    if (tile_i8()) {
        if (pb <= 8)
            return dual ? KernelCfg{(const void *)q4_gemv_mb_kernel<8, true, NORM>, kMbThreads, 0, 1}
                        : KernelCfg{(const void *)q4_gemv_mb_kernel<8, false, NORM>, kMbThreads, 0, 1};
        return dual ? KernelCfg{(const void *)q4_gemv_mb_kernel<16, true, NORM>, kMbThreads, 0, 1}
                    : KernelCfg{(const void *)q4_gemv_mb_kernel<16, false, NORM>, kMbThreads, 0, 1};
    }
    if (pb <= 8)
        return dual ? KernelCfg{(const void *)q4_gemv_mbh_kernel<8, true, NORM>, kMbThreads, 0, 1}
                    : KernelCfg{(const void *)q4_gemv_mbh_kernel<8, false, NORM>, kMbThreads, 0, 1};
    return dual ? KernelCfg{(const void *)q4_gemv_mbh_kernel<16, true, NORM>, kMbThreads, 0, 1}
                : KernelCfg{(const void *)q4_gemv_mbh_kernel<16, false, NORM>, kMbThreads, 0, 1};
}
KernelCfg mb_cfg(int pb, bool dual, bool norm) { return norm ? mb_cfg_n<true>(pb, dual) : mb_cfg_n<false>(pb, dual); }

template <bool DUAL>
KernelCfg i8_cfg(int pb, bool norm) {
    if (norm) {
        if (pb <= 1) return KernelCfg{(const void *)q4_gemv_i8_kernel<1, DUAL, true>, kThreads, 0, kWarps};
        if (pb == 2) return KernelCfg{(const void *)q4_gemv_i8_kernel<2, DUAL, true>, kThreads, 0, kWarps};
        return KernelCfg{(const void *)q4_gemv_i8_kernel<4, DUAL, true>, kThreads, 0, kWarps};
    }
    if (pb <= 1) return KernelCfg{(const void *)q4_gemv_i8_kernel<1, DUAL, false>, kThreads, 0, kWarps};
    if (pb == 2) return KernelCfg{(const void *)q4_gemv_i8_kernel<2, DUAL, false>, kThreads, 0, kWarps};
    return KernelCfg{(const void *)q4_gemv_i8_kernel<4, DUAL, false>, kThreads, 0, kWarps};
}

KernelCfg i8tma_cfg(int pb) {
    using R = I8Ring;
    if (pb <= 1) return KernelCfg{(const void *)q4_gemv_i8_tma_kernel<1, R>, R::THREADS, R::SMEM_BYTES, R::WARPS};
    if (pb == 2) return KernelCfg{(const void *)q4_gemv_i8_tma_kernel<2, R>, R::THREADS, R::SMEM_BYTES, R::WARPS};
    return KernelCfg{(const void *)q4_gemv_i8_tma_kernel<4, R>, R::THREADS, R::SMEM_BYTES, R::WARPS};
}

// dual: the launch holds a SwiGLU task (kernels without the SwiGLU path need fewer registers).
// Smallest batch that runs on the tile path.  Default 3: measured on the
// Qwen3-8B step, the tile path takes B = 3..4 at a third of the batch-1 int8
// kernel's time and ties it at B = 2.  Q4RDNA_TILE_MIN_BATCH (1, 2, 3 or 5)
// overrides it for A/B measurements.
int tile_min_batch() {
    static const int v = [] {
        const char *e = std::getenv("Q4RDNA_TILE_MIN_BATCH");
        const int t = (e != nullptr && *e != '\0') ? std::atoi(e) : 3;
        return std::max(1, std::min(t, kMaxPassBatch + 1));
    }();
    return v;
}

// norm: the launch holds a fused-RMSNorm task (occupancy and grids are taken
// from the kernels without it; the norm kernels use the same registers +- 5).
KernelCfg kernel_cfg(int v, int pb, bool dual = true, bool norm = false) {
    if (pb >= tile_min_batch()) return mb_cfg(pb, dual, norm);
    switch (v) {
        case kI8Tma: return i8tma_cfg(pb);
        case kLdg:
            return pb <= 2 ? KernelCfg{(const void *)q4_gemv_kernel<1>, kThreads, 0, kWarps}
                           : KernelCfg{(const void *)q4_gemv_kernel<2>, kThreads, 0, kWarps};
        default: return dual ? i8_cfg<true>(pb, norm) : i8_cfg<false>(pb, norm);
    }
}

struct DeviceInfo {
    int sms = 0;
    int occ[kVariants][kBatchClasses][2] = {};  // resident CTAs per SM: variant, batch class, SwiGLU (0: unknown)
};
std::mutex g_dev_mutex;
DeviceInfo g_dev[kMaxDevices];

bool device_info(DeviceInfo &out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return false;
    std::lock_guard<std::mutex> lock(g_dev_mutex);
    DeviceInfo &d = g_dev[dev];
    if (d.sms == 0) {
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return false;
        d.sms = sms;
    }
    const int v = variant();
    for (int bc = 0; bc < kBatchClasses; ++bc)
        for (int du = 0; du < 2; ++du) {
            if (d.occ[v][bc][du] != 0) continue;
            const KernelCfg k = kernel_cfg(v, class_batch(bc), du != 0);
            if (k.smem > 48 * 1024 &&
                cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, k.smem) != cudaSuccess)
                return false;
            int o = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, k.fn, k.threads, k.smem) != cudaSuccess)
                return false;
            d.occ[v][bc][du] = std::max(o, 1);
        }
    out = d;
    return true;
}

int env_split() {
    // LLAMA_Q4_RDNA_COOP was the reference's split-K width (q4rdna.cu:578-589);
    // here it forces the split-K factor.
    const char *v = std::getenv("LLAMA_Q4_RDNA_COOP");
    if (v == nullptr || *v == '\0') return 0;
    const int s = std::atoi(v);
    return s > 0 ? s : 0;
}

struct Split {
    int S, Gs;
};

Split make_split(int G, int requested) {
    requested = std::max(1, std::min(requested, G));
    const int Gs = (G + requested - 1) / requested;
    return Split{(G + Gs - 1) / Gs, Gs};
}

// Selector: enough work items to give every resident warp about one item.
// The warp count comes from the live occupancy of this build; the per-shape
// tuning table is measured separately and can override it through cfg/env.
int select_split_for(int N, int K, int B, int op, const DeviceInfo &d) {
    (void)op;
    const int G = K / Q4_GROUP;
    const int RB = (N + Q4_BLOCK_ROWS - 1) / Q4_BLOCK_ROWS;
    const int pb = B;
    const bool dual = op == Q4RDNA_OP_SWIGLU;
    const long long warps =
        (long long)d.sms * d.occ[variant()][batch_class(pb)][dual] * kernel_cfg(variant(), pb, dual).warps;
    long long S = (warps + RB - 1) / RB;
    return make_split(G, (int)std::min<long long>(S, G)).S;
}

int resolve_split(int N, int K, int B, int op, const q4rdna_cfg *cfg, const DeviceInfo &d) {
    const int G = K / Q4_GROUP;
    int req = cfg != nullptr && cfg->split > 0 ? cfg->split : env_split();
    if (req <= 0) req = select_split_for(N, K, B, op, d);
    if (N > (int)(65536 / sizeof(unsigned)) * Q4_BLOCK_ROWS) req = 1;
    return make_split(G, req).S;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// Single-call workspaces start with a fixed ticket area, so the partial sums of
// any later call (any shape) never land on a ticket: every call leaves all
// tickets at zero, which is the only state a call relies on.
constexpr size_t kTicketArea = 65536;  // 16384 row blocks = 2,097,152 rows
constexpr int kMaxSplitRows = (int)(kTicketArea / sizeof(unsigned)) * Q4_BLOCK_ROWS;

size_t partial_bytes(int N, int B, int S, int op) {
    const int planes = op == Q4RDNA_OP_SWIGLU ? 2 : 1;
    return (size_t)S * planes * B * N * sizeof(float);
}

// Fused RMSNorm with S > 1: one sum of h^2 per (row block, split, batch column).
size_t sumsq_bytes(int N, int B, int S) {
    const int RB = (N + Q4_BLOCK_ROWS - 1) / Q4_BLOCK_ROWS;
    return (size_t)RB * S * B * sizeof(float);
}

// Workspace of one q4rdna_gemv* call: ticket area + partials + the RMSNorm sums
// (reserved for every call, so one size query serves both; 0 when S == 1).
size_t ws_bytes_for(int N, int B, int S, int op) {
    return S <= 1 ? 0 : kTicketArea + partial_bytes(N, B, S, op) + sumsq_bytes(N, B, S);
}

// Workspace of one plan task: its own tickets + partials (+ RMSNorm sums), fixed
// for the plan's life.
size_t plan_ws_bytes_for(int N, int B, int S, int op, bool norm) {
    if (S <= 1) return 0;
    const int RB = (N + Q4_BLOCK_ROWS - 1) / Q4_BLOCK_ROWS;
    return align256((size_t)RB * sizeof(unsigned)) + align256(partial_bytes(N, B, S, op)) +
           (norm ? align256(sumsq_bytes(N, B, S)) : 0);
}

// Work items per resident warp (or tile-path CTA) that a plan's split-K choice
// aims at; Q4RDNA_PLAN_ITEMS overrides the default for A/B measurements.
double plan_items_per_worker() {
    const char *e = std::getenv("Q4RDNA_PLAN_ITEMS");
    const double v = (e != nullptr && *e != '\0') ? std::atof(e) : 0.0;
    return v > 0.0 ? std::min(v, 1024.0) : 2.0;
}

// The fused RMSNorm runs in the int8 batch-1 kernel and the tile path, not in
// the A/B variants (Q4RDNA_KERNEL=ldg|i8tma).
bool norm_supported(int B) { return B >= tile_min_batch() || variant() == kI8; }

bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

q4rdna_status check_shape(int N, int K, int B) {
    if (N <= 0 || K <= 0) return Q4RDNA_ERR_INVALID_ARGUMENT;
    if (N % Q4_TILE_ROWS != 0 || K % Q4_GROUP != 0) return Q4RDNA_ERR_SHAPE;
    if (B < 1 || B > Q4RDNA_MAX_BATCH) return Q4RDNA_ERR_UNSUPPORTED;
    return Q4RDNA_OK;
}

int grid_for(long long items, int pb, bool dual, const DeviceInfo &d) {
    const KernelCfg k = kernel_cfg(variant(), pb, dual);
    const long long want = (items + k.warps - 1) / k.warps;
    const long long cap = (long long)d.sms * d.occ[variant()][batch_class(pb)][dual];
    return (int)std::max<long long>(1, std::min(want, cap));
}

// pb: batch columns of the launch (1..16).
q4rdna_status launch(const Launch &L, int grid, int pb, bool dual, cudaStream_t stream, bool norm = false) {
    const KernelCfg k = kernel_cfg(variant(), pb, dual, norm);
    Launch arg = L;
    void *args[] = {&arg};
    if (cudaLaunchKernel(k.fn, dim3(grid), dim3(k.threads), args, (size_t)k.smem, stream) != cudaSuccess)
        return Q4RDNA_ERR_CUDA;
    if (cudaGetLastError() != cudaSuccess) return Q4RDNA_ERR_CUDA;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return Q4RDNA_OK;
}

q4rdna_status gemv_common(int op, const uint8_t *w, const uint8_t *w2, const float *x, const float *add, float *y,
                          int N, int K, int B, const q4rdna_cfg *cfg, void *ws, size_t ws_bytes,
                          cudaStream_t stream, const float *gn = nullptr, float eps = 0.0f) {
    q4rdna_status st = check_shape(N, K, B);
    if (st != Q4RDNA_OK) return st;
    if (w == nullptr || x == nullptr || y == nullptr) return Q4RDNA_ERR_INVALID_ARGUMENT;
    if (op == Q4RDNA_OP_ADD && add == nullptr) return Q4RDNA_ERR_INVALID_ARGUMENT;
    if (op == Q4RDNA_OP_SWIGLU && w2 == nullptr) return Q4RDNA_ERR_INVALID_ARGUMENT;
    if (!aligned(w, 16) || (w2 && !aligned(w2, 16)) || !aligned(x, 8) || !aligned(y, 4) || (add && !aligned(add, 4)) ||
        (gn && !aligned(gn, 8)))
        return Q4RDNA_ERR_ALIGNMENT;
    if (gn != nullptr && !norm_supported(B)) return Q4RDNA_ERR_UNSUPPORTED;
    DeviceInfo d;
    if (!device_info(d)) return Q4RDNA_ERR_DEVICE;
    const int G = K / Q4_GROUP;
    const int RB = (N + Q4_BLOCK_ROWS - 1) / Q4_BLOCK_ROWS;
    Split sp = make_split(G, resolve_split(N, K, B, op, cfg, d));
    if (N > kMaxSplitRows) sp = make_split(G, 1);  // beyond the ticket area: no split
    unsigned *ticket = nullptr;
    float *part = nullptr;
    if (sp.S > 1) {
        const size_t need = ws_bytes_for(N, B, sp.S, op);
        if (ws == nullptr || ws_bytes < need || !aligned(ws, 256)) return Q4RDNA_ERR_WORKSPACE;
        ticket = static_cast<unsigned *>(ws);
        part = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + kTicketArea);
    }
    // One launch for the whole batch: B < tile_min_batch() on the batch-1 kernels, the rest
    // on the tile path; the weights are streamed once.
    Launch L{};
    L.table = nullptr;
    L.ntasks = 1;
    L.B = B;
    Task &T = L.one;
    T.w = w;
    T.w2 = w2;
    T.x = x;
    T.add = add;
    T.y = y;
    T.part = part;
    T.ticket = ticket;
    T.N = N; T.K = K; T.G = G; T.RB = RB; T.S = sp.S; T.Gs = sp.Gs; T.op = op; T.nmirror = 0;
    T.item_begin = 0;
    T.gn = gn;
    T.eps = eps;
    T.nss = (gn != nullptr && sp.S > 1) ? part + partial_bytes(N, B, sp.S, op) / sizeof(float) : nullptr;
    L.total_items = (long long)RB * sp.S;
    const bool dual = op == Q4RDNA_OP_SWIGLU;
    return launch(L, grid_for(L.total_items, B, dual, d), B, dual, stream, gn != nullptr);
}

}  // namespace q4

using namespace q4;

// Flag exchange that closes a fused gather: after the plan kernel (stream
// order), lane p raises this rank's flag at rank p, then waits, bounded, for
// rank p's flag of this epoch here.
struct GatherSignal {
    uint32_t *peer[kMaxMirrors];  // every rank's flag array, as mapped in this process
    uint32_t *local;              // this rank's flag array
    int world, rank;
    uint32_t epoch;
};
constexpr int kGatherTries = 1 << 22;  // x ~0.5 us sleep: about 2 s
constexpr unsigned kFaultGatherTimeout = 2u;

__global__ void q4_gather_signal_kernel(const __grid_constant__ GatherSignal a) {
    const int p = threadIdx.x;
    if (p >= a.world) return;
    // the plan kernel's stores (peer ones included) precede this kernel in stream
    // order; the system-scope fence orders them before the flag for the peers
    __threadfence_system();
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.peer[p] + a.rank), "r"(a.epoch) : "memory");
    int i = 0;
    for (; i < kGatherTries; ++i) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a.local + p) : "memory");
        if ((int)(v - a.epoch) >= 0) break;
        __nanosleep(500);
    }
    if (i == kGatherTries) atomicOr(&g_fault, kFaultGatherTimeout);
}

// Segment counts.  Plan runs default to one launch: with the plan-wide split
// choice the items are large and few per warp, and segment launches that
// overlap (two streams) leave SMs idle between segments (Qwen3-8B step: 631 us
// as one launch, 705 us as 2, 750 us as 4).
// q4rdna_plan_run_host's default segment counts.  A segment's copies over PCIe
// take a fraction of its compute time (one whole-buffer copy of the step's
// activations about 0.16), and each extra launch ends with a tail of idle SMs,
// so few graded segments win:
// - output copies: weights 1, 2, 1; the middle segment's copies hide behind
//   the end segments' compute (Qwen3-8B step, B = 1: e2e 792 us at 3, 959 at
//   6, 1116 at 8);
// - outputs stored straight into the host buffer: weights 1, g (host_growth);
//   the second segment's input copy hides behind the first one's compute
//   (712 us at 2 segments, 773 at 3, 843 at 4, with g = 2).
constexpr int kHostSegments = 3;
constexpr int kHostSegmentsDirect = 2;

// q4rdna_plan_run_host stores outputs straight into a mapped pinned host
// buffer unless Q4RDNA_HOST_DIRECT=0.
bool host_direct() {
    static const bool v = [] {
        const char *e = std::getenv("Q4RDNA_HOST_DIRECT");
        return e == nullptr || std::strcmp(e, "0") != 0;
    }();
    return v;
}

// Growth of consecutive run_host segments with direct outputs (weights g^s):
// segment s + 1's input copy must hide behind segment s's compute, and a
// whole-buffer input copy takes about 0.16 of the step's compute, so a larger
// g shrinks the exposed first copy until the second one stops hiding.
// Qwen3-8B step, B = 1, 2 segments: e2e - device 80 us at g = 2, 71 at 4, 96
// at 6.  Q4RDNA_HOST_GROWTH overrides it.
double host_growth() {
    static const double v = [] {
        const char *e = std::getenv("Q4RDNA_HOST_GROWTH");
        const double g = (e != nullptr && *e != '\0') ? std::atof(e) : 0.0;
        return g >= 1.0 ? std::min(g, 64.0) : 4.0;
    }();
    return v;
}

// Device address of run_host's output buffer when the whole [yh, yh + yb) is
// pinned host memory mapped for the device (both ends map, at the same
// distance as on the host), else null: the outputs are then copied.
uint8_t *mapped_output(const void *yh, size_t yb) {
    if (yh == nullptr || yb == 0 || !host_direct()) return nullptr;
    void *a = nullptr, *b = nullptr;
    uint8_t *r = nullptr;
    if (cudaHostGetDevicePointer(&a, const_cast<void *>(yh), 0) == cudaSuccess &&
        cudaHostGetDevicePointer(&b, static_cast<uint8_t *>(const_cast<void *>(yh)) + yb - 1, 0) == cudaSuccess &&
        static_cast<uint8_t *>(b) - static_cast<uint8_t *>(a) == (ptrdiff_t)(yb - 1))
        r = static_cast<uint8_t *>(a);
    cudaGetLastError();  // a pageable or unmapped buffer is not an error here
    return r;
}

// q4rdna_plan_run_host replays a captured CUDA graph unless Q4RDNA_HOST_GRAPH=0.
bool host_graph() {
    static const bool v = [] {
        const char *e = std::getenv("Q4RDNA_HOST_GRAPH");
        return e == nullptr || std::strcmp(e, "0") != 0;
    }();
    return v;
}


// Device copy of a task table in launch order: tasks with the longest items
// first (stable), item_begin renumbered from 0.  The persistent kernels take
// items round-robin, so the last round then consists of the shortest items
// (longest-processing-time-first list scheduling); results do not depend on
// the order.
Task *upload_tasks(std::vector<Task> t) {
    std::stable_sort(t.begin(), t.end(), [](const Task &a, const Task &b) {
        const long long ca = (long long)a.Gs * (a.op == Q4RDNA_OP_SWIGLU ? 2 : 1);
        const long long cb = (long long)b.Gs * (b.op == Q4RDNA_OP_SWIGLU ? 2 : 1);
        return ca > cb;
    });
    long long items = 0;
    for (Task &T : t) {
        T.item_begin = items;
        items += (long long)T.RB * T.S;
    }
    Task *d = nullptr;
    if (cudaMalloc(&d, sizeof(Task) * t.size()) != cudaSuccess) return nullptr;
    if (cudaMemcpy(d, t.data(), sizeof(Task) * t.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(d);
        return nullptr;
    }
    return d;
}

struct q4rdna_plan {
    int device = -1;
    int count = 0, B = 1, nb = 1, grid = 1;
    bool dual = false;  // the plan holds a SwiGLU task
    bool norm = false;  // the plan holds a fused-RMSNorm task
    long long items = 0;
    Task *table = nullptr;     // device
    void *workspace = nullptr; // device
    size_t ws_bytes = 0;
    uint64_t weight_bytes = 0, algo_bytes = 0;
    std::vector<Task> host;    // task table as uploaded (no gather)
    // q4rdna_plan_run_host: consecutive task ranges with their own device tables
    struct Segment {
        int first = 0, count = 0;
        long long items = 0;
        int grid = 1;
        Task *table = nullptr;  // item_begin rebased to the segment
        Task *gtable[2] = {nullptr, nullptr};  // the same with the gather's mirrors, per gathered buffer
        size_t x_lo = 0, x_hi = 0, y_lo = 0, y_hi = 0;  // byte ranges from x_dev / y_dev
        cudaEvent_t x_ready = nullptr, y_ready = nullptr;
    };
    std::vector<Segment> segs;
    int seg_request = -1;
    bool seg_graded = false;  // segments cut by graded weights (run_host) or equal ones
    bool seg_direct = false;  // run_host: outputs stored straight into the mapped host buffer
    const void *seg_yh = nullptr;
    int run_segments = 1;  // q4rdna_plan_run: segment launches (1 = one launch, the default)
    const void *seg_x = nullptr, *seg_y = nullptr;
    // q4rdna_plan_run_host: the whole copy/launch sequence as one CUDA graph,
    // keyed by the buffers it was captured with (rebuilt when they change)
    struct HostGraph {
        const void *xh = nullptr, *xd = nullptr, *yd = nullptr, *yh = nullptr;
        size_t xb = 0, yb = 0;
        cudaGraphExec_t exec = nullptr;
        uint64_t launches = 0;  // kernel launches one replay performs
    } hg;
    cudaStream_t cap = nullptr;  // capture stream
    cudaStream_t h2d = nullptr, d2h = nullptr;
    cudaStream_t comp[2] = {nullptr, nullptr};  // segments alternate, so one's tail overlaps the next
    cudaEvent_t start = nullptr, done = nullptr;
    // fused gather (q4rdna_plan_set_gather): one task table per gathered buffer
    Task *gtable[2] = {nullptr, nullptr};
    std::vector<Task> ghost[2];
    GatherSignal sig{};
    uint32_t epoch = 0;
    bool gather = false;
    // Q4_K descriptors (format Q4RDNA_FORMAT_Q4K): their own task table and
    // launch, after the Q4_RDNA launch on the same stream
    std::vector<q4k::Task> q4k_host;
    q4k::Task *q4k_table = nullptr;
    long long q4k_items = 0;
};

namespace {
q4rdna_status build_segments(q4rdna_plan *p, int want, const uint8_t *xd, size_t xb, const uint8_t *yd,
                             size_t yb, bool graded = false, const uint8_t *yh = nullptr);
q4rdna_status launch_segments(q4rdna_plan *plan, cudaStream_t cs, const uint8_t *xh, uint8_t *xd, const uint8_t *yd,
                              uint8_t *yh, int par = -1);
}  // namespace

extern "C" {

const char *q4rdna_status_string(q4rdna_status s) {
    switch (s) {
        case Q4RDNA_OK: return "ok";
        case Q4RDNA_ERR_INVALID_ARGUMENT: return "invalid argument";
        case Q4RDNA_ERR_SHAPE: return "unsupported shape (rows % 32, columns % 64)";
        case Q4RDNA_ERR_ALIGNMENT: return "misaligned pointer";
        case Q4RDNA_ERR_WORKSPACE: return "workspace missing or too small";
        case Q4RDNA_ERR_UNSUPPORTED: return "unsupported batch";
        case Q4RDNA_ERR_CUDA: return "CUDA error";
        case Q4RDNA_ERR_IO: return "sidecar I/O error";
        case Q4RDNA_ERR_FORMAT: return "invalid sidecar";
        case Q4RDNA_ERR_NOT_FOUND: return "tensor not found";
        case Q4RDNA_ERR_DEVICE: return "device error";
        case Q4RDNA_ERR_TOO_LARGE: return "size beyond the entry point's limit";
    }
    return "unknown status";
}

const char *q4rdna_version(void) { return "q4rdna-b200 0.1 (sm_100a)"; }

int q4rdna_select_split(int N, int K, int B, int op) {
    if (check_shape(N, K, B) != Q4RDNA_OK) return 0;
    DeviceInfo d;
    if (!device_info(d)) return 0;
    return resolve_split(N, K, B, op, nullptr, d);
}

size_t q4rdna_workspace_bytes(int N, int K, int B, int op, const q4rdna_cfg *cfg) {
    if (check_shape(N, K, B) != Q4RDNA_OK) return 0;
    DeviceInfo d;
    if (!device_info(d)) return 0;
    return ws_bytes_for(N, B, resolve_split(N, K, B, op, cfg, d), op);
}

q4rdna_status q4rdna_workspace_init(void *workspace, size_t bytes, q4rdna_stream_t stream) {
    if (bytes == 0) return Q4RDNA_OK;
    if (workspace == nullptr) return Q4RDNA_ERR_INVALID_ARGUMENT;
    return cudaMemsetAsync(workspace, 0, bytes, (cudaStream_t)stream) == cudaSuccess ? Q4RDNA_OK : Q4RDNA_ERR_CUDA;
}

q4rdna_status q4rdna_gemv(const uint8_t *tiles, const float *x, float *y, int N, int K, int B,
                          const q4rdna_cfg *cfg, void *workspace, size_t workspace_bytes, q4rdna_stream_t stream) {
    return gemv_common(Q4RDNA_OP_PLAIN, tiles, nullptr, x, nullptr, y, N, K, B, cfg, workspace, workspace_bytes,
                       (cudaStream_t)stream);
}

q4rdna_status q4rdna_gemv_add(const uint8_t *tiles, const float *x, const float *add, float *y, int N, int K, int B,
                              const q4rdna_cfg *cfg, void *workspace, size_t workspace_bytes,
                              q4rdna_stream_t stream) {
    return gemv_common(Q4RDNA_OP_ADD, tiles, nullptr, x, add, y, N, K, B, cfg, workspace, workspace_bytes,
                       (cudaStream_t)stream);
}

q4rdna_status q4rdna_gemv_swiglu(const uint8_t *up_tiles, const uint8_t *gate_tiles, const float *x, float *y,
                                 int N, int K, int B, const q4rdna_cfg *cfg, void *workspace,
                                 size_t workspace_bytes, q4rdna_stream_t stream) {
    return gemv_common(Q4RDNA_OP_SWIGLU, up_tiles, gate_tiles, x, nullptr, y, N, K, B, cfg, workspace,
                       workspace_bytes, (cudaStream_t)stream);
}

q4rdna_status q4rdna_gemv_rmsnorm(const uint8_t *tiles, const uint8_t *gate_tiles, const float *h,
                                  const float *norm_weight, float eps, const float *add, float *y, int N, int K,
                                  int B, int op, const q4rdna_cfg *cfg, void *workspace, size_t workspace_bytes,
                                  q4rdna_stream_t stream) {
    if (norm_weight == nullptr || !(eps >= 0.0f) || op < Q4RDNA_OP_PLAIN || op > Q4RDNA_OP_SWIGLU)
        return Q4RDNA_ERR_INVALID_ARGUMENT;
    return gemv_common(op, tiles, gate_tiles, h, add, y, N, K, B, cfg, workspace, workspace_bytes,
                       (cudaStream_t)stream, norm_weight, eps);
}

q4rdna_status q4rdna_dequant_f32(const uint8_t *tiles, float *W, int N, int K, q4rdna_stream_t stream) {
    q4rdna_status st = check_shape(N, K, 1);
    if (st != Q4RDNA_OK) return st;
    if (tiles == nullptr || W == nullptr) return Q4RDNA_ERR_INVALID_ARGUMENT;
    if (!aligned(tiles, 2) || !aligned(W, 4)) return Q4RDNA_ERR_ALIGNMENT;
    const long long n = (long long)N * (K / Q4_GROUP);
    q4_dequant_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(tiles, W, N, K);
    if (cudaGetLastError() != cudaSuccess) return Q4RDNA_ERR_CUDA;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return Q4RDNA_OK;
}

q4rdna_status plan_create_rdna(const q4rdna_gemv_desc *descs, int count, int B, q4rdna_plan **out) {
    if (out == nullptr || descs == nullptr || count <= 0) return Q4RDNA_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    if (B < 1 || B > Q4RDNA_MAX_BATCH) return Q4RDNA_ERR_UNSUPPORTED;
    DeviceInfo d;
    if (!device_info(d)) return Q4RDNA_ERR_DEVICE;
    std::vector<Task> host(count);
    std::vector<size_t> ws_off(count);
    size_t ws_total = 0;
    long long items = 0;
    uint64_t wbytes = 0, abytes = 0;
    // Split-K only as far as the whole plan needs it: every split adds partial
    // stores, a fence and a reduction per item, which on the Qwen3-8B step cost
    // more than the imbalance of unsplit items (624 us per step unsplit, 949 us
    // with ~64 KB items).  Each task gets the split that gives the plan about
    // plan_items_per_worker() items per resident warp (CTA on the tile path).
    long long total_rb = 0;
    bool any_dual_task = false;
    for (int i = 0; i < count; ++i) {
        if (descs[i].N > 0) total_rb += (descs[i].N + Q4_BLOCK_ROWS - 1) / Q4_BLOCK_ROWS;
        any_dual_task = any_dual_task || descs[i].op == Q4RDNA_OP_SWIGLU;
    }
    const long long workers = (long long)d.sms * d.occ[variant()][batch_class(B)][any_dual_task] *
                              kernel_cfg(variant(), B, any_dual_task).warps;
    const double want_items = plan_items_per_worker() * (double)workers;
    const int plan_split = total_rb > 0 ? (int)std::max(1.0, std::ceil(want_items / (double)total_rb)) : 1;
    // Tail split (Q4RDNA_TAIL_SPLIT = S > 1, A/B measurements): the tasks with
    // the cheapest items, about one item per worker of them, are split S ways,
    // so that the plan's last round (items run longest first) is made of
    // smaller items.
    std::vector<int> tail_req(count, 0);
    if (const char *ts = std::getenv("Q4RDNA_TAIL_SPLIT")) {
        const int S = std::atoi(ts);
        if (S > 1 && plan_split == 1) {
            std::vector<int> order(count);
            for (int i = 0; i < count; ++i) order[i] = i;
            auto cost = [&](int i) {
                return (long long)(descs[i].K / Q4_GROUP) * (descs[i].op == Q4RDNA_OP_SWIGLU ? 2 : 1);
            };
            std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return cost(a) < cost(b); });
            long long acc = 0;
            for (int i : order) {
                if (acc >= workers) break;
                if (descs[i].split > 0 || descs[i].N <= 0) continue;
                tail_req[i] = S;
                acc += (long long)(descs[i].N + Q4_BLOCK_ROWS - 1) / Q4_BLOCK_ROWS * S;
            }
        }
    }
    for (int i = 0; i < count; ++i) {
        const q4rdna_gemv_desc &e = descs[i];
        q4rdna_status st = check_shape(e.N, e.K, B);
        if (st != Q4RDNA_OK) return st;
        if (e.op < Q4RDNA_OP_PLAIN || e.op > Q4RDNA_OP_SWIGLU) return Q4RDNA_ERR_INVALID_ARGUMENT;
        if (e.tiles == nullptr || e.x == nullptr || e.y == nullptr) return Q4RDNA_ERR_INVALID_ARGUMENT;
        if (e.op == Q4RDNA_OP_ADD && e.add == nullptr) return Q4RDNA_ERR_INVALID_ARGUMENT;
        if (e.op == Q4RDNA_OP_SWIGLU && e.gate_tiles == nullptr) return Q4RDNA_ERR_INVALID_ARGUMENT;
        if (!aligned(e.tiles, 16) || (e.gate_tiles && !aligned(e.gate_tiles, 16)) || !aligned(e.x, 8) ||
            !aligned(e.y, 4) || (e.add && !aligned(e.add, 4)) || (e.norm_weight && !aligned(e.norm_weight, 8)))
            return Q4RDNA_ERR_ALIGNMENT;
        if (e.norm_weight != nullptr && !norm_supported(B)) return Q4RDNA_ERR_UNSUPPORTED;
        const int planes = e.op == Q4RDNA_OP_SWIGLU ? 2 : 1;
        const int G = e.K / Q4_GROUP;
        const int RB = (e.N + Q4_BLOCK_ROWS - 1) / Q4_BLOCK_ROWS;
        const int req = e.split > 0 ? e.split : std::min(tail_req[i] > 0 ? tail_req[i] : plan_split, G);
        const Split sp = make_split(G, req);
        Task &T = host[i];
        T.w = e.tiles; T.w2 = e.gate_tiles; T.x = e.x; T.add = e.add; T.y = e.y;
        T.part = nullptr; T.ticket = nullptr;
        T.N = e.N; T.K = e.K; T.G = G; T.RB = RB; T.S = sp.S; T.Gs = sp.Gs; T.op = e.op; T.nmirror = 0;
        T.item_begin = items;
        T.gn = e.norm_weight;
        T.eps = e.norm_eps;
        items += (long long)RB * sp.S;
        ws_off[i] = ws_total;
        ws_total += plan_ws_bytes_for(e.N, B, sp.S, e.op, e.norm_weight != nullptr);
        wbytes += (uint64_t)planes * Q4_TENSOR_BYTES(e.N, e.K);
        abytes += (uint64_t)planes * Q4_TENSOR_BYTES(e.N, e.K) + 4ull * e.K * B + 4ull * e.N * B +
                  (e.op == Q4RDNA_OP_ADD ? 4ull * e.N * B : 0ull);
    }
    q4rdna_plan *p = new (std::nothrow) q4rdna_plan();
    if (p == nullptr) return Q4RDNA_ERR_CUDA;
    cudaGetDevice(&p->device);
    if (ws_total > 0 && cudaMalloc(&p->workspace, ws_total) != cudaSuccess) { delete p; return Q4RDNA_ERR_CUDA; }
    if (ws_total > 0 && cudaMemset(p->workspace, 0, ws_total) != cudaSuccess) { q4rdna_plan_destroy(p); return Q4RDNA_ERR_CUDA; }
    for (int i = 0; i < count; ++i) {
        Task &T = host[i];
        if (T.S > 1) {
            uint8_t *base = static_cast<uint8_t *>(p->workspace) + ws_off[i];
            T.ticket = reinterpret_cast<unsigned *>(base);
            T.part = reinterpret_cast<float *>(base + align256((size_t)T.RB * sizeof(unsigned)));
            if (T.gn != nullptr)
                T.nss = reinterpret_cast<float *>(base + align256((size_t)T.RB * sizeof(unsigned)) +
                                                  align256(partial_bytes(T.N, B, T.S, T.op)));
        }
    }
    if ((p->table = upload_tasks(host)) == nullptr) {
        q4rdna_plan_destroy(p);
        return Q4RDNA_ERR_CUDA;
    }
    bool any_dual = false;
    for (int i = 0; i < count; ++i) any_dual = any_dual || descs[i].op == Q4RDNA_OP_SWIGLU;
    p->count = count; p->B = B; p->nb = B; p->items = items; p->dual = any_dual;
    for (int i = 0; i < count; ++i) p->norm = p->norm || descs[i].norm_weight != nullptr;
    p->host = host;
    p->grid = grid_for(items, B, any_dual, d);
    p->ws_bytes = ws_total; p->weight_bytes = wbytes; p->algo_bytes = abytes;
    *out = p;
    return Q4RDNA_OK;
}

// Plans with Q4_K descriptors: the Q4_RDNA ones go through plan_create_rdna
// (in their original order), the Q4_K ones get their own task table.
q4rdna_status q4rdna_plan_create(const q4rdna_gemv_desc *descs, int count, int B, q4rdna_plan **out) {
    if (out == nullptr || descs == nullptr || count <= 0) return Q4RDNA_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    std::vector<q4rdna_gemv_desc> rd;
    std::vector<q4k::Task> kt;
    long long kitems = 0;
    uint64_t kw = 0, ka = 0;
    for (int i = 0; i < count; ++i) {
        const q4rdna_gemv_desc &e = descs[i];
        if (e.format == Q4RDNA_FORMAT_Q4RDNA) {
            rd.push_back(e);
        } else if (e.format == Q4RDNA_FORMAT_Q4K) {
            q4k::Task T;
            long long items = 0;
            const q4rdna_status st = q4k_build_task(e, B, kitems, T, items);
            if (st != Q4RDNA_OK) return st;
            kt.push_back(T);
            kitems += items;
            const uint64_t w = q4rdna_q4k_bytes(e.N, e.K);
            kw += w;
            ka += w + 4ull * e.K * B + 4ull * e.N * B + (e.op == Q4RDNA_OP_ADD ? 4ull * e.N * B : 0ull);
        } else {
            return Q4RDNA_ERR_INVALID_ARGUMENT;
        }
    }
    if (B < 1 || B > Q4RDNA_MAX_BATCH) return Q4RDNA_ERR_UNSUPPORTED;
    q4rdna_plan *p = nullptr;
    if (!rd.empty()) {
        const q4rdna_status st = plan_create_rdna(rd.data(), (int)rd.size(), B, &p);
        if (st != Q4RDNA_OK) return st;
    } else {
        p = new (std::nothrow) q4rdna_plan();
        if (p == nullptr) return Q4RDNA_ERR_CUDA;
        cudaGetDevice(&p->device);
        p->count = 0; p->B = B; p->nb = B;
    }
    if (!kt.empty()) {
        if (cudaMalloc(&p->q4k_table, sizeof(q4k::Task) * kt.size()) != cudaSuccess ||
            cudaMemcpy(p->q4k_table, kt.data(), sizeof(q4k::Task) * kt.size(), cudaMemcpyHostToDevice) !=
                cudaSuccess) {
            q4rdna_plan_destroy(p);
            return Q4RDNA_ERR_CUDA;
        }
        p->q4k_host = kt;
        p->q4k_items = kitems;
        p->weight_bytes += kw;
        p->algo_bytes += ka;
    }
    *out = p;
    return Q4RDNA_OK;
}

namespace {
q4rdna_status launch_q4k(q4rdna_plan *plan, cudaStream_t stream) {
    if (plan->q4k_host.empty()) return Q4RDNA_OK;
    return q4k_launch_tasks(plan->q4k_table, nullptr, (int)plan->q4k_host.size(), plan->B, plan->q4k_items, stream);
}
}  // namespace

q4rdna_status q4rdna_plan_run(q4rdna_plan *plan, q4rdna_stream_t stream) {
    if (plan == nullptr) return Q4RDNA_ERR_INVALID_ARGUMENT;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != plan->device) return Q4RDNA_ERR_DEVICE;
    const int nseg = std::max(1, plan->run_segments);
    const bool segmented = nseg > 1 && plan->count > 1;
    if (segmented) {
        const int want = std::min(nseg, plan->count);
        if (plan->seg_request != want || plan->seg_graded) {
            const q4rdna_status st = build_segments(plan, want, nullptr, 0, nullptr, 0);
            if (st != Q4RDNA_OK) return st;
        }
    }
    if (!plan->gather) {
        q4rdna_status st = Q4RDNA_OK;
        if (segmented) {
            st = launch_segments(plan, (cudaStream_t)stream, nullptr, nullptr, nullptr, nullptr);
        } else if (plan->count > 0) {
            Launch L{};
            L.table = plan->table;
            L.ntasks = plan->count;
            L.B = plan->B;
            L.total_items = plan->items;
            st = launch(L, plan->grid, plan->nb, plan->dual, (cudaStream_t)stream, plan->norm);
        }
        if (st != Q4RDNA_OK) return st;
        return launch_q4k(plan, (cudaStream_t)stream);
    }
    const uint32_t epoch = plan->epoch + 1;
    q4rdna_status st;
    if (segmented) {
        st = launch_segments(plan, (cudaStream_t)stream, nullptr, nullptr, nullptr, nullptr, (int)(epoch & 1));
    } else {
        Launch L{};
        L.table = plan->gtable[epoch & 1];
        L.ntasks = plan->count;
        L.B = plan->B;
        L.total_items = plan->items;
        st = launch(L, plan->grid, plan->nb, plan->dual, (cudaStream_t)stream, plan->norm);
    }
    if (st != Q4RDNA_OK) return st;
    GatherSignal sg = plan->sig;
    sg.epoch = epoch;
    void *args[] = {&sg};
    if (cudaLaunchKernel((const void *)q4_gather_signal_kernel, dim3(1), dim3(32), args, 0, (cudaStream_t)stream) !=
        cudaSuccess)
        return Q4RDNA_ERR_CUDA;
    if (cudaGetLastError() != cudaSuccess) return Q4RDNA_ERR_CUDA;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    plan->epoch = epoch;
    return Q4RDNA_OK;
}

q4rdna_status q4rdna_plan_set_gather(q4rdna_plan *plan, int world, int rank, const float *y_base,
                                     size_t rank_floats, float *const *gathered0, float *const *gathered1,
                                     uint32_t *const *flags) {
    if (plan == nullptr || y_base == nullptr || gathered0 == nullptr || gathered1 == nullptr || flags == nullptr)
        return Q4RDNA_ERR_INVALID_ARGUMENT;
    if (world < 2 || world > kMaxMirrors || rank < 0 || rank >= world || plan->gather)
        return Q4RDNA_ERR_INVALID_ARGUMENT;
    if (!plan->q4k_host.empty() || plan->count == 0) return Q4RDNA_ERR_UNSUPPORTED;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != plan->device) return Q4RDNA_ERR_DEVICE;
    for (int p = 0; p < world; ++p)
        if (gathered0[p] == nullptr || gathered1[p] == nullptr || flags[p] == nullptr ||
            !aligned(gathered0[p], 4) || !aligned(gathered1[p], 4) || !aligned(flags[p], 4))
            return Q4RDNA_ERR_INVALID_ARGUMENT;
    // every output block [B][N] must lie inside this rank's slice
    for (const Task &T : plan->host) {
        if (T.y < y_base) return Q4RDNA_ERR_INVALID_ARGUMENT;
        const size_t off = (size_t)(T.y - y_base);
        if (off + (size_t)plan->B * T.N > rank_floats) return Q4RDNA_ERR_INVALID_ARGUMENT;
    }
    for (int par = 0; par < 2; ++par) {
        float *const *g = par == 0 ? gathered0 : gathered1;
        std::vector<Task> t = plan->host;
        for (Task &T : t) {
            const size_t off = (size_t)(T.y - y_base);
            T.nmirror = world;
            for (int p = 0; p < world; ++p) T.mirror[p] = g[p] + (size_t)rank * rank_floats + off;
        }
        plan->ghost[par] = t;
        if ((plan->gtable[par] = upload_tasks(t)) == nullptr) {
            for (Task *&gt : plan->gtable) {
                if (gt) cudaFree(gt);
                gt = nullptr;
            }
            return Q4RDNA_ERR_CUDA;
        }
    }
    GatherSignal &sg = plan->sig;
    for (int p = 0; p < world; ++p) sg.peer[p] = flags[p];
    sg.local = flags[rank];
    sg.world = world;
    sg.rank = rank;
    plan->epoch = 0;
    plan->gather = true;
    plan->seg_request = -1;  // segments are rebuilt with the gather's tables
    return Q4RDNA_OK;
}

}  // extern "C"

namespace {

// Cuts the plan into `want` runs of consecutive tasks and gives each its own
// device task table, events and byte ranges.  Equal weight bytes per run, or
// with `graded` weights 2^min(s, want - 1 - s): small runs at both ends, so
// that the first input copy and the last output copy are short.  With `yh`
// (run_host's output buffer) mapped into the device's address space, every
// task also stores its outputs there (its one mirror), so no output copies
// remain; the runs then grow 2^s, so each input copy hides behind the
// previous run's compute.
q4rdna_status build_segments(q4rdna_plan *p, int want, const uint8_t *xd, size_t xb, const uint8_t *yd,
                             size_t yb, bool graded, const uint8_t *yh) {
    for (auto &sg : p->segs) {
        if (sg.table) cudaFree(sg.table);
        for (Task *t : sg.gtable)
            if (t) cudaFree(t);
        if (sg.x_ready) cudaEventDestroy(sg.x_ready);
        if (sg.y_ready) cudaEventDestroy(sg.y_ready);
    }
    p->segs.clear();
    p->seg_request = -1;
    if (p->hg.exec) {  // the graph holds the old segments' tables and events
        cudaGraphExecDestroy(p->hg.exec);
        p->hg = q4rdna_plan::HostGraph{};
    }
    DeviceInfo d;
    if (!device_info(d)) return Q4RDNA_ERR_DEVICE;
    const int n = p->count;
    want = std::max(1, std::min(want, n));
    uint8_t *yh_dev = graded && xd != nullptr ? mapped_output(yh, yb) : nullptr;
    const bool direct = yh_dev != nullptr;
    uint64_t total = 0;
    for (const Task &T : p->host) total += (uint64_t)T.N * T.K * (T.op == Q4RDNA_OP_SWIGLU ? 2 : 1);
    std::vector<double> cum(want);  // cumulative share of the weights after run s
    double wsum = 0;
    for (int s = 0; s < want; ++s) {
        wsum += !graded ? 1.0
                : direct ? std::pow(host_growth(), (double)std::min(s, 30))
                         : std::ldexp(1.0, std::min(std::min(s, want - 1 - s), 30));
        cum[s] = wsum;
    }
    int first = 0;
    uint64_t acc = 0;
    for (int s = 0; s < want && first < n; ++s) {
        int last = first;  // exclusive end
        const uint64_t goal = (uint64_t)((double)total * (cum[s] / wsum));
        while (last < n && (last == first || acc < goal || s == want - 1)) {
            const Task &T = p->host[last];
            acc += (uint64_t)T.N * T.K * (T.op == Q4RDNA_OP_SWIGLU ? 2 : 1);
            ++last;
        }
        q4rdna_plan::Segment sg;
        sg.first = first;
        sg.count = last - first;
        sg.x_lo = sg.y_lo = SIZE_MAX;
        std::vector<Task> t(p->host.begin() + first, p->host.begin() + last);
        const long long base = t.front().item_begin;
        for (Task &T : t) {
            const uint8_t *x = reinterpret_cast<const uint8_t *>(T.x);
            const uint8_t *y = reinterpret_cast<const uint8_t *>(T.y);
            const size_t xn = (size_t)p->B * T.K * sizeof(float), yn = (size_t)p->B * T.N * sizeof(float);
            if (xd == nullptr) continue;  // device-only segments: no copy ranges
            if (x < xd || x + xn > xd + xb || y < yd || y + yn > yd + yb) return Q4RDNA_ERR_INVALID_ARGUMENT;
            sg.x_lo = std::min(sg.x_lo, (size_t)(x - xd));
            sg.x_hi = std::max(sg.x_hi, (size_t)(x - xd) + xn);
            sg.y_lo = std::min(sg.y_lo, (size_t)(y - yd));
            sg.y_hi = std::max(sg.y_hi, (size_t)(y - yd) + yn);
            if (direct) {
                T.nmirror = 1;
                T.mirror[0] = reinterpret_cast<float *>(yh_dev + (y - yd));
            }
        }
        const long long end = last < n ? p->host[last].item_begin : p->items;
        sg.items = end - base;
        sg.grid = grid_for(sg.items, p->B, p->dual, d);
        p->segs.push_back(sg);  // owned by the plan from here on (freed on failure paths below)
        q4rdna_plan::Segment &g = p->segs.back();
        if ((g.table = upload_tasks(t)) == nullptr ||
            cudaEventCreateWithFlags(&g.x_ready, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&g.y_ready, cudaEventDisableTiming) != cudaSuccess)
            return Q4RDNA_ERR_CUDA;
        for (int par = 0; p->gather && par < 2; ++par) {
            std::vector<Task> gt(p->ghost[par].begin() + first, p->ghost[par].begin() + last);
            if ((g.gtable[par] = upload_tasks(gt)) == nullptr) return Q4RDNA_ERR_CUDA;
        }
        first = last;
    }
    // the segments' ranges must be disjoint: a later segment's input copy may
    // land while an earlier segment still reads, and outputs leave early
    for (size_t a = 0; xd != nullptr && a < p->segs.size(); ++a)
        for (size_t b = a + 1; b < p->segs.size(); ++b) {
            const auto &A = p->segs[a], &Bs = p->segs[b];
            if (A.x_lo < Bs.x_hi && Bs.x_lo < A.x_hi) return Q4RDNA_ERR_INVALID_ARGUMENT;
            if (A.y_lo < Bs.y_hi && Bs.y_lo < A.y_hi) return Q4RDNA_ERR_INVALID_ARGUMENT;
        }
    if (p->h2d == nullptr &&
        (cudaStreamCreateWithFlags(&p->h2d, cudaStreamNonBlocking) != cudaSuccess ||
         cudaStreamCreateWithFlags(&p->d2h, cudaStreamNonBlocking) != cudaSuccess ||
         cudaStreamCreateWithFlags(&p->comp[0], cudaStreamNonBlocking) != cudaSuccess ||
         cudaStreamCreateWithFlags(&p->comp[1], cudaStreamNonBlocking) != cudaSuccess ||
         cudaEventCreateWithFlags(&p->start, cudaEventDisableTiming) != cudaSuccess ||
         cudaEventCreateWithFlags(&p->done, cudaEventDisableTiming) != cudaSuccess))
        return Q4RDNA_ERR_CUDA;
    p->seg_request = want;
    p->seg_graded = graded;
    p->seg_direct = direct;
    p->seg_yh = yh;
    p->seg_x = xd;
    p->seg_y = yd;
    return Q4RDNA_OK;
}

}  // namespace

extern "C" {

}  // extern "C"

namespace {

// Runs the plan's segments, alternating between the two library streams, after
// prior work on cs; cs waits for the end.  With host buffers (xh != null) each
// segment's input copy precedes it on the copy stream and its output copy
// follows it on the other copy stream.
q4rdna_status launch_segments(q4rdna_plan *plan, cudaStream_t cs, const uint8_t *xh, uint8_t *xd, const uint8_t *yd,
                              uint8_t *yh, int par) {
    const bool copies = xh != nullptr;
    if (cudaEventRecord(plan->start, cs) != cudaSuccess ||
        cudaStreamWaitEvent(plan->comp[0], plan->start, 0) != cudaSuccess ||
        cudaStreamWaitEvent(plan->comp[1], plan->start, 0) != cudaSuccess)
        return Q4RDNA_ERR_CUDA;
    const bool out_copies = copies && !plan->seg_direct;  // direct: the kernels store into yh
    if (copies && cudaStreamWaitEvent(plan->h2d, plan->start, 0) != cudaSuccess) return Q4RDNA_ERR_CUDA;
    if (out_copies && cudaStreamWaitEvent(plan->d2h, plan->start, 0) != cudaSuccess) return Q4RDNA_ERR_CUDA;
    for (auto &sg : plan->segs) {
        if (!copies) break;
        if (cudaMemcpyAsync(xd + sg.x_lo, xh + sg.x_lo, sg.x_hi - sg.x_lo, cudaMemcpyHostToDevice, plan->h2d) !=
                cudaSuccess ||
            cudaEventRecord(sg.x_ready, plan->h2d) != cudaSuccess)
            return Q4RDNA_ERR_CUDA;
    }
    for (size_t i = 0; i < plan->segs.size(); ++i) {
        auto &sg = plan->segs[i];
        // segments alternate between two streams: segment i + 1 starts on the
        // SMs that segment i's last items leave idle
        cudaStream_t c = plan->comp[i & 1];
        if (copies && cudaStreamWaitEvent(c, sg.x_ready, 0) != cudaSuccess) return Q4RDNA_ERR_CUDA;
        Launch L{};
        L.table = par >= 0 ? sg.gtable[par] : sg.table;  // par: gathered buffer of a gather run
        L.ntasks = sg.count;
        L.B = plan->B;
        L.total_items = sg.items;
        const q4rdna_status st = launch(L, sg.grid, plan->nb, plan->dual, c, plan->norm);
        if (st != Q4RDNA_OK) return st;
        if (cudaEventRecord(sg.y_ready, c) != cudaSuccess) return Q4RDNA_ERR_CUDA;
        if (!out_copies) continue;
        if (cudaStreamWaitEvent(plan->d2h, sg.y_ready, 0) != cudaSuccess ||
            cudaMemcpyAsync(yh + sg.y_lo, yd + sg.y_lo, sg.y_hi - sg.y_lo, cudaMemcpyDeviceToHost, plan->d2h) !=
                cudaSuccess)
            return Q4RDNA_ERR_CUDA;
    }
    if (out_copies) {
        if (cudaEventRecord(plan->done, plan->d2h) != cudaSuccess || cudaStreamWaitEvent(cs, plan->done, 0) != cudaSuccess)
            return Q4RDNA_ERR_CUDA;
    } else {
        // the last segment of each stream ends that stream's work
        const size_t n = plan->segs.size();
        for (size_t i = n >= 2 ? n - 2 : 0; i < n; ++i)
            if (cudaStreamWaitEvent(cs, plan->segs[i].y_ready, 0) != cudaSuccess) return Q4RDNA_ERR_CUDA;
    }
    return Q4RDNA_OK;
}

}  // namespace

extern "C" {

q4rdna_status q4rdna_plan_run_host(q4rdna_plan *plan, const void *x_host, void *x_dev, size_t x_bytes,
                                   const void *y_dev, void *y_host, size_t y_bytes, int segments,
                                   q4rdna_stream_t stream) {
    if (plan == nullptr || x_host == nullptr || x_dev == nullptr || y_dev == nullptr || y_host == nullptr ||
        segments < 0)
        return Q4RDNA_ERR_INVALID_ARGUMENT;
    if (plan->gather) return Q4RDNA_ERR_UNSUPPORTED;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != plan->device) return Q4RDNA_ERR_DEVICE;
    if (!plan->q4k_host.empty()) {
        // plans with Q4_K tensors: one copy in, the run, one copy out (not overlapped)
        cudaStream_t cs = (cudaStream_t)stream;
        if (cudaMemcpyAsync(x_dev, x_host, x_bytes, cudaMemcpyHostToDevice, cs) != cudaSuccess)
            return Q4RDNA_ERR_CUDA;
        const q4rdna_status st = q4rdna_plan_run(plan, stream);
        if (st != Q4RDNA_OK) return st;
        if (cudaMemcpyAsync(y_host, y_dev, y_bytes, cudaMemcpyDeviceToHost, cs) != cudaSuccess)
            return Q4RDNA_ERR_CUDA;
        return Q4RDNA_OK;
    }
    const int want =
        segments != 0 ? segments : (mapped_output(y_host, y_bytes) != nullptr ? kHostSegmentsDirect : kHostSegments);
    if (plan->seg_request != std::max(1, std::min(want, plan->count)) || !plan->seg_graded || plan->seg_x != x_dev ||
        plan->seg_y != y_dev || plan->seg_yh != y_host) {
        const q4rdna_status st = build_segments(plan, want, static_cast<const uint8_t *>(x_dev), x_bytes,
                                                static_cast<const uint8_t *>(y_dev), y_bytes, true,
                                                static_cast<const uint8_t *>(y_host));
        if (st != Q4RDNA_OK) return st;
    } else {
        for (const auto &sg : plan->segs)
            if (sg.x_hi > x_bytes || sg.y_hi > y_bytes) return Q4RDNA_ERR_INVALID_ARGUMENT;
    }
    if (!host_graph()) {
        return launch_segments(plan, (cudaStream_t)stream, static_cast<const uint8_t *>(x_host),
                               static_cast<uint8_t *>(x_dev), static_cast<const uint8_t *>(y_dev),
                               static_cast<uint8_t *>(y_host));
    }
    // One graph replay per call: a plan of S segments issues about 10 S copies,
    // launches and event operations, which at S = 8 cost more host time than
    // the GPU needs for the whole step.
    auto &hg = plan->hg;
    if (hg.exec == nullptr || hg.xh != x_host || hg.xd != x_dev || hg.yd != y_dev || hg.yh != y_host ||
        hg.xb != x_bytes || hg.yb != y_bytes) {
        if (hg.exec) cudaGraphExecDestroy(hg.exec);
        hg = q4rdna_plan::HostGraph{};
        if (plan->cap == nullptr && cudaStreamCreateWithFlags(&plan->cap, cudaStreamNonBlocking) != cudaSuccess)
            return Q4RDNA_ERR_CUDA;
        if (cudaStreamBeginCapture(plan->cap, cudaStreamCaptureModeRelaxed) != cudaSuccess) return Q4RDNA_ERR_CUDA;
        const uint64_t before = g_launches.load();
        const q4rdna_status st = launch_segments(plan, plan->cap, static_cast<const uint8_t *>(x_host),
                                                 static_cast<uint8_t *>(x_dev), static_cast<const uint8_t *>(y_dev),
                                                 static_cast<uint8_t *>(y_host));
        const uint64_t captured = g_launches.load() - before;
        g_launches.fetch_sub(captured, std::memory_order_relaxed);  // counted per replay below
        cudaGraph_t g = nullptr;
        const cudaError_t ec = cudaStreamEndCapture(plan->cap, &g);
        if (st != Q4RDNA_OK || ec != cudaSuccess || g == nullptr) {
            if (g) cudaGraphDestroy(g);
            cudaGetLastError();
            return st != Q4RDNA_OK ? st : Q4RDNA_ERR_CUDA;
        }
        cudaGraphExec_t ex = nullptr;
        const cudaError_t ei = cudaGraphInstantiate(&ex, g, 0);
        cudaGraphDestroy(g);
        if (ei != cudaSuccess) return Q4RDNA_ERR_CUDA;
        hg.exec = ex;
        hg.xh = x_host; hg.xd = x_dev; hg.yd = y_dev; hg.yh = y_host; hg.xb = x_bytes; hg.yb = y_bytes;
        hg.launches = captured;
    }
    if (cudaGraphLaunch(hg.exec, (cudaStream_t)stream) != cudaSuccess) return Q4RDNA_ERR_CUDA;
    g_launches.fetch_add(hg.launches, std::memory_order_relaxed);
    return Q4RDNA_OK;
}

q4rdna_status q4rdna_plan_set_segments(q4rdna_plan *plan, int segments) {
    if (plan == nullptr || segments < 0) return Q4RDNA_ERR_INVALID_ARGUMENT;
    plan->run_segments = segments == 0 ? 1 : segments;
    return Q4RDNA_OK;
}

int q4rdna_plan_gather_parity(const q4rdna_plan *plan) {
    if (plan == nullptr || !plan->gather || plan->epoch == 0) return -1;
    return (int)(plan->epoch & 1u);
}

q4rdna_status q4rdna_ipc_alloc(size_t bytes, void **dev_ptr, unsigned char handle[Q4RDNA_IPC_HANDLE_BYTES]) {
    if (bytes == 0 || dev_ptr == nullptr || handle == nullptr) return Q4RDNA_ERR_INVALID_ARGUMENT;
    static_assert(sizeof(cudaIpcMemHandle_t) == Q4RDNA_IPC_HANDLE_BYTES, "IPC handle size");
    void *p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return Q4RDNA_ERR_CUDA;
    cudaIpcMemHandle_t h;
    if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaFree(p);
        return Q4RDNA_ERR_CUDA;
    }
    std::memcpy(handle, &h, sizeof(h));
    *dev_ptr = p;
    return Q4RDNA_OK;
}

q4rdna_status q4rdna_ipc_open(const unsigned char handle[Q4RDNA_IPC_HANDLE_BYTES], void **dev_ptr) {
    if (handle == nullptr || dev_ptr == nullptr) return Q4RDNA_ERR_INVALID_ARGUMENT;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void *p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return Q4RDNA_ERR_CUDA;
    *dev_ptr = p;
    return Q4RDNA_OK;
}

q4rdna_status q4rdna_ipc_close(void *dev_ptr) {
    if (dev_ptr == nullptr) return Q4RDNA_ERR_INVALID_ARGUMENT;
    return cudaIpcCloseMemHandle(dev_ptr) == cudaSuccess ? Q4RDNA_OK : Q4RDNA_ERR_CUDA;
}

q4rdna_status q4rdna_ipc_free(void *dev_ptr) {
    if (dev_ptr == nullptr) return Q4RDNA_ERR_INVALID_ARGUMENT;
    return cudaFree(dev_ptr) == cudaSuccess ? Q4RDNA_OK : Q4RDNA_ERR_CUDA;
}

q4rdna_status q4rdna_plan_get_info(const q4rdna_plan *plan, q4rdna_plan_info *info) {
    if (plan == nullptr || info == nullptr) return Q4RDNA_ERR_INVALID_ARGUMENT;
    info->count = plan->count + (int)plan->q4k_host.size();
    info->batch = plan->B;
    info->items = plan->items + plan->q4k_items;
    info->grid = plan->grid;
    info->weight_bytes = plan->weight_bytes;
    info->algo_bytes = plan->algo_bytes;
    info->workspace_bytes = plan->ws_bytes;
    return Q4RDNA_OK;
}

void q4rdna_plan_destroy(q4rdna_plan *plan) {
    if (plan == nullptr) return;
    if (plan->hg.exec) cudaGraphExecDestroy(plan->hg.exec);
    if (plan->cap) cudaStreamDestroy(plan->cap);
    if (plan->table) cudaFree(plan->table);
    if (plan->q4k_table) cudaFree(plan->q4k_table);
    for (auto &sg : plan->segs) {
        if (sg.table) cudaFree(sg.table);
        for (Task *t : sg.gtable)
            if (t) cudaFree(t);
        if (sg.x_ready) cudaEventDestroy(sg.x_ready);
        if (sg.y_ready) cudaEventDestroy(sg.y_ready);
    }
    if (plan->h2d) cudaStreamDestroy(plan->h2d);
    for (cudaStream_t c : plan->comp)
        if (c) cudaStreamDestroy(c);
    if (plan->d2h) cudaStreamDestroy(plan->d2h);
    if (plan->start) cudaEventDestroy(plan->start);
    if (plan->done) cudaEventDestroy(plan->done);
    for (Task *t : plan->gtable)
        if (t) cudaFree(t);
    if (plan->workspace) cudaFree(plan->workspace);
    delete plan;
}

uint64_t q4rdna_launch_count(void) { return g_launches.load() + q4k_launch_count(); }

uint32_t q4rdna_take_fault(void) {
    unsigned v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_fault, sizeof(v)) != cudaSuccess) return 0xffffffffu;
    if (v != 0) cudaMemcpyToSymbol(g_fault, &zero, sizeof(zero));
    return v;
}

}  // extern "C"
