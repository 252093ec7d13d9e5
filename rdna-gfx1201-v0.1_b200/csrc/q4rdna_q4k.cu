// Q4_K GEMV for sm_100a: the tensors that the reference's qkv-fallback scope
// (source/q4rdna.cu:685-691) leaves in llama.cpp's block_q4_K format, and the
// Q4_K GEMV the reference bench times beside its own
// (source/q4rdna_gemv_bench.hip:93-135).
//
// Format (source/q4rdna_cpu_experiment.cpp:17, 102-135): one block holds 256
// weights of one row in 144 bytes: fp16 d, fp16 dmin, 12 bytes of 6-bit
// scales and mins, then 128 quant bytes; byte 16 + 32c + i holds weight
// 64c + i (low nibble) and 64c + 32 + i (high nibble), unsigned.
// weight = d * scale_s * q - dmin * min_s for sub-block s = k / 32.
//
// Kernel (HBM-bound: 4.5 bits per weight):
//   * one CTA of 8 warps owns a work item = 64 rows x one activation column;
//     warp w owns rows 8w .. 8w + 7 of it and streams them in steps of 8
//     blocks (2048 columns).  Lane (bo, j) = (lane / 4, lane % 4) owns block bo
//     of the step and its 32 quant bytes 32j .. 32j + 31, i.e. the two
//     sub-blocks 2j (low nibbles) and 2j + 1 (high nibbles), for every row;
//   * the CTA prepares the step's activations once, in shared memory: per
//     sub-block of 32 it scales x by a power of two so that |x| max lies in
//     [2^22, 2^23), rounds to integers X and stores their bytes 0, 1, 2 as
//     three byte planes (X = L0 + 256 L1 + 65536 L2, L0 and L1 unsigned, L2
//     signed), with the sub-block's scale-back 2^-e and sum of X 2^-e.
//     Double-buffered, one barrier per step;
//   * per row and sub-block the exact integer sums sum q * L are dp4a chains
//     (quant bytes masked to low nibbles, or high nibbles times 16) started on
//     the float bias 1.5 * 2^23, so that each sum reads back as f32 with one
//     subtract; then y += (d * scale * 2^-e) sum q X - (dmin * min) sum X 2^-e;
//   * rows travel to shared memory by cp.async, kAhead rows ahead per warp
//     across step and item boundaries (no registers held by loads in flight,
//     hardware waits only); the 32
//     lane partials of the 8 rows are added by a fixed butterfly, so results
//     do not depend on the grid.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <mutex>
#include <vector>

#include "q4rdna.h"
#include "q4rdna_q4k.h"

namespace q4k {

constexpr int kBlock = 256;
constexpr int kBlockBytes = 144;
constexpr int kWarps = 8;
constexpr int kThreads = 32 * kWarps;
constexpr int kRowsPerWarp = 8;
constexpr int kRowsPerItem = kWarps * kRowsPerWarp;  // 64
constexpr int kStepBlocks = 8;
constexpr int kStepK = kStepBlocks * kBlock;  // 2048 activations per step
constexpr uint32_t kMagicI = 0x4B400000u;     // 1.5 * 2^23
constexpr float kMagicF = 12582912.0f;

struct Launch {
    const Task *table;  // null: the single task `one`
    Task one;
    int ntasks;
    int B;
    long long total_items;
};

// One (item, step) of a CTA's sequence.
struct Cursor {
    int task;
    int b;          // activation column
    int row0;       // first row of the item
    int step;       // 0 .. steps - 1
    int steps;
    long long item;
    bool valid;
};

__device__ __forceinline__ const Task &task_at(const Launch &L, int i) { return L.table ? L.table[i] : L.one; }

__device__ __forceinline__ int find_task(const Launch &L, long long item) {
    int lo = 0, hi = L.ntasks - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (task_at(L, mid).item_begin <= item) lo = mid; else hi = mid - 1;
    }
    return lo;
}

__device__ __forceinline__ Cursor cursor_for(const Launch &L, long long item) {
    Cursor c{};
    c.item = item;
    c.valid = item < L.total_items;
    if (!c.valid) return c;
    c.task = find_task(L, item);
    const Task &T = task_at(L, c.task);
    const long long local = item - T.item_begin;
    c.b = (int)(local % L.B);
    c.row0 = (int)(local / L.B) * kRowsPerItem;
    c.step = 0;
    c.steps = (T.nb + kStepBlocks - 1) / kStepBlocks;
    return c;
}

__device__ __forceinline__ Cursor advance(const Launch &L, const Cursor &c) {
    if (c.step + 1 < c.steps) {
        Cursor n = c;
        ++n.step;
        return n;
    }
    return cursor_for(L, c.item + gridDim.x);
}

// Step buffer: the activation byte planes of 2048 columns and, per sub-block
// pair owned by one lane, (2^-e, sum X 2^-e) of both sub-blocks.
struct __align__(16) Stage {
    uint4 plane[3][128];  // [byte plane][chunk_slot(c)]: 16 columns per chunk c
    float4 us[32];        // lane (bo, j): (2^-e, sum X 2^-e) of sub-blocks 8 bo + 2j, 8 bo + 2j + 1
};

// Chunk c (columns 16c .. 16c + 15 of the step) is stored at slot
// (c % 4) * 32 + c / 4: lane l reads its four chunks 4l .. 4l + 3 at slots
// i * 32 + l, consecutive across the warp (no bank conflicts).
__device__ __forceinline__ int chunk_slot(int c) { return (c & 3) * 32 + (c >> 2); }

__device__ __forceinline__ uint32_t dp4a_uu(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t dp4a_us(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// 16-byte asynchronous copy global -> shared (LDGSTS); valid = false zero-fills
// the destination without reading (gmem must still be a valid address).
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool valid) {
    const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sa), "l"(gmem), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// One row of one step: 8 consecutive blocks, 72 chunks of 16 bytes.
constexpr int kRowChunks = kStepBlocks * kBlockBytes / 16;
// Rows in flight per warp, and ring slots (one more, so that a slot is never
// refilled while its row is being read).
constexpr int kAhead = 4;
constexpr int kSlots = kAhead + 1;

struct RowRegs {
    uint4 h, q0, q1;  // block header; quant bytes 32j .. 32j + 15 and 32j + 16 .. 32j + 31
};

// Where a warp's rows of one (item, step) start: computed once per step, so
// that issuing a row is a multiply-add and three predicated copies.
struct RowStream {
    const uint8_t *base;  // the warp's first row at the step's first block
    long long stride;     // bytes between rows
    int nrows;            // rows of the warp inside the tensor (0 .. kRowsPerWarp)
    int nchunks;          // 16-byte chunks of a row inside the tensor (0 .. kRowChunks)
};

__device__ __forceinline__ RowStream row_stream(const Launch &L, const Cursor &c, int wrow, const uint8_t *safe) {
    RowStream rs{safe, 0, 0, 0};
    if (!c.valid) return rs;
    const Task &T = task_at(L, c.task);
    const int n0 = c.row0 + wrow;
    const int blk0 = c.step * kStepBlocks;
    rs.nrows = max(0, min(kRowsPerWarp, T.N - n0));
    if (rs.nrows == 0) return rs;
    rs.stride = (long long)T.nb * kBlockBytes;
    rs.base = T.w + (long long)n0 * rs.stride + (long long)blk0 * kBlockBytes;
    rs.nchunks = min(kStepBlocks, T.nb - blk0) * (kBlockBytes / 16);
    return rs;
}

// Issue the copies of row `row` of a row stream into a ring slot; rows past
// N, blocks past the row's end and an exhausted cursor are zero-filled, which
// makes them contribute exactly 0 (d = dmin = 0).
__device__ __forceinline__ void issue_row(uint4 *slot, const RowStream &rs, int row, int lane, const uint8_t *safe) {
    const bool rok = row < rs.nrows;
    const uint8_t *base = rs.base + (rok ? row * rs.stride : 0);
#pragma unroll
    for (int r = 0; r < (kRowChunks + 31) / 32; ++r) {
        const int ch = lane + 32 * r;
        if (ch < kRowChunks) {
            const bool ok = rok && ch < rs.nchunks;
            cp_async16(slot + ch, ok ? base + 16 * ch : safe, ok);
        }
    }
}

__device__ __forceinline__ void read_row(RowRegs &r, const uint4 *slot, int bo, int j) {
    const uint4 *b = slot + bo * (kBlockBytes / 16);
    r.h = b[0];
    r.q0 = b[1 + 2 * j];
    r.q1 = b[2 + 2 * j];
}

// Activations of a step: thread t copies columns 8t .. 8t + 7 (zero past K).
__device__ __forceinline__ void issue_x(float4 *xraw, const Launch &L, const Cursor &c, int t) {
    const float *safe = task_at(L, 0).x;
    const float *p = safe;
    bool ok = false;
    if (c.valid) {
        const Task &T = task_at(L, c.task);
        const int k = c.step * kStepK + 8 * t;
        ok = k < T.K;
        if (ok) p = T.x + (size_t)c.b * T.K + k;
    }
    cp_async16(xraw + 2 * t, p, ok);
    cp_async16(xraw + 2 * t + 1, ok ? p + 4 : safe, ok);
}

struct XRegs {
    float4 a, b;
};

// Prepare this thread's 8 columns (a quarter of sub-block t / 4) into st.
__device__ __forceinline__ void prep(Stage &st, const XRegs &v, int t) {
    const float x[8] = {v.a.x, v.a.y, v.a.z, v.a.w, v.b.x, v.b.y, v.b.z, v.b.w};
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(x[i]));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    // biased exponent of the sub-block maximum, clamped so that the scale and
    // its inverse are normal floats; |x| * 2^(149 - eb) < 2^23
    const int eb = max((int)(__float_as_uint(m) >> 23), 27);
    const float s = __uint_as_float((uint32_t)(276 - eb) << 23);  // 2^(149 - eb)
    const float u = __uint_as_float((uint32_t)(eb - 22) << 23);   // 2^(eb - 149)
    int X[8];
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        // rint(x * s) in [-2^23, 2^23 - 1]: byte 2 is then a valid s8 limb
        X[i] = min(__float2int_rn(x[i] * s), 0x7FFFFF);
        sum += X[i];
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    // byte planes: word (X[4h] .. X[4h+3]) of plane p holds byte p of each
    uint32_t pl[3][2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint32_t a = (uint32_t)X[4 * h], b = (uint32_t)X[4 * h + 1];
        const uint32_t c = (uint32_t)X[4 * h + 2], d = (uint32_t)X[4 * h + 3];
        const uint32_t ab0 = __byte_perm(a, b, 0x0040), cd0 = __byte_perm(c, d, 0x0040);  // [a0 b0 . .]
        const uint32_t ab1 = __byte_perm(a, b, 0x0051), cd1 = __byte_perm(c, d, 0x0051);
        const uint32_t ab2 = __byte_perm(a, b, 0x0062), cd2 = __byte_perm(c, d, 0x0062);
        pl[0][h] = __byte_perm(ab0, cd0, 0x5410);
        pl[1][h] = __byte_perm(ab1, cd1, 0x5410);
        pl[2][h] = __byte_perm(ab2, cd2, 0x5410);
    }
    const int slot = chunk_slot(t >> 1);
#pragma unroll
    for (int p = 0; p < 3; ++p)
        reinterpret_cast<uint2 *>(&st.plane[p][slot])[t & 1] = make_uint2(pl[p][0], pl[p][1]);
    if ((t & 3) == 0) {
        const int sb = t >> 2;  // sub-block of the step, 0 .. 63
        reinterpret_cast<float2 *>(&st.us[sb >> 1])[sb & 1] = make_float2(u, (float)sum * u);
    }
}

// Scales and mins of sub-blocks 2j and 2j + 1 from the 12 scale bytes
// (h.y = bytes 0-3, h.z = 4-7, h.w = 8-11), source/q4rdna_cpu_experiment.cpp:102-110:
// j < 2: scale = s[i] & 63, min = s[i + 4] & 63 (i = 2j, 2j + 1);
// j >= 2: scale = (s[i + 4] & 15) | (s[i - 4] >> 6) << 4,
//         min = (s[i + 4] >> 4) | (s[i] >> 6) << 4.
// Both sub-blocks of a lane are adjacent bytes, handled as one 16-bit pair,
// with lane-constant byte selectors, shifts and masks (no per-lane branch).
struct ScaleMin {
    float sc0, sc1, m0, m1;
};

struct ScaleSel {
    uint32_t low;    // prmt selector: the pair's low-part bytes (from h.y / h.z, or from h.w)
    uint32_t high;   // prmt selector: the pair's bytes s[2jj], s[2jj + 1] of a word
    uint32_t mask1;  // 0x3F3F (j < 2) or 0x0F0F
    uint32_t mask2;  // 0 (j < 2) or 0x3030: the two high bits
    uint32_t mshift; // 0 (j < 2) or 4: mins take the high nibbles of h.w
};

__device__ __forceinline__ ScaleSel scale_sel(int j) {
    const uint32_t jj = (uint32_t)(j & 1), lo = j < 2;
    ScaleSel q;
    q.high = (2 * jj) | ((2 * jj + 1) << 4);
    q.low = lo ? q.high : ((4 + 2 * jj) | ((5 + 2 * jj) << 4));
    q.mask1 = lo ? 0x3F3Fu : 0x0F0Fu;
    q.mask2 = lo ? 0u : 0x3030u;
    q.mshift = lo ? 0u : 4u;
    return q;
}

__device__ __forceinline__ ScaleMin scale_min(const uint4 &h, const ScaleSel &q) {
    const uint32_t sc = (__byte_perm(h.y, h.w, q.low) & q.mask1) | ((__byte_perm(h.y, 0u, q.high) >> 2) & q.mask2);
    const uint32_t mn =
        ((__byte_perm(h.z, h.w, q.low) >> q.mshift) & q.mask1) | ((__byte_perm(h.z, 0u, q.high) >> 2) & q.mask2);
    ScaleMin r;
    // byte -> 2^23 + byte as a float, minus 2^23: exact
    r.sc0 = __uint_as_float(__byte_perm(sc, 0x4B000000u, 0x7440)) - 8388608.0f;
    r.sc1 = __uint_as_float(__byte_perm(sc, 0x4B000000u, 0x7441)) - 8388608.0f;
    r.m0 = __uint_as_float(__byte_perm(mn, 0x4B000000u, 0x7440)) - 8388608.0f;
    r.m1 = __uint_as_float(__byte_perm(mn, 0x4B000000u, 0x7441)) - 8388608.0f;
    return r;
}

// Lane's activation planes for one step: lo = columns 64j .. 64j + 31 of its
// block (sub-block 2j), hi = 64j + 32 .. 64j + 63 (sub-block 2j + 1).
struct XPlanes {
    uint32_t lo[3][8], hi[3][8];
    float u0, xs0, u1s, xs1;  // 2^-e and sum X 2^-e of sub-blocks 2j, 2j + 1 (u1s = 2^-e / 16)
};

__device__ __forceinline__ void load_planes(XPlanes &xp, const Stage &st, int lane) {
#pragma unroll
    for (int p = 0; p < 3; ++p) {
        const uint4 c0 = st.plane[p][0 * 32 + lane], c1 = st.plane[p][1 * 32 + lane];
        const uint4 c2 = st.plane[p][2 * 32 + lane], c3 = st.plane[p][3 * 32 + lane];
        xp.lo[p][0] = c0.x; xp.lo[p][1] = c0.y; xp.lo[p][2] = c0.z; xp.lo[p][3] = c0.w;
        xp.lo[p][4] = c1.x; xp.lo[p][5] = c1.y; xp.lo[p][6] = c1.z; xp.lo[p][7] = c1.w;
        xp.hi[p][0] = c2.x; xp.hi[p][1] = c2.y; xp.hi[p][2] = c2.z; xp.hi[p][3] = c2.w;
        xp.hi[p][4] = c3.x; xp.hi[p][5] = c3.y; xp.hi[p][6] = c3.z; xp.hi[p][7] = c3.w;
    }
    const float4 us = st.us[lane];
    xp.u0 = us.x; xp.xs0 = us.y;
    xp.u1s = us.z * 0.0625f; xp.xs1 = us.w;
}

// The lane's contribution of one row to y: both sub-blocks of its quant bytes.
// The lane's contribution of one row to y: both sub-blocks of its quant bytes.
// Per sub-block, S = sum q X comes from the three exact limb sums (each read
// back from the 1.5 * 2^23 bias with one subtract) and is rounded once to f32;
// then y += (d * scale * 2^-e) S - (dmin * min) (sum X 2^-e).  The two terms
// can partly cancel (both grow with the activations, w = d*scale*q - dmin*min
// can be small); the rounding is 2^-24 of each term, a few times
// 2^-24 sum |w x| for any weights, which stays below the activation rounding
// of 2^-24 max|x| per sub-block.
__device__ __forceinline__ float row_dot(const RowRegs &r, const XPlanes &xp, const ScaleSel &ss) {
    const uint32_t q[8] = {r.q0.x, r.q0.y, r.q0.z, r.q0.w, r.q1.x, r.q1.y, r.q1.z, r.q1.w};
    uint32_t a0 = kMagicI, a1 = kMagicI, a2 = kMagicI;  // sub-block 2j, planes 0..2
    uint32_t b0 = kMagicI, b1 = kMagicI, b2 = kMagicI;  // sub-block 2j + 1 (codes x 16)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t lo = q[i] & 0x0F0F0F0Fu, hi = q[i] & 0xF0F0F0F0u;
        a0 = dp4a_uu(lo, xp.lo[0][i], a0);
        a1 = dp4a_uu(lo, xp.lo[1][i], a1);
        a2 = dp4a_us(lo, xp.lo[2][i], a2);
        b0 = dp4a_uu(hi, xp.hi[0][i], b0);
        b1 = dp4a_uu(hi, xp.hi[1][i], b1);
        b2 = dp4a_us(hi, xp.hi[2][i], b2);
    }
    const float sa = fmaf(65536.0f, __uint_as_float(a2) - kMagicF,
                          fmaf(256.0f, __uint_as_float(a1) - kMagicF, __uint_as_float(a0) - kMagicF));
    const float sb = fmaf(65536.0f, __uint_as_float(b2) - kMagicF,
                          fmaf(256.0f, __uint_as_float(b1) - kMagicF, __uint_as_float(b0) - kMagicF));
    const float2 dd = __half22float2(*reinterpret_cast<const __half2 *>(&r.h.x));  // (d, dmin)
    const ScaleMin sm = scale_min(r.h, ss);
    float acc = (dd.x * sm.sc0 * xp.u0) * sa;
    acc = fmaf(dd.x * sm.sc1 * xp.u1s, sb, acc);
    acc = fmaf(-(dd.y * sm.m0), xp.xs0, acc);
    acc = fmaf(-(dd.y * sm.m1), xp.xs1, acc);
    return acc;
}

// Sum of the kRowsPerWarp row partials over the warp in a fixed order: a
// butterfly halves the rows each lane holds, then the lanes that share a row
// add up.  Row r ends in lanes r * kLanesPerRow .. (r + 1) * kLanesPerRow - 1.
constexpr int kLanesPerRow = 32 / kRowsPerWarp;

__device__ __forceinline__ float warp_rows_sum(float (&v)[kRowsPerWarp], int lane) {
    int m = 16;
#pragma unroll
    for (int half = kRowsPerWarp / 2; half >= 1; half >>= 1, m >>= 1) {
        const bool up = (lane & m) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float send = up ? v[i] : v[i + half];
            const float keep = up ? v[i + half] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
        }
    }
    float s = v[0];
#pragma unroll
    for (int o = kLanesPerRow / 2; o >= 1; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    return s;
}

struct __align__(16) Smem {
    Stage stage[2];                                    // activation planes, per step
    float4 xraw[2][2 * kThreads];                      // raw activations of a step
    uint4 ring[kWarps][kSlots][kRowChunks];            // rows in flight, per warp
};

__global__ void __launch_bounds__(kThreads, 2) q4k_gemv_kernel(const __grid_constant__ Launch L) {
    extern __shared__ __align__(16) unsigned char q4k_smem_raw[];
    Smem &sm = *reinterpret_cast<Smem *>(q4k_smem_raw);
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int bo = lane >> 2, j = lane & 3;
    const int wrow = warp * kRowsPerWarp;
    const ScaleSel ssel = scale_sel(j);
    Cursor cur = cursor_for(L, blockIdx.x);
    if (!cur.valid) return;
    uint4(&ring)[kSlots][kRowChunks] = sm.ring[warp];
    const uint8_t *safe = task_at(L, 0).w;  // a valid address for zero-fill copies
    // Prologue: the first step's activations, then the warp's first kAhead rows.
    // Every thread commits one copy group per row it consumes, so that
    // cp.async.wait_group kAhead - 1 before row u means "row u has landed".
    issue_x(sm.xraw[0], L, cur, t);
    cp_async_commit();
    RowStream rs_cur = row_stream(L, cur, wrow, safe);
#pragma unroll
    for (int i = 0; i < kAhead; ++i) {
        issue_row(ring[i], rs_cur, i, lane, safe);
        cp_async_commit();
    }
    cp_async_wait<kAhead>();
    float acc[kRowsPerWarp];
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) acc[i] = 0.f;
    int buf = 0, slot = 0;
    while (cur.valid) {
        {
            const float4 *xr = sm.xraw[buf];
            XRegs xv{xr[2 * t], xr[2 * t + 1]};
            prep(sm.stage[buf], xv, t);
        }
        const Cursor nxt = advance(L, cur);
        const RowStream rs_nxt = row_stream(L, nxt, wrow, safe);
        __syncthreads();
        XPlanes xp;
        load_planes(xp, sm.stage[buf], lane);
#pragma unroll
        for (int i = 0; i < kRowsPerWarp; ++i) {
            cp_async_wait<kAhead - 1>();
            // the row's chunks were copied by all lanes of the warp: after every
            // lane's wait, the barrier makes them visible to each other, and it
            // orders the previous row's reads before this row's refill of that slot
            __syncwarp();
            RowRegs r;
            read_row(r, ring[slot], bo, j);
            // refill: kAhead rows ahead, in this step or the next (step or item)
            const int fill = slot + kAhead < kSlots ? slot + kAhead : slot + kAhead - kSlots;
            if (i + kAhead < kRowsPerWarp) issue_row(ring[fill], rs_cur, i + kAhead, lane, safe);
            else issue_row(ring[fill], rs_nxt, i + kAhead - kRowsPerWarp, lane, safe);
            // the next step's activations travel with the first row's group
            if (i == 0) issue_x(sm.xraw[buf ^ 1], L, nxt, t);
            cp_async_commit();
            slot = slot + 1 < kSlots ? slot + 1 : 0;
            acc[i] += row_dot(r, xp, ssel);
        }
        if (cur.step + 1 == cur.steps) {
            const Task &T = task_at(L, cur.task);
            const float v = warp_rows_sum(acc, lane);
            const int n = cur.row0 + wrow + lane / kLanesPerRow;
            if (lane % kLanesPerRow == 0 && n < T.N) {
                float out = v;
                if (T.op == Q4RDNA_OP_ADD) out += T.add[(size_t)cur.b * T.N + n];
                T.y[(size_t)cur.b * T.N + n] = out;
            }
#pragma unroll
            for (int i = 0; i < kRowsPerWarp; ++i) acc[i] = 0.f;
        }
        cur = nxt;
        rs_cur = rs_nxt;
        buf ^= 1;
    }
    cp_async_wait<0>();
}

// Dense W[N][K], one thread per weight of a block (debug and parity).
__global__ void q4k_dequant_kernel(const uint8_t *blocks, float *W, int nb) {
    const long long blk = blockIdx.x;  // row * nb + block
    const int i = threadIdx.x, c = i >> 6, w = i & 63;
    const uint8_t *p = blocks + blk * kBlockBytes;
    const float d = __half2float(*reinterpret_cast<const __half *>(p));
    const float dmin = __half2float(*reinterpret_cast<const __half *>(p + 2));
    const int idx = 2 * c + (w >> 5);
    const uint8_t *s = p + 4;
    int sc, mn;
    if (idx < 4) {
        sc = s[idx] & 63;
        mn = s[idx + 4] & 63;
    } else {
        sc = (s[idx + 4] & 15) | ((s[idx - 4] >> 6) << 4);
        mn = (s[idx + 4] >> 4) | ((s[idx] >> 6) << 4);
    }
    const uint8_t qb = p[16 + 32 * c + (w & 31)];
    const int q = (w < 32) ? (qb & 15) : (qb >> 4);
    // d * scale * q is exact; the subtraction is the only rounding, as in the reference
    W[blk * kBlock + i] = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)mn));
}

// ---- host side ----

int device_sms_occ(int *sms) {
    static std::mutex mu;
    static std::vector<std::pair<int, int>> cache;  // per device: (sms, CTAs per SM)
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    std::lock_guard<std::mutex> lock(mu);
    if ((int)cache.size() <= dev) cache.resize(dev + 1, {0, 0});
    if (cache[dev].first == 0) {
        int n = 0, occ = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
        if (cudaFuncSetAttribute(q4k_gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(Smem)) !=
            cudaSuccess)
            return 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, q4k_gemv_kernel, kThreads, sizeof(Smem)) !=
            cudaSuccess)
            return 0;
        cache[dev] = {n, std::max(occ, 1)};
    }
    *sms = cache[dev].first;
    return cache[dev].second;
}

bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

}  // namespace q4k

namespace q4k_host {
std::atomic<unsigned long long> g_q4k_launches{0};
}

q4rdna_status q4k_build_task(const q4rdna_gemv_desc &e, int B, long long item_begin, q4k::Task &T, long long &items) {
    if (e.N <= 0 || e.K <= 0 || e.K % q4k::kBlock != 0) return Q4RDNA_ERR_SHAPE;
    if (B < 1 || B > Q4RDNA_MAX_BATCH) return Q4RDNA_ERR_UNSUPPORTED;
    if (e.op != Q4RDNA_OP_PLAIN && e.op != Q4RDNA_OP_ADD) return Q4RDNA_ERR_UNSUPPORTED;
    if (e.norm_weight != nullptr || e.gate_tiles != nullptr) return Q4RDNA_ERR_UNSUPPORTED;
    if (e.tiles == nullptr || e.x == nullptr || e.y == nullptr) return Q4RDNA_ERR_INVALID_ARGUMENT;
    if (e.op == Q4RDNA_OP_ADD && e.add == nullptr) return Q4RDNA_ERR_INVALID_ARGUMENT;
    if (!q4k::aligned(e.tiles, 16) || !q4k::aligned(e.x, 16) || !q4k::aligned(e.y, 4) ||
        (e.add && !q4k::aligned(e.add, 4)))
        return Q4RDNA_ERR_ALIGNMENT;
    T = q4k::Task{};
    T.w = e.tiles; T.x = e.x; T.add = e.op == Q4RDNA_OP_ADD ? e.add : nullptr; T.y = e.y;
    T.N = e.N; T.K = e.K; T.nb = e.K / q4k::kBlock; T.op = e.op;
    T.item_begin = item_begin;
    T.row_items = (e.N + q4k::kRowsPerItem - 1) / q4k::kRowsPerItem;
    items = (long long)T.row_items * B;
    return Q4RDNA_OK;
}

q4rdna_status q4k_launch_tasks(const q4k::Task *table, const q4k::Task *one, int ntasks, int B, long long items,
                               cudaStream_t stream) {
    if (items <= 0) return Q4RDNA_OK;
    int sms = 0;
    const int occ = q4k::device_sms_occ(&sms);
    if (occ == 0) return Q4RDNA_ERR_DEVICE;
    q4k::Launch L{};
    L.table = table;
    if (one) L.one = *one;
    L.ntasks = ntasks;
    L.B = B;
    L.total_items = items;
    const long long grid = std::min<long long>(items, (long long)sms * occ);
    void *args[] = {&L};
    if (cudaLaunchKernel((const void *)q4k::q4k_gemv_kernel, dim3((unsigned)grid), dim3(q4k::kThreads), args,
                         sizeof(q4k::Smem), stream) != cudaSuccess)
        return Q4RDNA_ERR_CUDA;
    if (cudaGetLastError() != cudaSuccess) return Q4RDNA_ERR_CUDA;
    q4k_host::g_q4k_launches.fetch_add(1, std::memory_order_relaxed);
    return Q4RDNA_OK;
}

unsigned long long q4k_launch_count() { return q4k_host::g_q4k_launches.load(std::memory_order_relaxed); }

extern "C" {

size_t q4rdna_q4k_bytes(int N, int K) {
    if (N <= 0 || K <= 0 || K % q4k::kBlock != 0) return 0;
    return (size_t)N * (K / q4k::kBlock) * q4k::kBlockBytes;
}

q4rdna_status q4rdna_q4k_gemv(const uint8_t *blocks, const float *x, const float *add, float *y, int N, int K, int B,
                              q4rdna_stream_t stream) {
    q4rdna_gemv_desc e{};
    e.tiles = blocks; e.x = x; e.add = add; e.y = y; e.N = N; e.K = K;
    e.op = add != nullptr ? Q4RDNA_OP_ADD : Q4RDNA_OP_PLAIN;
    q4k::Task T;
    long long items = 0;
    const q4rdna_status st = q4k_build_task(e, B, 0, T, items);
    if (st != Q4RDNA_OK) return st;
    return q4k_launch_tasks(nullptr, &T, 1, B, items, (cudaStream_t)stream);
}

q4rdna_status q4rdna_q4k_dequant_f32(const uint8_t *blocks, float *W, int N, int K, q4rdna_stream_t stream) {
    if (blocks == nullptr || W == nullptr) return Q4RDNA_ERR_INVALID_ARGUMENT;
    if (N <= 0 || K <= 0 || K % q4k::kBlock != 0) return Q4RDNA_ERR_SHAPE;
    const long long n = (long long)N * (K / q4k::kBlock);
    if (n > 0x7fffffffLL) return Q4RDNA_ERR_TOO_LARGE;
    q4k::q4k_dequant_kernel<<<(unsigned)n, q4k::kBlock, 0, (cudaStream_t)stream>>>(blocks, W, K / q4k::kBlock);
    if (cudaGetLastError() != cudaSuccess) return Q4RDNA_ERR_CUDA;
    q4k_host::g_q4k_launches.fetch_add(1, std::memory_order_relaxed);
    return Q4RDNA_OK;
}

}  // extern "C"
