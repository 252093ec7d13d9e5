// Q4_RDNA group-64 GEMV for B200 (sm_100a): shared device helpers, the plan /
// single-call host side, and the fused tensor-parallel gather.
//
// The kernels live in the headers included below:
//   q4rdna_gemv_i8.cuh  the int8 group math for B = 1..2: a warp streams the four
//                       32-row tiles of a 128-row block with 128-bit loads into
//                       a register pipeline; int8 tensor-core MMAs (mma.sync
//                       m16n8k32) sum each group exactly;
//   q4rdna_gemv_cta.cuh B = 1..2, single calls and plans: one CTA item = 128 rows
//                       x a K-range split again over the CTA's 8 warps;
//   q4rdna_gemv_mb.cuh  B = 3..16: the tile path, one CTA work item of 128 rows,
//                       the full m16n8k32 fragment over the batch columns.
// Both scale each 64-element activation group by a power of two, round it to
// an integer X (|X| <= 2^30) and feed its four balanced base-256 digits to the
// int8 MMAs; the fp16 group scale is applied once per (row, group) in f32, as
// the reference does (source/q4rdna.cu:370-371).  Split-K partial sums go to a
// workspace; the last warp (or CTA) to finish a row block (arrival ticket) adds
// them in split order and applies the add / SwiGLU epilogue, so results are
// deterministic.
//
// Accumulation order of an output: exact int32 inside a group; groups of one
// split in ascending order, sum = fma(scale / 16, v * 2^e, sum) with v the
// recombined digit sums; splits in ascending split order in f32.
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
#include <type_traits>
#include <new>
#include <vector>

#include "q4rdna.h"
#include "q4rdna_q4k.h"
#include "q4rdna_tile.h"

namespace q4 {

constexpr int kWarps = 8;             // warps per CTA
constexpr int kThreads = kWarps * 32;

constexpr int kMaxWorld = 8;    // GPUs of one box
constexpr int kMaxMirrors = kMaxWorld + 1;  // every rank's gathered buffer + a host-mapped output (run_host)

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
    // tensor-core tile path (B >= kTcMinBatch, q4rdna_gemv_tc.cuh)
    uint8_t *img;       // the prepared activation: one operand image per chunk of 4 groups
    float *csum;        // fused RMSNorm: sum of h^2 per [chunk][BP]
    long long chunk_begin;  // first prep-kernel CTA of this task
    int rbi;            // row blocks per work item (2 on the tile path without SwiGLU, else 1)
    int pad3;
};

struct Launch {
    const Task *table;  // device array of ntasks tasks, or null: use `one`
    Task one;
    int ntasks;
    int B;
    long long total_items;
    long long total_chunks;  // tensor-core tile path: prep-kernel CTAs
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

__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
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

__device__ __forceinline__ const Task &find_task(const Launch &L, long long item) {
    if (L.table == nullptr) return L.one;
    int lo = 0, hi = L.ntasks - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (L.table[mid].item_begin <= item) lo = mid; else hi = mid - 1;
    }
    return L.table[lo];
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

// Device-side fault flags, read and cleared by q4rdna_take_fault (bit 1: a fused
// gather stopped waiting for a peer's flag).
__device__ unsigned int g_fault;

#include "q4rdna_gemv_i8.cuh"
#include "q4rdna_gemv_cta.cuh"
#include "q4rdna_gemv_mb.cuh"
#include "q4rdna_gemv_tc.cuh"

// ------------------------------------------------------------------ host side

constexpr int kMaxDevices = 64;
constexpr int kTileMinBatch = 3;  // B >= 3 runs on the tile path (q4rdna_gemv_mb.cuh)
constexpr int kTcMinBatch = 8;    // B >= 8: the tensor-core tile path (q4rdna_gemv_tc.cuh)
std::atomic<uint64_t> g_launches{0};

struct KernelCfg {
    const void *fn;
    int threads;
};

// Tile-path launch class: 0 -> B = 3..8 (BP = 8), 1 -> B = 9..16 (BP = 16).
int tile_class(int pb) { return pb <= 8 ? 0 : 1; }

template <bool NORM>
KernelCfg mb_cfg_n(int pb, bool dual) {
    if (pb <= 8)
        return dual ? KernelCfg{(const void *)q4_gemv_mb_kernel<8, true, NORM>, kMbThreads}
                    : KernelCfg{(const void *)q4_gemv_mb_kernel<8, false, NORM>, kMbThreads};
    return dual ? KernelCfg{(const void *)q4_gemv_mb_kernel<16, true, NORM>, kMbThreads}
                : KernelCfg{(const void *)q4_gemv_mb_kernel<16, false, NORM>, kMbThreads};
}

// The tile path (B >= 3).  dual: the launch holds a SwiGLU task; norm: a
// fused-RMSNorm task.  Kernels compiled without those paths need fewer
// registers.  Occupancy and grids are taken from the kernels without a norm
// (the norm kernels use the same registers +- 5).
KernelCfg tile_cfg(int pb, bool dual = true, bool norm = false) {
    return norm ? mb_cfg_n<true>(pb, dual) : mb_cfg_n<false>(pb, dual);
}

// The CTA-split kernel (B = 1..2); cl: the clustered single-call variant.
template <bool NORM, bool CL>
const void *cta_kernel_n(int pb, bool dual) {
    if (pb <= 1)
        return dual ? (const void *)q4_gemv_cta_kernel<1, true, NORM, CL>
                    : (const void *)q4_gemv_cta_kernel<1, false, NORM, CL>;
    return dual ? (const void *)q4_gemv_cta_kernel<2, true, NORM, CL> : (const void *)q4_gemv_cta_kernel<2, false, NORM, CL>;
}
const void *cta_kernel(int pb, bool dual, bool norm, bool cl = false) {
    if (cl) return norm ? cta_kernel_n<true, true>(pb, dual) : cta_kernel_n<false, true>(pb, dual);
    return norm ? cta_kernel_n<true, false>(pb, dual) : cta_kernel_n<false, false>(pb, dual);
}

struct DeviceInfo {
    int sms = 0;
    int occ_tile[2][2] = {};  // tile path: resident CTAs per SM by tile class, SwiGLU (0: unknown)
    int occ_cta[2][2] = {};   // CTA-split kernel: by B - 1, SwiGLU
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
    for (int i = 0; i < 2; ++i)
        for (int du = 0; du < 2; ++du) {
            int o = 0;
            if (d.occ_tile[i][du] == 0) {
                const KernelCfg k = tile_cfg(i == 0 ? 8 : 16, du != 0);
                if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, k.fn, k.threads, 0) != cudaSuccess) return false;
                d.occ_tile[i][du] = std::max(o, 1);
            }
            if (d.occ_cta[i][du] == 0) {
                if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, cta_kernel(i + 1, du != 0, false), kThreads, 0) !=
                    cudaSuccess)
                    return false;
                d.occ_cta[i][du] = std::max(o, 1);
            }
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

// Tensor-core tile path: K-ranges of whole chunks (Gs a multiple of kTcCG), so
// that every range starts at a chunk of the prepared activation.
int tc_chunks(int G) { return (G + kTcCG - 1) / kTcCG; }
Split make_split_tc(int G, int requested) {
    const int nch = tc_chunks(G);
    requested = std::max(1, std::min(requested, nch));
    const int Gs = (nch + requested - 1) / requested * kTcCG;
    return Split{(G + Gs - 1) / Gs, Gs};
}
Split split_of(int G, int requested, int B) {
    return B >= kTcMinBatch ? make_split_tc(G, requested) : make_split(G, requested);
}

// Row blocks per work item: two on the tensor-core tile path (one with SwiGLU,
// whose up and gate tiles fill the item's two A-blocks), else one.
int rows_per_item(int B, int op) { return B >= kTcMinBatch && op != Q4RDNA_OP_SWIGLU ? 2 : 1; }
long long task_items(const Task &T) { return (long long)((T.RB + T.rbi - 1) / T.rbi) * T.S; }

// CTAs resident at once: the CTA-split kernel (B = 1..2), the tensor-core
// tile path (one CTA per SM) or the mma.sync tile path.
long long resident_ctas(int pb, bool dual, const DeviceInfo &d) {
    if (pb < kTileMinBatch) return (long long)d.sms * d.occ_cta[pb - 1][dual];
    if (pb >= kTcMinBatch) return d.sms;
    return (long long)d.sms * d.occ_tile[tile_class(pb)][dual];
}

// K-ranges per tensor for a B = 1..2 launch of RB row blocks in total on the
// CTA-split kernel: as many as fit in ONE wave of resident CTAs
// (RB * S <= SMs x CTAs per SM), but at least one group per warp (S <= G / 8).
// Measured on B200 (bench.py --single --single-sweep, B = 1, split 1..16, us
// per call), this rule picks the best split within 2% on every config shape:
// 4096x4096 S = 8 (6.9 us; best 6.8 at S = 4), 12288x4096 S = 3 (9.9 us, the
// best), 4096x12288 S = 9 (10.3 us; best 10.1 at S = 8), 1024x4096 S = 8
// (5.5 us; best 5.4), gate+up 12288x4096 S = 3 (14.1 us, the best).  A second
// wave costs up to 50%: 12288x4096 at S = 4 (384 CTAs) 12.6 us, 4096x12288 at
// S = 10 (320 CTAs) 15.1 us.
int cta_split(long long total_rb, int G, long long ctas) {
    const long long S = std::min<long long>(total_rb > 0 ? ctas / total_rb : 1, std::max(1, G / kWarps));
    return (int)std::max<long long>(S, 1);
}

// Clusters of S CTA-split CTAs (a single call's row blocks) resident at once,
// from cudaOccupancyMaxActiveClusters; cached per device, batch, SwiGLU and S.
int active_clusters(int pb, bool dual, int S) {
    static std::mutex mu;
    static int cache[kMaxDevices][2][2][kMaxClusterSplit + 1] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices || S < 2 || S > kMaxClusterSplit) return 0;
    std::lock_guard<std::mutex> lock(mu);
    int &c = cache[dev][pb > 1][dual][S];
    if (c == 0) {
        cudaLaunchConfig_t lc = {};
        lc.gridDim = dim3((unsigned)S * 64);
        lc.blockDim = dim3(kThreads);
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = (unsigned)S;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        lc.attrs = at;
        lc.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, cta_kernel(pb, dual, false, true), &lc) != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
        c = std::max(n, -1);  // -1: no cluster of this size fits
        if (c == 0) c = -1;
    }
    return std::max(c, 0);
}

// Selector of single calls at B = 1..2: the one-wave rule above with at most
// kMaxClusterSplit K-ranges, so that the call runs as clusters (one per row
// block), lowered until all the row blocks' clusters are resident at once.
// Measured on B200 (bench.py --single --single-sweep, us per call): 12288x4096
// runs 9.4 us at S = 2 and 13.2 us at S = 3, where 96 clusters of 3 no longer
// fit in one wave; on the tile path (B = 3..16) about one item per resident CTA.
int select_split_for(int N, int K, int B, int op, const DeviceInfo &d) {
    const int G = K / Q4_GROUP;
    const int RB = (N + Q4_BLOCK_ROWS - 1) / Q4_BLOCK_ROWS;
    const bool dual = op == Q4RDNA_OP_SWIGLU;
    const long long ctas = resident_ctas(B, dual, d);
    if (B < kTileMinBatch) {
        for (int req = std::min(cta_split(RB, G, ctas), kMaxClusterSplit); req > 1; --req) {
            const int S = make_split(G, req).S;
            if (S > 1 && S <= kMaxClusterSplit && RB <= active_clusters(B, dual, S)) return S;
        }
        return 1;
    }
    if (B >= kTcMinBatch) {  // about one item per SM
        const long long items = (RB + rows_per_item(B, op) - 1) / rows_per_item(B, op);
        return make_split_tc(G, (int)std::min<long long>((ctas + items - 1) / items, G)).S;
    }
    const long long S = (ctas + RB - 1) / RB;
    return make_split(G, (int)std::min<long long>(S, G)).S;
}

Split resolve(int N, int K, int B, int op, const q4rdna_cfg *cfg, const DeviceInfo &d) {
    const int G = K / Q4_GROUP;
    int req = cfg != nullptr && cfg->split > 0 ? cfg->split : env_split();
    if (req <= 0) req = select_split_for(N, K, B, op, d);
    if (N > (int)(65536 / sizeof(unsigned)) * Q4_BLOCK_ROWS) req = 1;
    return split_of(G, req, B);
}
int resolve_split(int N, int K, int B, int op, const q4rdna_cfg *cfg, const DeviceInfo &d) {
    return resolve(N, K, B, op, cfg, d).S;
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

// Tensor-core tile path: the prepared activation of one task (operand images
// of every chunk, then the RMSNorm chunk sums when `norm`).
int tc_bp(int pb) { return pb <= 8 ? 8 : 16; }
size_t tc_img_bytes(int K, int pb) {
    return align256((size_t)tc_chunks(K / Q4_GROUP) * (tc_bp(pb) == 8 ? Tc<8>::CHUNK : Tc<16>::CHUNK));
}
size_t tc_prep_bytes(int K, int pb, bool norm) {
    return tc_img_bytes(K, pb) + (norm ? align256((size_t)tc_chunks(K / Q4_GROUP) * tc_bp(pb) * sizeof(float)) : 0);
}

// Workspace of one q4rdna_gemv* call: ticket area + partials + the RMSNorm sums
// (reserved for every call, so one size query serves both; nothing when S == 1),
// then, on the tensor-core tile path, the prepared activation -- after the
// ticket area even when S == 1, so that no call writes over the tickets.
size_t ws_split_bytes(int N, int B, int S, int op) {
    return S <= 1 ? 0 : kTicketArea + partial_bytes(N, B, S, op) + sumsq_bytes(N, B, S);
}
size_t ws_prep_offset(int N, int B, int S, int op) {
    return align256(S <= 1 ? kTicketArea : ws_split_bytes(N, B, S, op));
}
// A single call at B < kTileMinBatch with 2..kMaxClusterSplit K-ranges runs
// as thread-block clusters that add their K-ranges in distributed shared
// memory (launch_cta): no tickets, no partial sums, no workspace.
bool cluster_call(int B, int S) { return B < kTileMinBatch && S > 1 && S <= kMaxClusterSplit; }

size_t ws_bytes_for(int N, int K, int B, int S, int op) {
    if (cluster_call(B, S)) return 0;
    if (B < kTcMinBatch) return ws_split_bytes(N, B, S, op);
    return ws_prep_offset(N, B, S, op) + tc_prep_bytes(K, B, true);
}

// Workspace of one plan task: its own tickets + partials (+ RMSNorm sums), fixed
// for the plan's life; on the tensor-core tile path the prepared activation
// follows.
size_t plan_split_bytes(int N, int B, int S, int op, bool norm) {
    if (S <= 1) return 0;
    const int RB = (N + Q4_BLOCK_ROWS - 1) / Q4_BLOCK_ROWS;
    return align256((size_t)RB * sizeof(unsigned)) + align256(partial_bytes(N, B, S, op)) +
           (norm ? align256(sumsq_bytes(N, B, S)) : 0);
}
size_t plan_ws_bytes_for(int N, int K, int B, int S, int op, bool norm) {
    return plan_split_bytes(N, B, S, op, norm) + (B >= kTcMinBatch ? tc_prep_bytes(K, B, norm) : 0);
}

// Work items per resident CTA that a tile-path plan's split-K choice aims at
// (every split costs partial stores, a fence, an arrival ticket and a
// reduction per item).
constexpr double kPlanItemsPerWorker = 2.0;

bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

q4rdna_status check_shape(int N, int K, int B) {
    if (N <= 0 || K <= 0) return Q4RDNA_ERR_INVALID_ARGUMENT;
    if (N % Q4_TILE_ROWS != 0 || K % Q4_GROUP != 0) return Q4RDNA_ERR_SHAPE;
    if (B < 1 || B > Q4RDNA_MAX_BATCH) return Q4RDNA_ERR_UNSUPPORTED;
    return Q4RDNA_OK;
}

// Persistent grid of a tile-path launch: one CTA per item up to the resident CTAs.
int grid_for(long long items, int pb, bool dual, const DeviceInfo &d) {
    return (int)std::max<long long>(1, std::min(items, resident_ctas(pb, dual, d)));
}

// pb: batch columns of the launch (3..16).
q4rdna_status launch(const Launch &L, int grid, int pb, bool dual, cudaStream_t stream, bool norm = false) {
    const KernelCfg k = tile_cfg(pb, dual, norm);
    Launch arg = L;
    void *args[] = {&arg};
    if (cudaLaunchKernel(k.fn, dim3(grid), dim3(k.threads), args, 0, stream) != cudaSuccess)
        return Q4RDNA_ERR_CUDA;
    if (cudaGetLastError() != cudaSuccess) return Q4RDNA_ERR_CUDA;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return Q4RDNA_OK;
}

// The CTA-split kernel (q4rdna_gemv_cta.cuh, B = 1..2): one CTA per item of
// L (total_items CTAs); overlap: programmatic dependent launch.
q4rdna_status launch_cta(const Launch &L, int pb, bool dual, bool norm, cudaStream_t stream, bool overlap = false) {
    Launch arg = L;
    void *args[] = {&arg};
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)L.total_items);
    lc.blockDim = dim3(kThreads);
    lc.stream = stream;
    cudaLaunchAttribute at[2];
    int na = 0;
    if (overlap) {
        at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    // a single call with 2..8 K-ranges: one cluster of S CTAs per row block
    const bool cl = L.table == nullptr && L.one.S > 1 && L.one.S <= kMaxClusterSplit;
    if (cl) {
        at[na].id = cudaLaunchAttributeClusterDimension;
        at[na].val.clusterDim.x = (unsigned)L.one.S;
        at[na].val.clusterDim.y = 1;
        at[na].val.clusterDim.z = 1;
        ++na;
    }
    lc.attrs = na > 0 ? at : nullptr;
    lc.numAttrs = na;
    if (cudaLaunchKernelExC(&lc, cta_kernel(pb, dual, norm, cl), args) != cudaSuccess) return Q4RDNA_ERR_CUDA;
    if (cudaGetLastError() != cudaSuccess) return Q4RDNA_ERR_CUDA;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return Q4RDNA_OK;
}

// The tensor-core tile path: q4_tc_prep_kernel over L's chunks, then the
// persistent q4_tc_gemv_kernel (one CTA per SM), launched as a programmatic
// dependent of the prep kernel so that its weight copies start while the prep
// kernel finishes.  overlap: the prep kernel is itself a programmatic
// dependent of the previous kernel of the stream.
template <int BP>
const void *tc_gemv_fn(bool dual) {
    return dual ? (const void *)q4_tc_gemv_kernel<BP, true> : (const void *)q4_tc_gemv_kernel<BP, false>;
}

bool tc_attributes() {
    static std::mutex mu;
    static bool done[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return false;
    std::lock_guard<std::mutex> lock(mu);
    if (done[dev]) return true;
    for (int dual = 0; dual < 2; ++dual) {
        if (cudaFuncSetAttribute(tc_gemv_fn<8>(dual != 0), cudaFuncAttributeMaxDynamicSharedMemorySize, Tc<8>::SMEM) !=
                cudaSuccess ||
            cudaFuncSetAttribute(tc_gemv_fn<16>(dual != 0), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 Tc<16>::SMEM) != cudaSuccess)
            return false;
    }
    done[dev] = true;
    return true;
}

q4rdna_status launch_tc(const Launch &L, int pb, bool dual, cudaStream_t stream, bool overlap = false) {
    DeviceInfo d;
    if (!device_info(d)) return Q4RDNA_ERR_DEVICE;
    if (!tc_attributes()) return Q4RDNA_ERR_CUDA;
    if (L.total_items <= 0 || L.total_chunks <= 0) return Q4RDNA_ERR_INVALID_ARGUMENT;
    const int bp = tc_bp(pb);
    Launch arg = L;
    void *args[] = {&arg};
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t pc = {};
    pc.gridDim = dim3((unsigned)L.total_chunks);
    pc.blockDim = dim3(128);
    pc.stream = stream;
    if (overlap) {
        pc.attrs = at;
        pc.numAttrs = 1;
    }
    const void *prep = bp == 8 ? (const void *)q4_tc_prep_kernel<8> : (const void *)q4_tc_prep_kernel<16>;
    if (cudaLaunchKernelExC(&pc, prep, args) != cudaSuccess) return Q4RDNA_ERR_CUDA;
    cudaLaunchConfig_t mc = {};
    mc.gridDim = dim3((unsigned)std::min<long long>(L.total_items, d.sms));
    mc.blockDim = dim3(kTcThreads);
    mc.dynamicSmemBytes = bp == 8 ? Tc<8>::SMEM : Tc<16>::SMEM;
    mc.stream = stream;
    mc.attrs = at;
    mc.numAttrs = 1;
    if (cudaLaunchKernelExC(&mc, bp == 8 ? tc_gemv_fn<8>(dual) : tc_gemv_fn<16>(dual), args) != cudaSuccess)
        return Q4RDNA_ERR_CUDA;
    if (cudaGetLastError() != cudaSuccess) return Q4RDNA_ERR_CUDA;
    g_launches.fetch_add(2, std::memory_order_relaxed);
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
    DeviceInfo d;
    if (!device_info(d)) return Q4RDNA_ERR_DEVICE;
    const int G = K / Q4_GROUP;
    const int RB = (N + Q4_BLOCK_ROWS - 1) / Q4_BLOCK_ROWS;
    Split sp = resolve(N, K, B, op, cfg, d);
    if (N > kMaxSplitRows) sp = split_of(G, 1, B);  // beyond the ticket area: no split
    const bool tc = B >= kTcMinBatch;
    unsigned *ticket = nullptr;
    float *part = nullptr;
    uint8_t *prep = nullptr;
    if ((sp.S > 1 && !cluster_call(B, sp.S)) || tc) {
        const size_t need = ws_bytes_for(N, K, B, sp.S, op);
        if (ws == nullptr || ws_bytes < need || !aligned(ws, 256)) return Q4RDNA_ERR_WORKSPACE;
        if (sp.S > 1) {
            ticket = static_cast<unsigned *>(ws);
            part = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + kTicketArea);
        }
        if (tc) prep = static_cast<uint8_t *>(ws) + ws_prep_offset(N, B, sp.S, op);
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
    T.rbi = rows_per_item(B, op);
    T.chunk_begin = 0;
    T.img = prep;
    T.csum = (tc && gn != nullptr) ? reinterpret_cast<float *>(prep + tc_img_bytes(K, B)) : nullptr;
    L.total_items = task_items(T);
    L.total_chunks = tc_chunks(G);
    const bool dual = op == Q4RDNA_OP_SWIGLU;
    if (tc)
        return launch_tc(L, B, dual, stream, cfg != nullptr && (cfg->flags & Q4RDNA_CFG_OVERLAP_PREVIOUS));
    if (B < kTileMinBatch)  // one CTA per (row block, K-range) (q4rdna_gemv_cta.cuh)
        return launch_cta(L, B, dual, gn != nullptr, stream,
                          cfg != nullptr && (cfg->flags & Q4RDNA_CFG_OVERLAP_PREVIOUS));
    return launch(L, grid_for(L.total_items, B, dual, d), B, dual, stream, gn != nullptr);
}

}  // namespace q4

using namespace q4;

// Flag exchange that closes a fused gather: after the plan kernel (stream
// order), lane p raises this rank's flag at rank p, then waits, bounded, for
// rank p's flag of this epoch here.
struct GatherSignal {
    uint32_t *peer[kMaxWorld];    // every rank's flag array, as mapped in this process
    uint32_t *local;              // this rank's flag array
    int world, rank;
    uint32_t epoch;
    int tries;                    // flag polls before the wait gives up (~0.5 us each)
};
constexpr int kGatherTries = 1 << 22;  // x ~0.5 us sleep: about 2 s
constexpr unsigned kFaultGatherTimeout = 2u;

__global__ void q4_gather_signal_kernel(const __grid_constant__ GatherSignal a) {
    // the next plan, when launched with programmatic dependent launch, may start
    // streaming its weights now; it reads nothing else before this kernel ends
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int p = threadIdx.x;
    if (p >= a.world) return;
    // the plan kernel's stores (peer ones included) precede this kernel in stream
    // order; the system-scope fence orders them before the flag for the peers
    __threadfence_system();
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.peer[p] + a.rank), "r"(a.epoch) : "memory");
    int i = 0;
    for (; i < a.tries; ++i) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a.local + p) : "memory");
        if ((int)(v - a.epoch) >= 0) break;
        __nanosleep(500);
    }
    if (i == a.tries) atomicOr(&g_fault, kFaultGatherTimeout);
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

// Kernels whose output stores suit a mapped host buffer: the CTA-split kernel
// (B = 1..2) and the tensor-core tile path (B >= 8) store whole 128-byte runs
// of a row block; the mma.sync tile path (B = 3..7) stores 4-byte scattered
// values, which cost one PCIe transaction each (e2e 7.3 ms at B = 4 against
// 1.45 ms on the device), so it keeps the output copies.
bool direct_batch(int B) { return B < kTileMinBatch || B >= kTcMinBatch; }

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
    long long items = 0, chunks = 0;
    for (Task &T : t) {
        T.item_begin = items;
        items += task_items(T);
        T.chunk_begin = chunks;
        chunks += tc_chunks(T.G);
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
    bool cta = false;   // B = 1..2: the CTA-split kernel (one CTA per item), else the tile path
    bool tc = false;    // B >= kTcMinBatch: the tensor-core tile path (prep kernel + GEMV kernel)
    long long chunks = 0;  // tensor-core tile path: chunks of all tasks (prep-kernel CTAs)
    bool overlap = false;  // q4rdna_plan_set_flags(Q4RDNA_CFG_OVERLAP_PREVIOUS): programmatic dependent launch
    long long items = 0;
    Task *table = nullptr;     // device
    void *workspace = nullptr; // device
    size_t ws_bytes = 0;
    uint64_t weight_bytes = 0, algo_bytes = 0;
    std::vector<Task> host;    // task table as uploaded (no gather)
    // q4rdna_plan_run_host: consecutive task ranges with their own device tables
    struct Segment {
        int first = 0, count = 0;
        long long items = 0, chunks = 0;
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
    // q4rdna_plan_run_host with Q4_K tasks: their launch is one more segment,
    // with its own input copy (first on the copy stream) and output copy,
    // beside the Q4_RDNA segments
    struct KSeg {
        bool on = false;
        size_t x_lo = 0, x_hi = 0, y_lo = 0, y_hi = 0;  // byte ranges from x_dev / y_dev
        cudaEvent_t x_ready = nullptr, y_ready = nullptr;
    } kseg;
};

namespace {
// One launch of (a segment of) a plan on its kernel.
q4rdna_status plan_launch(const q4rdna_plan *plan, const Launch &L, int grid, cudaStream_t stream) {
    if (plan->cta) return launch_cta(L, plan->nb, plan->dual, plan->norm, stream, plan->overlap);
    if (plan->tc) return launch_tc(L, plan->nb, plan->dual, stream, plan->overlap);
    return launch(L, grid, plan->nb, plan->dual, stream, plan->norm);
}

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
    return ws_bytes_for(N, K, B, resolve_split(N, K, B, op, cfg, d), op);
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
    long long items = 0, chunks = 0;
    uint64_t wbytes = 0, abytes = 0;
    // Split-K only as far as the whole plan needs it.  B = 1..2 (the CTA-split
    // kernel, one CTA per (row block, K-range)): as many K-ranges per tensor as
    // fit one wave of resident CTAs over all the plan's row blocks, at least one
    // group per warp (cta_split) -- the Qwen3-8B step's 10944 row blocks run
    // unsplit.  B = 3..16 (the tile path): about kPlanItemsPerWorker items per
    // resident CTA.
    long long total_rb = 0;
    bool any_dual_task = false;
    for (int i = 0; i < count; ++i) {
        if (descs[i].N > 0) total_rb += (descs[i].N + Q4_BLOCK_ROWS - 1) / Q4_BLOCK_ROWS;
        any_dual_task = any_dual_task || descs[i].op == Q4RDNA_OP_SWIGLU;
    }
    const bool cta = B < kTileMinBatch;
    const bool tc = B >= kTcMinBatch;
    const long long ctas = resident_ctas(B, any_dual_task, d);
    const double want_items = kPlanItemsPerWorker * (double)ctas;
    // the tensor-core path's items hold two row blocks (one with SwiGLU)
    const double item_rb = tc ? 2.0 : 1.0;
    const int tile_split =
        total_rb > 0 ? (int)std::max(1.0, std::ceil(want_items * item_rb / (double)total_rb)) : 1;
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
        const int planes = e.op == Q4RDNA_OP_SWIGLU ? 2 : 1;
        const int G = e.K / Q4_GROUP;
        const int RB = (e.N + Q4_BLOCK_ROWS - 1) / Q4_BLOCK_ROWS;
        const int req = e.split > 0 ? e.split : cta ? cta_split(total_rb, G, ctas) : std::min(tile_split, G);
        const Split sp = split_of(G, req, B);
        Task &T = host[i];
        T.w = e.tiles; T.w2 = e.gate_tiles; T.x = e.x; T.add = e.add; T.y = e.y;
        T.part = nullptr; T.ticket = nullptr;
        T.N = e.N; T.K = e.K; T.G = G; T.RB = RB; T.S = sp.S; T.Gs = sp.Gs; T.op = e.op; T.nmirror = 0;
        T.item_begin = items;
        T.gn = e.norm_weight;
        T.eps = e.norm_eps;
        T.rbi = rows_per_item(B, e.op);
        T.chunk_begin = chunks;
        T.img = nullptr;
        T.csum = nullptr;
        items += task_items(T);
        chunks += tc_chunks(G);
        ws_off[i] = ws_total;
        ws_total += plan_ws_bytes_for(e.N, e.K, B, sp.S, e.op, e.norm_weight != nullptr);
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
        if (tc) {  // the prepared activation follows the split workspace
            uint8_t *prep = static_cast<uint8_t *>(p->workspace) + ws_off[i] +
                            plan_split_bytes(T.N, B, T.S, T.op, T.gn != nullptr);
            T.img = prep;
            if (T.gn != nullptr) T.csum = reinterpret_cast<float *>(prep + tc_img_bytes(T.K, B));
        }
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
    p->cta = cta;
    p->tc = tc;
    p->chunks = chunks;
    p->grid = cta ? (int)std::min<long long>(items, INT32_MAX) : grid_for(items, B, any_dual, d);
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

// The flag exchange that closes run `epoch` of a gather plan (after its GEMV
// launches, in stream order).
static q4rdna_status launch_signal(q4rdna_plan *plan, uint32_t epoch, cudaStream_t stream) {
    GatherSignal sg = plan->sig;
    sg.epoch = epoch;
    void *args[] = {&sg};
    if (cudaLaunchKernel((const void *)q4_gather_signal_kernel, dim3(1), dim3(32), args, 0, stream) != cudaSuccess)
        return Q4RDNA_ERR_CUDA;
    if (cudaGetLastError() != cudaSuccess) return Q4RDNA_ERR_CUDA;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    plan->epoch = epoch;
    return Q4RDNA_OK;
}

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
            L.total_chunks = plan->chunks;
            st = plan_launch(plan, L, plan->grid, (cudaStream_t)stream);
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
        L.total_chunks = plan->chunks;
        st = plan_launch(plan, L, plan->grid, (cudaStream_t)stream);
    }
    if (st != Q4RDNA_OK) return st;
    return launch_signal(plan, epoch, (cudaStream_t)stream);
}

q4rdna_status q4rdna_plan_set_gather(q4rdna_plan *plan, int world, int rank, const float *y_base,
                                     size_t rank_floats, float *const *gathered0, float *const *gathered1,
                                     uint32_t *const *flags) {
    if (plan == nullptr || y_base == nullptr || gathered0 == nullptr || gathered1 == nullptr || flags == nullptr)
        return Q4RDNA_ERR_INVALID_ARGUMENT;
    if (world < 2 || world > kMaxWorld || rank < 0 || rank >= world || plan->gather)
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
    if (sg.tries <= 0) sg.tries = kGatherTries;
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
    uint8_t *yh_dev = graded && xd != nullptr && direct_batch(p->B) ? mapped_output(yh, yb) : nullptr;
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
        for (const Task &T : t) sg.chunks += tc_chunks(T.G);
        sg.grid = grid_for(sg.items, p->B, p->dual, d);
        p->segs.push_back(sg);  // owned by the plan from here on (freed on failure paths below)
        q4rdna_plan::Segment &g = p->segs.back();
        if ((g.table = upload_tasks(t)) == nullptr ||
            cudaEventCreateWithFlags(&g.x_ready, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&g.y_ready, cudaEventDisableTiming) != cudaSuccess)
            return Q4RDNA_ERR_CUDA;
        for (int par = 0; p->gather && par < 2; ++par) {
            std::vector<Task> gt(p->ghost[par].begin() + first, p->ghost[par].begin() + last);
            if (direct)  // the gather's mirrors, then the host-mapped output
                for (size_t k = 0; k < gt.size(); ++k) {
                    const Task &T = p->host[first + k];
                    gt[k].mirror[gt[k].nmirror] =
                        reinterpret_cast<float *>(yh_dev + (reinterpret_cast<const uint8_t *>(T.y) - yd));
                    gt[k].nmirror += 1;
                }
            if ((g.gtable[par] = upload_tasks(gt)) == nullptr) return Q4RDNA_ERR_CUDA;
        }
        first = last;
    }
    // the Q4_K tasks of a run_host plan: one segment of their own
    p->kseg.on = false;
    if (xd != nullptr && !p->q4k_host.empty()) {
        auto &k = p->kseg;
        k.x_lo = k.y_lo = SIZE_MAX;
        k.x_hi = k.y_hi = 0;
        for (const q4k::Task &T : p->q4k_host) {
            const uint8_t *x = reinterpret_cast<const uint8_t *>(T.x);
            const uint8_t *y = reinterpret_cast<const uint8_t *>(T.y);
            const size_t xn = (size_t)p->B * T.K * sizeof(float), yn = (size_t)p->B * T.N * sizeof(float);
            if (x < xd || x + xn > xd + xb || y < yd || y + yn > yd + yb) return Q4RDNA_ERR_INVALID_ARGUMENT;
            k.x_lo = std::min(k.x_lo, (size_t)(x - xd));
            k.x_hi = std::max(k.x_hi, (size_t)(x - xd) + xn);
            k.y_lo = std::min(k.y_lo, (size_t)(y - yd));
            k.y_hi = std::max(k.y_hi, (size_t)(y - yd) + yn);
        }
        if ((k.x_ready == nullptr && cudaEventCreateWithFlags(&k.x_ready, cudaEventDisableTiming) != cudaSuccess) ||
            (k.y_ready == nullptr && cudaEventCreateWithFlags(&k.y_ready, cudaEventDisableTiming) != cudaSuccess))
            return Q4RDNA_ERR_CUDA;
        // ranges shared with a Q4_RDNA segment (say q/k/v in Q4_K reading the
        // same x as a Q4_RDNA tensor) cannot overlap: run_host then copies in,
        // runs and copies out the whole plan
        k.on = true;
        for (const auto &sg : p->segs)
            if ((k.x_lo < sg.x_hi && sg.x_lo < k.x_hi) || (k.y_lo < sg.y_hi && sg.y_lo < k.y_hi)) k.on = false;
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
    const bool kseg = copies && plan->kseg.on;  // the Q4_K tasks' segment (copies both ways)
    if (copies && cudaStreamWaitEvent(plan->h2d, plan->start, 0) != cudaSuccess) return Q4RDNA_ERR_CUDA;
    if ((out_copies || kseg) && cudaStreamWaitEvent(plan->d2h, plan->start, 0) != cudaSuccess) return Q4RDNA_ERR_CUDA;
    if (kseg) {  // its inputs first: the Q4_K kernel then runs beside the first Q4_RDNA segment
        const auto &k = plan->kseg;
        if (cudaMemcpyAsync(xd + k.x_lo, xh + k.x_lo, k.x_hi - k.x_lo, cudaMemcpyHostToDevice, plan->h2d) !=
                cudaSuccess ||
            cudaEventRecord(k.x_ready, plan->h2d) != cudaSuccess)
            return Q4RDNA_ERR_CUDA;
    }
    for (auto &sg : plan->segs) {
        if (!copies) break;
        if (cudaMemcpyAsync(xd + sg.x_lo, xh + sg.x_lo, sg.x_hi - sg.x_lo, cudaMemcpyHostToDevice, plan->h2d) !=
                cudaSuccess ||
            cudaEventRecord(sg.x_ready, plan->h2d) != cudaSuccess)
            return Q4RDNA_ERR_CUDA;
    }
    if (kseg) {
        const auto &k = plan->kseg;
        cudaStream_t c = plan->comp[1];
        if (cudaStreamWaitEvent(c, k.x_ready, 0) != cudaSuccess) return Q4RDNA_ERR_CUDA;
        const q4rdna_status st = launch_q4k(plan, c);
        if (st != Q4RDNA_OK) return st;
        if (cudaEventRecord(k.y_ready, c) != cudaSuccess || cudaStreamWaitEvent(plan->d2h, k.y_ready, 0) != cudaSuccess ||
            cudaMemcpyAsync(yh + k.y_lo, yd + k.y_lo, k.y_hi - k.y_lo, cudaMemcpyDeviceToHost, plan->d2h) != cudaSuccess)
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
        L.total_chunks = sg.chunks;
        const q4rdna_status st = plan_launch(plan, L, sg.grid, c);
        if (st != Q4RDNA_OK) return st;
        if (cudaEventRecord(sg.y_ready, c) != cudaSuccess) return Q4RDNA_ERR_CUDA;
        if (!out_copies) continue;
        if (cudaStreamWaitEvent(plan->d2h, sg.y_ready, 0) != cudaSuccess ||
            cudaMemcpyAsync(yh + sg.y_lo, yd + sg.y_lo, sg.y_hi - sg.y_lo, cudaMemcpyDeviceToHost, plan->d2h) !=
                cudaSuccess)
            return Q4RDNA_ERR_CUDA;
    }
    if (out_copies || kseg) {  // every output copy is on the copy-out stream
        if (cudaEventRecord(plan->done, plan->d2h) != cudaSuccess || cudaStreamWaitEvent(cs, plan->done, 0) != cudaSuccess)
            return Q4RDNA_ERR_CUDA;
    }
    if (!out_copies) {
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
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != plan->device) return Q4RDNA_ERR_DEVICE;
    auto whole = [&]() -> q4rdna_status {  // one copy in, the run, one copy out
        cudaStream_t cs = (cudaStream_t)stream;
        if (cudaMemcpyAsync(x_dev, x_host, x_bytes, cudaMemcpyHostToDevice, cs) != cudaSuccess)
            return Q4RDNA_ERR_CUDA;
        const q4rdna_status st = q4rdna_plan_run(plan, stream);
        if (st != Q4RDNA_OK) return st;
        if (cudaMemcpyAsync(y_host, y_dev, y_bytes, cudaMemcpyDeviceToHost, cs) != cudaSuccess)
            return Q4RDNA_ERR_CUDA;
        return Q4RDNA_OK;
    };
    if (!plan->q4k_host.empty() && plan->count == 0) return whole();  // Q4_K tensors only
    const int want = segments != 0 ? segments
                                   : (direct_batch(plan->B) && mapped_output(y_host, y_bytes) != nullptr ? kHostSegmentsDirect
                                                                                                          : kHostSegments);
    if (plan->seg_request != std::max(1, std::min(want, plan->count)) || !plan->seg_graded || plan->seg_x != x_dev ||
        plan->seg_y != y_dev || plan->seg_yh != y_host) {
        const q4rdna_status st = build_segments(plan, want, static_cast<const uint8_t *>(x_dev), x_bytes,
                                                static_cast<const uint8_t *>(y_dev), y_bytes, true,
                                                static_cast<const uint8_t *>(y_host));
        if (st != Q4RDNA_OK) return st;
    } else {
        for (const auto &sg : plan->segs)
            if (sg.x_hi > x_bytes || sg.y_hi > y_bytes) return Q4RDNA_ERR_INVALID_ARGUMENT;
        if (plan->kseg.on && (plan->kseg.x_hi > x_bytes || plan->kseg.y_hi > y_bytes)) return Q4RDNA_ERR_INVALID_ARGUMENT;
    }
    if (!plan->q4k_host.empty() && !plan->kseg.on) return whole();  // Q4_K ranges shared with Q4_RDNA ones
    if (plan->gather) {
        // a gather plan: the segments store into every rank's gathered buffer
        // (and the host buffer when it is mapped), then the flag exchange; the
        // run's epoch changes per call, so these are direct launches
        const uint32_t epoch = plan->epoch + 1;
        const q4rdna_status st = launch_segments(plan, (cudaStream_t)stream, static_cast<const uint8_t *>(x_host),
                                                 static_cast<uint8_t *>(x_dev), static_cast<const uint8_t *>(y_dev),
                                                 static_cast<uint8_t *>(y_host), (int)(epoch & 1));
        if (st != Q4RDNA_OK) return st;
        return launch_signal(plan, epoch, (cudaStream_t)stream);
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
        const uint64_t before = g_launches.load(), before_k = q4k_launch_count();
        const q4rdna_status st = launch_segments(plan, plan->cap, static_cast<const uint8_t *>(x_host),
                                                 static_cast<uint8_t *>(x_dev), static_cast<const uint8_t *>(y_dev),
                                                 static_cast<uint8_t *>(y_host));
        // launches recorded by the capture are counted per replay below (the
        // Q4_K counter's share comes off this one: the sum stays exact)
        const uint64_t captured = (g_launches.load() - before) + (q4k_launch_count() - before_k);
        g_launches.fetch_sub(captured, std::memory_order_relaxed);
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

q4rdna_status q4rdna_plan_run_many(q4rdna_plan *const *plans, int count, q4rdna_stream_t stream) {
    if (plans == nullptr || count < 0) return Q4RDNA_ERR_INVALID_ARGUMENT;
    for (int i = 0; i < count; ++i) {
        const q4rdna_status st = q4rdna_plan_run(plans[i], stream);
        if (st != Q4RDNA_OK) return st;
    }
    return Q4RDNA_OK;
}

q4rdna_status q4rdna_plan_set_flags(q4rdna_plan *plan, int flags) {
    if (plan == nullptr || (flags & ~Q4RDNA_CFG_OVERLAP_PREVIOUS) != 0) return Q4RDNA_ERR_INVALID_ARGUMENT;
    plan->overlap = (flags & Q4RDNA_CFG_OVERLAP_PREVIOUS) != 0;
    return Q4RDNA_OK;
}

q4rdna_status q4rdna_plan_set_segments(q4rdna_plan *plan, int segments) {
    if (plan == nullptr || segments < 0) return Q4RDNA_ERR_INVALID_ARGUMENT;
    plan->run_segments = segments == 0 ? 1 : segments;
    return Q4RDNA_OK;
}

q4rdna_status q4rdna_plan_set_gather_timeout(q4rdna_plan *plan, uint32_t microseconds) {
    if (plan == nullptr) return Q4RDNA_ERR_INVALID_ARGUMENT;
    // one poll is a flag load plus a ~0.5 us sleep hint
    const uint64_t t = microseconds == 0 ? (uint64_t)kGatherTries : (uint64_t)microseconds * 2u;
    plan->sig.tries = (int)std::min<uint64_t>(std::max<uint64_t>(t, 1), (uint64_t)1 << 30);
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
    if (plan->kseg.x_ready) cudaEventDestroy(plan->kseg.x_ready);
    if (plan->kseg.y_ready) cudaEventDestroy(plan->kseg.y_ready);
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
