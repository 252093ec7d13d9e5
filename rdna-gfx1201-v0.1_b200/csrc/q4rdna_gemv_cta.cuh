// CTA-split GEMV for B = 1..2 (included into q4rdna_gemv.cu inside namespace
// q4, after q4rdna_gemv_i8.cuh): every single call and every plan at B <= 2.
//
// A lone GEMV has too few rows to keep every warp busy with whole-K items: a
// warp streams one group (4.3 KB) per DRAM round trip, so an item of 64 groups
// takes ~60 us whatever the matrix size.  Here one CTA work item is one
// 128-row block x one K-range of Gs groups, and the CTA's 8 warps split that
// range again (Gw groups each), so the whole matrix is in flight at once:
//   * every warp streams its groups through the batch-1 kernel's register
//     pipeline and int8 MMAs (mma_step_i8), with its own activation prep;
//   * the 8 warps' sums meet in shared memory, added in warp order;
//   * with S > 1 CTA K-ranges, each CTA stores its partial sums to the
//     workspace and the last CTA to arrive at the row block (arrival ticket)
//     adds them in ascending order with all 256 threads and applies the add /
//     SwiGLU epilogue; a single call with S <= 8 instead runs each row block's
//     CTAs as one cluster and adds the sums through distributed shared memory.
// Accumulation order of an output: exact int32 inside a group; the groups of a
// warp in ascending order, sum = fma(scale / 16, v * 2^e, sum); warps in
// ascending order; CTA K-ranges in ascending order.  The fused RMSNorm's sum of
// h^2 follows the same order (groups, warps, K-ranges), and its scale
// 1 / sqrt(sum / K + eps) multiplies each output once, before the epilogue.
// Deterministic: no data atomics.
//
// A large plan (the Qwen3-8B step: 10944 row blocks) is one wave after another
// of these CTAs; measured on B200 it matches the persistent warp-item design it
// replaced (625 vs 630 us per step) and beats it when the rows per tensor are
// few (a tensor-parallel rank's shards: 325 vs 379 us at 2 ranks, 95 vs 137 us
// at 8).
//
// Programmatic dependent launch (Q4RDNA_CFG_OVERLAP_PREVIOUS): every CTA lets
// the next kernel of the stream launch at once, and waits for the previous
// kernel (griddepcontrol.wait) after its first weight step is in flight and
// before any read of x, the workspace or add and any store.  Launched without
// the attribute, both instructions do nothing.

// The launch is the plans' Launch: one task (single call) or a task table; an
// item is one CTA, item_begin counts CTA items (RB * S per task).

template <int BB>
__device__ __forceinline__ void cta_fetch_x(const Task &T, int B, int g, int lane, float2 (&xv)[BB]) {
#pragma unroll
    for (int b = 0; b < BB; ++b)
        xv[b] = b < B ? __ldg(reinterpret_cast<const float2 *>(T.x + (size_t)b * T.K + (size_t)g * Q4_GROUP) + lane)
                      : make_float2(0.0f, 0.0f);
}

// Single calls with 2..8 K-ranges run each row block's K-range CTAs as one
// thread-block cluster: the CTAs write their sums into the first CTA's shared
// memory (distributed shared memory) and meet at one cluster barrier, instead
// of a round trip through the workspace and an arrival ticket.  The first CTA
// then adds the K-ranges in ascending order, as the last-arrival path does, so
// the outputs are the same bits either way.
constexpr int kMaxClusterSplit = 8;

template <int BB>
struct CtaSmem {
    I8X<BB> xs[kWarps][2];
    float red[kWarps][2][4][BB][32];  // [warp][plane][q][b][lane]
    float ssq[kWarps][BB];            // fused RMSNorm: each warp's sum of h^2 per batch column
    float cpart[kMaxClusterSplit][2][4 * BB * 32];  // cluster path, first CTA: [K-range][plane][output]
    float cssq[kMaxClusterSplit][BB];               // cluster path, first CTA: sums of h^2 per K-range
    unsigned last;
};

// Stores v into the shared memory of the cluster's CTA 0 at the address that
// p has in this CTA.
__device__ __forceinline__ void st_cluster0(const float *p, float v) {
    uint32_t a = (uint32_t)__cvta_generic_to_shared(p), r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(r) : "r"(a));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(r), "f"(v) : "memory");
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// One CTA item of task T: row block rb, K-range sc.  NORM: the kernel has the
// fused-RMSNorm path (used by tasks with a norm weight, T.gn != null).  CL: the
// launch is clustered by row block (K-range sc = cluster rank sc).
template <int BB, bool DUAL, bool NORM, bool CL>
__device__ __forceinline__ void cta_item(const Task &T, int B, int rb, int sc, CtaSmem<BB> &sm) {
    constexpr int planes = DUAL ? 2 : 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int Gw = (T.Gs + kWarps - 1) / kWarps;
    const int gc1 = min((sc + 1) * T.Gs, T.G);
    const int g0 = sc * T.Gs + warp * Gw;
    const int ng = max(0, min(Gw, gc1 - g0));
    const int grp = lane >> 2, c = lane & 3, t = grp >> 1, h = grp & 1;

    float acc[2][4][BB];
#pragma unroll
    for (int pl = 0; pl < 2; ++pl)
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int b = 0; b < BB; ++b) acc[pl][q][b] = 0.0f;
    const bool norm = NORM && T.gn != nullptr;
    float iss[BB];  // fused RMSNorm: this warp's sum of h^2 per batch column, groups ascending
#pragma unroll
    for (int b = 0; b < BB; ++b) iss[b] = 0.0f;

    if (ng > 0) {
        I8Sel sel;
        {
            const int n = lane >> 2;  // this lane's B column
            sel.a = sel_one(n >> 1, (n & 1) ? 0 : 1);
            sel.b2 = sel_one(n >> 1, 2);
            sel.b3 = sel_one(n >> 1, 3);
            sel.bcol_odd = n & 1;
        }
        // rows past N read the block's first row tile (always present): every
        // load stays in bounds, and those rows are never stored
        int tile_row = rb * Q4_BLOCK_TILES + t;
        if (tile_row >= (T.N >> 5)) tile_row = rb * Q4_BLOCK_TILES;
        const size_t off = ((size_t)tile_row * T.G + g0) * Q4_TILE_BYTES;
        const uint8_t *base0 = T.w + off;
        const uint8_t *base1 = DUAL ? T.w2 + off : base0;
        const int nsteps = ng * planes;
        auto step_tile = [&](int st) -> const uint8_t * {
            const int tt = DUAL ? (st & 1) : 0, gl = DUAL ? (st >> 1) : st;
            return (tt ? base1 : base0) + (size_t)gl * Q4_TILE_BYTES;
        };
        I8X<BB>(&xs)[2] = sm.xs[warp];
        StepBufI8 buf;
        load_step_i8(buf, base0, c, h);  // weights: not written by the previous kernels
        asm volatile("griddepcontrol.wait;" ::: "memory");
        // fused RMSNorm: the group is prepared as h * g (g = 1 without a norm weight)
        auto fetch_g = [&](int g) -> float2 {
            return norm ? __ldg(reinterpret_cast<const float2 *>(T.gn + (size_t)g * Q4_GROUP) + lane)
                        : make_float2(1.0f, 1.0f);
        };
        float2 xv[BB], gv = NORM ? fetch_g(g0) : make_float2(1.0f, 1.0f);
        cta_fetch_x<BB>(T, B, g0, lane, xv);
#pragma unroll
        for (int b = 0; b < BB; ++b) prep_group_i8<NORM>(xv[b], gv, norm, xs[0].xq[b], &xs[0].up[b], &xs[0].ss[b], lane);
        if (ng > 1) {
            cta_fetch_x<BB>(T, B, g0 + 1, lane, xv);
            if (NORM) gv = fetch_g(g0 + 1);
        }
        __syncwarp();
        int par = 0;
        for (int st = 0; st < nsteps; ++st) {
            const int tt = DUAL ? (st & 1) : 0, gl = DUAL ? (st >> 1) : st;
            // the last step refills from its own tile (in bounds, never used)
            RegSource src(buf, step_tile(st + 1 < nsteps ? st + 1 : st), c, h);
            if (tt == 0) {
                mma_step_i8<BB>(src, xs[par], acc[0], lane, sel);
                if (NORM) {
#pragma unroll
                    for (int b = 0; b < BB; ++b) iss[b] += xs[par].ss[b];
                }
                if (gl + 1 < ng) {
                    // the next group's activation into the other buffer
#pragma unroll
                    for (int b = 0; b < BB; ++b)
                        prep_group_i8<NORM>(xv[b], gv, norm, xs[par ^ 1].xq[b], &xs[par ^ 1].up[b],
                                            &xs[par ^ 1].ss[b], lane);
                    if (gl + 2 < ng) {
                        cta_fetch_x<BB>(T, B, g0 + gl + 2, lane, xv);
                        if (NORM) gv = fetch_g(g0 + gl + 2);
                    }
                }
            } else {
                mma_step_i8<BB>(src, xs[par], acc[DUAL ? 1 : 0], lane, sel);
            }
            if (!DUAL || tt == 1) {
                __syncwarp();
                par ^= 1;
            }
        }
    } else {
        asm volatile("griddepcontrol.wait;" ::: "memory");
    }

    // the warps' sums meet in shared memory
#pragma unroll
    for (int pl = 0; pl < planes; ++pl)
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int b = 0; b < BB; ++b) sm.red[warp][pl][q][b][lane] = acc[pl][q][b];
    if (NORM && lane == 0) {
#pragma unroll
        for (int b = 0; b < BB; ++b) sm.ssq[warp][b] = iss[b];
    }
    __syncthreads();
    // fused RMSNorm: the CTA's sum of h^2 of batch column b over its K-range, warps ascending
    auto cta_sumsq = [&](int b) -> float {
        float q = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) q += sm.ssq[w][b];
        return q;
    };

    // thread -> outputs (q, b, ln) of the block: row = tile (ln >> 3) of the
    // block, row in tile 16 ((ln >> 2) & 1) + (ln & 3) + 4 q
    constexpr int kOut = 4 * BB * 32;
    const size_t split_stride = (size_t)planes * B * T.N;
    for (int o = threadIdx.x; o < kOut; o += kThreads) {
        const int ln = o & 31, b = (o >> 5) % BB, q = o / (32 * BB);
        if (b >= B) continue;
        const int lt = ln >> 3, lh = (ln >> 2) & 1, lc = ln & 3;
        const int row = (rb * Q4_BLOCK_TILES + lt) * Q4_TILE_ROWS + 16 * lh + lc + 4 * q;
        if (row >= T.N) continue;
        float v[planes];
#pragma unroll
        for (int pl = 0; pl < planes; ++pl) {
            float s = 0.0f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) s += sm.red[w][pl][q][b][ln];
            v[pl] = s;
        }
        const size_t idx = (size_t)b * T.N + row;
        if (T.S == 1) {
            if (norm) {
                const float r = norm_scale(T, cta_sumsq(b));
#pragma unroll
                for (int pl = 0; pl < planes; ++pl) v[pl] *= r;
            }
            put_y(T, idx, finish(v[0], v[planes - 1], T.op, T.add, idx));
        } else if (CL) {
#pragma unroll
            for (int pl = 0; pl < planes; ++pl) st_cluster0(&sm.cpart[sc][pl][o], v[pl]);
        } else {
#pragma unroll
            for (int pl = 0; pl < planes; ++pl) __stcg(&T.part[(size_t)sc * split_stride + (size_t)pl * B * T.N + idx], v[pl]);
        }
    }
    if (T.S == 1) return;

    if (CL) {
        // the cluster's CTAs meet once; CTA 0 adds the K-ranges in ascending order
        if (norm && threadIdx.x < B) st_cluster0(&sm.cssq[sc][threadIdx.x], cta_sumsq(threadIdx.x));
        cluster_sync_all();
        if (sc != 0) return;
        for (int o = threadIdx.x; o < kOut; o += kThreads) {
            const int ln = o & 31, b = (o >> 5) % BB, q = o / (32 * BB);
            if (b >= B) continue;
            const int lt = ln >> 3, lh = (ln >> 2) & 1, lc = ln & 3;
            const int row = (rb * Q4_BLOCK_TILES + lt) * Q4_TILE_ROWS + 16 * lh + lc + 4 * q;
            if (row >= T.N) continue;
            float v[planes];
#pragma unroll
            for (int pl = 0; pl < planes; ++pl) {
                float s = 0.0f;
                for (int sp = 0; sp < T.S; ++sp) s += sm.cpart[sp][pl][o];
                v[pl] = s;
            }
            if (norm) {  // the K-ranges' sums of h^2 in ascending order
                float q2 = 0.0f;
                for (int sp = 0; sp < T.S; ++sp) q2 += sm.cssq[sp][b];
                const float r = norm_scale(T, q2);
#pragma unroll
                for (int pl = 0; pl < planes; ++pl) v[pl] *= r;
            }
            const size_t idx = (size_t)b * T.N + row;
            put_y(T, idx, finish(v[0], v[planes - 1], T.op, T.add, idx));
        }
        return;
    }

    // K-ranges of several CTAs: the last one to arrive adds them in order
    if (norm && threadIdx.x < B) __stcg(&T.nss[((size_t)rb * T.S + sc) * B + threadIdx.x], cta_sumsq(threadIdx.x));
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) sm.last = atomicAdd(&T.ticket[rb], 1u) == (unsigned)(T.S - 1) ? 1u : 0u;
    __syncthreads();
    if (sm.last == 0) return;
    __threadfence();
    for (int o = threadIdx.x; o < Q4_BLOCK_ROWS * BB; o += kThreads) {
        const int r = o % Q4_BLOCK_ROWS, b = o / Q4_BLOCK_ROWS;
        const int row = rb * Q4_BLOCK_ROWS + r;
        if (b >= B || row >= T.N) continue;
        const size_t idx = (size_t)b * T.N + row;
        float v[planes];
#pragma unroll
        for (int pl = 0; pl < planes; ++pl) {
            float s = 0.0f;
            for (int sp = 0; sp < T.S; ++sp) s += __ldcg(&T.part[(size_t)sp * split_stride + (size_t)pl * B * T.N + idx]);
            v[pl] = s;
        }
        if (norm) {  // the splits' sums of h^2 in ascending split order
            const float r = norm_scale(T, split_sumsq(T, rb, b, B));
#pragma unroll
            for (int pl = 0; pl < planes; ++pl) v[pl] *= r;
        }
        put_y(T, idx, finish(v[0], v[planes - 1], T.op, T.add, idx));
    }
    if (threadIdx.x == 0) atomicExch(&T.ticket[rb], 0u);
}

// One CTA per item (not persistent).  HAS_DUAL = false: the launch holds no
// SwiGLU task; NORM = false: no fused-RMSNorm task; those paths are compiled
// out.  CL: a single call launched as clusters of S CTAs (one per row block).
template <int BB, bool HAS_DUAL, bool NORM, bool CL>
__global__ void __launch_bounds__(kThreads, 2) q4_gemv_cta_kernel(const __grid_constant__ Launch L) {
    __shared__ CtaSmem<BB> sm;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const long long it = blockIdx.x;
    const Task &T = find_task(L, it);
    const int local = (int)(it - T.item_begin);
    const int rb = local / T.S, sc = local % T.S;
    if (HAS_DUAL && T.op == Q4RDNA_OP_SWIGLU)
        cta_item<BB, true, NORM, CL>(T, L.B, rb, sc, sm);
    else
        cta_item<BB, false, NORM, CL>(T, L.B, rb, sc, sm);
}
