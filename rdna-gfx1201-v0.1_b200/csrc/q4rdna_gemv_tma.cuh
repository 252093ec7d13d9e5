// TMA-ring variant of the GEMV (included into q4rdna_gemv.cu inside namespace q4).
//
// Same work items, lane mapping and tensor-core math as q4_gemv_kernel, but the
// tiles reach the SM by bulk copies (cp.async.bulk, the TMA engine) into a
// per-warp ring of shared-memory stages instead of by 128-bit register loads.
// A stage holds, for the item's four 32-row tiles, CHUNK consecutive steps (one
// contiguous run of CHUNK*1088 bytes per tile row for a plain tensor; up and
// gate tiles alternate for SwiGLU).  So HBM sees long contiguous bursts whatever order the
// MMA fragments need, and each warp keeps up to STAGES - 1 stages in flight
// with no registers spent on them.
//
// Pipeline per warp (no inter-warp synchronisation): lane 0 is the producer.
// Chunk q of the warp's flat chunk sequence (its items in order, each split into
// chunks) goes to stage q % STAGES, whose mbarrier expects the chunk's
// bytes.  All 32 lanes wait on that barrier (bounded), compute, __syncwarp, and
// lane 0 refills the stage with chunk q + STAGES.  Every wait has an
// iteration limit: on expiry the kernel records a fault code in g_fault, waits
// (again bounded) for its own copies still in flight, and returns.

// Ring shape: STAGES stages per warp, each holding CHUNK steps (a step is one
// group of one tensor) for the item's four row tiles; WARPS warps per CTA,
// MINB CTAs per SM.
template <int STAGES_, int CHUNK_, int WARPS_, int MINB_>
struct RingCfg {
    static constexpr int STAGES = STAGES_, CHUNK = CHUNK_, WARPS = WARPS_, MINB = MINB_;
    static constexpr int THREADS = WARPS * 32;
    static constexpr int ROW_STRIDE = CHUNK * Q4_TILE_BYTES;
    static constexpr int STAGE_BYTES = Q4_BLOCK_TILES * ROW_STRIDE;
    static constexpr int SMEM_BYTES = WARPS * STAGES * STAGE_BYTES;
};
using RingA = RingCfg<3, 2, 8, 1>;   // 209 KB, 8 warps/SM
using RingB = RingCfg<2, 1, 8, 2>;   //  70 KB per CTA, 16 warps/SM
using RingC = RingCfg<3, 1, 8, 2>;   // 104 KB per CTA, 16 warps/SM
using RingD = RingCfg<2, 1, 16, 1>;  // 139 KB, 16 warps in one CTA
constexpr int kWaitTries = 1 << 21;  // x ~1 us suspend hint per try: about 2 s
constexpr unsigned kFaultWaitTimeout = 1u;

__device__ unsigned int g_fault;

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(1000u)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with `parity`; the result is the same in every lane.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    bool ok = false;
    for (int i = 0; i < kWaitTries && !ok; ++i) ok = mbar_try(bar, parity);
    return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Global -> this CTA's shared memory, completion counted on `bar` (no multicast).
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const uint8_t *src, uint32_t bytes, uint32_t bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(policy)
        : "memory");
}

struct ItemGeom {
    int rb, sp, g0, ng, nsteps, nchunks;
    bool dual;
};

// Steps of an item: groups in order; for SwiGLU each group is two steps (up, gate).
template <int CHUNK>
__device__ __forceinline__ ItemGeom item_geom(const Task &T, long long local) {
    ItemGeom g;
    g.rb = (int)(local / T.S);
    g.sp = (int)(local % T.S);
    g.g0 = g.sp * T.Gs;
    g.ng = min(T.Gs, T.G - g.g0);
    g.dual = T.op == Q4RDNA_OP_SWIGLU;
    g.nsteps = g.ng * (g.dual ? 2 : 1);
    g.nchunks = (g.nsteps + CHUNK - 1) / CHUNK;
    return g;
}

// Producer (lane 0): chunk `ch` (steps ch*CHUNK ...) of item `it` into the stage
// at `stage` / `bar`.  Step u of the chunk for row tile t lands at
// stage + t * ROW_STRIDE + u * 1088.  Consecutive plain steps of one row tile are
// adjacent in HBM and go as one copy; SwiGLU steps alternate tensors and go one
// tile per copy.  Rows past N are not copied.
template <class R>
__device__ __forceinline__ void issue_chunk(const Launch &L, long long it, int ch, uint32_t stage, uint32_t bar,
                                            uint64_t policy) {
    const Task &T = find_task(L, it);
    const ItemGeom g = item_geom<R::CHUNK>(T, it - T.item_begin);
    const int rows_tiles = T.N >> 5;
    const int s0 = ch * R::CHUNK;
    const int ns = min(R::CHUNK, g.nsteps - s0);
    int valid_rows = 0;
    for (int t = 0; t < Q4_BLOCK_TILES; ++t)
        if (g.rb * Q4_BLOCK_TILES + t < rows_tiles) ++valid_rows;
    mbar_arrive_expect(bar, (uint32_t)(valid_rows * ns * Q4_TILE_BYTES));
    for (int t = 0; t < valid_rows; ++t) {
        const size_t row_off = (size_t)(g.rb * Q4_BLOCK_TILES + t) * T.G;
        const uint32_t dst = stage + t * R::ROW_STRIDE;
        if (!g.dual) {
            bulk_g2s(dst, T.w + (row_off + g.g0 + s0) * Q4_TILE_BYTES, ns * Q4_TILE_BYTES, bar, policy);
        } else {
            for (int u = 0; u < ns; ++u) {
                const int st = s0 + u;
                const uint8_t *src = ((st & 1) ? T.w2 : T.w) + (row_off + g.g0 + (st >> 1)) * Q4_TILE_BYTES;
                bulk_g2s(dst + u * Q4_TILE_BYTES, src, Q4_TILE_BYTES, bar, policy);
            }
        }
    }
}

// One group of one tensor from a staged tile (`tile` = this lane's row tile in
// the stage): the same fragment mapping and accumulation order as compute_step.
template <int NB>
__device__ __forceinline__ void mma_group_smem(const uint8_t *tile, int c, int h, const WarpSmem<NB> &sm,
                                               float (&acc)[4][NB][2], int lane, const uint32_t (&sel)[NB],
                                               const int (&xrow)[NB], const int (&urow)[NB]) {
    float D[4][NB][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int nb = 0; nb < NB; ++nb)
#pragma unroll
            for (int r = 0; r < 4; ++r) D[j][nb][r] = 0.0f;
    const uint8_t *qp = tile + Q4_SCALE_BYTES + 32 * c + 16 * h;
    const int c4 = lane & 3;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        const uint4 cur = *reinterpret_cast<const uint4 *>(qp + 128 * m);
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
    const uint8_t *sp = tile + 32 * h + 4 * (c & 1);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t w = *reinterpret_cast<const uint32_t *>(sp + 8 * j);
        const float2 sc = __half22float2(*reinterpret_cast<const __half2 *>(&w));
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
            const float u = sm.up[urow[nb]];
            acc[j][nb][0] = fmaf(sc.x * u, D[j][nb][0] + D[j][nb][1], acc[j][nb][0]);
            acc[j][nb][1] = fmaf(sc.y * u, D[j][nb][2] + D[j][nb][3], acc[j][nb][1]);
        }
    }
}

template <int NB, class R>
__global__ void __launch_bounds__(R::THREADS, R::MINB) q4_gemv_tma_kernel(const __grid_constant__ Launch L) {
    extern __shared__ __align__(128) uint8_t stages_smem[];
    __shared__ __align__(8) uint64_t bars[R::WARPS][R::STAGES];
    __shared__ WarpSmem<NB> xsm[R::WARPS];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long nw = (long long)gridDim.x * R::WARPS;
    const long long first = (long long)blockIdx.x * R::WARPS + warp;
    uint8_t *ring = stages_smem + (size_t)warp * R::STAGES * R::STAGE_BYTES;
    const uint32_t ring_s = smem_addr(ring);
    const uint32_t bar0 = smem_addr(&bars[warp][0]);  // stage q's barrier at bar0 + 8q
    if (lane == 0) {
#pragma unroll
        for (int q = 0; q < R::STAGES; ++q) mbar_init(bar0 + 8 * q);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncwarp();
    const uint64_t policy = evict_first_policy();
    WarpSmem<NB> &sm = xsm[warp];

    // Producer cursor over the warp's chunk sequence (lane 0 issues, every lane
    // tracks the cursor so the number of chunks in flight is warp-uniform).
    long long p_it = first;
    int p_ch = 0, p_nch = 0;
    if (p_it < L.total_items) {
        const Task &T = find_task(L, p_it);
        p_nch = item_geom<R::CHUNK>(T, p_it - T.item_begin).nchunks;
    }
    auto produce = [&](int slot) {
        if (lane == 0) {
            // the warp's generic reads of this stage are done (__syncwarp before
            // every refill); order them before the async-proxy writes
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue_chunk<R>(L, p_it, p_ch, ring_s + slot * R::STAGE_BYTES, bar0 + 8 * slot, policy);
        }
        if (++p_ch >= p_nch) {
            p_it += nw;
            p_ch = 0;
            if (p_it < L.total_items) {
                const Task &T = find_task(L, p_it);
                p_nch = item_geom<R::CHUNK>(T, p_it - T.item_begin).nchunks;
            }
        }
    };
    int issued = 0;
    for (int q = 0; q < R::STAGES && p_it < L.total_items; ++q, ++issued) produce(q);

    uint32_t phase = 0;
    int consumed = 0;
    bool fault = false;
    const int grp = lane >> 2, c = lane & 3, t = grp >> 1, h = grp & 1;
    for (long long it = first; it < L.total_items && !fault; it += nw) {
        const Task &T = find_task(L, it);
        const ItemGeom g = item_geom<R::CHUNK>(T, it - T.item_begin);
        const int B = L.B;
        const int tile_row = g.rb * Q4_BLOCK_TILES + t;
        const bool valid = tile_row < (T.N >> 5);
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
        float acc[2][4][NB][2];
#pragma unroll
        for (int q = 0; q < 2; ++q)
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int nb = 0; nb < NB; ++nb) acc[q][j][nb][0] = acc[q][j][nb][1] = 0.0f;
        float2 xv[2 * NB];
#pragma unroll
        for (int b = 0; b < 2 * NB; ++b)
            xv[b] = b < B ? __ldg(reinterpret_cast<const float2 *>(T.x + (size_t)b * T.K + (size_t)g.g0 * Q4_GROUP) + lane)
                          : make_float2(0.0f, 0.0f);

        int st = 0;  // next step of this item
        for (int ch = 0; ch < g.nchunks; ++ch) {
            const int slot = consumed % R::STAGES;
            if (!mbar_wait(bar0 + 8 * slot, (phase >> slot) & 1u)) { fault = true; break; }
            phase ^= 1u << slot;
            ++consumed;
            const uint8_t *tile = ring + slot * R::STAGE_BYTES + t * R::ROW_STRIDE;
            const int ns = min(R::CHUNK, g.nsteps - st);
            for (int u = 0; u < ns; ++u, ++st) {
                const int tt = g.dual ? (st & 1) : 0;
                const int gl = g.dual ? (st >> 1) : st;
                if (tt == 0) {
                    // this group's activation -> smem; fetch the next group's
                    __syncwarp();
#pragma unroll
                    for (int b = 0; b < 2 * NB; ++b)
                        if (b < B) prep_group(xv[b], sm.xq[b], &sm.up[b], lane);
                    if (gl + 1 < g.ng) {
#pragma unroll
                        for (int b = 0; b < 2 * NB; ++b)
                            if (b < B)
                                xv[b] = __ldg(reinterpret_cast<const float2 *>(
                                                  T.x + (size_t)b * T.K + (size_t)(g.g0 + gl + 1) * Q4_GROUP) + lane);
                    }
                    __syncwarp();
                }
                if (tt)
                    mma_group_smem<NB>(tile + u * Q4_TILE_BYTES, c, h, sm, acc[1], lane, sel, xrow, urow);
                else
                    mma_group_smem<NB>(tile + u * Q4_TILE_BYTES, c, h, sm, acc[0], lane, sel, xrow, urow);
            }
            __syncwarp();
            if (p_it < L.total_items) {
                produce(slot);
                ++issued;
            }
        }
        if (fault) break;
        if (g.dual)
            finish_item<NB, true>(T, g.rb, g.sp, B, acc, lane, valid, tile_row, h, c);
        else
            finish_item<NB, false>(T, g.rb, g.sp, B, reinterpret_cast<float(&)[1][4][NB][2]>(acc), lane, valid,
                                   tile_row, h, c);
    }
    if (fault) {
        if (lane == 0) atomicOr(&g_fault, kFaultWaitTimeout);
        // Let this warp's own copies still in flight land before the CTA exits.
        for (; consumed < issued; ++consumed) {
            const int slot = consumed % R::STAGES;
            mbar_wait(bar0 + 8 * slot, (phase >> slot) & 1u);
            phase ^= 1u << slot;
        }
    }
}
