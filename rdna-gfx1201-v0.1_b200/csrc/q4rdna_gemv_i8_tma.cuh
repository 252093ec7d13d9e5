// int8 GEMV with the TMA ring (included into q4rdna_gemv.cu inside namespace q4,
// after q4rdna_gemv_tma.cuh and q4rdna_gemv_i8.cuh).
//
// The math is mma_step_i8 reading staged tiles (SmemSource); the tiles reach
// shared memory by cp.async.bulk copies issued by lane 0 into a per-warp ring
// of R::STAGES stages of R::CHUNK steps (see q4rdna_gemv_tma.cuh for the ring
// protocol, bounded waits and the fault path).  Unlike that kernel, the
// producer keeps the geometry of the item it is copying (row bases, steps,
// SwiGLU flag) and computes it once per item with 32-bit arithmetic, so a
// refill costs lane 0 a handful of instructions instead of a task search.

// Producer cursor: the item being copied and its geometry.
struct I8Producer {
    long long it;          // item index (>= total: done)
    int ch, nch;           // next chunk, chunks of the item
    int nsteps, rows;      // steps of the item, valid row tiles (1..4)
    bool dual;
    const uint8_t *base;   // row tile 0 of the item at its first group, tensor w
    long long w2off;       // w2 - w (SwiGLU)
    size_t row_stride;     // bytes between consecutive row tiles: G * 1088
};

template <int CHUNK>
__device__ __forceinline__ void producer_load(const Launch &L, I8Producer &p) {
    if (p.it >= L.total_items) return;
    const Task &T = find_task(L, p.it);
    const int local = (int)(p.it - T.item_begin);
    const int rb = local / T.S, sp = local % T.S;
    const int g0 = sp * T.Gs, ng = min(T.Gs, T.G - g0);
    p.dual = T.op == Q4RDNA_OP_SWIGLU;
    p.nsteps = ng * (p.dual ? 2 : 1);
    p.nch = (p.nsteps + CHUNK - 1) / CHUNK;
    p.ch = 0;
    p.rows = min(Q4_BLOCK_TILES, (T.N >> 5) - rb * Q4_BLOCK_TILES);
    p.row_stride = (size_t)T.G * Q4_TILE_BYTES;
    p.base = T.w + ((size_t)rb * Q4_BLOCK_TILES * T.G + g0) * Q4_TILE_BYTES;
    p.w2off = p.dual ? (long long)(T.w2 - T.w) : 0;
}

// Lane 0: copy the cursor's next chunk into the stage at `stage` / `bar`.
template <class R>
__device__ __forceinline__ void producer_issue(const I8Producer &p, uint32_t stage, uint32_t bar, uint64_t policy) {
    const int s0 = p.ch * R::CHUNK;
    const int ns = min(R::CHUNK, p.nsteps - s0);
    mbar_arrive_expect(bar, (uint32_t)(p.rows * ns * Q4_TILE_BYTES));
    for (int t = 0; t < p.rows; ++t) {
        const uint8_t *row = p.base + t * p.row_stride;
        const uint32_t dst = stage + t * R::ROW_STRIDE;
        if (!p.dual) {
            bulk_g2s(dst, row + (size_t)s0 * Q4_TILE_BYTES, ns * Q4_TILE_BYTES, bar, policy);
        } else {
            for (int u = 0; u < ns; ++u) {
                const int st = s0 + u;
                const uint8_t *src = row + (size_t)(st >> 1) * Q4_TILE_BYTES + ((st & 1) ? p.w2off : 0);
                bulk_g2s(dst + u * Q4_TILE_BYTES, src, Q4_TILE_BYTES, bar, policy);
            }
        }
    }
}

// The ring variant takes no fused-RMSNorm task (the host refuses them).
template <int BB>
__device__ const float kNoSumsq[BB] = {};

// 70 KB per CTA, 3 CTAs (24 warps) per SM, one group in flight per warp: the
// fastest ring shape measured on B200 (the register kernel is faster still).
using I8Ring = RingCfg<2, 1, 8, 3>;

template <int BB, class R>
__global__ void __launch_bounds__(R::THREADS, R::MINB) q4_gemv_i8_tma_kernel(const __grid_constant__ Launch L) {
    extern __shared__ __align__(128) uint8_t stages_smem[];
    __shared__ __align__(8) uint64_t bars[R::WARPS][R::STAGES];
    __shared__ I8X<BB> xsm[R::WARPS];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long nw = (long long)gridDim.x * R::WARPS;
    const long long first = (long long)blockIdx.x * R::WARPS + warp;
    if (first >= L.total_items) return;
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
    I8X<BB> &sm = xsm[warp];
    I8Sel sel;
    {
        const int n = lane >> 2;  // this lane's B column
        sel.a = sel_one(n >> 1, (n & 1) ? 0 : 1);
        sel.b = sel_one(n >> 1, 2);
        sel.bcol_odd = n & 1;
    }
    const int grp = lane >> 2, c = lane & 3, t = grp >> 1, h = grp & 1;

    I8Producer p;
    p.it = first;
    producer_load<R::CHUNK>(L, p);  // every lane keeps the cursor, lane 0 issues
    auto produce = [&](int slot) {
        if (lane == 0) {
            // the warp's generic reads of this stage are done (__syncwarp before
            // every refill); order them before the async-proxy writes
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            producer_issue<R>(p, ring_s + slot * R::STAGE_BYTES, bar0 + 8 * slot, policy);
        }
        if (++p.ch >= p.nch) {
            p.it += nw;
            producer_load<R::CHUNK>(L, p);
        }
    };
    int issued = 0;
    for (int q = 0; q < R::STAGES && p.it < L.total_items; ++q, ++issued) produce(q);

    float2 xv[BB];
    {
        const Task &T = find_task(L, first);
        const int local = (int)(first - T.item_begin);
        const int g0 = (local % T.S) * T.Gs;
#pragma unroll
        for (int b = 0; b < BB; ++b)
            xv[b] = b < L.B ? __ldg(reinterpret_cast<const float2 *>(T.x + (size_t)b * T.K + (size_t)g0 * Q4_GROUP) + lane)
                            : make_float2(0.0f, 0.0f);
    }
    uint32_t phase = 0;
    int consumed = 0;
    bool fault = false;
    for (long long it = first; it < L.total_items && !fault; it += nw) {
        const Task &T = find_task(L, it);
        const int local = (int)(it - T.item_begin);
        const int rb = local / T.S, s = local % T.S;
        const int g0 = s * T.Gs, ng = min(T.Gs, T.G - g0);
        const bool dual = T.op == Q4RDNA_OP_SWIGLU;
        const int nsteps = ng * (dual ? 2 : 1);
        const int tile_row = rb * Q4_BLOCK_TILES + t;
        const bool valid = tile_row < (T.N >> 5);
        const long long nit = it + nw;
        const Task *nT = nit < L.total_items ? &find_task(L, nit) : nullptr;
        int ng0 = 0;
        if (nT) ng0 = ((int)(nit - nT->item_begin) % nT->S) * nT->Gs;

        float acc[2][4][BB];
#pragma unroll
        for (int pl = 0; pl < 2; ++pl)
#pragma unroll
            for (int q = 0; q < 4; ++q)
#pragma unroll
                for (int b = 0; b < BB; ++b) acc[pl][q][b] = 0.0f;

        int st = 0;
        const int nch = (nsteps + R::CHUNK - 1) / R::CHUNK;
        for (int ch = 0; ch < nch; ++ch) {
            const int slot = consumed % R::STAGES;
            if (!mbar_wait(bar0 + 8 * slot, (phase >> slot) & 1u)) { fault = true; break; }
            phase ^= 1u << slot;
            ++consumed;
            const uint8_t *tile = ring + slot * R::STAGE_BYTES + t * R::ROW_STRIDE;
            const int ns = min(R::CHUNK, nsteps - st);
            for (int u = 0; u < ns; ++u, ++st) {
                const int tt = dual ? (st & 1) : 0, gl = dual ? (st >> 1) : st;
                if (tt == 0) {
                    __syncwarp();
#pragma unroll
                    for (int b = 0; b < BB; ++b)
                        if (b < L.B)
                            prep_group_i8<false>(xv[b], make_float2(0.0f, 0.0f), false, sm.xq[b], &sm.up[b], &sm.ss[b],
                                                 lane);
#pragma unroll
                    for (int b = 0; b < BB; ++b) {
                        if (b >= L.B) continue;
                        if (gl + 1 < ng)
                            xv[b] = __ldg(reinterpret_cast<const float2 *>(T.x + (size_t)b * T.K +
                                                                           (size_t)(g0 + gl + 1) * Q4_GROUP) + lane);
                        else if (nT)
                            xv[b] = __ldg(reinterpret_cast<const float2 *>(nT->x + (size_t)b * nT->K +
                                                                           (size_t)ng0 * Q4_GROUP) + lane);
                    }
                    __syncwarp();
                }
                SmemSource src(tile + u * Q4_TILE_BYTES, c, h);
                if (tt)
                    mma_step_i8<BB>(src, sm, acc[1], lane, sel);
                else
                    mma_step_i8<BB>(src, sm, acc[0], lane, sel);
            }
            __syncwarp();
            if (p.it < L.total_items) {
                produce(slot);
                ++issued;
            }
        }
        if (fault) break;
        if (dual)
            finish_rows_i8<BB, true, false>(T, rb, s, L.B, acc, kNoSumsq<BB>, lane, valid, tile_row, h, c);
        else
            finish_rows_i8<BB, false, false>(T, rb, s, L.B, acc, kNoSumsq<BB>, lane, valid, tile_row, h, c);
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
