// Tensor-core tile path for B = 8..16 activation columns on sm_100a (included
// into q4rdna_gemv.cu inside namespace q4, after q4rdna_gemv_i8.cuh).
//
// At eight or more columns every weight meets enough activations that the
// product is a dense contraction, so it runs on the 5th-generation tensor
// cores: tcgen05.mma kind::i8 issued by one thread, operands in shared memory,
// int32 accumulators in tensor memory (TMEM).
//
// Two kernels per launch:
//
// q4_tc_prep_kernel: one CTA per chunk of 4 groups (256 columns of K) of every
//   task.  It turns the chunk of x (times the norm weight for a fused RMSNorm
//   task) into the B operand of the MMAs, once, for all row blocks:
//   * per batch column the chunk's largest |x| sets a power-of-two scale so
//     that X = rint(x * 2^(156 - E)) has |X| <= 2^30 (act_exponent/act_scale,
//     the activation scaling of the batch-1 kernel); X is written as its four
//     balanced base-256 digits (act_digits), each an s8;
//   * the digits form an MN-major canonical operand image: MMA row n = 4 b + d
//     (batch column b, digit d), K = 32 column pairs per plane, plane "lo" for
//     the even columns 2i and plane "hi" for the odd columns 2i + 1; byte
//     (n, i) of a plane sits at n % 16 + 16 (i % 8) + 128 (i / 8) + 512 (n / 16),
//     so the four digits of (b, i) are one 32-bit word;
//   * after the 4 groups' images, 16 f32 factors 2^(E - 156) (0 for padded
//     columns); for a fused-RMSNorm task also the chunk's sum of h^2 per column.
//
// q4_tc_gemv_kernel: persistent, one CTA per SM, warp-specialised.  A work item
//   is two "A-blocks" x one K-range of whole chunks: two 128-row blocks of a
//   tensor, or, for SwiGLU, the up and the gate tiles of one row block.
//   * warp 0: cp.async.bulk copies of the raw tiles (per row tile, 4 groups =
//     4352 contiguous bytes; lanes 0..7 one copy each) and of the chunk's
//     operand image (lane 8) into a ring of shared-memory stages, completion
//     counted on mbarriers;
//   * warps 4..7: unpack.  A stored byte holds row r's columns 2i (low nibble)
//     and 2i + 1 (high nibble); w & 0xF0F0F0F0 and (w << 4) & 0xF0F0F0F0 are
//     exactly 16 * code as s8 for the odd and the even column.  The tile's
//     bytes for pair column i and rows 16h..16h+15 are 16 contiguous bytes, so
//     one 16-byte load yields one 16-byte slice of each of two MN-major A
//     planes (128 rows x 32 K): byte (m, i) at m % 16 + 16 (i % 8) + 128 (i / 8)
//     + 576 (m / 16).  The 576-byte stride of a 16-row slab (512 + 64) keeps
//     both the loads and the stores free of bank conflicts;
//   * warps 1..3 (one lane each, group n on warp 1 + n % 3): per group and
//     A-block two MMAs, M = 128, N = 4 BP, K = 32 (plane lo, then plane hi),
//     into a TMEM slot that already holds the bias 0x4B400000 in every word.
//     The int32 sums of a group stay below 2^22 in magnitude, so each
//     accumulator word, read as an f32, is exactly 1.5 * 2^23 + S;
//   * warps 8..23: epilogue, one TMEM lane (= one row) per thread: 2 A-blocks
//     x 2 halves of the batch columns x 4 lane quarters (a warp reaches the
//     TMEM lanes 32 (warp % 4) ..).  Per group: tcgen05.ld of the row's words,
//     the bias written back with tcgen05.st (the slot is then ready for the
//     next group), the digit sums recombined as ((S3 256 + S2) 256 + S1) 256
//     + S0 and accumulated with fma(scale / 16, X * 2^(E - 156), acc), the
//     factor 2^(E - 156) being the (group, column) one of the prepared image.
//
// Accumulation order of an output: exact int32 per (group, digit); digits
// combined in f32 (three roundings); groups of a K-range ascending with
// fma(scale / 16, X * factor, acc); K-ranges of a split row block ascending
// (last CTA to arrive).  The tolerance against the fp64 oracle is the
// suite's normwise bound; the order is not the reference's CPU order, which
// a tensor-core contraction cannot keep.
//
// Synchronisation: every wait is bounded (about one second, %globaltimer);
// on expiry the waiting role sets bit 2 of the fault flag
// (q4rdna_take_fault), stops, and the CTA drains its copies and MMAs (bounded
// again), frees its TMEM and exits: the outputs of that launch are then
// invalid.  No data atomics; the split arrival tickets are reset by the last
// CTA, as in the other kernels.

constexpr int kTcCG = 4;                                 // groups per chunk
constexpr int kTcRA = 2;                                 // A-blocks per work item
constexpr int kTcSpan = kTcCG * Q4_TILE_BYTES;           // one row tile, one chunk: 4352 B
constexpr int kTcRawW = kTcRA * Q4_BLOCK_TILES * kTcSpan;  // raw weight bytes of a stage: 34816
constexpr int kTcSlab = 576;                             // 16 rows x 32 K of an A plane + 64 B
constexpr int kTcAPlane = 8 * kTcSlab;                   // 128 rows x 32 K
constexpr int kTcABlock = 2 * kTcAPlane;                 // planes lo and hi
constexpr int kTcAStage = kTcRA * kTcABlock;             // one group, both A-blocks
constexpr int kTcFac = kTcCG * 16 * 4;                   // f32 factors [group][16 columns] per chunk
// warp roles: 0 copies, 1..3 MMA issue, 4..7 unpack, 8..23 epilogue (A-block x
// half of the batch columns x TMEM lane quarter).  24 warps, six per SM
// sub-partition (80 registers per thread).
constexpr int kTcMmaWarp0 = 1, kTcMmaWarps = 3, kTcUnpackWarp0 = 4, kTcUnpackWarps = 4, kTcEpiWarp0 = 8,
              kTcEpiWarps = 16;
constexpr int kTcWarps = 24;
constexpr int kTcThreads = kTcWarps * 32;
constexpr uint32_t kTcBias = 0x4B400000u;                // f32 1.5 * 2^23
constexpr float kTcBiasF = 12582912.0f;
constexpr uint64_t kTcWaitNs = 1000000000ull;            // bounded waits: 1 s
constexpr unsigned kFaultTileWait = 4u;                  // q4rdna_take_fault bit 2

template <int BP>
struct Tc {
    static constexpr int NCOL = 4 * BP;                  // MMA N: four digits per batch column
    static constexpr int IMGP = NCOL * 32;               // one plane of a group's operand image
    static constexpr int IMG = 2 * IMGP;                 // a group's operand image
    static constexpr int CHUNK = kTcCG * IMG + kTcFac;   // a chunk of the prepared activation
    static constexpr int RAW = kTcRawW + CHUNK;          // one stage of the copy ring
    static constexpr int NRAW = BP == 8 ? 3 : 2;         // raw stages in flight
    // TMEM accumulator slots (one group each) and unpacked A stages.  The
    // unpack warps reuse A stage n % NA after the MMAs of group n - NA, which
    // they learn from that group's TMEM slot barrier: NA <= NSL keeps that
    // barrier within one phase of the wait.
    static constexpr int NSL = BP == 8 ? 8 : 4;
    static constexpr int NA = BP == 8 ? 5 : 4;
    static constexpr int TCOLS = NSL * kTcRA * NCOL;     // all 512 TMEM columns
    static_assert(NA <= NSL, "A-stage reuse waits on the TMEM slot barrier");
    static constexpr int OFF_A = NRAW * RAW;
    static constexpr int OFF_X = OFF_A + NA * kTcAStage;  // SwiGLU gate sums [BP][128]
    static constexpr int OFF_BAR = OFF_X + BP * Q4_BLOCK_ROWS * 4;
    static constexpr int NBAR = 2 * NRAW + NA + 2 * NSL + 2 * kTcMmaWarps + 1;
    static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;  // TMEM address, last-CTA flag, norm scales
    static constexpr int SMEM = OFF_MISC + 16 + BP * 4;
    // instruction descriptor: D s32, A and B s8, both MN-major, N = NCOL, M = 128
    static constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | (1u << 16) |
                                      ((uint32_t)(NCOL >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
    static_assert(SMEM <= 232448, "shared memory of the tile kernel");
    static_assert(RAW % 16 == 0 && OFF_A % 16 == 0 && OFF_X % 16 == 0, "16-byte aligned stages");
};

// ------------------------------------------------------------ PTX wrappers

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits until the phase of the given parity has completed; false after about
// one second (the caller records the fault and stops).
__device__ __noinline__ bool mbar_wait_slow(uint32_t bar, uint32_t parity) {
    const uint64_t t0 = global_ns();
    for (uint32_t n = 1;; ++n) {
        if (mbar_try(bar, parity)) return true;
        if ((n & 63u) == 0 && global_ns() - t0 > kTcWaitNs) return false;
    }
}
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    return mbar_try(bar, parity) || mbar_wait_slow(bar, parity);
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    // no swizzle; LBO = stride of 8-element K blocks, SBO = stride of 16-element
    // M/N blocks (bytes >> 4); version 1 (bits 46..47)
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

__device__ __forceinline__ void tc_mma_i8(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, 1, 0;\n tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}" ::"r"(d),
        "l"(adesc), "l"(bdesc), "r"(idesc)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_ld_x16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_x32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_st_bias_x16(uint32_t taddr) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr), "r"(kTcBias) : "memory");
}
__device__ __forceinline__ void tmem_st_bias_x32(uint32_t taddr) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr), "r"(kTcBias) : "memory");
}
__device__ __forceinline__ void tmem_st_bias_x64(uint32_t taddr) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr), "r"(kTcBias) : "memory");
}

template <int NCOL>
__device__ __forceinline__ void tmem_bias(uint32_t taddr) {
    if constexpr (NCOL == 16) tmem_st_bias_x16(taddr);
    else if constexpr (NCOL == 32) tmem_st_bias_x32(taddr);
    else tmem_st_bias_x64(taddr);
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ------------------------------------------------------------ work items

__device__ __forceinline__ const Task &find_task_chunk(const Launch &L, long long chunk) {
    if (L.table == nullptr) return L.one;
    int lo = 0, hi = L.ntasks - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (L.table[mid].chunk_begin <= chunk) lo = mid; else hi = mid - 1;
    }
    return L.table[lo];
}

struct TcItem {
    const Task *T;
    int rb0;   // first row block
    int nab;   // A-blocks holding rows (1 or 2)
    bool dual; // A-blocks are the up and gate tiles of row block rb0
    int sc;    // K-range (split) index
    int g0, g1;  // groups [g0, g1), g0 a multiple of kTcCG
};

template <bool HAS_DUAL>
__device__ __forceinline__ TcItem tc_item(const Launch &L, long long it) {
    const Task &T = find_task(L, it);
    const int local = (int)(it - T.item_begin);
    TcItem I;
    I.T = &T;
    I.dual = HAS_DUAL && T.op == Q4RDNA_OP_SWIGLU;
    const int rbp = local / T.S;
    I.sc = local % T.S;
    I.rb0 = I.dual ? rbp : rbp * kTcRA;
    I.nab = I.dual ? 2 : min(kTcRA, T.RB - I.rb0);
    I.g0 = I.sc * T.Gs;
    I.g1 = min(T.G, I.g0 + T.Gs);
    return I;
}

// ------------------------------------------------------------ prep kernel

template <int BP>
__global__ void __launch_bounds__(128) q4_tc_prep_kernel(const __grid_constant__ Launch L) {
    using S = Tc<BP>;
    __shared__ __align__(16) uint8_t img[S::CHUNK];
    __shared__ float wmax[4][BP], wss[4][BP];
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const Task &T = find_task_chunk(L, blockIdx.x);
    const int c = (int)(blockIdx.x - T.chunk_begin);
    const int g0 = c * kTcCG, ng = min(kTcCG, T.G - g0);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool norm = T.gn != nullptr;
    const int B = L.B;
    asm volatile("griddepcontrol.wait;" ::: "memory");  // x comes from the previous kernel
    const size_t kk = (size_t)(g0 + w) * Q4_GROUP + 2 * lane;  // columns 2i, 2i + 1 of group g0 + w (i = lane)
    const bool have = w < ng;
    const float2 gv = (norm && have) ? __ldg(reinterpret_cast<const float2 *>(T.gn + kk)) : make_float2(1.0f, 1.0f);
    float2 v[BP];
#pragma unroll
    for (int b = 0; b < BP; ++b) {
        v[b] = (have && b < B) ? __ldg(reinterpret_cast<const float2 *>(T.x + (size_t)b * T.K + kk))
                               : make_float2(0.0f, 0.0f);
        float q = fmaf(v[b].x, v[b].x, v[b].y * v[b].y);
        v[b].x *= gv.x;
        v[b].y *= gv.y;
        float m = fmaxf(fabsf(v[b].x), fabsf(v[b].y));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            q += __shfl_xor_sync(0xffffffffu, q, o);
        }
        if (lane == 0) {
            wmax[w][b] = m;
            wss[w][b] = q;
        }
    }
    __syncthreads();
#pragma unroll
    for (int b = 0; b < BP; ++b) {
        const float f = act_scale(act_exponent(wmax[w][b]));  // per (group, column)
        const uint32_t d0 = act_digits(__float2int_rn(v[b].x * f));
        const uint32_t d1 = act_digits(__float2int_rn(v[b].y * f));
        // MMA row n = 4 b + d, K index i = lane: word (b, i) at 4 (b % 4) + 16 (i % 8) + 128 (i / 8) + 512 (b / 4)
        const int off = w * S::IMG + 4 * (b & 3) + 16 * (lane & 7) + 128 * (lane >> 3) + 512 * (b >> 2);
        *reinterpret_cast<uint32_t *>(img + off) = d0;
        *reinterpret_cast<uint32_t *>(img + off + S::IMGP) = d1;
    }
    if (threadIdx.x < kTcCG * 16) {  // factor of (group gg, column b); 0 for padded columns
        const int gg = threadIdx.x >> 4, b = threadIdx.x & 15;
        reinterpret_cast<float *>(img + kTcCG * S::IMG)[threadIdx.x] =
            b < B ? act_unscale(act_exponent(wmax[gg][b < BP ? b : 0])) : 0.0f;
    }
    if (norm && threadIdx.x < BP) {
        const int b = threadIdx.x;
        T.csum[(size_t)c * BP + b] = ((wss[0][b] + wss[1][b]) + wss[2][b]) + wss[3][b];
    }
    __syncthreads();
    uint4 *dst = reinterpret_cast<uint4 *>(T.img + (size_t)c * S::CHUNK);
    const uint4 *src = reinterpret_cast<const uint4 *>(img);
    for (int i = threadIdx.x; i < S::CHUNK / 16; i += 128) dst[i] = src[i];
}

// ------------------------------------------------------------ GEMV kernel

template <int BP, bool HAS_DUAL>
__global__ void __launch_bounds__(kTcThreads, 1) q4_tc_gemv_kernel(const __grid_constant__ Launch L) {
    using S = Tc<BP>;
    constexpr int NCOL = S::NCOL, NRAW = S::NRAW, NA = S::NA, NSL = S::NSL;
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t *raw = smem;
    uint8_t *abuf = smem + S::OFF_A;
    float *xch = reinterpret_cast<float *>(smem + S::OFF_X);
    const uint32_t bar0 = smem_u32(smem + S::OFF_BAR);
    // mbarriers (8 bytes each).  Group n of the CTA's sequence uses A stage
    // n % NA and TMEM slot n % NSL; its MMAs are issued by MMA warp n % kTcMmaWarps (a
    // tcgen05.mma or commit holds its issuing thread for about a hundred
    // cycles, so one thread cannot keep up with the stream),
    // whose one commit per group (mma_done) tells the epilogue that the slot
    // holds the sums and the unpack warps that the A stage may be rewritten;
    // each group's warp also commits to its chunk's raw_empty (the chunk's
    // operand image has been read).  A waiter never falls two phases behind a
    // barrier: the next phase of each barrier it waits on needs the waiter's
    // own progress first.
    auto raw_full = [&](int s) { return bar0 + 8u * s; };                        // copies landed
    auto raw_empty = [&](int s) { return bar0 + 8u * (NRAW + s); };              // unpacked, image read
    auto a_full = [&](int s) { return bar0 + 8u * (2 * NRAW + s); };             // A stage unpacked
    auto mma_done = [&](int s) { return bar0 + 8u * (2 * NRAW + NA + s); };      // slot's MMAs complete
    auto acc_empty = [&](int s) { return bar0 + 8u * (2 * NRAW + NA + NSL + s); };  // slot read
    auto drain = [&](int s) { return bar0 + 8u * (2 * NRAW + NA + 2 * NSL + s); };    // issuer s's last MMAs
    const uint32_t epi_bar = bar0 + 8u * (2 * NRAW + NA + 2 * NSL + kTcMmaWarps);  // the epilogue warps meet here
    // the MMA warps take their waits in group order: group n's warp starts its
    // waits once group n - 1's warp has passed its own (phase n / kTcMmaWarps of
    // turn(n % kTcMmaWarps)), so that no waiter is ever a phase ahead of a barrier;
    // the MMAs themselves overlap
    auto turn = [&](int j) { return bar0 + 8u * (2 * NRAW + NA + 2 * NSL + kTcMmaWarps + 1 + j); };
    // the completion of group n's MMAs is phase n / NSL of mma_done(n % NSL)
    auto wait_group = [&](uint32_t n) { return mbar_wait(mma_done(n % NSL), (n / NSL) & 1u); };
    uint32_t *misc = reinterpret_cast<uint32_t *>(smem + S::OFF_MISC);  // [0] TMEM address, [1] last-CTA flag
    float *nrm = reinterpret_cast<float *>(smem + S::OFF_MISC + 16);

    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(misc)),
                     "r"((uint32_t)S::TCOLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (threadIdx.x == 32) {
        for (int s = 0; s < NRAW; ++s) {
            mbar_init(raw_full(s), 1);
            mbar_init(raw_empty(s), kTcUnpackWarps + kTcCG);  // unpack warps, one commit per group
        }
        for (int s = 0; s < NA; ++s) mbar_init(a_full(s), kTcUnpackWarps);
        for (int s = 0; s < NSL; ++s) {
            mbar_init(mma_done(s), 1);
            mbar_init(acc_empty(s), kTcEpiWarps);
        }
        for (int s = 0; s < kTcMmaWarps; ++s) {
            mbar_init(drain(s), 1);
            mbar_init(turn(s), 1);
        }
        mbar_arrive(turn(0));  // group 0 has no predecessor
        mbar_init(epi_bar, kTcEpiWarps);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = misc[0];
    const int epi = warp - kTcEpiWarp0;  // epilogue warp index 0..15
    constexpr int HB = BP / 2;           // batch columns of one epilogue thread
    if (epi >= 0) {
        // every accumulator word of this warp's lanes and columns starts at the bias
        const uint32_t lanes = (uint32_t)(32 * (warp & 3)) << 16;
        const int set = epi >> 3, half = (epi >> 2) & 1;
        for (int ts = 0; ts < NSL; ++ts)
            tmem_bias<NCOL / 2>(tmem + lanes + ts * kTcRA * NCOL + set * NCOL + half * (NCOL / 2));
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();

    bool ok = true;
    if (warp == 0) {
        // ---------------------------------------------------------- producer
        // The whole warp walks the chunks; lanes 0..7 issue the 8 tile-run
        // copies of a chunk and lane 8 its operand image, so that the copies of
        // a chunk are issued at once (one thread spends a few hundred cycles per
        // cp.async.bulk and cannot keep up with the stream on its own).
        uint32_t rit = 0;
        bool waited = false;
        for (long long it = blockIdx.x; ok && it < L.total_items; it += gridDim.x) {
            const TcItem I = tc_item<HAS_DUAL>(L, it);
            const Task &T = *I.T;
            const int rtiles = T.N / Q4_TILE_ROWS;
            for (int g = I.g0; g < I.g1; g += kTcCG, ++rit) {
                const int ng = min(kTcCG, I.g1 - g);
                const int s = rit % NRAW;
                bool free_stage = true;
                if (lane == 0) free_stage = mbar_wait(raw_empty(s), ((rit / NRAW) & 1u) ^ 1u);
                if (!__shfl_sync(0xffffffffu, free_stage, 0)) { ok = false; break; }
                const uint32_t dst = smem_u32(raw + (size_t)s * S::RAW);
                if (lane == 0) {
                    uint32_t bytes = S::CHUNK;
                    for (int a = 0; a < I.nab; ++a) {
                        const int rb = I.dual ? I.rb0 : I.rb0 + a;
                        for (int t = 0; t < Q4_BLOCK_TILES; ++t)
                            if (rb * Q4_BLOCK_TILES + t < rtiles) bytes += (uint32_t)ng * Q4_TILE_BYTES;
                    }
                    mbar_expect_tx(raw_full(s), bytes);
                }
                __syncwarp();
                if (lane < kTcRA * Q4_BLOCK_TILES) {
                    const int a = lane >> 2, t = lane & 3;
                    const int rb = I.dual ? I.rb0 : I.rb0 + a;
                    const int rt = rb * Q4_BLOCK_TILES + t;
                    if (a < I.nab && rt < rtiles)
                        bulk_g2s(dst + (uint32_t)((a * Q4_BLOCK_TILES + t) * kTcSpan),
                                 ((I.dual && a == 1) ? T.w2 : T.w) + ((size_t)rt * T.G + g) * Q4_TILE_BYTES,
                                 (uint32_t)ng * Q4_TILE_BYTES, raw_full(s));
                } else if (lane == kTcRA * Q4_BLOCK_TILES) {
                    if (!waited) {  // the operand image is written by the prep kernel
                        asm volatile("griddepcontrol.wait;" ::: "memory");
                        waited = true;
                    }
                    bulk_g2s(dst + kTcRawW, T.img + (size_t)(g / kTcCG) * S::CHUNK, S::CHUNK, raw_full(s));
                }
            }
        }
        if (!ok && lane == 0) atomicOr(&g_fault, kFaultTileWait);
        // no copy may still be landing when the CTA leaves
        if (lane == 0)
            for (uint32_t k = rit > (uint32_t)NRAW ? rit - NRAW : 0; k < rit; ++k)
                mbar_wait(raw_full(k % NRAW), (k / NRAW) & 1u);
    } else if (warp < kTcUnpackWarp0) {
        // ---------------------------------------------------------- MMA issue (warp 1 + j: groups n % kTcMmaWarps == j)
        const int j = warp - kTcMmaWarp0;
        if (lane == 0) {
            uint32_t rit = 0, ait = 0;
            bool issued = false;
            for (long long it = blockIdx.x; ok && it < L.total_items; it += gridDim.x) {
                const TcItem I = tc_item<HAS_DUAL>(L, it);
                for (int g = I.g0; ok && g < I.g1; g += kTcCG, ++rit) {
                    const int ng = min(kTcCG, I.g1 - g);
                    const int s = rit % NRAW;
                    const uint32_t img = smem_u32(raw + (size_t)s * S::RAW + kTcRawW);
                    for (int gi = 0; gi < ng; ++gi, ++ait) {
                        if ((int)(ait % kTcMmaWarps) != j) continue;
                        const int as = ait % NA, ts = ait % NSL;
                        if (!mbar_wait(turn(j), (ait / kTcMmaWarps) & 1u) || !mbar_wait(raw_full(s), (rit / NRAW) & 1u) ||
                            !mbar_wait(a_full(as), (ait / NA) & 1u) ||
                            !mbar_wait(acc_empty(ts), ((ait / NSL) & 1u) ^ 1u)) {
                            ok = false;
                            break;
                        }
                        mbar_arrive(turn((j + 1) % kTcMmaWarps));  // group ait + 1's warp may wait now
                        tc_fence_after();
                        const uint32_t A = smem_u32(abuf + (size_t)as * kTcAStage);
                        for (int a = 0; a < I.nab; ++a) {
                            const uint32_t d = tmem + (uint32_t)(ts * kTcRA * NCOL + a * NCOL);
                            for (int p = 0; p < 2; ++p)
                                tc_mma_i8(d, smem_desc(A + a * kTcABlock + p * kTcAPlane, 128, kTcSlab),
                                          smem_desc(img + gi * S::IMG + p * S::IMGP, 128, 512), S::IDESC);
                        }
                        tc_commit(mma_done(ts));
                        // this group's MMAs have read the chunk's image (a commit covers only
                        // the committing thread's MMAs; in a short last chunk the last group
                        // stands in for the missing ones)
                        for (int c = (gi == ng - 1 ? kTcCG - ng : 0); c >= 0; --c) tc_commit(raw_empty(s));
                        issued = true;
                    }
                }
            }
            if (!ok) atomicOr(&g_fault, kFaultTileWait);
            // every MMA of this warp has completed before the TMEM is freed
            if (issued) {
                tc_commit(drain(j));
                mbar_wait(drain(j), 0);
            }
        }
    } else if (warp < kTcEpiWarp0) {
        // ---------------------------------------------------------- unpack
        const int ut = threadIdx.x - 32 * kTcUnpackWarp0;
        const int loc = ut & 63;
        const int pi = ((loc >> 3) << 2) | (loc & 3), ph16 = (loc >> 2) & 1;  // pair column i, row half h
        uint32_t rit = 0, ait = 0;
        for (long long it = blockIdx.x; ok && it < L.total_items; it += gridDim.x) {
            const TcItem I = tc_item<HAS_DUAL>(L, it);
            for (int g = I.g0; ok && g < I.g1; g += kTcCG, ++rit) {
                const int ng = min(kTcCG, I.g1 - g);
                const int s = rit % NRAW;
                if (!mbar_wait(raw_full(s), (rit / NRAW) & 1u)) { ok = false; break; }
                const uint8_t *rs = raw + (size_t)s * S::RAW;
                for (int gi = 0; gi < ng; ++gi, ++ait) {
                    const int as = ait % NA;
                    // the A stage is free once the MMAs of group ait - NA have completed
                    if (ait >= (uint32_t)NA && !wait_group(ait - NA)) { ok = false; break; }
                    uint8_t *A = abuf + (size_t)as * kTcAStage;
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int a = u >> 1, t = ((u & 1) << 1) | (ut >> 6);
                        const uint4 w = *reinterpret_cast<const uint4 *>(
                            rs + (a * Q4_BLOCK_TILES + t) * kTcSpan + gi * Q4_TILE_BYTES + Q4_SCALE_BYTES + 32 * pi +
                            16 * ph16);
                        uint4 lo, hi;
                        lo.x = (w.x << 4) & 0xF0F0F0F0u; hi.x = w.x & 0xF0F0F0F0u;
                        lo.y = (w.y << 4) & 0xF0F0F0F0u; hi.y = w.y & 0xF0F0F0F0u;
                        lo.z = (w.z << 4) & 0xF0F0F0F0u; hi.z = w.z & 0xF0F0F0F0u;
                        lo.w = (w.w << 4) & 0xF0F0F0F0u; hi.w = w.w & 0xF0F0F0F0u;
                        uint8_t *dst = A + a * kTcABlock + (2 * t + ph16) * kTcSlab + (pi >> 3) * 128 + (pi & 7) * 16;
                        *reinterpret_cast<uint4 *>(dst) = lo;
                        *reinterpret_cast<uint4 *>(dst + kTcAPlane) = hi;
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) mbar_arrive(a_full(as));
                }
                __syncwarp();
                if (ok && lane == 0) mbar_arrive(raw_empty(s));
            }
        }
        if (!ok && lane == 0) atomicOr(&g_fault, kFaultTileWait);
    } else {
        // ---------------------------------------------------------- epilogue
        // warp (set, half, quarter q): row m = 32 q + lane of A-block `set`,
        // batch columns half * BP / 2 .. + BP / 2
        const int set = epi >> 3, half = (epi >> 2) & 1, q = warp & 3;
        const int m = 32 * q + lane;  // row within the row block = TMEM lane
        const int b0 = half * HB;
        const uint32_t lanes = (uint32_t)(32 * q) << 16;
        asm volatile("griddepcontrol.wait;" ::: "memory");  // add, norm sums, operand factors and outputs
        uint32_t ait = 0, eph = 0;
        // the epilogue warps' meeting point (an mbarrier, so that the wait is bounded)
        auto epi_sync = [&]() -> bool {
            __syncwarp();
            if (lane == 0) mbar_arrive(epi_bar);
            const bool r = mbar_wait(epi_bar, eph);
            eph ^= 1u;
            return r;
        };
        for (long long it = blockIdx.x; ok && it < L.total_items; it += gridDim.x) {
            const TcItem I = tc_item<HAS_DUAL>(L, it);
            const Task &T = *I.T;
            // this row's tile and its fp16 scales (read through L2, behind the
            // copy warp's bulk copy of the same tiles)
            const int rbm = I.dual ? I.rb0 : I.rb0 + set;
            const int rt = rbm * Q4_BLOCK_TILES + q;
            const bool have_row = (I.dual || set < I.nab) && rt < T.N / Q4_TILE_ROWS;
            const uint8_t *srow = ((I.dual && set == 1) ? T.w2 : T.w) +
                                  (size_t)(have_row ? rt : 0) * T.G * Q4_TILE_BYTES + 2 * lane;
            auto scale_of = [&](int g) -> float {
                return have_row ? __half2float(__ldg(reinterpret_cast<const __half *>(srow + (size_t)g * Q4_TILE_BYTES))) *
                                      0.0625f
                                : 0.0f;
            };
            float acc[HB];
#pragma unroll
            for (int b = 0; b < HB; ++b) acc[b] = 0.0f;
            float sc_next = scale_of(I.g0);
            for (int g = I.g0; g < I.g1; ++g, ++ait) {
                const int ts = ait % NSL;
                const float sc = sc_next;
                if (g + 1 < I.g1) sc_next = scale_of(g + 1);
                // factors 2^(E - 156) of this group's columns (from the prepared image)
                const float4 *fg = reinterpret_cast<const float4 *>(
                    T.img + (size_t)(g / kTcCG) * S::CHUNK + kTcCG * S::IMG + ((g % kTcCG) * 16 + b0) * 4);
                if (!mbar_wait(mma_done(ts), (ait / NSL) & 1u)) { ok = false; break; }
                tc_fence_after();
                const uint32_t taddr = tmem + lanes + (uint32_t)(ts * kTcRA * NCOL + set * NCOL + half * (NCOL / 2));
                // four batch columns (16 words) per load
#pragma unroll
                for (int h = 0; h < HB / 4; ++h) {
                    uint32_t v[16];
                    tmem_ld_x16(taddr + 16 * h, v);
                    const float4 f4 = __ldg(fg + h);
                    const float fac[4] = {f4.x, f4.y, f4.z, f4.w};
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float f0 = __uint_as_float(v[4 * j]) - kTcBiasF;
                        const float f1 = __uint_as_float(v[4 * j + 1]) - kTcBiasF;
                        const float f2 = __uint_as_float(v[4 * j + 2]) - kTcBiasF;
                        const float f3 = __uint_as_float(v[4 * j + 3]) - kTcBiasF;
                        const float X = fmaf(fmaf(fmaf(f3, 256.0f, f2), 256.0f, f1), 256.0f, f0);
                        // X * 2^(E - 156) first: scale / 16 * 2^(E - 156) can be subnormal
                        acc[4 * h + j] = fmaf(sc, X * fac[j], acc[4 * h + j]);
                    }
                }
                tmem_bias<NCOL / 2>(taddr);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(acc_empty(ts));
            }
            if (!ok) break;

            // ------------------------------------------------ item outputs
            const int B = L.B;
            const bool norm = T.gn != nullptr;
            const int row = rbm * Q4_BLOCK_ROWS + m;
            const bool mine = (I.dual || set < I.nab) && row < T.N;
            const int nb = max(0, min(HB, B - b0));  // real batch columns of this thread
            const int nch = (T.G + kTcCG - 1) / kTcCG;
            auto norm_scales = [&]() {  // 1 / sqrt(mean(h^2) + eps) per batch column, chunks ascending
                if (epi == 0 && lane < BP) {
                    float ssum = 0.0f;
                    for (int c = 0; c < nch; ++c) ssum += T.csum[(size_t)c * BP + lane];
                    nrm[lane] = norm_scale(T, ssum);
                }
            };
            if (T.S == 1) {
                if (norm) norm_scales();
                if (I.dual && set == 1) {
#pragma unroll
                    for (int j = 0; j < HB; ++j) xch[(b0 + j) * Q4_BLOCK_ROWS + m] = acc[j];
                }
                if ((norm || I.dual) && !epi_sync()) { ok = false; break; }
                if (mine && (!I.dual || set == 0))
                    for (int j = 0; j < nb; ++j) {
                        const int b = b0 + j;
                        const float r = norm ? nrm[b] : 1.0f;
                        const float gate = I.dual ? xch[b * Q4_BLOCK_ROWS + m] : acc[j];
                        const size_t idx = (size_t)b * T.N + row;
                        put_y(T, idx, finish(acc[j] * r, gate * r, T.op, T.add, idx));
                    }
                if ((norm || I.dual) && !epi_sync()) { ok = false; break; }
                continue;
            }
            // K-ranges of several CTAs: partial sums, then the last CTA adds them in order
            const int planes = I.dual ? 2 : 1;
            const size_t split_stride = (size_t)planes * B * T.N;
            const int plane = I.dual ? set : 0;
            if (mine)
                for (int j = 0; j < nb; ++j)
                    __stcg(&T.part[(size_t)I.sc * split_stride + (size_t)plane * B * T.N + (size_t)(b0 + j) * T.N + row],
                           acc[j]);
            __threadfence();
            if (!epi_sync()) { ok = false; break; }
            if (epi == 0 && lane == 0) misc[1] = atomicAdd(&T.ticket[I.rb0], 1u) == (unsigned)(T.S - 1) ? 1u : 0u;
            if (!epi_sync()) { ok = false; break; }
            if (misc[1] == 0) continue;
            __threadfence();
            if (norm) norm_scales();
            if (!epi_sync()) { ok = false; break; }
            if (mine && (!I.dual || set == 0))
                for (int j = 0; j < nb; ++j) {
                    const size_t idx = (size_t)(b0 + j) * T.N + row;
                    float v[2] = {0.0f, 0.0f};
                    for (int pl = 0; pl < planes; ++pl) {
                        float sum = 0.0f;
                        for (int sp = 0; sp < T.S; ++sp)
                            sum += __ldcg(&T.part[(size_t)sp * split_stride + (size_t)pl * B * T.N + idx]);
                        v[pl] = sum;
                    }
                    const float r = norm ? nrm[b0 + j] : 1.0f;
                    put_y(T, idx, finish(v[0] * r, v[planes - 1] * r, T.op, T.add, idx));
                }
            if (!epi_sync()) { ok = false; break; }
            if (epi == 0 && lane == 0) atomicExch(&T.ticket[I.rb0], 0u);
        }
        if (!ok && lane == 0) atomicOr(&g_fault, kFaultTileWait);
        // no TMEM access of this warp is outstanding when the TMEM is freed
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)S::TCOLS)
                     : "memory");
    }
}
