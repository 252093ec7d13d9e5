// TMA-ring primitives (included into q4rdna_gemv.cu inside namespace q4):
// mbarriers with bounded waits, bulk global->shared copies, and the ring shape
// used by q4_gemv_i8_tma_kernel (q4rdna_gemv_i8_tma.cuh).
//
// The tiles reach the SM by bulk copies (cp.async.bulk, the TMA engine) into a
// per-warp ring of shared-memory stages instead of by 128-bit register loads.
// A stage holds, for the item's four 32-row tiles, CHUNK consecutive steps (one
// contiguous run of CHUNK*1088 bytes per tile row for a plain tensor; up and
// gate tiles alternate for SwiGLU), and each warp keeps up to STAGES - 1 stages
// in flight with no registers spent on them.
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

