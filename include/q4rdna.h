/*
 * q4rdna.h - C ABI of the B200 (sm_100a) Q4_RDNA group-64 decode GEMV.
 *
 * Plain pointers and sizes only.  Every device pointer is a CUDA device address
 * on the current device; streams are cudaStream_t (declared here as an opaque
 * pointer so the header needs no CUDA include).  All compute entry points are
 * stream-ordered and never synchronise; they return a status and never abort.
 *
 * Weights use the reference's packed layout unchanged (32-row x 64-column
 * tiles of 1088 bytes; see q4rdna_tile.h), so a tensor is N*K*34/64 bytes
 * with N % 32 == 0 and K % 64 == 0.  Activations x are f32 [B][K] (column b at
 * x + b*K); outputs y are f32 [B][N].
 *
 * Reference interfaces these replace (paths inside davidchen-rocm/RDNA-gfx1201-v0.1):
 *   source/q4rdna.cuh:5-24       ggml_cuda_q4rdna_mul_mat / _mul_mat_add / _mul_mat_glu
 *   source/q4rdna.cu:119-179     q4rdna_initialize (sidecar load + validation)
 *   source/q4rdna.cu:578-680     q4rdna_launch and its split selector
 *   source/q4rdna.cu:682-709     q4rdna_find / q4rdna_count (name registry, hits)
 *   source/q4rdna.cu:73-112      launch counter and exit-time shape histogram
 */
#ifndef Q4RDNA_H
#define Q4RDNA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default) /* the library builds with -fvisibility=hidden */
#endif

typedef struct CUstream_st *q4rdna_stream_t; /* == cudaStream_t */

typedef enum q4rdna_status {
    Q4RDNA_OK = 0,
    Q4RDNA_ERR_INVALID_ARGUMENT = 1, /* null pointer, non-positive size, unknown op */
    Q4RDNA_ERR_SHAPE = 2,            /* N % 32 != 0, K % 64 != 0, or shape mismatch */
    Q4RDNA_ERR_ALIGNMENT = 3,        /* tiles not 16-byte aligned, x/y/add not 8-byte aligned */
    Q4RDNA_ERR_WORKSPACE = 4,        /* workspace missing or smaller than q4rdna_workspace_bytes */
    Q4RDNA_ERR_UNSUPPORTED = 5,      /* batch B outside [1, Q4RDNA_MAX_BATCH] */
    Q4RDNA_ERR_CUDA = 6,             /* a CUDA call failed (launch, copy, allocation) */
    Q4RDNA_ERR_IO = 7,               /* sidecar file missing, unreadable or truncated */
    Q4RDNA_ERR_FORMAT = 8,           /* sidecar header or entry fails validation */
    Q4RDNA_ERR_NOT_FOUND = 9,        /* tensor name not in the sidecar */
    Q4RDNA_ERR_DEVICE = 10,          /* wrong or unavailable CUDA device */
    Q4RDNA_ERR_TOO_LARGE = 11        /* size beyond a fixed limit of the entry point */
} q4rdna_status;

#define Q4RDNA_MAX_BATCH 16

/* Which epilogue a GEMV applies (reference kernels' use_add / use_gate). */
typedef enum q4rdna_op {
    Q4RDNA_OP_PLAIN = 0,  /* y = W x                      (q4rdna.cu:713-745) */
    Q4RDNA_OP_ADD = 1,    /* y = W x + add                (q4rdna.cu:747-767) */
    Q4RDNA_OP_SWIGLU = 2  /* y = (W_up x) * silu(W_gate x) (q4rdna.cu:769-793) */
} q4rdna_op;

/* Launch options.  split = 0 lets the selector choose the split-K factor;
 * split > 0 forces it (clamped to [1, K/64]).  flags: Q4RDNA_CFG_* bits. */
typedef struct q4rdna_cfg {
    int split;
    int flags;
    int reserved[6];
} q4rdna_cfg;

/* Single calls at B = 1..2: let the GEMV start streaming its first weights
 * while the previous kernel on the stream finishes (programmatic dependent
 * launch).  Everything the previous kernels write (x, y, add, the
 * workspace) is touched only after they complete; only the weight tiles are
 * read early, so the caller guarantees that no kernel still running on the
 * stream writes them (true for weights loaded once, e.g. a sidecar). */
#define Q4RDNA_CFG_OVERLAP_PREVIOUS 1

const char *q4rdna_status_string(q4rdna_status s);
/* Library version string. */
const char *q4rdna_version(void);

/* Split-K factor the selector would use for (N, K, B, op) on the current device. */
int q4rdna_select_split(int N, int K, int B, int op);

/* Device workspace a single GEMV needs: split-K partial sums plus arrival
 * tickets (0 when the chosen split is 1 and B < 8, and at B <= 2 for splits
 * up to 8, whose K-ranges meet in a thread-block cluster: the default
 * selector's choice, so the name-keyed operators allocate nothing per stream
 * unless LLAMA_Q4_RDNA_COOP forces a larger split), and at B >= 8 (the
 * tensor-core tile path) also the activation prepared for the tensor cores
 * (4 bytes per element of x, plus a small per-chunk table).  A workspace must
 * be zero-filled once when it is allocated (q4rdna_workspace_init); every call
 * leaves its tickets zeroed again.  Calls that share a workspace must be
 * ordered on one stream. */
size_t q4rdna_workspace_bytes(int N, int K, int B, int op, const q4rdna_cfg *cfg);
q4rdna_status q4rdna_workspace_init(void *workspace, size_t bytes, q4rdna_stream_t stream);

/* y = W x.  Replaces the launch inside ggml_cuda_q4rdna_mul_mat
 * (source/q4rdna.cu:736-741, q4rdna_launch<false,false>). */
q4rdna_status q4rdna_gemv(const uint8_t *tiles, const float *x, float *y, int N, int K, int B,
                          const q4rdna_cfg *cfg, void *workspace, size_t workspace_bytes,
                          q4rdna_stream_t stream);

/* y = W x + add, add f32 [B][N].  Replaces source/q4rdna.cu:760-763
 * (q4rdna_launch<false,true>). */
q4rdna_status q4rdna_gemv_add(const uint8_t *tiles, const float *x, const float *add, float *y,
                              int N, int K, int B, const q4rdna_cfg *cfg, void *workspace,
                              size_t workspace_bytes, q4rdna_stream_t stream);

/* y = (W_up x) * silu(W_gate x), both tensors N x K, streamed by one kernel.
 * Replaces source/q4rdna.cu:785-788 (q4rdna_launch<true,false>). */
q4rdna_status q4rdna_gemv_swiglu(const uint8_t *up_tiles, const uint8_t *gate_tiles, const float *x,
                                 float *y, int N, int K, int B, const q4rdna_cfg *cfg,
                                 void *workspace, size_t workspace_bytes, q4rdna_stream_t stream);

/* The GEMV with its input produced by RMSNorm in the same kernel:
 *   y = W (h * g) / sqrt(mean(h^2) + eps) [+ add | * silu(...) for SwiGLU]
 * per batch column, h f32 [B][K] the raw hidden state, g = norm_weight f32 [K]
 * (8-byte aligned).  This is the ggml rms_norm + mul pair that feeds the
 * reference's mul_mat nodes (the llama.cpp graph before
 * llama-cpp-q4rdna-integration.patch:17-19), fused into the weight stream: the
 * sum of h^2 is taken while the activation groups are prepared, and the scale
 * is applied once per output (after the split-K reduction when S > 1, splits
 * in ascending order).  op, gate_tiles and add as in q4rdna_gemv_swiglu /
 * q4rdna_gemv_add; the workspace is sized by q4rdna_workspace_bytes. */
q4rdna_status q4rdna_gemv_rmsnorm(const uint8_t *tiles, const uint8_t *gate_tiles, const float *h,
                                  const float *norm_weight, float eps, const float *add, float *y, int N, int K,
                                  int B, int op, const q4rdna_cfg *cfg, void *workspace, size_t workspace_bytes,
                                  q4rdna_stream_t stream);

/* y = W x without any allocation and without a workspace argument.  No
 * counterpart in the reference.  For callers that cannot call cudaMalloc: an
 * operator hook inside a host framework (like the llama.cpp mul_mat hook) gets
 * only its input and output tensors, device memory belongs to the framework's
 * pool, and allocating there would stall the device and bypass the framework's
 * memory accounting.  The split-K scratch is a fixed array of
 * Q4RDNA_NOALLOC_SCRATCH_BYTES inside this library, held by every GPU that
 * loads it until the process exits.  Calls whose split-K scratch would not fit
 * return Q4RDNA_ERR_TOO_LARGE.  Results equal q4rdna_gemv's for the same cfg.
 * The first call on a device looks up the array's device address (a one-time
 * set-up per device); make that first call before any stream capture.  All
 * calls on a device share the one array, so calls that overlap on the GPU (on
 * different streams, or from several threads) race and must be serialised by
 * the caller. */
#define Q4RDNA_NOALLOC_SCRATCH_BYTES (8u << 20)
q4rdna_status q4rdna_gemv_noalloc(const uint8_t *tiles, const float *x, float *y, int N, int K, int B,
                                  const q4rdna_cfg *cfg, q4rdna_stream_t stream);

/* Debug: dense row-major W[N][K] = fp16 scale * int4 code, bit-exact (an fp16
 * scale times an integer in [-8, 7] is exact in f32).  No reference
 * counterpart; it is the dequantisation the reference kernels perform inline
 * (source/q4rdna.cu:346-371). */
q4rdna_status q4rdna_dequant_f32(const uint8_t *tiles, float *W, int N, int K, q4rdna_stream_t stream);

/* ---- Q4_K rows: the tensors the reference leaves on llama.cpp's stock path ----
 * The qkv-fallback scope (source/q4rdna.cu:685-691, LLAMA_Q4_RDNA_SCOPE)
 * routes attn_q/k/v to the caller's Q4_K kernel; the reference bench times a
 * Q4_K GEMV (q4_k_gemv, source/q4rdna_gemv_bench.hip:93-135) beside its own.
 * These entry points run such tensors on the GPU with the same stream and
 * status conventions.  Layout (source/q4rdna_cpu_experiment.cpp:17, 102-135):
 * a row is K/256 blocks of 144 bytes (fp16 d, fp16 dmin, 12 bytes of 6-bit
 * scales and mins, 128 bytes of unsigned nibbles); weight = d * scale * q -
 * dmin * min per 32-column sub-block.  K % 256 == 0; blocks 16-byte aligned,
 * x 16-byte aligned, y and add 4-byte aligned; x must be finite. */
#define Q4RDNA_Q4K_BLOCK 256
#define Q4RDNA_Q4K_BLOCK_BYTES 144

/* Bytes of an N x K Q4_K tensor (0 for a bad shape). */
size_t q4rdna_q4k_bytes(int N, int K);

/* y = W x (+ add when add != NULL), x f32 [B][K], y and add f32 [B][N],
 * B in [1, Q4RDNA_MAX_BATCH].  No workspace and no allocation. */
q4rdna_status q4rdna_q4k_gemv(const uint8_t *blocks, const float *x, const float *add, float *y, int N, int K,
                              int B, q4rdna_stream_t stream);

/* Debug: dense row-major W[N][K], bit-exact with the reference's
 * dequantize_q4_k (source/q4rdna_cpu_experiment.cpp:112-135) on IEEE fp16
 * decoding of d and dmin. */
q4rdna_status q4rdna_q4k_dequant_f32(const uint8_t *blocks, float *W, int N, int K, q4rdna_stream_t stream);

/* ---- multi-GEMV plans: many independent GEMVs in one persistent launch ----
 * One descriptor per GEMV; all share the batch B.  gate_tiles is used only by
 * Q4RDNA_OP_SWIGLU, add only by Q4RDNA_OP_ADD.  The plan copies the
 * descriptor table to the device once and owns its workspace; the caller keeps
 * the buffers alive and rewrites x in place between runs.  No reference
 * counterpart: the reference launches one kernel per mul_mat node. */
typedef struct q4rdna_gemv_desc {
    const uint8_t *tiles;
    const uint8_t *gate_tiles;
    const float *x;
    const float *add;
    float *y;
    int N;
    int K;
    int op;
    int split; /* 0 = selector */
    /* fused RMSNorm (q4rdna_gemv_rmsnorm): norm weight [K] or NULL; x is then the raw input h */
    const float *norm_weight;
    float norm_eps;
    /* weight format of `tiles`: Q4RDNA_FORMAT_Q4RDNA (0, the default) or
     * Q4RDNA_FORMAT_Q4K (ggml block_q4_K rows; op PLAIN or ADD, no norm) */
    int format;
} q4rdna_gemv_desc;

typedef enum q4rdna_format {
    Q4RDNA_FORMAT_Q4RDNA = 0, /* 32 x 64 tiles of 1088 bytes (q4rdna.cu:20-24) */
    Q4RDNA_FORMAT_Q4K = 1     /* ggml block_q4_K: 144 bytes per 256 weights of a row */
} q4rdna_format;

typedef struct q4rdna_plan q4rdna_plan;
typedef struct q4rdna_plan_info {
    int count;             /* GEMVs in the plan */
    int batch;             /* B */
    int64_t items;         /* warp work items per run */
    int grid;              /* CTAs launched per run */
    uint64_t weight_bytes; /* packed weight bytes streamed per run */
    uint64_t algo_bytes;   /* weights + activations + outputs (+ add) per run */
    size_t workspace_bytes;
} q4rdna_plan_info;

q4rdna_status q4rdna_plan_create(const q4rdna_gemv_desc *descs, int count, int B, q4rdna_plan **out);
q4rdna_status q4rdna_plan_run(q4rdna_plan *plan, q4rdna_stream_t stream);
q4rdna_status q4rdna_plan_get_info(const q4rdna_plan *plan, q4rdna_plan_info *info);
void q4rdna_plan_destroy(q4rdna_plan *plan);

/* One plan run from host memory, with the transfers overlapped with the GEMVs.
 * [x_dev, x_dev + x_bytes) must hold every descriptor's activations and
 * x_host mirrors it byte for byte; [y_dev, y_dev + y_bytes) must hold every
 * output and y_host receives it byte for byte (pinned host memory lets the
 * copies run asynchronously).  The plan is cut into `segments` runs of
 * consecutive descriptors (0: 2 with direct output stores, see below, else 3)
 * whose weight bytes are graded, in proportion to 2^min(s, segments - 1 - s):
 * small runs at both ends.  Segment s's
 * activations are copied in on a library copy stream, its GEMVs wait for that
 * copy only, and its outputs are copied out on a second copy stream as soon
 * as they are written.  Consecutive segments run on two library streams, so a
 * segment starts on the SMs the previous one leaves idle.  Only the first
 * (smallest) segment's input copy and the last (smallest) segment's output
 * copy are not hidden behind the weight stream.  When y_host is pinned host
 * memory mapped for the device (cudaHostAlloc / cudaMallocHost, or registered
 * as mapped), the kernels also store their outputs straight into it, so no
 * output copies remain and the runs grow instead; a pageable y_host
 * keeps the output copies (Q4RDNA_HOST_DIRECT=0 forces them); with direct
 * stores the runs' weight bytes grow as 4^s (Q4RDNA_HOST_GROWTH).  y_dev receives
 * the outputs either way.  The whole sequence is
 * captured once into a CUDA graph (per set of buffers) and replayed, so a call
 * costs one graph launch of host time (Q4RDNA_HOST_GRAPH=0: direct launches).
 * The first call with a given set of buffers does the capture; make it outside
 * any stream capture of the caller.  The
 * segments' activation ranges must not overlap, nor their output ranges.
 * Q4_K descriptors (Q4RDNA_FORMAT_Q4K) form one more segment: their
 * activations are copied in first, their launch runs beside the first Q4_RDNA
 * segment and their outputs are copied out (never stored straight into
 * y_host).  When the Q4_K descriptors' byte range of activations or of
 * outputs meets a Q4_RDNA segment's, the call instead copies all of x in,
 * runs the plan and copies all of y out; placing the Q4_K tensors' inputs and
 * outputs apart (say first in both buffers) keeps the overlap.
 * With a fused gather (q4rdna_plan_set_gather) the segments also store into
 * every rank's gathered buffer and the run ends with the flag exchange; y_host
 * then receives this rank's outputs (its y buffer), and the calls are direct
 * launches (no graph).
 * Ordered after prior work on `stream`; `stream` waits for the last copy.  No
 * synchronisation; calls on one plan must not overlap.  No reference
 * counterpart (the reference keeps activations on the GPU). */
q4rdna_status q4rdna_plan_run_host(q4rdna_plan *plan, const void *x_host, void *x_dev, size_t x_bytes,
                                   const void *y_dev, void *y_host, size_t y_bytes, int segments,
                                   q4rdna_stream_t stream);

/* Launch options of the plan's runs: Q4RDNA_CFG_OVERLAP_PREVIOUS lets each
 * run start streaming its weights while the previous kernel on the stream
 * finishes (programmatic dependent launch), as for single calls; the caller
 * guarantees that no kernel still running on the stream writes the plan's
 * weight tiles.  B = 1..2 plans only (others ignore it).  0 clears it. */
q4rdna_status q4rdna_plan_set_flags(q4rdna_plan *plan, int flags);

/* Runs plans[0], plans[1], ... in order on `stream`, each exactly as
 * q4rdna_plan_run does (with its fused gather, if set): one host call for a
 * sequence of dependent plans, e.g. a decoder layer's stages under tensor
 * parallelism.  Stops at the first failing plan and returns its status. */
q4rdna_status q4rdna_plan_run_many(q4rdna_plan *const *plans, int count, q4rdna_stream_t stream);

/* How q4rdna_plan_run executes the plan: as `segments` launches of consecutive
 * descriptors (about equal weight bytes) that alternate between two library
 * streams and are joined to `stream` at the end.  1 (the default; also 0) =
 * one launch, which is the fastest with the plan's own split-K choice; more
 * segments pay off only for plans whose descriptors force small items.
 * Results are identical.  With a gather (q4rdna_plan_set_gather) the flag
 * exchange follows the last segment. */
q4rdna_status q4rdna_plan_set_segments(q4rdna_plan *plan, int segments);

/* ---- tensor parallelism: the all-gather fused into the plan kernel ----
 * Replaces the NCCL all-gather of the row-sharded decode step (one process per
 * GPU, each owning rows [r*N/P, (r+1)*N/P) of every tensor; the reference is
 * single-GPU, so there is no reference counterpart).  The plan's outputs of a
 * rank form one buffer of rank_floats floats starting at y_base (every
 * descriptor's y lies inside it).  gathered0[p] / gathered1[p] are rank p's two
 * gathered buffers of world * rank_floats floats (peer addresses mapped in this
 * process with q4rdna_ipc_open, this rank's own at index rank); flags[p] is rank
 * p's array of `world` u32 arrival flags, zero-initialised.  After this call,
 * run n (1-based) of the plan stores every output also into slice `rank` of
 * every rank's gathered buffer n % 2 (plain peer stores from the GEMV
 * epilogue, no multicast), then raises its flag at every rank and waits, at
 * most about 2 s, until every rank's run n has landed here.  On expiry bit 1 of
 * q4rdna_take_fault is set.  Every rank must run the plan the same number of
 * times.  world is 2..8. */
q4rdna_status q4rdna_plan_set_gather(q4rdna_plan *plan, int world, int rank, const float *y_base,
                                     size_t rank_floats, float *const *gathered0, float *const *gathered1,
                                     uint32_t *const *flags);
/* Bound of the fused gather's flag wait: a run stops waiting for the peers'
 * flags after about `microseconds` (0: the default, about 2 s), sets bit 1 of
 * q4rdna_take_fault and returns, so a rank that never arrives shows up on the
 * host as a fault flag instead of a hung stream.  The wait is a polling loop
 * with ~0.5 us sleeps, so the bound is approximate.  May be called before or
 * after q4rdna_plan_set_gather.  No reference counterpart. */
q4rdna_status q4rdna_plan_set_gather_timeout(q4rdna_plan *plan, uint32_t microseconds);
/* Gathered buffer (0 or 1) that the plan's last run filled; -1 before the first
 * run or without a gather. */
int q4rdna_plan_gather_parity(const q4rdna_plan *plan);

/* Device memory shareable with the other processes of the box (cudaMalloc +
 * CUDA IPC), zero-filled: the gathered buffers and flags above. */
#define Q4RDNA_IPC_HANDLE_BYTES 64
q4rdna_status q4rdna_ipc_alloc(size_t bytes, void **dev_ptr, unsigned char handle[Q4RDNA_IPC_HANDLE_BYTES]);
q4rdna_status q4rdna_ipc_open(const unsigned char handle[Q4RDNA_IPC_HANDLE_BYTES], void **dev_ptr);
/* Unmaps a q4rdna_ipc_open mapping. */
q4rdna_status q4rdna_ipc_close(void *dev_ptr);
/* Frees a q4rdna_ipc_alloc allocation (after every peer closed its mapping). */
q4rdna_status q4rdna_ipc_free(void *dev_ptr);

/* Packs a row-major bf16 matrix [N][K] (device memory, 16-byte aligned) into
 * Q4_RDNA tiles (N*K*34/64 bytes, 2-byte aligned) on the GPU, byte for byte what
 * the reference packer writes for the tensor.  Replaces the per-tensor loop of
 * source/q4rdna_sidecar_pack.cpp:262-279 (scale search :140-179, quantiser
 * :126-129); source/pack_q4rdna_sidecar.py:44-73 writes the same bytes.  The
 * container (header, entries, alignment) is written by the host
 * (q4rdna.format.write_sidecar). */
q4rdna_status q4rdna_pack_bf16(const uint16_t *bf16, uint8_t *tiles, int N, int K, q4rdna_stream_t stream);

/* ---- sidecar (the reference's .q4rdna container, byte layout unchanged) ----
 * Header 48 B, entries 96 B, data at data_offset (source/q4rdna.cu:26-50).
 * Validation follows source/q4rdna.cu:131-152.  The whole data region is
 * uploaded to one device buffer owned by the handle. */
typedef struct q4rdna_sidecar q4rdna_sidecar;

q4rdna_status q4rdna_sidecar_open(const char *path, int device, q4rdna_sidecar **out);
void q4rdna_sidecar_close(q4rdna_sidecar *sc);
int q4rdna_sidecar_count(const q4rdna_sidecar *sc);
q4rdna_status q4rdna_sidecar_entry(const q4rdna_sidecar *sc, int index, char name_out[64], int *rows,
                                   int *cols, uint64_t *relative_offset);
/* Device address of a tensor's tiles and its shape (q4rdna_find, q4rdna.cu:700-704). */
q4rdna_status q4rdna_sidecar_find(const q4rdna_sidecar *sc, const char *name, int *rows, int *cols,
                                  const uint8_t **tiles);

/* ---- the reference's operator surface, keyed by ggml tensor name ----
 * These carry the semantics of ggml_cuda_q4rdna_mul_mat / _mul_mat_add /
 * _mul_mat_glu (source/q4rdna.cuh:5-24): return 1 when the work was enqueued on
 * `stream`, 0 when the caller must use its stock kernel (sidecar unset, tensor
 * out of scope or unknown, shape mismatch, other device).  The process-wide
 * registry loads lazily from LLAMA_Q4_RDNA_SIDECAR on the first call, onto the
 * device current at that call; LLAMA_Q4_RDNA_SCOPE (ffn | qkv-fallback |
 * hotspot | attn) filters by name as in source/q4rdna.cu:685-696.
 * weight_ne0 = K (columns) and weight_ne1 = N (rows) of the ggml weight tensor;
 * x_ne0 must equal K and y_ne0 (elements of dst) must equal N.  Batch 1. */
int q4rdna_mul_mat(const char *weight_name, int64_t weight_ne0, int64_t weight_ne1, const float *x,
                   int64_t x_ne0, float *y, int64_t y_ne0, q4rdna_stream_t stream);
int q4rdna_mul_mat_add(const char *weight_name, int64_t weight_ne0, int64_t weight_ne1, const float *x,
                       int64_t x_ne0, const float *add, int64_t add_nelements, float *y,
                       int64_t y_nelements, q4rdna_stream_t stream);
int q4rdna_mul_mat_glu(const char *up_name, int64_t up_ne0, int64_t up_ne1, const char *gate_name,
                       int64_t gate_ne0, int64_t gate_ne1, const float *x, int64_t x_ne0, float *y,
                       int64_t y_nelements, q4rdna_stream_t stream);

/* Counters (source/q4rdna.cu:73-112): kernels launched by this library, and per
 * sidecar tensor the number of operator hits. */
uint64_t q4rdna_launch_count(void);
uint64_t q4rdna_registry_hits(const char *weight_name);
/* Device-side fault flags of the GEMV kernels since the last call, then cleared
 * (synchronises the device).  Bit 1: a fused gather (q4rdna_plan_set_gather)
 * stopped waiting for a peer's flag (q4rdna_plan_set_gather_timeout), so the
 * gathered buffer of that run is incomplete; the GEMV outputs of this rank
 * (y) are complete.  Bit 2: a wait inside the tensor-core tile kernel (B >= 8)
 * ran out (about 1 s) and the kernel stopped; the outputs of that launch are
 * invalid and the workspaces it used must be re-initialised
 * (q4rdna_workspace_init) or the plans re-created.  Bit 0 is no longer set by
 * any kernel.  0 = no fault; 0xffffffff = the flag could not be read.  No
 * reference counterpart (the reference kernels never wait). */
uint32_t q4rdna_take_fault(void);
/* Prints the reference's exit-time summary to stderr (also run at exit once the
 * registry has loaded); LLAMA_Q4_RDNA_TRACE adds per-tensor hit lines. */
void q4rdna_report_stats(void);
/* Drops the process-wide registry (frees its device memory and workspaces)
 * and the no-alloc entry point's cached scratch addresses.  For tests, and
 * after a cudaDeviceReset. */
void q4rdna_registry_reset(void);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif /* Q4RDNA_H */
