// q4rdna_gemv_noalloc: the plain GEMV for callers that cannot allocate device
// memory.
//
// Who needs it: a drop-in operator hook such as llama.cpp's
// ggml_cuda_q4rdna_mul_mat gets its activation and output from the host
// framework and has no workspace argument.  Device memory there belongs to the
// framework's own pool; cudaMalloc from inside the hook would stall the device
// and hide memory from the framework's accounting, and some runtimes forbid any
// allocation once start-up is over.  Such callers pass only inputs and outputs;
// the split-K scratch comes from a fixed array that lives in this library.
//
// The scratch is a file-scope __device__ array of Q4RDNA_NOALLOC_SCRATCH_BYTES
// (8 MiB).  Every GPU that loads the library holds it until the process exits.
// Host code must not pass the array's name to a kernel: on the host that name
// is only a stand-in, not a device address.  The device address is looked up
// once per device with cudaGetSymbolAddress, with that device current, on the
// first call made on it.  A device reset (cudaDeviceReset) reloads the module
// and can move the array, so q4rdna_registry_reset also forgets the cached
// addresses (noalloc_forget_devices); call it after a reset.
#include <cuda_runtime.h>

#include <mutex>

#include "q4rdna.h"
#include "q4rdna_tile.h"

namespace {

constexpr int kMaxDevices = 64;

// Split-K scratch shared by every q4rdna_gemv_noalloc call on a device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[Q4RDNA_NOALLOC_SCRATCH_BYTES];

std::mutex g_mutex;
void *g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch for the current device (set-up on first use).
q4rdna_status scratch_for_current_device(void **out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return Q4RDNA_ERR_DEVICE;
    std::lock_guard<std::mutex> lock(g_mutex);
    if (g_scratch_addr[dev] == nullptr) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
            cudaGetLastError();
            return Q4RDNA_ERR_CUDA;
        }
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return Q4RDNA_OK;
}

}  // namespace

// Drops the cached device addresses (called by q4rdna_registry_reset).
void noalloc_forget_devices() {
    std::lock_guard<std::mutex> lock(g_mutex);
    for (void *&p : g_scratch_addr) p = nullptr;
}

extern "C" q4rdna_status q4rdna_gemv_noalloc(const uint8_t *tiles, const float *x, float *y, int N, int K, int B,
                                              const q4rdna_cfg *cfg, q4rdna_stream_t stream) {
    if (tiles == nullptr || x == nullptr || y == nullptr) return Q4RDNA_ERR_INVALID_ARGUMENT;
    if (N <= 0 || K <= 0) return Q4RDNA_ERR_INVALID_ARGUMENT;
    if (N % Q4_TILE_ROWS != 0 || K % Q4_GROUP != 0) return Q4RDNA_ERR_SHAPE;
    if (B < 1 || B > Q4RDNA_MAX_BATCH) return Q4RDNA_ERR_UNSUPPORTED;
    const size_t need = q4rdna_workspace_bytes(N, K, B, Q4RDNA_OP_PLAIN, cfg);
    if (need > Q4RDNA_NOALLOC_SCRATCH_BYTES) return Q4RDNA_ERR_TOO_LARGE;
    void *scratch = nullptr;
    if (need > 0) {
        const q4rdna_status st = scratch_for_current_device(&scratch);
        if (st != Q4RDNA_OK) return st;
        // The split-K arrival tickets at the head of the scratch must start at
        // zero; clear them on the caller's stream before the kernel runs.
        const size_t tickets = (size_t)((N + Q4_BLOCK_ROWS - 1) / Q4_BLOCK_ROWS) * sizeof(unsigned);
        if (cudaMemsetAsync(scratch, 0, tickets, (cudaStream_t)stream) != cudaSuccess) return Q4RDNA_ERR_CUDA;
    }
    return q4rdna_gemv(tiles, x, y, N, K, B, cfg, scratch, need > 0 ? Q4RDNA_NOALLOC_SCRATCH_BYTES : 0, stream);
}
