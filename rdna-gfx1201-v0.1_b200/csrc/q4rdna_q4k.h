// Q4_K task table shared by the Q4_K kernel (q4rdna_q4k.cu) and the plans
// (q4rdna_gemv.cu) that hold Q4_K tensors beside Q4_RDNA ones.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "q4rdna.h"

namespace q4k {

struct Task {
    const uint8_t *w;   // N rows of nb blocks
    const float *x;     // [B][K]
    const float *add;   // [B][N] or null
    float *y;           // [B][N]
    int N, K, nb, op;
    long long item_begin;  // first item of this task
    int row_items;         // ceil(N / kRowsPerItem)
    int pad;
};

}  // namespace q4k

// Validates a Q4_K descriptor and fills its task; items = work items it adds.
q4rdna_status q4k_build_task(const q4rdna_gemv_desc &e, int B, long long item_begin, q4k::Task &T, long long &items);
// One launch over `ntasks` tasks (device table, or the single host task `one`).
q4rdna_status q4k_launch_tasks(const q4k::Task *table, const q4k::Task *one, int ntasks, int B, long long items,
                               cudaStream_t stream);
// Q4_K kernel launches so far (added to q4rdna_launch_count).
unsigned long long q4k_launch_count();
