// Q4_RDNA packed-format constants and index math, shared by host and device.
//
// Format (fixed by the reference: source/q4rdna.cu:20-24, writer
// source/q4rdna_sidecar_pack.cpp:268-278, reader source/q4rdna.cu:346-370):
//   * a tile covers 32 rows x 64 columns (one 64-weight group per row) in 1088 B;
//   * bytes [0, 64): 32 little-endian fp16 scales, row lane r at byte 2r;
//   * byte 64 + 32*i + r: row r, columns 2i (low nibble) and 2i+1 (high nibble),
//     two's-complement int4 in [-8, 7];
//   * tile index = row_tile * groups + group, so the tiles of one 32-row band
//     form one contiguous K-stream of groups*1088 bytes.
#pragma once
#include <stdint.h>

#define Q4_GROUP 64          // weights per scale
#define Q4_TILE_ROWS 32      // rows per tile
#define Q4_TILE_BYTES 1088   // 64 B scales + 1024 B codes
#define Q4_SCALE_BYTES 64
// Packed bytes of an N x K tensor: N*K*34/64 (source/q4rdna.cu:149).
#define Q4_TENSOR_BYTES(N, K) ((uint64_t)(N) * (uint64_t)(K) * 34u / 64u)

// Rows handled by one warp work item: four 32-row tiles (see q4rdna_gemv.cu).
#define Q4_BLOCK_ROWS 128
#define Q4_BLOCK_TILES 4

#ifdef __cplusplus
static inline uint64_t q4_tile_offset(uint64_t row_tile, uint64_t groups, uint64_t group) {
    return (row_tile * groups + group) * (uint64_t)Q4_TILE_BYTES;
}
#endif
