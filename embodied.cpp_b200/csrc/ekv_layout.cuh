// ekv_layout.cuh -- device-side layout of the paged KV pool, shared by every kernel.
//
// HBM layout (one cudaMalloc per pool, all regions 1024-byte aligned):
//
//   prefix arena  [n_layers][n_blocks][2 (K,V)][kv_heads] tiles
//     bf16 tile : block_tokens x head_dim bf16 stored as [rows/8][D*2/W chunks][8 rows][W bytes]
//                 with the tcgen05 shared-memory swizzle already applied (Swizzle<log2(W/16),4,3>,
//                 W = 128, 64 or 32 bytes). One contiguous copy of a block lands in shared
//                 memory as a canonical K-major operand (K) or MN-major operand (V) tile.
//     Q8_0 tile : qs int8 [block_tokens][head_dim] (16-byte units XOR-swizzled by row, see
//                 q8_qs_off) followed by fp16 scales [block_tokens][head_dim/32]; a gather
//                 re-interleaves them into ggml's block_q8_0 {d, qs[32]} bytes.
//   suffix arena  [n_layers][max_seqs][2][kv_heads] tiles of suffix_rows bf16 rows, in the
//                 same swizzled bf16 tile layout (suffix_rows = suffix_tokens rounded up to 16, so
//                 the tiles of consecutive heads stack into one MMA operand with 16-aligned columns).
//   seq table     int32 block_tables[max_seqs][max_blocks_per_seq], int32 seq_lens[max_seqs]
//   status word   int32[4]: [0] first error code, [1..3] details of that error
#pragma once

#include <cstdint>

namespace ekv {

struct PoolView {
    uint8_t *prefix;          // prefix arena
    uint8_t *suffix;          // suffix arena
    int32_t *block_tables;    // [max_seqs][max_blocks_per_seq]
    int32_t *seq_lens;        // [max_seqs]
    int32_t *status;          // [4]
    int32_t dtype;            // EKV_DTYPE_BF16 / EKV_DTYPE_Q8_0
    int32_t block_tokens;
    int32_t n_blocks;
    int32_t kv_heads;
    int32_t head_dim;
    int32_t n_layers;
    int32_t max_seqs;
    int32_t max_blocks_per_seq;
    int32_t suffix_rows;      // rows per suffix tile (multiple of 16), 0 = none
    int32_t swz_bytes;        // W: row bytes of one swizzle chunk (128, 64 or 32)
    int32_t bt_shift;         // log2(block_tokens) when it is a power of two, else -1
    int64_t tile_bytes;       // bytes of one (layer, block, kv, head) prefix tile
    int64_t suffix_tile_bytes;// bytes of one (layer, seq, kv, head) suffix tile
};

// Error codes written into status[0] by kernels (first error wins).
enum : int32_t {
    DEV_ERR_BAD_BLOCK = 1,     // block-table entry outside [0, n_blocks)
    DEV_ERR_BAD_SEQ = 2,       // sequence id outside [0, max_seqs)
    DEV_ERR_BAD_POS = 3,       // position outside the sequence's blocks
    DEV_ERR_TIMEOUT = 4,       // bounded mbarrier wait ran out
    DEV_ERR_F16_RANGE = 5,     // a value beyond the f16 range met an f16 operand (Q8_0 pools)
};

__host__ __device__ inline int swizzle_bytes_for(int head_dim) {
    const int row = head_dim * 2;
    return (row % 128 == 0) ? 128 : (row % 64 == 0) ? 64 : 32;
}

// Swizzle<B,4,3> on an offset inside a 1024-byte-aligned frame: the 16-byte unit index
// (bits 4..4+B) is XORed with bits 7..7+B. mask = W/16 - 1.
__host__ __device__ inline uint32_t swz(uint32_t off, uint32_t mask) {
    return off ^ (((off >> 7) & mask) << 4);
}

// Byte offset of element (row, d) inside a bf16 tile of head_dim D and swizzle chunk width W.
// Row-group-major: [row / 8][chunk = 2d / W][row % 8][W bytes], swizzled inside each 8 x W atom.
// The rows of one block (or any run of whole 8-row groups) are one contiguous byte range, and
// in shared memory the tile is a canonical tcgen05 operand: K-major with 8-row groups at
// SBO = (2D/W) * 8W bytes (K), or MN-major with D-chunks at LBO = 8W and the same SBO (V).
__host__ __device__ inline uint32_t tile_elem_off(int row, int d, int D, int W) {
    const int nch = D * 2 / W;
    const int byte = d * 2;
    const int chunk = byte / W;
    const int wb = byte - chunk * W;
    return (uint32_t)((row >> 3) * nch + chunk) * (uint32_t)(8 * W) +
           swz((uint32_t)((row & 7) * W + wb), (uint32_t)(W / 16 - 1));
}

// Byte offset of int8 element (row, d) in the qs plane of a Q8_0 tile: rows of D bytes whose
// 16-byte units are XOR-swizzled by the row (unit ^ (row & m), m = min(D/16, 8) - 1), so that
// 8 consecutive rows of one 16-byte column fall in 8 different shared-memory bank groups.
__host__ __device__ inline uint32_t q8_qs_off(int row, int d, int D) {
    const int units = D / 16;
    const int m = (units < 8 ? units : 8) - 1;
    return (uint32_t)(row * D + (((d >> 4) ^ (row & m)) << 4) + (d & 15));
}

__host__ __device__ inline int64_t prefix_tile_index(const PoolView &p, int layer, int block, int kv,
                                                      int head) {
    return (((int64_t)layer * p.n_blocks + block) * 2 + kv) * p.kv_heads + head;
}

__host__ __device__ inline int64_t suffix_tile_index(const PoolView &p, int layer, int seq, int kv,
                                                      int head) {
    return (((int64_t)layer * p.max_seqs + seq) * 2 + kv) * p.kv_heads + head;
}

#ifdef __CUDACC__
__device__ inline void report_error(int32_t *status, int32_t code, int32_t a, int32_t b, int32_t c) {
    if (atomicCAS(status, 0, code) == 0) {
        status[1] = a;
        status[2] = b;
        status[3] = c;
    }
}
#endif

}  // namespace ekv
