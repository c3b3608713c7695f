// ekv_cache_kernels.cu -- append / gather kernels of the paged pool.
//
// Append replaces the per-step ggml_concat + cont copies of the reference
// (models/pi05.cpp:406-412) and the LingBot slot scatter
// (kernels/lingbot/lingbot_flex_attn_cuda.cu:626-649): each new K/V row is written once, into
// the block its position maps to. bf16 rows move as 16-byte vectors into the swizzled tile
// layout; Q8_0 pools quantise each 32-element group on the way (gguf-py quants.py:378-393:
// d = amax/127, id = 1/d, q = roundf(x*id), fp16 d), with IEEE division and no FMA contraction
// so the bytes match the CPU rule exactly.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "ekv_device.cuh"
#include "ekv_internal.h"

namespace ekv {
namespace {

constexpr int kThreads = 256;

// Resolve (seq, position) of batch element b, row r to the destination tile base of
// (layer, kv, head) and the row inside the block. Returns false when the row is skipped.
__device__ __forceinline__ bool prefix_dest(const PoolView &p, int layer, int seq, int pos, int &blk,
                                            int &rib) {
    if (seq < 0 || seq >= p.max_seqs) {
        report_error(p.status, DEV_ERR_BAD_SEQ, seq, pos, 0);
        return false;
    }
    if (pos < 0 || pos >= p.seq_lens[seq]) {
        report_error(p.status, DEV_ERR_BAD_POS, seq, pos, p.seq_lens[seq]);
        return false;
    }
    blk = lookup_block(p, seq, pos / p.block_tokens);
    rib = pos % p.block_tokens;
    return blk >= 0;
}

// Rows per CTA of the bf16 prefix append and of the suffix append (a suffix is a few dozen rows per
// request, so its CTAs take fewer rows: one warp per (row, K|V) pair keeps enough CTAs in flight), and
// 16-byte loads a lane keeps in flight before its stores.
constexpr int kRowsPerCta = 16;
constexpr int kSuffixRowsPerCta = 4;
constexpr int kUnitsPerLane = 8;

// Move one (row, K|V) of kv_heads x head_dim bf16 elements from a packed source row to the swizzled
// tiles at row `rib` (tile of head h at tile0 + h * tile_bytes), by one warp: consecutive lanes take
// consecutive 16-byte units of the source row, up to kUnitsPerLane loads in flight per lane.
__device__ __forceinline__ void move_row_bf16(const uint4 *__restrict__ src, uint8_t *tile0, int64_t tile_bytes,
                                              int rib, const PoolView &p, int lane) {
    const int dh8 = p.head_dim / 8, upk = p.kv_heads * dh8;
    for (int u0 = lane; u0 < upk; u0 += 32 * kUnitsPerLane) {
        uint4 val[kUnitsPerLane];
#pragma unroll
        for (int j = 0; j < kUnitsPerLane; ++j)
            if (u0 + 32 * j < upk) val[j] = __ldg(src + u0 + 32 * j);
#pragma unroll
        for (int j = 0; j < kUnitsPerLane; ++j) {
            const int u = u0 + 32 * j;
            if (u < upk) {
                const int h = u / dh8, d0 = (u - h * dh8) * 8;
                *(uint4 *)(tile0 + h * tile_bytes + tile_elem_off(rib, d0, p.head_dim, p.swz_bytes)) = val[j];
            }
        }
    }
}

// bf16 append: a CTA moves `rows` (at most kRowsPerCta) rows of one batch element. One thread per row
// resolves the row's destination block (sequence length and block-table reads) into shared memory; then
// each warp takes (row, K|V) pairs and moves them with move_row_bf16.
__global__ void append_bf16_kernel(PoolView p, int layer, const int32_t *__restrict__ seq_ids,
                                   const int32_t *__restrict__ dst_pos, const int32_t *__restrict__ n_rows,
                                   const int32_t *__restrict__ src_row, int max_rows, int rows,
                                   const uint4 *__restrict__ k, const uint4 *__restrict__ v) {
    __shared__ int s_blk[kRowsPerCta], s_rib[kRowsPerCta];
    const int b = blockIdx.y;
    const int r0 = blockIdx.x * rows;
    const int nr = min(rows, min(max_rows, n_rows[b]) - r0);
    if (nr <= 0) return;
    if ((int)threadIdx.x < nr) {
        int blk, rib = 0;
        if (!prefix_dest(p, layer, seq_ids[b], dst_pos[b] + r0 + (int)threadIdx.x, blk, rib)) blk = -1;
        s_blk[threadIdx.x] = blk;
        s_rib[threadIdx.x] = rib;
    }
    __syncthreads();
    const int upk = p.kv_heads * (p.head_dim / 8);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int64_t row0 = (int64_t)src_row[b] + r0;
    for (int pr = warp; pr < 2 * nr; pr += blockDim.x / 32) {
        const int r = pr >> 1, kv = pr & 1;
        const int blk = s_blk[r];
        if (blk < 0) continue;
        move_row_bf16((kv ? v : k) + (row0 + r) * upk, p.prefix + prefix_tile_index(p, layer, blk, kv, 0) * p.tile_bytes,
                      p.tile_bytes, s_rib[r], p, lane);
    }
}

// Q8_0 append: one thread quantises one 32-element group of one (row, kv, head).
__global__ void append_q8_kernel(PoolView p, int layer, const int32_t *__restrict__ seq_ids,
                                 const int32_t *__restrict__ dst_pos, const int32_t *__restrict__ n_rows,
                                 const int32_t *__restrict__ src_row, int max_rows,
                                 const uint4 *__restrict__ k, const uint4 *__restrict__ v) {
    const int b = blockIdx.y;
    const int groups = p.head_dim / 32;
    const int units_per_row = 2 * p.kv_heads * groups;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int r = (int)(idx / units_per_row);
    if (r >= max_rows || r >= n_rows[b]) return;
    const int u = (int)(idx - (int64_t)r * units_per_row);
    const int kv = u / (p.kv_heads * groups);
    const int rem = u - kv * (p.kv_heads * groups);
    const int h = rem / groups;
    const int g = rem - h * groups;
    // the group's 64 source bytes are requested before the destination is resolved (block table
    // lookups), so the two memory latencies overlap instead of adding up
    const int64_t src = (((int64_t)src_row[b] + r) * p.kv_heads + h) * p.head_dim + g * 32;
    const uint4 *s = (kv ? v : k) + src / 8;
    uint4 raw[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) raw[i] = __ldg(s + i);
    int blk, rib;
    if (!prefix_dest(p, layer, seq_ids[b], dst_pos[b] + r, blk, rib)) return;
    float x[32];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 w = raw[i];
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            x[i * 8 + j * 2] = __uint_as_float(ww[j] << 16);
            x[i * 8 + j * 2 + 1] = __uint_as_float(ww[j] & 0xffff0000u);
        }
    }
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[j]));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    uint32_t qw[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        uint32_t word = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int qv = (int)roundf(__fmul_rn(x[j * 4 + e], id));
            word |= ((uint32_t)(uint8_t)(int8_t)qv) << (8 * e);
        }
        qw[j] = word;
    }
    uint8_t *tile = p.prefix + prefix_tile_index(p, layer, blk, kv, h) * p.tile_bytes;
    *(uint4 *)(tile + q8_qs_off(rib, g * 32, p.head_dim)) = make_uint4(qw[0], qw[1], qw[2], qw[3]);
    *(uint4 *)(tile + q8_qs_off(rib, g * 32 + 16, p.head_dim)) = make_uint4(qw[4], qw[5], qw[6], qw[7]);
    uint16_t *sdst = (uint16_t *)(tile + (int64_t)p.block_tokens * p.head_dim) + rib * groups + g;
    *sdst = __half_as_ushort(__float2half_rn(d));
}

// Suffix slot write (bf16, swizzled tile of suffix_rows rows): a CTA moves kSuffixRowsPerCta rows of one
// batch element, one warp per (row, K|V) pair.
__global__ void append_suffix_kernel(PoolView p, int layer, const int32_t *__restrict__ seq_ids, int n_rows,
                                     const uint4 *__restrict__ k, const uint4 *__restrict__ v) {
    const int b = blockIdx.y;
    const int r0 = blockIdx.x * kSuffixRowsPerCta;
    const int nr = min(kSuffixRowsPerCta, n_rows - r0);
    const int seq = seq_ids[b];
    if (seq < 0 || seq >= p.max_seqs) {
        if (threadIdx.x == 0) report_error(p.status, DEV_ERR_BAD_SEQ, seq, r0, 1);
        return;
    }
    const int upk = p.kv_heads * (p.head_dim / 8);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    for (int pr = warp; pr < 2 * nr; pr += blockDim.x / 32) {
        const int r = pr >> 1, kv = pr & 1;
        move_row_bf16((kv ? v : k) + ((int64_t)b * n_rows + r0 + r) * upk,
                      p.suffix + suffix_tile_index(p, layer, seq, kv, 0) * p.suffix_tile_bytes, p.suffix_tile_bytes,
                      r0 + r, p, lane);
    }
}

// Gather of bf16 tiles (prefix or suffix) back to [rows][kv_heads][head_dim].
__global__ void gather_bf16_kernel(PoolView p, int layer, int seq, int pos0, int n_rows, int from_suffix,
                                   int as_f32, void *k_out, void *v_out) {
    const int per_head = p.head_dim / 8;
    const int units_per_row = 2 * p.kv_heads * per_head;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int r = (int)(idx / units_per_row);
    if (r >= n_rows) return;
    const int u = (int)(idx - (int64_t)r * units_per_row);
    const int kv = u / (p.kv_heads * per_head);
    const int rem = u - kv * (p.kv_heads * per_head);
    const int h = rem / per_head;
    const int d0 = (rem - h * per_head) * 8;
    const uint8_t *tile;
    uint32_t off;
    if (from_suffix) {
        tile = p.suffix + suffix_tile_index(p, layer, seq, kv, h) * p.suffix_tile_bytes;
        off = tile_elem_off(r, d0, p.head_dim, p.swz_bytes);
    } else {
        const int pos = pos0 + r;
        const int blk = lookup_block(p, seq, pos / p.block_tokens);
        if (blk < 0) return;
        tile = p.prefix + prefix_tile_index(p, layer, blk, kv, h) * p.tile_bytes;
        off = tile_elem_off(pos % p.block_tokens, d0, p.head_dim, p.swz_bytes);
    }
    const uint4 val = *(const uint4 *)(tile + off);
    const int64_t dst = ((int64_t)r * p.kv_heads + h) * p.head_dim + d0;
    if (!as_f32) {
        ((uint4 *)(kv ? v_out : k_out))[dst / 8] = val;
    } else {
        float *o = (float *)(kv ? v_out : k_out) + dst;
        const uint32_t w[4] = {val.x, val.y, val.z, val.w};
        float4 a, c;
        a.x = __uint_as_float(w[0] << 16); a.y = __uint_as_float(w[0] & 0xffff0000u);
        a.z = __uint_as_float(w[1] << 16); a.w = __uint_as_float(w[1] & 0xffff0000u);
        c.x = __uint_as_float(w[2] << 16); c.y = __uint_as_float(w[2] & 0xffff0000u);
        c.z = __uint_as_float(w[3] << 16); c.w = __uint_as_float(w[3] & 0xffff0000u);
        ((float4 *)o)[0] = a;
        ((float4 *)o)[1] = c;
    }
}

// Gather of Q8_0 tiles: NATIVE re-interleaves ggml block_q8_0 {d, qs[32]} (34 bytes, 2-byte
// aligned); F32 dequantises x = qs * d (gguf-py quants.py:395-401).
__global__ void gather_q8_kernel(PoolView p, int layer, int seq, int pos0, int n_rows, int as_f32,
                                 void *k_out, void *v_out) {
    const int groups = p.head_dim / 32;
    const int units_per_row = 2 * p.kv_heads * groups;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int r = (int)(idx / units_per_row);
    if (r >= n_rows) return;
    const int u = (int)(idx - (int64_t)r * units_per_row);
    const int kv = u / (p.kv_heads * groups);
    const int rem = u - kv * (p.kv_heads * groups);
    const int h = rem / groups;
    const int g = rem - h * groups;
    const int pos = pos0 + r;
    const int blk = lookup_block(p, seq, pos / p.block_tokens);
    if (blk < 0) return;
    const int rib = pos % p.block_tokens;
    const uint8_t *tile = p.prefix + prefix_tile_index(p, layer, blk, kv, h) * p.tile_bytes;
    const uint16_t dbits = *((const uint16_t *)(tile + (int64_t)p.block_tokens * p.head_dim) + rib * groups + g);
    const uint4 q0 = *(const uint4 *)(tile + q8_qs_off(rib, g * 32, p.head_dim));
    const uint4 q1 = *(const uint4 *)(tile + q8_qs_off(rib, g * 32 + 16, p.head_dim));
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    const int64_t blk_out = ((int64_t)r * p.kv_heads + h) * groups + g;
    if (!as_f32) {
        uint16_t *o = (uint16_t *)((uint8_t *)(kv ? v_out : k_out) + blk_out * 34);
        o[0] = dbits;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            o[1 + 2 * j] = (uint16_t)(w[j] & 0xffffu);
            o[2 + 2 * j] = (uint16_t)(w[j] >> 16);
        }
    } else {
        const float d = f16_bits_to_f32(dbits);
        float *o = (float *)(kv ? v_out : k_out) + blk_out * 32;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float4 f;
            f.x = (float)(int8_t)(w[j] & 0xff) * d;
            f.y = (float)(int8_t)((w[j] >> 8) & 0xff) * d;
            f.z = (float)(int8_t)((w[j] >> 16) & 0xff) * d;
            f.w = (float)(int8_t)(w[j] >> 24) * d;
            ((float4 *)o)[j] = f;
        }
    }
}

int grid_for(int64_t units) { return (int)((units + kThreads - 1) / kThreads); }

int launch_status() { return cudaGetLastError() == cudaSuccess ? EKV_OK : EKV_ERR_CUDA; }

}  // namespace

int launch_append(const PoolView &p, int layer, int n_batch, const int32_t *seq_ids, const int32_t *dst_pos,
                  const int32_t *n_rows, const int32_t *src_row, int max_rows, const void *k, const void *v,
                  cudaStream_t s) {
    if (((uintptr_t)k | (uintptr_t)v) & 15) return EKV_ERR_INVALID_ARG;
    if (n_batch > 65535) return EKV_ERR_INVALID_ARG;
    if (p.dtype == EKV_DTYPE_BF16) {
        // rows per CTA: 16, or fewer where that leaves under two CTAs per SM (a long chunk of one request)
        int sms = 148, dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        int rows = kRowsPerCta;
        while (rows > 4 && (int64_t)((max_rows + rows - 1) / rows) * n_batch < 2 * sms) rows /= 2;
        append_bf16_kernel<<<dim3((max_rows + rows - 1) / rows, n_batch), kThreads, 0, s>>>(
            p, layer, seq_ids, dst_pos, n_rows, src_row, max_rows, rows, (const uint4 *)k, (const uint4 *)v);
    } else {
        const int64_t units = (int64_t)max_rows * 2 * p.kv_heads * (p.head_dim / 32);
        append_q8_kernel<<<dim3(grid_for(units), n_batch), kThreads, 0, s>>>(
            p, layer, seq_ids, dst_pos, n_rows, src_row, max_rows, (const uint4 *)k, (const uint4 *)v);
    }
    note_launches(1);
    return launch_status();
}

int launch_append_suffix(const PoolView &p, int layer, int n_batch, const int32_t *seq_ids, int n_rows,
                         const void *k, const void *v, cudaStream_t s) {
    if (((uintptr_t)k | (uintptr_t)v) & 15) return EKV_ERR_INVALID_ARG;
    if (n_batch > 65535 || p.suffix_rows == 0) return EKV_ERR_INVALID_ARG;
    append_suffix_kernel<<<dim3((n_rows + kSuffixRowsPerCta - 1) / kSuffixRowsPerCta, n_batch), kThreads, 0, s>>>(
        p, layer, seq_ids, n_rows, (const uint4 *)k, (const uint4 *)v);
    note_launches(1);
    return launch_status();
}

int launch_gather(const PoolView &p, int layer, int seq, int pos0, int n_rows, int format, void *k_out,
                  void *v_out, cudaStream_t s) {
    if (p.dtype == EKV_DTYPE_BF16) {
        if (((uintptr_t)k_out | (uintptr_t)v_out) & 15) return EKV_ERR_INVALID_ARG;
        const int64_t units = (int64_t)n_rows * 2 * p.kv_heads * (p.head_dim / 8);
        gather_bf16_kernel<<<grid_for(units), kThreads, 0, s>>>(p, layer, seq, pos0, n_rows, 0,
                                                               format == EKV_GATHER_F32, k_out, v_out);
    } else {
        if (((uintptr_t)k_out | (uintptr_t)v_out) & (format == EKV_GATHER_F32 ? 15 : 1)) return EKV_ERR_INVALID_ARG;
        const int64_t units = (int64_t)n_rows * 2 * p.kv_heads * (p.head_dim / 32);
        gather_q8_kernel<<<grid_for(units), kThreads, 0, s>>>(p, layer, seq, pos0, n_rows,
                                                             format == EKV_GATHER_F32, k_out, v_out);
    }
    note_launches(1);
    return launch_status();
}

int launch_gather_suffix(const PoolView &p, int layer, int seq, int n_rows, int format, void *k_out,
                         void *v_out, cudaStream_t s) {
    if (((uintptr_t)k_out | (uintptr_t)v_out) & 15) return EKV_ERR_INVALID_ARG;
    if (p.suffix_rows == 0) return EKV_ERR_INVALID_ARG;
    const int64_t units = (int64_t)n_rows * 2 * p.kv_heads * (p.head_dim / 8);
    gather_bf16_kernel<<<grid_for(units), kThreads, 0, s>>>(p, layer, seq, 0, n_rows, 1,
                                                           format == EKV_GATHER_F32, k_out, v_out);
    note_launches(1);
    return launch_status();
}

}  // namespace ekv
