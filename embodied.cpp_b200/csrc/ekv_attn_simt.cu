// ekv_attn_simt.cu -- one-warp-per-query-row attention on CUDA cores.
//
// A deliberately plain kernel over the same paged layout and mask predicate as the tensor-core
// kernel: every lane owns head_dim/32 output columns, each key's dot product is a warp
// reduction, the softmax is the online (running max / running sum) form. It exists as an
// independent GPU cross-check of the tensor-core path (selected with EKV_ALGO_SIMT); K/V are
// read exactly (Q8_0 dequantised in f32), so it agrees with the CPU oracle to f32 rounding.
#include "ekv_device.cuh"
#include "ekv_internal.h"

namespace ekv {
namespace {

constexpr int kWarps = 4;
constexpr int kMaxPerLane = 8;  // head_dim <= 256

struct KeySrc {
    const uint8_t *tile;  // K or V tile base
    int row, rows;        // row within the tile, rows of the tile (bf16 layouts)
    bool q8;
};

__device__ __forceinline__ float load_elem(const PoolView &p, const KeySrc &s, int d) {
    if (!s.q8) {
        const uint16_t h = *(const uint16_t *)(s.tile + tile_elem_off(s.row, d, p.head_dim, p.swz_bytes));
        return bf16_bits_to_f32(h);
    }
    const int8_t q = *(const int8_t *)(s.tile + q8_qs_off(s.row, d, p.head_dim));
    const uint16_t db = *((const uint16_t *)(s.tile + (int64_t)p.block_tokens * p.head_dim) +
                          s.row * (p.head_dim / 32) + d / 32);
    return (float)q * f16_bits_to_f32(db);
}

__global__ void attn_simt_kernel(AttnArgs a) {
    const PoolView &p = a.pool;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int64_t row_id = (int64_t)blockIdx.x * kWarps + warp;
    const int64_t n_rows = (int64_t)a.n_batch * a.q_tokens * a.q_heads;
    if (row_id >= n_rows) return;
    const int h = (int)(row_id % a.q_heads);
    const int t = (int)((row_id / a.q_heads) % a.q_tokens);
    const int b = (int)(row_id / ((int64_t)a.q_heads * a.q_tokens));
    const int g = h / a.group;
    const int D = p.head_dim;
    const SeqKeys sk = resolve_seq(p, a.use_prefix, a.seq_ids, a.prefix_len, a.prefix_valid, a.span_begin,
                                   a.span_end, b);
    if (!sk.ok && lane == 0) report_error(p.status, DEV_ERR_BAD_SEQ, b, a.seq_ids[b], 2);
    const MaskDesc m = mask_desc(a, b);

    float qv[kMaxPerLane], acc[kMaxPerLane];
    const uint16_t *qrow = a.q + (((int64_t)b * a.q_tokens + t) * a.q_heads + h) * D;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
        const int d = lane + 32 * i;
        qv[i] = d < D ? bf16_bits_to_f32(qrow[d]) : 0.0f;
        acc[i] = 0.0f;
    }
    float mrun = -INFINITY, lrun = 0.0f;
    const int n_suffix = sk.ok ? a.suffix_len : 0;
    const int n_prefix = sk.ok ? sk.n_prefix : 0;
    int cached_idx = -1, cached_blk = -1;
    for (int k = 0; k < n_prefix + n_suffix; ++k) {
        bool vis;
        KeySrc ks, vs;
        if (k < n_prefix) {
            vis = prefix_allowed(m, t, k, sk.prefix_valid, sk.span_b, sk.span_e);
            if (!vis) continue;
            const int idx = k / p.block_tokens;
            if (idx != cached_idx) {
                cached_idx = idx;
                cached_blk = lookup_block(p, sk.seq, idx);
            }
            if (cached_blk < 0) continue;
            const bool q8 = p.dtype == EKV_DTYPE_Q8_0;
            ks.tile = p.prefix + prefix_tile_index(p, a.layer, cached_blk, 0, g) * p.tile_bytes;
            vs.tile = p.prefix + prefix_tile_index(p, a.layer, cached_blk, 1, g) * p.tile_bytes;
            ks.row = vs.row = k % p.block_tokens;
            ks.rows = vs.rows = p.block_tokens;
            ks.q8 = vs.q8 = q8;
        } else {
            const int s = k - n_prefix;
            vis = suffix_allowed(m, t, s, a.suffix_len, n_prefix);
            if (!vis) continue;
            ks.tile = p.suffix + suffix_tile_index(p, a.layer, sk.seq, 0, g) * p.suffix_tile_bytes;
            vs.tile = p.suffix + suffix_tile_index(p, a.layer, sk.seq, 1, g) * p.suffix_tile_bytes;
            ks.row = vs.row = s;
            ks.rows = vs.rows = p.suffix_rows;
            ks.q8 = vs.q8 = false;
        }
        float dot = 0.0f;
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) {
            const int d = lane + 32 * i;
            if (d < D) dot += qv[i] * load_elem(p, ks, d);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
        const float x = dot * a.scale_log2;
        const float mnew = fmaxf(mrun, x);
        const float alpha = exp2f(mrun - mnew);
        const float pr = exp2f(x - mnew);
        lrun = lrun * alpha + pr;
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) {
            const int d = lane + 32 * i;
            if (d < D) acc[i] = acc[i] * alpha + pr * load_elem(p, vs, d);
        }
        mrun = mnew;
    }
    const float inv = lrun > 0.0f ? 1.0f / lrun : 0.0f;
    const int64_t obase = (((int64_t)b * a.q_tokens + t) * a.q_heads + h) * D;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
        const int d = lane + 32 * i;
        if (d >= D) continue;
        const float o = acc[i] * inv;
        if (a.out_dtype == EKV_DTYPE_F32)
            ((float *)a.out)[obase + d] = o;
        else
            ((uint16_t *)a.out)[obase + d] = f32_to_bf16_bits(o);
    }
}

}  // namespace

int launch_attention_simt(const AttnArgs &a, cudaStream_t s) {
    const int64_t n_rows = (int64_t)a.n_batch * a.q_tokens * a.q_heads;
    const int64_t grid = (n_rows + kWarps - 1) / kWarps;
    if (grid > 0x7fffffff) return EKV_ERR_INVALID_ARG;
    attn_simt_kernel<<<(unsigned)grid, kWarps * 32, 0, s>>>(a);
    if (cudaGetLastError() != cudaSuccess) return EKV_ERR_CUDA;
    note_launches(1);
    return EKV_OK;
}

}  // namespace ekv
