// ekv_attn_common.cuh -- device helpers shared by the attention kernels (one-CTA and CTA-pair):
// closed-form key-visibility words, paged-block indexing, Q8_0 -> f16 and bf16 -> f16 conversion.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "ekv_device.cuh"
#include "ekv_internal.h"

namespace ekv {
namespace {

constexpr long long kWaitBudget = 4000000000LL;  // clock cycles (~2-3 s) before giving up
constexpr int kBM = 128;                          // query rows per CTA (TMEM lanes)
constexpr int kMaxSplits = 8;
constexpr int kDq = 256;  // dequantising threads (Q8_0): 8 warps, two per SM sub-partition

// Key-split count for `units` work units (one CTA or CTA pair each) over `slots` concurrent units,
// `max_tiles` key tiles per unit: minimises waves x (per-unit fixed cost + tiles per split x tile
// cost) + a merge pass when split. The costs are in tile-times, measured on B200: a unit's set-up
// and epilogue (Q load, table, O write) take about five tile-times, the merge about two.
inline int choose_split_count(int64_t units, int max_tiles, int slots) {
    constexpr double kFixed = 5.0, kMerge = 2.0;
    slots = slots > 0 ? slots : 1;
    int best = 1;
    double best_cost = 1e30;
    for (int s = 1; s <= kMaxSplits; ++s) {
        const int per = (max_tiles + s - 1) / s;
        if (s > 1 && per < 2) break;
        const double waves = (double)((units * s + slots - 1) / slots);
        const double cost = waves * (kFixed + per) + (s > 1 ? kMerge : 0.0);
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = s;
        }
    }
    return best;
}

// Bits of the keys [lo, hi) inside the 32-key word starting at key w0.
__device__ __forceinline__ uint32_t range_bits(int lo, int hi, int w0) {
    const int a = max(lo - w0, 0), b = min(hi - w0, 32);
    if (b <= a) return 0u;
    const uint32_t upto_b = b >= 32 ? 0xffffffffu : ((1u << b) - 1u);
    const uint32_t below_a = (1u << a) - 1u;  // a < 32 here
    return upto_b & ~below_a;
}

// Visibility of keys [w0, w0+32) for query token t, from key ranges (no per-key loop):
// the predicate of prefix_allowed / suffix_allowed in closed form.
__device__ __forceinline__ uint32_t vis_word(const MaskDesc &m, bool suffix, int w0, int t, int prefix_valid,
                                             int span_b, int span_e, int suffix_len) {
    if (suffix) {
        int hi = suffix_len;
        if (m.flags & EKV_MASK_SUFFIX_CAUSAL) hi = min(hi, t + 1);
        if ((m.flags & EKV_MASK_SUFFIX_PREFIX_LM) && t == 0) hi = min(hi, 1);
        return range_bits(0, hi, w0);
    }
    uint32_t bits = range_bits(0, prefix_valid, w0);
    if (m.flags & EKV_MASK_SPAN_ONLY) bits &= range_bits(span_b, span_e, w0);
    if (m.flags & EKV_MASK_SPAN_EXCLUDE) bits &= ~range_bits(span_b, span_e, w0);
    if (m.flags & EKV_MASK_BLOCK_CAUSAL) {
        const int qc = m.q_chunk0 + t / m.chunk_tokens;
        const int kc_lo = max(qc - m.window_chunks + 1, max(w0, 0) / m.chunk_stride);
        const int kc_hi = min(qc, (w0 + 31) / m.chunk_stride);
        uint32_t win = 0u;
        for (int kc = kc_lo; kc <= kc_hi; ++kc)
            win |= range_bits(kc * m.chunk_stride, kc * m.chunk_stride + m.chunk_tokens, w0);
        bits &= win;
    }
    return bits;
}


// Table index of key k, and the key's row inside its block (shift/mask for power-of-two blocks).
__device__ __forceinline__ int block_index(const PoolView &p, int k, int &rib) {
    if (p.bt_shift >= 0) {
        rib = k & (p.block_tokens - 1);
        return k >> p.bt_shift;
    }
    const int idx = k / p.block_tokens;
    rib = k - idx * p.block_tokens;
    return idx;
}

__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t w) {
    const __half2 h2 = __floats2half2_rn(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
    return *(const uint32_t *)&h2;
}

// 16 Q8_0 values (int8) and their fp16 block scale -> 16 f16 values in registers
__device__ __forceinline__ void dequant16(const uint4 q, uint32_t dbits, uint4 &lo, uint4 &hi) {
    const __half2 scale = __halves2half2(__ushort_as_half((uint16_t)dbits), __ushort_as_half((uint16_t)dbits));
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    uint32_t o[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t u = w[i] ^ 0x80808080u;                 // int8 -> uint8 (q + 128)
        uint32_t e01 = __byte_perm(u, 0x64646464u, 0x5140);    // f16 (1024 + u0, 1024 + u1)
        uint32_t e23 = __byte_perm(u, 0x64646464u, 0x5342);
        __half2 h01 = __hmul2(__hsub2(*(__half2 *)&e01, bias), scale);  // exact q, one rounding
        __half2 h23 = __hmul2(__hsub2(*(__half2 *)&e23, bias), scale);
        o[2 * i] = *(uint32_t *)&h01;
        o[2 * i + 1] = *(uint32_t *)&h23;
    }
    lo = make_uint4(o[0], o[1], o[2], o[3]);
    hi = make_uint4(o[4], o[5], o[6], o[7]);
}

[[maybe_unused]] __device__ __forceinline__ uint4 bf16x8_to_f16x8(uint4 v) {
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2 h2 = __floats2half2_rn(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u));
        w[i] = *(const uint32_t *)&h2;
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}


}  // namespace
}  // namespace ekv
