// ekv_device.cuh -- device helpers shared by the cache and attention kernels: number formats,
// the mask predicate, and addressing of keys in the paged pool.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/ekv.h"
#include "ekv_internal.h"
#include "ekv_layout.cuh"

namespace ekv {

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) {
    return __uint_as_float((uint32_t)h << 16);
}

__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

// Round-to-nearest-even f32 -> bf16, NaN kept quiet: the rule of gguf-py quants.py:204-213.
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float x) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

// Mask predicate: may query token q (0-based within the call) attend key k of the sequence?
// Prefix keys are [0, n_prefix), suffix keys follow. Semantics per mode:
//   padding ......... prefix keys >= prefix_valid are masked  (models/smolvla.cpp:707-716)
//   SPAN_ONLY/EXCLUDE prefix key inside/outside [span_b, span_e) (models/groot_n1.cpp:708-718)
//   BLOCK_CAUSAL .... key chunk kc = k / chunk_stride (slots past chunk_tokens invalid), query
//                     chunk qc = q_chunk0 + q / chunk_tokens, visible iff qc-window < kc <= qc
//   SUFFIX_CAUSAL ... suffix key s visible iff s <= q          (models/smolvla.cpp:718-720)
//   SUFFIX_PREFIX_LM  query 0 sees suffix key 0 only           (models/hy_vla.cpp:2355-2367)
//   FLEX_SELF ....... flex_self_allowed over per-token metadata words (models/lingbot_va.cpp:9336-9344)
//   FLEX_CROSS ...... flex_cross_allowed: query sequence valid and equal to the key's (:9346-9348)
struct MaskDesc {
    int32_t flags, chunk_tokens, chunk_stride, window_chunks, q_chunk0;
    const int32_t *flex;  // this batch element's metadata words (flex_meta + b * flex_stride), or null
    int32_t flex_q0, flex_k0, flex_window;
    const uint32_t *bits;  // kMaskBits: this batch element's visibility rows, or null
    int32_t bits_words;    // 32-bit words per query row
};

constexpr int32_t kFlexFlags = EKV_MASK_FLEX_SELF | EKV_MASK_FLEX_CROSS;
// Internal (not settable through ekv_attn_params): prefix-key visibility from an explicit bitmask,
// bit k % 32 of word [t][k / 32] of the batch element's rows -- a ggml 0 / -inf mask tensor
// converted by the ggml op surface.
constexpr int32_t kMaskBits = 1 << 30;
// Flags under which a tile's visibility is taken per row from vis_word.
constexpr int32_t kVisWordFlags = kFlexFlags | kMaskBits;

// A pair of metadata words (EKV_FLEX_META) under the FLEX flags of `flags`.
__host__ __device__ __forceinline__ bool flex_allowed(int32_t flags, uint32_t qm, uint32_t km, int32_t window) {
    const uint32_t qs = qm >> 24, ks = km >> 24;
    if (qs == 0u || qs != ks) return false;  // padding query, or another sequence
    if (flags & EKV_MASK_FLEX_SELF) {
        const int32_t qf = (int32_t)(qm & 0x7FFFFFu), kf = (int32_t)(km & 0x7FFFFFu);
        const bool qc = (qm >> 23) & 1u, kc = (km >> 23) & 1u;
        const bool clean2clean = qc && kc && kf <= qf;
        const bool noise2clean = !qc && kc && kf < qf;
        const bool noise2noise = !qc && !kc && kf == qf;
        const int32_t df = qf > kf ? qf - kf : kf - qf;
        if (!((clean2clean || noise2clean || noise2noise) && df <= window)) return false;
    }
    return true;
}

// The mask description of batch element b of a call.
__device__ __forceinline__ MaskDesc mask_desc(const AttnArgs &a, int b) {
    MaskDesc m;
    m.flags = a.mask_flags;
    m.chunk_tokens = a.chunk_tokens;
    m.chunk_stride = a.chunk_stride;
    m.window_chunks = a.window_chunks;
    m.q_chunk0 = a.q_chunk0;
    m.flex = (a.mask_flags & kFlexFlags) ? a.flex_meta + (int64_t)b * a.flex_stride : nullptr;
    m.flex_q0 = a.flex_q0;
    m.flex_k0 = a.flex_k0;
    m.flex_window = a.flex_window;
    m.bits = (a.mask_flags & kMaskBits)
                 ? a.mask_bits + (int64_t)(b % a.mask_bits_nb) * a.q_tokens * a.mask_bits_words
                 : nullptr;
    m.bits_words = a.mask_bits_words;
    return m;
}

// Visibility bits of keys [w0, w0 + 32) for query token t under kMaskBits (w0 >= 0).
__device__ __forceinline__ uint32_t mask_bits_word(const MaskDesc &m, int t, int w0) {
    const uint32_t *row = m.bits + (int64_t)t * m.bits_words;
    const int wi = w0 >> 5, sh = w0 & 31;
    const uint32_t lo = wi < m.bits_words ? __ldg(row + wi) : 0u;
    if (sh == 0) return lo;
    const uint32_t hi = wi + 1 < m.bits_words ? __ldg(row + wi + 1) : 0u;
    return (lo >> sh) | (hi << (32 - sh));
}

__device__ __forceinline__ bool flex_key_allowed(const MaskDesc &m, int q, int key_index) {
    if (!(m.flags & kFlexFlags)) return true;
    return flex_allowed(m.flags, (uint32_t)__ldg(m.flex + m.flex_q0 + q), (uint32_t)__ldg(m.flex + m.flex_k0 + key_index),
                        m.flex_window);
}

__device__ __forceinline__ bool prefix_allowed(const MaskDesc &m, int q, int k, int prefix_valid,
                                               int span_b, int span_e) {
    if (k >= prefix_valid) return false;
    if (!flex_key_allowed(m, q, k)) return false;
    const bool in_span = k >= span_b && k < span_e;
    if ((m.flags & EKV_MASK_SPAN_ONLY) && !in_span) return false;
    if ((m.flags & EKV_MASK_SPAN_EXCLUDE) && in_span) return false;
    if (m.flags & EKV_MASK_BLOCK_CAUSAL) {
        const int kc = k / m.chunk_stride;
        if (k - kc * m.chunk_stride >= m.chunk_tokens) return false;
        const int qc = m.q_chunk0 + q / m.chunk_tokens;
        if (kc > qc || qc - kc >= m.window_chunks) return false;
    }
    return true;
}

__device__ __forceinline__ bool suffix_allowed(const MaskDesc &m, int q, int s, int suffix_len, int n_prefix) {
    if (s >= suffix_len) return false;
    if (!flex_key_allowed(m, q, n_prefix + s)) return false;
    if ((m.flags & EKV_MASK_SUFFIX_CAUSAL) && s > q) return false;
    if ((m.flags & EKV_MASK_SUFFIX_PREFIX_LM) && q == 0 && s != 0) return false;
    return true;
}

// Per-sequence key ranges of an attention call, resolved from the optional arrays.
struct SeqKeys {
    int seq;          // pool sequence slot (validated)
    int n_prefix;     // prefix keys in use
    int prefix_valid; // prefix keys below this are not padding
    int span_b, span_e;
    bool ok;
};

__device__ __forceinline__ SeqKeys resolve_seq(const PoolView &p, int use_prefix,
                                               const int32_t *seq_ids, const int32_t *prefix_len,
                                               const int32_t *prefix_valid, const int32_t *span_begin,
                                               const int32_t *span_end, int b) {
    SeqKeys r;
    r.seq = seq_ids[b];
    r.ok = r.seq >= 0 && r.seq < p.max_seqs;
    if (!r.ok) {
        r.seq = 0;
        r.n_prefix = r.prefix_valid = r.span_b = r.span_e = 0;
        return r;
    }
    const int len = p.seq_lens[r.seq];
    int np = prefix_len ? prefix_len[b] : len;
    if (!use_prefix) np = 0;
    if (np > len || np < 0) {
        r.ok = false;
        np = 0;
    }
    r.n_prefix = np;
    int pv = prefix_valid ? prefix_valid[b] : np;
    r.prefix_valid = pv < 0 ? 0 : (pv > np ? np : pv);
    r.span_b = span_begin ? span_begin[b] : 0;
    r.span_e = span_end ? span_end[b] : 0;
    return r;
}

// Physical block of table entry `idx` of `seq`, or -1 (and an error report) when out of range.
__device__ __forceinline__ int lookup_block(const PoolView &p, int seq, int idx) {
    if (idx < 0 || idx >= p.max_blocks_per_seq) {
        report_error(p.status, DEV_ERR_BAD_POS, seq, idx, 0);
        return -1;
    }
    const int blk = p.block_tables[(int64_t)seq * p.max_blocks_per_seq + idx];
    if (blk < 0 || blk >= p.n_blocks) {
        report_error(p.status, DEV_ERR_BAD_BLOCK, seq, idx, blk);
        return -1;
    }
    return blk;
}

}  // namespace ekv
