/*
 * ekv_oracle.h -- CPU restatement of the reference path (TEST INFRASTRUCTURE ONLY).
 *
 * This header belongs to the oracle: the checker that the CUDA library is compared against,
 * and the timed CPU baseline. Only tests/, __graft_entry__.smoke() and bench.py's CPU legs
 * may load it. The product library (include/ekv.h) never links or calls anything here.
 *
 * What is restated, and from where (paths are inside the Embodied.cpp project):
 *   - BF16 rounding ........ gguf-py quants.py:204-213 (RNE, NaN forced quiet), which is the
 *                            same rule as ggml_compute_fp32_to_bf16 in ggml-impl.h
 *   - Q8_0 blocks .......... gguf-py quants.py:378-401 + np_roundf quants.py:43-47, stated there
 *                            to be bit-exact with quantize_row_q8_0_ref in ggml-quants.c
 *   - masked attention ..... models/pi05.cpp:406-421 (concat, K*Q in F32, soft_max_ext with
 *                            scale, V*attn), fully-masked rows give 0 as in
 *                            models/lingbot_va.cpp:9467-9511 and
 *                            kernels/lingbot/lingbot_flex_attn_cuda.cu:1010-1031
 *   - masks ................ padding + causal suffix models/smolvla.cpp:705-725; prefix-LM
 *                            row-0 suffix models/hy_vla.cpp:2355-2367; GR00T text/image spans
 *                            models/groot_n1.cpp:708-718; block-causal + window in the shape of
 *                            models/lingbot_va.cpp:9336-9344 (BASELINE config 4 form)
 *
 * Pinning: the BF16 and Q8_0 rules are checked against vectors produced by the installed
 * gguf-py package (tests/golden/make_golden.py); the attention is checked against the LingBot
 * smoke vectors (formula inputs of lingbot_flex_attn_cuda.cu:1034-1047, reference result
 * computed in float64) and against a float64 restatement of itself.
 */
#ifndef EKV_ORACLE_H
#define EKV_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- number formats ---- */
uint16_t ekvo_f32_to_bf16(float x);
float ekvo_bf16_to_f32(uint16_t h);
uint16_t ekvo_f32_to_f16(float x);
float ekvo_f16_to_f32(uint16_t h);
void ekvo_f32_to_bf16_n(const float *x, uint16_t *out, int64_t n);
void ekvo_bf16_to_f32_n(const uint16_t *x, float *out, int64_t n);

/* Q8_0: n must be a multiple of 32; out holds n/32 blocks of 34 bytes {fp16 d; int8 qs[32]}. */
void ekvo_quantize_q8_0(const float *x, int64_t n, uint8_t *out);
void ekvo_dequantize_q8_0(const uint8_t *blocks, int64_t n, float *out);

/* ---- masks ---- */
enum {
    EKVO_MASK_SUFFIX_CAUSAL    = 1 << 0, /* suffix key s visible to query token q iff s <= q   */
    EKVO_MASK_SUFFIX_PREFIX_LM = 1 << 1, /* query token 0 sees only suffix key 0               */
    EKVO_MASK_SPAN_ONLY        = 1 << 2, /* prefix key visible iff inside [span_begin,span_end) */
    EKVO_MASK_SPAN_EXCLUDE     = 1 << 3, /* prefix key visible iff outside the span            */
    EKVO_MASK_BLOCK_CAUSAL     = 1 << 4, /* chunked prefix: causal across chunks + window      */
    EKVO_MASK_FLEX_SELF        = 1 << 5, /* LingBot flex_self_allowed over token metadata      */
    EKVO_MASK_FLEX_CROSS       = 1 << 6  /* LingBot flex_cross_allowed (text keys)             */
};

typedef struct ekvo_seq {
    int32_t n_prefix;     /* keys in the cached prefix region (padding included)            */
    int32_t prefix_valid; /* prefix keys at index >= prefix_valid are padding (masked)      */
    int32_t span_begin;   /* special span inside the prefix (GR00T image tokens)            */
    int32_t span_end;
    int32_t n_suffix;     /* keys after the prefix (this step's appended suffix)            */
    /* FLEX masks: metadata words of this sequence, packed as EKV_FLEX_META of include/ekv.h:
     * bits 31-24 sequence id + 1 (0 = padding), bit 23 noise id (1 = clean), bits 22-0 frame id */
    const int32_t *flex_meta;
} ekvo_seq;

typedef struct ekvo_mask {
    int32_t flags;
    int32_t chunk_tokens;  /* BLOCK_CAUSAL: valid tokens per chunk                         */
    int32_t chunk_stride;  /* BLOCK_CAUSAL: key-index stride of one chunk (>= chunk_tokens) */
    int32_t window_chunks; /* BLOCK_CAUSAL: chunks visible, the query's own one included    */
    int32_t q_chunk0;      /* BLOCK_CAUSAL: key-chunk index of query token 0's chunk         */
    int32_t flex_q0;       /* FLEX: metadata index of query token 0                          */
    int32_t flex_k0;       /* FLEX: metadata index of key 0 (prefix keys, then suffix keys)   */
    int32_t flex_window;   /* FLEX_SELF: window_size, the largest visible frame distance       */
} ekvo_mask;

/* 1 if query token q (0-based within the call) may attend key k (prefix keys first). */
int ekvo_allowed(const ekvo_mask *m, const ekvo_seq *s, int32_t q, int32_t k);

/* ---- attention ----
 * q:   [B][Tq][Hq][D] f32
 * k,v: [B][Lk_max][Hkv][D] f32, key order = prefix keys then suffix keys
 * dense_mask (optional, may be NULL): additive f32 [B][Tq][Lk_max] applied after the scale,
 *   as ggml_soft_max_ext does; combined with the structural mask above.
 * out: [B][Tq][Hq][D] f32. Rows with no allowed key are written as 0.
 * q head h reads kv head h / (Hq / Hkv) (ggml mul_mat broadcast of src0 over ne2).
 */
typedef struct ekvo_attn_args {
    int32_t B, Tq, Hq, Hkv, D, Lk_max;
    float scale;
    const float *q, *k, *v, *dense_mask;
    const ekvo_seq *seqs; /* [B] */
    ekvo_mask mask;
    float *out;
} ekvo_attn_args;

/* Rows (b, t, h) = rows[3 i .. 3 i + 2] only, into out[i][D]: the same arithmetic as
 * ekvo_attention_f32 for a sample of a large call's query rows. */
int ekvo_attention_rows(const ekvo_attn_args *a, int32_t n_rows, const int32_t *rows, float *out, int n_threads);

/* float32 arithmetic with the softmax sum in double, as ggml's CPU soft_max does. */
int ekvo_attention_f32(const ekvo_attn_args *a, int n_threads);
/* everything in double: the cross-check for the f32 restatement. */
int ekvo_attention_f64(const ekvo_attn_args *a, double *out);

/* ---- timed CPU baseline over a Q8_0 / bf16 cache in ggml's natural layout ----
 * Runs `n_calls` attention calls; call c uses query block q + c*q_call_stride and
 * cached keys of layer (c % n_layers). The cache holds, per request b and layer l,
 * n_prefix[b] prefix rows [tok][Hkv][D] either as ggml block_q8_0 (kv_is_q8 = 1) or bf16,
 * plus a bf16 suffix of n_suffix rows. Output f32 [B][Tq][Hq][D] per call is overwritten.
 */
typedef struct ekvo_cache_args {
    int32_t B, Tq, Hq, Hkv, D, n_layers, kv_is_q8, max_prefix, n_suffix;
    float scale;
    const int32_t *n_prefix;     /* [B] */
    const int32_t *prefix_valid; /* [B] */
    const uint8_t *prefix_k, *prefix_v; /* [n_layers][B][max_prefix][Hkv] rows (q8_0 or bf16) */
    const uint16_t *suffix_k, *suffix_v; /* [n_layers][B][n_suffix][Hkv][D] bf16 */
    const uint16_t *q;                   /* [n_calls][B][Tq][Hq][D] bf16 */
    int32_t n_calls;
    float *out;                          /* [B][Tq][Hq][D] */
} ekvo_cache_args;

int ekvo_cache_attention_run(const ekvo_cache_args *a, int n_threads);

const char *ekvo_version(void);

#ifdef __cplusplus
}
#endif
#endif
