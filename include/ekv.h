/*
 * ekv.h -- C-ABI of the B200 paged KV-cache + masked-attention library (libekv.so).
 *
 * The library is the GPU backend for the denoise-loop attention of Embodied.cpp: action-chunk
 * (or video-chunk) queries attending over a cached prefix KV. It replaces, in the reference
 * (paths inside the Embodied.cpp project):
 *   - the per-step prefix/suffix concat + permute copies        models/pi05.cpp:406-412
 *   - the attention triple mul_mat(K,Q) / soft_max_ext / mul_mat(V,attn)
 *                                                              models/pi05.cpp:414-421,
 *                                                              models/groot_n1.cpp:346-363
 *   - ggml_flash_attn_ext with a concatenated prefix            models/hy_vla.cpp:1067-1076
 *   - the slot KV store + device kernels of LingBot-VA          models/lingbot_va.cpp:8740-8997,
 *                                                              kernels/lingbot/lingbot_flex_attn_cuda.h:13-266
 *
 * Conventions (kept from kernels/lingbot/lingbot_flex_attn_cuda.h:13-266): plain C, caller-owned
 * device buffers, asynchronous launches on the given stream, an int status return
 * (0 = success, negative = error). Launch-time validation errors return before anything is
 * enqueued. Errors found by kernels (bad block ids, out-of-range positions, wait budgets) are
 * written to the pool's device status word and read with ekv_pool_status().
 *
 * Threading: one pool per device; calls on one pool are not re-entrant (the caller serialises,
 * as the reference server's single request loop does, serving/vla-server.cpp:240-523).
 * Different pools/devices are independent.
 */
#ifndef EKV_H
#define EKV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *ekv_stream_t; /* same type as cudaStream_t; NULL = legacy stream */

/* ---- status codes ---- */
#define EKV_OK 0
#define EKV_ERR_INVALID_ARG (-1)  /* bad pointer, size or configuration                */
#define EKV_ERR_CUDA (-2)         /* a CUDA runtime call failed                        */
#define EKV_ERR_POOL_EXHAUSTED (-3)/* not enough free blocks; pool left unchanged       */
#define EKV_ERR_NO_SEQ (-4)       /* sequence id unknown or not live                   */
#define EKV_ERR_RANGE (-5)        /* position / length outside the sequence or slot    */
#define EKV_ERR_UNSUPPORTED (-6)  /* shape or dtype this build does not handle         */
#define EKV_ERR_DEVICE (-7)       /* a kernel reported a bad index (see ekv_pool_status) */
#define EKV_ERR_TIMEOUT (-8)      /* a kernel's bounded wait ran out                   */
#define EKV_ERR_ALLOC (-9)        /* device or host allocation failed                  */

/* ---- dtypes (values follow ggml's enum ggml_type where one exists) ---- */
#define EKV_DTYPE_F32 0
#define EKV_DTYPE_F16 1
#define EKV_DTYPE_Q8_0 8   /* ggml block_q8_0: {fp16 d; int8 qs[32]}, gguf-py quants.py:378-401 */
#define EKV_DTYPE_BF16 30

/* ---- pool ---- */
typedef struct ekv_pool_config {
    int32_t device;             /* CUDA device ordinal                                      */
    int32_t dtype;              /* paged prefix storage: EKV_DTYPE_BF16 or EKV_DTYPE_Q8_0    */
    int32_t block_tokens;       /* tokens per block: multiple of 8, at most 256              */
    int32_t n_blocks;           /* physical blocks per layer                                */
    int32_t kv_heads;           /* Hkv                                                       */
    int32_t head_dim;           /* D: multiple of 16 (bf16) or 32 (Q8_0), at most 256        */
    int32_t n_layers;
    int32_t max_seqs;           /* sequence slots                                           */
    int32_t max_blocks_per_seq; /* block-table width                                        */
    int32_t suffix_tokens;      /* bf16 suffix slot per (sequence, layer); 0 = no slots      */
} ekv_pool_config;

typedef struct ekv_pool ekv_pool;

typedef struct ekv_pool_info {
    size_t bytes_total;         /* device bytes owned by the pool                           */
    size_t bytes_prefix;        /* paged block arena                                        */
    size_t bytes_suffix;        /* suffix slot arena                                        */
    size_t block_bytes;         /* bytes of one (layer, block) for K and V of all heads      */
    int32_t free_blocks;
    int32_t live_seqs;
    void *prefix_base;          /* device pointers, for tests and integration               */
    void *suffix_base;
    int32_t *block_tables;      /* device int32 [max_seqs][max_blocks_per_seq]               */
    int32_t *seq_lens;          /* device int32 [max_seqs] token length of each sequence     */
} ekv_pool_info;

/* Create a pool on cfg->device. Replaces the per-layer cache tensors of the reference
 * (pi0.5 graph tensors models/pi05.cpp:833-839; LingBotKVCache::init
 * models/lingbot_va.cpp:8751-8763). Device memory is zeroed. */
int ekv_pool_create(const ekv_pool_config *cfg, ekv_pool **out);
int ekv_pool_destroy(ekv_pool *pool);
int ekv_pool_get_info(const ekv_pool *pool, ekv_pool_info *info);
/* Read (and clear) the device status word: *code receives EKV_OK or the first kernel error:
 * 1 block-table entry outside the pool, 2 sequence id outside [0, max_seqs), 3 position outside the
 * sequence's blocks, 4 a bounded internal wait ran out, 5 a bf16 query or suffix value beyond the f16
 * range met an f16 operand (Q8_0 pools compute in f16). */
int ekv_pool_status(ekv_pool *pool, int32_t *code, ekv_stream_t stream);
/* Upload host-side block tables / lengths changed since the last sync (stream-ordered). */
int ekv_pool_sync(ekv_pool *pool, ekv_stream_t stream);

/* ---- sequences and block tables ----
 * Blocks are handed out lowest free index first, the order LingBotKVCache::allocate_slots_into
 * uses for free slots (models/lingbot_va.cpp:8803-8805, :8826-8829). */
int ekv_seq_create(ekv_pool *pool, int32_t *seq_id);
/* Return all blocks of the sequence to the free list (block reuse after request completion). */
int ekv_seq_free(ekv_pool *pool, int32_t seq_id);
/* Grow the sequence to n_tokens (allocating blocks); n_tokens below the length truncates and
 * frees whole trailing blocks. Fails with EKV_ERR_POOL_EXHAUSTED leaving the pool unchanged. */
int ekv_seq_resize(ekv_pool *pool, int32_t seq_id, int32_t n_tokens);
/* Install an explicit block table (e.g. a shuffled one); the blocks must be free. */
int ekv_seq_set_blocks(ekv_pool *pool, int32_t seq_id, const int32_t *blocks, int32_t n_blocks,
                       int32_t n_tokens);
/* Drop the oldest n_blocks blocks of the sequence (oldest-chunk eviction of a sliding window,
 * the role of LingBotKVCache::allocate_slots_into's oldest-id eviction,
 * models/lingbot_va.cpp:8806-8825). Later tokens move down by n_blocks*block_tokens. */
int ekv_seq_evict_front(ekv_pool *pool, int32_t seq_id, int32_t n_blocks);
/* ---- predicted tokens (LingBot-VA's rollout appends predicted K/V, attends, then rolls them back
 * before the clean K/V of the same chunk are appended: LingBotKVCache::update_with_workspace's
 * is_pred, restore and clear_pred, models/lingbot_va.cpp:8853-8886, 8946-8966). A sequence holds at
 * most one range of predicted tokens. ---- */
/* Grow the sequence by n_tokens at its tail (blocks as ekv_seq_resize allocates them); pred != 0 marks
 * them predicted. A predicted append extends the predicted range only when that range ends at the
 * tail (EKV_ERR_UNSUPPORTED otherwise); a clean append after predicted tokens leaves them inside. */
int ekv_seq_append_tokens(ekv_pool *pool, int32_t seq_id, int32_t n_tokens, int32_t pred);
/* Drop the predicted tokens (clear_pred). A predicted range at the tail is truncated (its blocks freed
 * as they empty), so the next append writes the clean tokens in place; a range inside the sequence
 * must start and end on block boundaries (its blocks leave the table and later tokens move down;
 * EKV_ERR_UNSUPPORTED otherwise). */
int ekv_seq_clear_pred(ekv_pool *pool, int32_t seq_id);
/* Roll back the last n_tokens appended (restore of the last update's slots): truncation. */
int ekv_seq_restore(ekv_pool *pool, int32_t seq_id, int32_t n_tokens);
/* The predicted range [*lo, *hi) in token positions (*lo == *hi == 0 when there is none). */
int ekv_seq_get_pred(const ekv_pool *pool, int32_t seq_id, int32_t *lo, int32_t *hi);

/* Host view of a sequence: length, block count, and up to `cap` block ids. */
int ekv_seq_get(const ekv_pool *pool, int32_t seq_id, int32_t *n_tokens, int32_t *n_blocks,
                int32_t *blocks, int32_t cap);

/* ---- data operations (device pointers, stream-ordered) ---- */

/* Append rows of K and V (bf16 [rows][kv_heads][head_dim]) into the paged prefix of layer
 * `layer`. For batch element i (device int32 arrays of n_batch entries): sequence seq_ids[i],
 * destination position dst_pos[i], n_rows[i] rows taken from row src_row[i] of k/v.
 * max_rows bounds every n_rows[i]. Q8_0 pools quantise on write (gguf-py rule, bit-exact).
 * Replaces ggml_concat of the prefix (models/pi05.cpp:406-407) and
 * lingbot_runtime_kv_update_f32 (kernels/lingbot/lingbot_flex_attn_cuda.cu:626-649,900-917). */
int ekv_append(ekv_pool *pool, int32_t layer, int32_t n_batch, const int32_t *seq_ids,
               const int32_t *dst_pos, const int32_t *n_rows, const int32_t *src_row,
               int32_t max_rows, const void *k, const void *v, ekv_stream_t stream);

/* Write n_rows bf16 rows per batch element into the suffix slot of (seq_ids[i], layer):
 * k/v are [n_batch][n_rows][kv_heads][head_dim]. The suffix is the per-step part of the keys
 * (the action tokens joined to the prefix by models/pi05.cpp:406-407 every layer-step). */
int ekv_append_suffix(ekv_pool *pool, int32_t layer, int32_t n_batch, const int32_t *seq_ids,
                      int32_t n_rows, const void *k, const void *v, ekv_stream_t stream);

#define EKV_GATHER_NATIVE 0   /* bf16 pool: the stored bf16; Q8_0 pool: ggml block_q8_0 bytes */
#define EKV_GATHER_F32 1      /* values as f32 (dequantised for Q8_0)                          */

/* Copy rows [pos0, pos0+n_rows) of one sequence's paged prefix (layer `layer`) into k_out /
 * v_out, laid out [n_rows][kv_heads][head_dim] (NATIVE Q8_0: [n_rows][kv_heads][head_dim/32]
 * blocks of 34 bytes). Replaces LingBotKVCache::compact_valid / lingbot_runtime_kv_gather_f32
 * (models/lingbot_va.cpp:8974-8996, kernels/lingbot/lingbot_flex_attn_cuda.cu:875-898). */
int ekv_gather(ekv_pool *pool, int32_t layer, int32_t seq_id, int32_t pos0, int32_t n_rows,
               int32_t format, void *k_out, void *v_out, ekv_stream_t stream);
/* Same for the bf16 suffix slot (format NATIVE = bf16, F32 = f32). */
int ekv_gather_suffix(ekv_pool *pool, int32_t layer, int32_t seq_id, int32_t n_rows,
                      int32_t format, void *k_out, void *v_out, ekv_stream_t stream);

/* ---- masked attention over the cache ---- */
#define EKV_MASK_SUFFIX_CAUSAL (1 << 0)    /* models/smolvla.cpp:718-720                    */
#define EKV_MASK_SUFFIX_PREFIX_LM (1 << 1) /* row 0 sees suffix key 0 only, hy_vla.cpp:2355-2367 */
#define EKV_MASK_SPAN_ONLY (1 << 2)        /* GR00T image mask, groot_n1.cpp:717            */
#define EKV_MASK_SPAN_EXCLUDE (1 << 3)     /* GR00T text mask, groot_n1.cpp:716             */
#define EKV_MASK_BLOCK_CAUSAL (1 << 4)     /* chunked prefix, causal across chunks + window */
/* LingBot-VA flex masks over per-token metadata (models/lingbot_va.cpp:9283-9348): every key k of
 * the call (prefix keys, then suffix keys) has the metadata word flex_meta[b * flex_stride +
 * flex_k0 + k], query token t the word flex_meta[b * flex_stride + flex_q0 + t], each word packed
 * by EKV_FLEX_META. FLEX_SELF: flex_self_allowed -- same sequence, and clean query to clean key of
 * an earlier or the same frame, noisy query to clean key of an earlier frame, or noisy query to
 * noisy key of the same frame, with |query frame - key frame| <= flex_window. FLEX_CROSS:
 * flex_cross_allowed -- the query's sequence is valid and equals the key's (text keys carry only
 * their sequence id). Both combine (AND) with the other flags. */
#define EKV_MASK_FLEX_SELF (1 << 5)
#define EKV_MASK_FLEX_CROSS (1 << 6)
/* Metadata word of a token: sequence id seq (0..254; a negative seq marks padding, which sees and
 * is seen by nothing), frame id frame (0 .. 2^23 - 1), clean = 1 for the clean copy of a token
 * (noise id 1 in the reference), 0 for its noisy copy. */
#define EKV_FLEX_META(seq, frame, clean)                                                              \
    ((int32_t)((seq) < 0 ? 0u                                                                     \
                         : ((((uint32_t)(seq) + 1u) << 24) | ((uint32_t)((clean) ? 1 : 0) << 23) |     \
                            ((uint32_t)(frame) & 0x7FFFFFu))))

typedef struct ekv_attn_params {
    int32_t layer;
    int32_t n_batch;        /* B                                                           */
    int32_t q_tokens;       /* Tq (query tokens per batch element)                         */
    int32_t q_heads;        /* Hq, a multiple of the pool's kv_heads (MQA / GQA / MHA)       */
    float scale;            /* softmax scale, 1/sqrt(head_dim) in every reference model      */
    int32_t mask_flags;     /* EKV_MASK_* bits                                              */
    int32_t chunk_tokens;   /* BLOCK_CAUSAL: valid tokens per chunk                          */
    int32_t chunk_stride;   /* BLOCK_CAUSAL: key positions per chunk (>= chunk_tokens)       */
    int32_t window_chunks;  /* BLOCK_CAUSAL: visible chunks, the query's own included        */
    int32_t q_chunk0;       /* BLOCK_CAUSAL: chunk index (in key positions) of query token 0 */
    int32_t suffix_len;     /* suffix-slot keys after the prefix (0 = none)                  */
    int32_t out_dtype;      /* EKV_DTYPE_BF16 or EKV_DTYPE_F32                               */
    int32_t use_prefix;     /* 0: attend the suffix only (self-attention layers)             */
    int32_t reserved;
    /* device int32 arrays of n_batch entries; NULL selects the default                    */
    const int32_t *seq_ids;      /* required                                               */
    const int32_t *prefix_len;   /* prefix keys used; default: the sequence length          */
    const int32_t *prefix_valid; /* keys >= prefix_valid are padding; default: prefix_len   */
    const int32_t *span_begin;   /* span for SPAN_ONLY / SPAN_EXCLUDE; default: empty       */
    const int32_t *span_end;
    /* FLEX_SELF / FLEX_CROSS: device int32 metadata words (EKV_FLEX_META), flex_stride words per
     * batch element; query token t reads word flex_q0 + t, key k word flex_k0 + k            */
    const int32_t *flex_meta;
    int32_t flex_stride;
    int32_t flex_q0;
    int32_t flex_k0;
    int32_t flex_window;         /* FLEX_SELF: the largest visible |query frame - key frame|  */
} ekv_attn_params;

/* Bytes of workspace that lets ekv_attention split long key ranges across CTAs; 0 means the
 * call never needs any. */
size_t ekv_attention_workspace_size(const ekv_pool *pool, const ekv_attn_params *p);

/* out[b][t][h][:] = softmax(scale * q.K^T + mask) V over the prefix keys of seq_ids[b] in
 * layer p->layer followed by p->suffix_len suffix-slot keys. q is bf16 [B][Tq][Hq][D]; out is
 * [B][Tq][Hq][D] in p->out_dtype. q head h reads kv head h / (Hq/Hkv), the ggml broadcast of
 * mul_mat (models/pi05.cpp:414). Rows without a visible key are 0
 * (models/lingbot_va.cpp:9503-9506). `workspace` may be NULL (no key splitting). q, out and
 * workspace must be 16-byte aligned (EKV_ERR_INVALID_ARG otherwise).
 * Replaces models/pi05.cpp:410-421 and ggml_flash_attn_ext (models/hy_vla.cpp:1075). */
int ekv_attention(ekv_pool *pool, const ekv_attn_params *p, const void *q, void *out,
                  void *workspace, size_t workspace_bytes, ekv_stream_t stream);

/* Attention without any device allocation, for callers that cannot call cudaMalloc where
 * attention runs (a controller or server that reserves its device memory at start-up and
 * forbids allocation on the control path, or a plugin host such as a ggml backend op callback
 * that has nowhere to put a workspace). It has no counterpart in the reference. The key-split
 * scratch lives in a fixed EKV_NOALLOC_SCRATCH_BYTES device array that every GPU loading the
 * library reserves until the process exits; a call whose ekv_attention_workspace_size exceeds
 * it returns EKV_ERR_RANGE. The first call on a device looks up the array's device address
 * (once per device); make that first call before any stream capture. All calls on a device
 * share the array: calls that overlap on the GPU race. Results equal ekv_attention's. */
#define EKV_NOALLOC_SCRATCH_BYTES (16u << 20)
int ekv_attention_noalloc(ekv_pool *pool, const ekv_attn_params *p, const void *q, void *out,
                          ekv_stream_t stream);

#define EKV_ALGO_TC 0      /* tcgen05 tensor cores (default): CTA pairs for head_dim 256 (128-key
                              tiles for bf16 calls of at most 8 pairs of 256 query rows where
                              EKV_ALGO_TC_PAIR supports the shape, 64-key tiles otherwise), the
                              one-CTA kernel for other head dims                              */
#define EKV_ALGO_SIMT 1    /* one-warp-per-row CUDA-core kernel, kept as a GPU cross-check   */
#define EKV_ALGO_TC_PAIR 2 /* head_dim 256 on CTA pairs (tcgen05 cta_group::2, 256 query rows
                              per pair, each K/V tile split between the two CTAs) with 128-key
                              tiles and Q in shared memory; needs a query group dividing 128 and
                              power-of-two blocks (EKV_ERR_UNSUPPORTED otherwise); other head
                              dims use the one-CTA kernel                                     */
#define EKV_ALGO_TC_CTA 3  /* the one-CTA tcgen05 kernel (128 query rows per CTA) for every
                              head dim                                                        */
#define EKV_ALGO_TC_PAIR64 4 /* head_dim 256 on CTA pairs with 64-key tiles and Q in tensor
                              memory (what EKV_ALGO_TC runs for Q8_0 pools at head_dim 256);
                              other head dims as EKV_ALGO_TC                                  */
#define EKV_ALGO_TC_HEADS 5 /* multi-head calls with few query tokens (GR00T's 17 x 32 heads,
                              models/groot_n1.cpp:328-364): four heads of one request per unit,
                              one per TMEM lane quarter, persistent CTAs streaming the four heads'
                              K/V of a block in one copy. Needs a bf16 pool, q_heads == kv_heads
                              (a multiple of 4), q_tokens <= 32, head_dim 48 or 64, 16/32/64-token
                              blocks and suffix_len <= 64 (EKV_ERR_UNSUPPORTED otherwise);
                              EKV_ALGO_TC picks it for such calls with at least 37 units    */
int ekv_attention_algo(ekv_pool *pool, const ekv_attn_params *p, const void *q, void *out,
                       void *workspace, size_t workspace_bytes, int32_t algo,
                       ekv_stream_t stream);

/* One layer-step of the denoise loop: attention whose suffix keys are this step's k_suffix /
 * v_suffix ([n_batch][suffix_len][kv_heads][head_dim] bf16, 16-byte aligned) -- the concat of
 * models/pi05.cpp:406-407 and the attention of :410-421 in one call. Same output as
 * ekv_append_suffix(pool, p->layer, p->n_batch, p->seq_ids, p->suffix_len, k_suffix, v_suffix)
 * followed by ekv_attention(pool, p, q, out, ...). At head_dim 256 the attention reads the suffix
 * straight from k_suffix / v_suffix and the pool's suffix slot is left as it was; at other head dims
 * the two calls run (the slot then holds this suffix). Use ekv_append_suffix where the slot must
 * hold it (ekv_gather_suffix). Nothing is enqueued when the arguments are invalid. */
int ekv_append_suffix_attention(ekv_pool *pool, const ekv_attn_params *p, const void *k_suffix,
                                const void *v_suffix, const void *q, void *out, void *workspace,
                                size_t workspace_bytes, ekv_stream_t stream);

/* ---- the layer-step's Q/K/V projection with RoPE, K/V straight into the pool ----
 * Replaces, per layer-step, models/pi05.cpp:391-407 (and :299-318 for the prefix layers' shape): q, k, v =
 * mul_mat(Wq | Wk | Wv, x_norm) over bf16 weights in ggml's layout ([rows of hidden], q_heads * head_dim,
 * kv_heads * head_dim and kv_heads * head_dim rows) and bf16 activations x [n_batch * tokens][hidden]
 * (row b * tokens + t), f32 accumulation; ggml_rope_ext in NEOX mode (freq_base rope_base, no scaling) on q
 * and k at positions[b * tokens + t]; results rounded to bf16. q goes to q_out [n_batch][tokens][q_heads]
 * [head_dim]. With k_out and v_out NULL, K and V go into the suffix slot rows 0 .. tokens - 1 of
 * (seq_ids[b], layer) -- the rows ekv_append_suffix writes, read by ekv_attention with suffix_len = tokens;
 * otherwise into k_out / v_out [n_batch][tokens][kv_heads][head_dim] (the buffers of
 * ekv_append_suffix_attention). head_dim 64, 128 or 256; hidden a multiple of 64; pointers 16-byte
 * aligned. */
int ekv_project_qkv_rope(ekv_pool *pool, int32_t layer, int32_t n_batch, const int32_t *seq_ids, int32_t tokens,
                         int32_t q_heads, int32_t hidden, const void *x, const void *wq, const void *wk, const void *wv,
                         const int32_t *positions, float rope_base, void *q_out, void *k_out, void *v_out,
                         ekv_stream_t stream);

/* ---- ggml op surface: GGML_OP_FLASH_ATTN_EXT on strided device tensors ----
 * Replaces ggml_flash_attn_ext (models/hy_vla.cpp:376-378, :439-441, :460, :492, :859 (GQA, mask);
 * models/lingbot_va.cpp:1263-1266) for a ggml backend that routes the op here: the tensors keep
 * ggml's order (ne[0] fastest) and byte strides, so permuted views are passed as they are.
 *   q    {D,  Tq, Hq,  B}     EKV_DTYPE_F32 / F16 / BF16
 *   k    {D,  Tk, Hkv, Bk}    same types; Hq % Hkv == 0 and B % Bk == 0 (head h reads KV head
 *   v    {Dv, Tk, Hkv, Bk}    h / (Hq / Hkv), batch b reads b / (B / Bk))
 *   mask {>= Tk, >= Tq, Mh, Mb} or NULL: F16 or F32 additive mask; row i of query i, broadcast
 *        over heads (h % Mh) and batch (b % Mb)
 *   dst  {Dv, Hq, Tq, B}      EKV_DTYPE_F32, any strides (the op's own result is contiguous)
 * score = scale * q.k, or logit_softcap * tanh(scale * q.k / logit_softcap) when logit_softcap != 0;
 * then + slope(h) * mask (slope = 1 when max_bias == 0, else the ALiBi slope of head h; needs a
 * mask); softmax over keys in f32; rows whose every score is -inf give 0. D <= 512, Dv <= 256.
 * Tensor cores: calls with D == Dv in {64, 128, 256}, logit_softcap == 0, max_bias == 0 and a mask
 * shared by the heads (Mh == 1) are staged into a workspace -- K/V as a one-layer bf16 pool in
 * 64-token blocks, Q as bf16 rows, the mask as visibility bits -- and run by the kernels of
 * ekv_attention (bf16 operands, f32 accumulation; tolerance as ekv_attention's bf16 path). A mask
 * whose visible entries are not all 0 is detected on the device while it is converted, and the call
 * is then redone exactly on the CUDA cores. Other calls run one warp per query row on the CUDA cores
 * (f32). ekv_flash_attn_ext stages into a workspace the library holds per device (grown on demand,
 * which waits for the device: make the first call of a shape outside graph capture; calls sharing it
 * must be stream-ordered); ekv_flash_attn_ext_ws takes the caller's. */
typedef struct ekv_tensor {
    void *data;     /* device pointer */
    int32_t type;   /* EKV_DTYPE_F32, EKV_DTYPE_F16 or EKV_DTYPE_BF16 */
    int64_t ne[4];
    int64_t nb[4];  /* bytes; nb[0] = element size for rows of consecutive elements */
} ekv_tensor;
int ekv_flash_attn_ext(const ekv_tensor *q, const ekv_tensor *k, const ekv_tensor *v, const ekv_tensor *mask,
                       float scale, float max_bias, float logit_softcap, const ekv_tensor *dst,
                       ekv_stream_t stream);
/* Workspace bytes the tensor-core route of this call needs (16-byte aligned), or 0 where the call
 * runs on the CUDA cores (or is invalid). */
size_t ekv_flash_attn_ext_workspace_size(const ekv_tensor *q, const ekv_tensor *k, const ekv_tensor *v,
                                         const ekv_tensor *mask, float max_bias, float logit_softcap,
                                         const ekv_tensor *dst);
/* ekv_flash_attn_ext with the caller's workspace (graph-capturable): EKV_ERR_RANGE when the size
 * reported above is non-zero and workspace_bytes is below it. */
int ekv_flash_attn_ext_ws(const ekv_tensor *q, const ekv_tensor *k, const ekv_tensor *v, const ekv_tensor *mask,
                          float scale, float max_bias, float logit_softcap, const ekv_tensor *dst, void *workspace,
                          size_t workspace_bytes, ekv_stream_t stream);

/* The ggml triple of models/pi05.cpp:414-418 (also models/smolvla.cpp and models/hy_vla.cpp expert
 * layers): kq = mul_mat(K, Q) at F32 precision, attn = soft_max_ext(kq, mask, scale, max_bias),
 * kqv = mul_mat(V, attn), fused into one call for a backend that recognises the pattern:
 *   k    {D,  Tk, Hkv, Bk}   q {D, Tq, Hq, B}   (head h reads K/V head h / (Hq / Hkv))
 *   v    {Tk, Dv, Hkv, Bk}   keys fastest: the ggml_permute(V, 1, 2, 0, 3) of :412
 *   mask {>= Tk, >= Tq, Mh, Mb} or NULL (F16 or F32), as for ekv_flash_attn_ext
 *   dst  {Dv, Tq, Hq, B}     EKV_DTYPE_F32, any strides: kqv before the permute of :419-420
 * Types, strides and limits as ekv_flash_attn_ext (no softcap). Rows whose every key is masked give
 * 0 (ggml's soft_max would give NaN there; the reference masks never produce such rows). */
int ekv_mul_mat_soft_max_mul_mat(const ekv_tensor *k, const ekv_tensor *q, const ekv_tensor *v,
                                 const ekv_tensor *mask, float scale, float max_bias, const ekv_tensor *dst,
                                 ekv_stream_t stream);
/* Workspace size and explicit-workspace form of the triple, as for ekv_flash_attn_ext. */
size_t ekv_mul_mat_soft_max_mul_mat_workspace_size(const ekv_tensor *k, const ekv_tensor *q, const ekv_tensor *v,
                                                   const ekv_tensor *mask, float max_bias, const ekv_tensor *dst);
int ekv_mul_mat_soft_max_mul_mat_ws(const ekv_tensor *k, const ekv_tensor *q, const ekv_tensor *v,
                                    const ekv_tensor *mask, float scale, float max_bias, const ekv_tensor *dst,
                                    void *workspace, size_t workspace_bytes, ekv_stream_t stream);

/* ---- batching scheduler over the pool ----
 * The reference serves one vla.PredictRequest at a time (serving/vla-server.cpp:240-523). The scheduler
 * queues requests (request_id of serving/vla.proto:33-71 and the prefix they produce), admits them
 * first come first served while sequence slots and blocks allow, runs every active request's next
 * denoise step in the same layer-step calls (a tick), and frees a request's blocks when its last step
 * is done, so later admissions reuse them. Per tick the caller: ekv_sched_begin_tick, appends the
 * prefix K/V of the admitted requests (ekv_append with the batch's admitted_* arrays, all layers), runs the
 * layer-steps (ekv_attn_params.seq_ids / prefix_valid = the batch's arrays, n_batch = n_batch), then
 * ekv_sched_end_tick. Host pointers in the batch stay valid until the next begin_tick; device arrays
 * are rewritten (stream-ordered) by it. One scheduler per pool; calls are not re-entrant. */
typedef struct ekv_sched ekv_sched;
typedef struct ekv_sched_batch {
    int32_t n_batch;                /* active requests this tick                                   */
    const uint64_t *request_ids;    /* host [n_batch]                                              */
    const int32_t *seq_ids_host;    /* host [n_batch]                                              */
    const int32_t *steps;           /* host [n_batch]: the denoise step each request runs this tick */
    const int32_t *seq_ids;         /* device [n_batch]: ekv_attn_params.seq_ids                    */
    const int32_t *prefix_valid;    /* device [n_batch]: ekv_attn_params.prefix_valid               */
    int32_t n_admitted;             /* requests admitted this tick (their prefix K/V are due)       */
    int32_t max_admitted_prefix;    /* the longest of their prefixes (ekv_append's max_rows)        */
    const int32_t *admitted_index;  /* host [n_admitted]: their positions in the batch              */
    const int32_t *admitted_seq_ids;    /* device [n_admitted]: ekv_append's seq_ids              */
    const int32_t *admitted_zeros;      /* device [n_admitted]: zeros (ekv_append's dst_pos)        */
    const int32_t *admitted_prefix_len; /* device [n_admitted]: ekv_append's n_rows               */
    const int32_t *admitted_src_row;    /* device [n_admitted]: ekv_append's src_row when the admitted
                                           requests' prefix rows are packed back to back in order */
    int32_t admitted_rows;              /* the packed rows in all                                  */
    int64_t blocks_reused;          /* blocks handed to this tick's admissions that a request held before */
    int32_t queued;                 /* requests still waiting                                       */
} ekv_sched_batch;
int ekv_sched_create(ekv_pool *pool, int32_t max_batch, int32_t n_steps, ekv_sched **out);
int ekv_sched_destroy(ekv_sched *sched);
/* Queue a request whose prefix has prefix_len tokens (keys >= prefix_valid are padding). */
int ekv_sched_submit(ekv_sched *sched, uint64_t request_id, int32_t prefix_len, int32_t prefix_valid);
int ekv_sched_begin_tick(ekv_sched *sched, ekv_sched_batch *batch, ekv_stream_t stream);
/* Every active request has run one more step; finished ones (up to cap ids into `finished`) free their
 * sequences. */
int ekv_sched_end_tick(ekv_sched *sched, uint64_t *finished, int32_t cap, int32_t *n_finished);
int ekv_sched_stats(const ekv_sched *sched, int64_t *completed, int64_t *blocks_reused, int32_t *active,
                    int32_t *queued);

/* ---- the sampler's per-step elementwise work (a denoise loop with no host round trip) ---- */
/* sample[i] += delta * velocity[i] over n f32 values: the product and the sum each rounded (no fused
 * multiply-add), then rounded to bf16 (nearest even) when bf16_round != 0. Replaces the Euler step of
 * pi0.5 (x_t + dt * velocity, models/pi05.cpp:856), GR00T's host-side action update (actions += dt *
 * velocity after a device-to-host copy every step, models/groot_n1.cpp:756-766) and
 * lingbot_scheduler_step_f32 (kernels/lingbot/lingbot_flex_attn_cuda.cu:40-52, 305-319). */
int ekv_flow_step_f32(float *sample, const float *velocity, int64_t n, float delta, int32_t bf16_round,
                      ekv_stream_t stream);
/* Classifier-free guidance in place over n f32 values: c = cond_in_out[i] (bf16-rounded when
 * bf16_round != 0); with use_guidance, u = uncond[i] (likewise rounded) and c = u + scale * (c - u)
 * (rounded again). Replaces lingbot_model_output_guidance_f32
 * (kernels/lingbot/lingbot_flex_attn_cuda.cu:54-73, 321-337). */
int ekv_guidance_f32(float *cond_in_out, const float *uncond, int64_t n, float scale, int32_t use_guidance,
                     int32_t bf16_round, ekv_stream_t stream);

/* Test hook for the kernels' failure path: with enable != 0, the next launch of the 64-key CTA-pair
 * kernel (head_dim 256 on Q8_0 pools, or EKV_ALGO_TC_PAIR64) has its MMA-issuing thread wait on a
 * barrier that nothing arrives on, and every wait of that launch gives up after about 10 ms (instead
 * of about 2 s). The launch records the kernel timeout in the pool's status word (ekv_pool_status),
 * writes zeros, drains its copies and MMAs in flight and returns; the context stays usable. No
 * counterpart in the reference. */
int ekv_debug_expire_wait(int32_t enable);

const char *ekv_version(void);
/* Kernels this library has launched in this process, on every device (a diagnostic: the difference
 * across a region of calls is the launches they made). */
uint64_t ekv_launch_count(void);
const char *ekv_strerror(int code);

#ifdef __cplusplus
}
#endif
#endif /* EKV_H */
