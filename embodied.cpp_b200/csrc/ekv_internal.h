// ekv_internal.h -- host-side pool object and the kernel launchers shared by the C-ABI.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <set>
#include <vector>

#include "../../include/ekv.h"
#include "ekv_layout.cuh"

struct ekv_pool {
    ekv_pool_config cfg{};
    ekv::PoolView view{};
    void *dev_base = nullptr;
    size_t bytes_total = 0, bytes_prefix = 0, bytes_suffix = 0;
    std::set<int32_t> free_blocks;  // lowest index first
    struct Seq {
        bool live = false;
        int32_t n_tokens = 0;
        std::vector<int32_t> blocks;
        int32_t pred_lo = 0, pred_hi = 0;  // predicted tokens [pred_lo, pred_hi), empty when equal
    };
    std::vector<Seq> seqs;
    std::set<int32_t> free_seq_ids;
    std::vector<uint8_t> dirty;    // per sequence: table/length changed since the last sync
    bool any_dirty = false;
    int32_t *h_status = nullptr;   // pinned, 4 ints
    int sms = 148;                 // SM count of the pool's device (key-split sizing)
};

namespace ekv {

struct AttnArgs {
    PoolView pool;
    int32_t layer, n_batch, q_tokens, q_heads, group;
    float scale_log2;  // scale * log2(e)
    int32_t mask_flags, chunk_tokens, chunk_stride, window_chunks, q_chunk0;
    int32_t suffix_len, out_dtype, use_prefix;
    const int32_t *seq_ids, *prefix_len, *prefix_valid, *span_begin, *span_end;
    // FLEX_SELF / FLEX_CROSS metadata (see ekv_attn_params)
    const int32_t *flex_meta;
    int32_t flex_stride, flex_q0, flex_k0, flex_window;
    const uint16_t *q;
    void *out;
    // key splitting (tensor-core kernel only)
    int32_t n_splits;
    float *ws_o;      // [units][128][D] unnormalised partial outputs
    float *ws_ml;     // [units][128][2] running max (log2 domain) and sum
    // this layer-step's suffix K/V read straight from the caller's [n_batch][suffix_len][kv_heads]
    // [head_dim] bf16 buffers instead of the pool's suffix slot (CTA-pair kernel only), or null
    const uint16_t *k_sfx, *v_sfx;
    // one-CTA kernel, bf16 at 128-key tiles: (request, KV head) units per CTA when a unit has at
    // most 64 query rows (the CTA's 128 rows hold several units, each seeing only its own keys);
    // 0 = one unit's 128-row tile per CTA
    int32_t pack;
    // 64-key CTA-pair kernel: clock cycles a bounded wait gives up after, and the test hook of
    // ekv_debug_expire_wait (1: the MMA-issuing thread waits on a barrier nothing arrives on)
    long long wait_budget;
    int32_t debug_stall;
    // kMaskBits (the ggml op surface): visibility rows [mask_bits_nb][q_tokens][mask_bits_words],
    // batch element b reading rows b % mask_bits_nb
    const uint32_t *mask_bits;
    int32_t mask_bits_words, mask_bits_nb;
};

constexpr long long kDefaultWaitBudget = 4000000000LL;  // clock cycles, about 2 s
constexpr long long kDebugWaitBudget = 20000000LL;      // about 10 ms
// Consumed by the next launch of the 64-key CTA-pair kernel (ekv_debug_expire_wait).
bool take_debug_stall();

// Kernels launched by this library in this process (ekv_launch_count); every launch site adds its
// launches after cudaLaunch* returned.
void note_launches(int n);

int launch_append(const PoolView &p, int layer, int n_batch, const int32_t *seq_ids,
                  const int32_t *dst_pos, const int32_t *n_rows, const int32_t *src_row,
                  int max_rows, const void *k, const void *v, cudaStream_t s);
int launch_append_suffix(const PoolView &p, int layer, int n_batch, const int32_t *seq_ids,
                         int n_rows, const void *k, const void *v, cudaStream_t s);
int launch_gather(const PoolView &p, int layer, int seq, int pos0, int n_rows, int format,
                  void *k_out, void *v_out, cudaStream_t s);
int launch_gather_suffix(const PoolView &p, int layer, int seq, int n_rows, int format,
                         void *k_out, void *v_out, cudaStream_t s);
int launch_attention_simt(const AttnArgs &a, cudaStream_t s);
// Which tcgen05 kernel runs a call at head_dim 256: Auto = the 128-key CTA-pair kernel
// (ekv_attn_pair128.cu) for bf16 pools where the call's shape allows it (query group dividing 128,
// power-of-two blocks), else the 64-key CTA-pair kernel (ekv_attn_pair.cu); Pair = the 128-key
// pair kernel or EKV_ERR_UNSUPPORTED; Pair64 = the 64-key pair kernel; OneCta = one CTA per 128
// query rows. Other head dims always run one CTA per 128 query rows.
// Heads = the multi-head small-query kernel (ekv_attn_heads.cu), which Auto also picks where
// heads_fits() holds and the call has at least a quarter of the SMs' worth of units.
enum class TcKernel { Auto, Pair, OneCta, Pair64, Heads };
int launch_attention_tc(const AttnArgs &a, cudaStream_t s, TcKernel k);
size_t attention_tc_workspace(const PoolView &p, const ekv_attn_params &prm, int max_prefix, int sms);
// CTA-pair kernel (head_dim 256); n_splits == 0 in `a` = choose from the workspace at a.ws_o
int launch_attention_pair(AttnArgs a, cudaStream_t s, size_t ws_bytes, int sms);
int pair_choose_splits(int64_t pair_units, int max_tiles, int sms);
// 128-key CTA-pair kernel (head_dim 256): EKV_ERR_UNSUPPORTED, with nothing enqueued, where the
// call's shape needs the 64-key pair kernel
int launch_attention_pair128(AttnArgs a, cudaStream_t s, size_t ws_bytes, int sms);
int pair128_choose_splits(int64_t pair_units, int max_tiles, int sms);
// Multi-head small-query kernel: four heads of one request per unit (MHA, <= 32 query tokens,
// head_dim 48 or 64, bf16 pool); EKV_ERR_UNSUPPORTED, with nothing enqueued, for other shapes.
bool heads_fits(const AttnArgs &a);
int heads_units(const AttnArgs &a);
int launch_attention_heads(const AttnArgs &a, cudaStream_t s, int sms);
// Q/K/V projection of one layer-step with RoPE NEOX (ekv_project.cu); k_out == nullptr writes K and V
// into the suffix slots of (seq_ids[b], layer)
int launch_project_qkv(const PoolView &p, int layer, int n_batch, const int32_t *seq_ids, int tokens, int q_heads,
                       int hidden, const void *x, const void *wq, const void *wk, const void *wv, const int32_t *positions,
                       float rope_base, void *q_out, void *k_out, void *v_out, cudaStream_t s);
// combine key-split partial outputs (head_dim of the pool) into a.out
int launch_merge_splits(const AttnArgs &a, int n_qtiles, cudaStream_t s);
#ifdef EKV_TRACE
int pair_debug_set_trace(unsigned long long *buf);
int pair128_debug_set_trace(unsigned long long *buf);
int heads_debug_set_trace(unsigned long long *buf);
int project_debug_set_trace(unsigned long long *buf);
#endif

}  // namespace ekv
