// ekv_attn_pair.cu -- masked attention over the paged KV pool on CTA pairs (tcgen05 cta_group::2),
// head_dim 256 (the pi0.5 action expert: 8 query heads over 1 KV head).
//
// Replaces the same reference ops as the one-CTA kernel (models/pi05.cpp:406-421: concat, permutes,
// mul_mat, soft_max_ext, mul_mat) for head_dim 256, where one SM's tensor memory holds one 128-row
// query tile at a time (S 2 x 64 + O 256 + Q 128 of its 512 columns). There, four CTAs per
// (request, KV head) each streamed every K/V byte through L2 into their SM and each Q8_0 block was
// dequantised four times. Here a cluster of two CTAs (ranks 0, 1) takes 256 query rows, rank r
// owning rows [256p + 128r, +128), and rank 0 issues every MMA for both with cta_group::2, M = 256:
//
//   S = Q K^T  N = 64 keys;  each CTA holds the K rows of keys [32r, 32r + 32) of the tile
//   O += P V   N = 256;      each CTA holds the V columns [128r, 128r + 128) of all 64 keys
//
// A, S, P and O of each CTA's 128 rows stay in its own tensor memory (same column addresses); B
// operands are split between the two CTAs' shared memory at the same offsets. Each CTA therefore
// copies (bf16) or dequantises (Q8_0) half of every K/V tile.
//
// Warps per CTA: 0-7 softmax (two per TMEM lane quarter, 32 columns each); 8 = MMA issue on rank 0,
// completion relay on rank 1 (bf16: forwards "my half landed" to rank 0's barriers); 9 = copy feeder;
// 10-17 = Q8_0 dequantisation. Rank 1's producers and softmax warps arrive on rank 0's barriers
// (mbarrier arrive at cluster scope); rank 0 signals MMA completion to both CTAs with one commit
// per CTA. Every wait is bounded; on expiry both CTAs record DEV_ERR_TIMEOUT and unwind through the
// closing cluster barrier, after rank 0's MMAs have finished.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "ekv_attn_common.cuh"
#include "ekv_device.cuh"
#include "ekv_internal.h"
#include "ekv_sm100.cuh"

namespace ekv {
namespace {

using namespace sm100;

template <bool Q8>
struct PairCfg {
    static constexpr int D = 256, BN = 64, W = 128;
    static constexpr uint32_t LAYOUT = 2u;       // 128-byte swizzle
    static constexpr int KH_ROWS = BN / 2;       // K rows per CTA
    static constexpr int VH_COLS = D / 2;        // V columns per CTA
    static constexpr int KH_BYTES = KH_ROWS * D * 2;  // 16 KB: [4 rg][4 chunk][8][128 B]
    static constexpr int VH_BYTES = BN * VH_COLS * 2; // 16 KB: [8 rg][2 chunk][8][128 B]
    static constexpr uint32_t K_SBO = (D * 2 / W) * 8 * W;        // 4096
    static constexpr uint32_t V_LBO = 8 * W;                      // 1024 (chunk stride along d)
    static constexpr uint32_t V_SBO = (VH_COLS * 2 / W) * 8 * W;  // 2048 (8-row group stride)
    static constexpr int NSTAGE = Q8 ? 4 : 6;
    // raw Q8_0 ring: per tile, K and V of this CTA's 32 key rows, then V of the peer's 32 rows
    // (int8 + fp16 scales)
    static constexpr int NRAW = Q8 ? 3 : 0;
    static constexpr int RAW_ROWB = D + D / 16;  // raw bytes per key row
    static constexpr int RAW_BYTES = 3 * KH_ROWS * RAW_ROWB;
    static constexpr int OFF_K = 0;
    static constexpr int OFF_V = NSTAGE * KH_BYTES;
    static constexpr int OFF_RAW = OFF_V + NSTAGE * VH_BYTES;
    static constexpr int OFF_BAR = OFF_RAW + NRAW * RAW_BYTES;
    static constexpr int BAR_BYTES = 512;
    static constexpr int OFF_XCH = OFF_BAR + BAR_BYTES;  // softmax pair exchange [2][2][128] + [2][128] floats
    static constexpr int OFF_TBL = OFF_XCH + 6 * kBM * 4;
    static constexpr int TBL_ROOM = (232448 - 1024 - OFF_TBL) / 8;
    static constexpr int TBL = TBL_ROOM > 512 ? 512 : TBL_ROOM;
    static constexpr int SMEM = OFF_TBL + TBL * 8 + 1024;
    static constexpr int QSTR = D * 2 + 16;  // Q staging row stride
    static constexpr int OSTR = D * 4 + 16;  // epilogue staging row stride (f32 worst case)
    static constexpr int SMW = 8;
    // 8 = MMA issue (rank 0); 9, 10 = K and V copy feeders; 11-18 = dequantisation (Q8_0) or
    // 11 = relay of the copies' completion (bf16)
    static constexpr int MMA_WARP = 8, TMA_WARP = 9, DQ_WARP0 = 11, RELAY_WARP = 11;
    static constexpr int THREADS = (SMW + 3) * 32 + (Q8 ? kDq : 32);
    static constexpr int TMEM_COLS = 512;
    static constexpr int S_COL = 0, O_COL = 2 * BN, Q_COL = 512 - D / 2;
    static_assert(O_COL + D <= Q_COL, "TMEM budget");
    static_assert(SMEM <= 232448, "shared-memory budget");
    static_assert(TBL >= 64, "block-table cache");
    static_assert(kBM * QSTR <= OFF_BAR && kBM * OSTR <= OFF_BAR, "Q and epilogue staging fit below the barriers");
    static_assert((D / 32) * 4 * kOutBox <= OFF_BAR, "epilogue boxes (f32) fit below the barriers");
};

// The MMA thread waits once per tile: a wait in the issuing thread costs about 220 cycles of idle
// tensor pipe (the issue queue is one MMA deep). After S(0) and S(1) (K_FULL), it issues for each j
// P.V(j) and then S(j + 2) behind it, both gated by PVK(j), which counts the V(j) and P(j) arrivals
// and the K(j + 2) arrivals of both CTAs. Rank 1's softmax and dequantisation warps arrive directly
// on rank 0's barriers; for bf16, each CTA's relay warp forwards its copies' completion (the copies
// signal per-stage barriers of their own CTA, which an aborting feeder can wait on). All arrivals
// release at CTA scope (mbar_arrive_remote).
enum {
    PB_K_FULL = 0,       // [6] bf16: this CTA's K half landed (forwarded by its relay warp)
    PB_KINIT = 6,        // [2] rank 0: both CTAs' K halves of tiles 0 and 1
    PB_STALL = 8,        // rank 0: never arrived on (ekv_debug_expire_wait)
                         // 9-11 unused
    PB_K_EMPTY = 12,     // [6] S(j) done (committed to both CTAs): K stage free, S(j) readable
    PB_V_FULL = 18,      // [6] bf16: this CTA's V half landed (forwarded by its relay warp)
                         // 24-29 unused
    PB_V_EMPTY = 30,     // [6] P.V(j) done (both CTAs): V stage free, P(j) consumed, O updated
    PB_RAW_FULL = 36,    // [3] raw Q8_0 stage landed (both feeders' copies)
    PB_RAW_EMPTY = 39,   // [3] raw Q8_0 stage read by the dequant warps
                         // 42-45 unused
                         // 46-47 unused
    PB_DONE = 48,
    PB_XCH = 49,         // [4] softmax pair exchange
    PB_PVK = 53,         // [6] rank 0: everything P.V(j) and the S(j + 2) issued behind it need --
                         //     V(j) and P(j) of both CTAs, and both K halves of tile j + 2
    PB_N = 59
};

// Barrier of rank 0 that the producers of K(t) arrive on: K(0) and K(1) on KINIT, later tiles on
// the barrier of the P.V two tiles earlier, so that the MMA thread waits once per tile. A tile past
// the end still arrives there (no data), so every phase completes.
__device__ __forceinline__ int pair_k_bar(int t, int ns) { return t < 2 ? PB_KINIT + t : PB_PVK + (t - 2) % ns; }
static_assert(PB_N * 8 + 16 <= 512, "barrier block");
static_assert(PB_PVK + 6 <= PB_N, "PVK covers the deepest stage ring");

__device__ __forceinline__ uint32_t stage_parity(int j, int ns) { return (uint32_t)(j / ns) & 1u; }

// Key-tile schedule of one CTA; both CTAs of a pair derive the same key range (from the pair's
// 256 rows) and their own query rows.
struct PairPlan {
    int b, g, pair, split, rank;
    int qrow0, rows_valid;  // this CTA's query rows (rows_valid may be 0 for rank 1)
    SeqKeys sk;
    int kbeg, np_tiles, ns_tiles, j0, j1, tbl_lo, tbl_n;
};

__device__ __forceinline__ PairPlan make_pair_plan(const AttnArgs &a) {
    constexpr int BN = 64;
    PairPlan pl;
    const int n_splits = a.n_splits > 1 ? a.n_splits : 1;
    pl.rank = (int)(blockIdx.x & 1u);
    const int unit = (int)(blockIdx.x >> 1);
    pl.pair = unit / n_splits;
    pl.split = unit - pl.pair * n_splits;
    pl.g = blockIdx.y;
    pl.b = blockIdx.z;
    const int rows_total = a.q_tokens * a.group;
    const int prow0 = pl.pair * 2 * kBM, prows = min(2 * kBM, rows_total - prow0);
    pl.qrow0 = prow0 + pl.rank * kBM;
    pl.rows_valid = max(0, min(kBM, rows_total - pl.qrow0));
    pl.sk = resolve_seq(a.pool, a.use_prefix, a.seq_ids, a.prefix_len, a.prefix_valid, a.span_begin, a.span_end, pl.b);
    pl.kbeg = 0;
    pl.np_tiles = 0;
    pl.ns_tiles = 0;
    if (pl.sk.ok) {
        int kb = 0, ke = pl.sk.prefix_valid;
        if (a.mask_flags & EKV_MASK_SPAN_ONLY) {
            kb = max(kb, pl.sk.span_b);
            ke = min(ke, pl.sk.span_e);
        }
        if (a.mask_flags & EKV_MASK_BLOCK_CAUSAL) {
            const int t_lo = prow0 / a.group, t_hi = (prow0 + prows - 1) / a.group;
            const int qc_lo = a.q_chunk0 + t_lo / a.chunk_tokens, qc_hi = a.q_chunk0 + t_hi / a.chunk_tokens;
            kb = max(kb, (qc_lo - a.window_chunks + 1) * a.chunk_stride);
            ke = min(ke, (qc_hi + 1) * a.chunk_stride);
        }
        if (ke > kb) {
            pl.kbeg = kb / BN * BN;
            pl.np_tiles = (ke - pl.kbeg + BN - 1) / BN;
        }
        pl.ns_tiles = (a.suffix_len + BN - 1) / BN;
    }
    const int n = pl.np_tiles + pl.ns_tiles;
    const int per = (n + n_splits - 1) / n_splits;
    pl.j0 = min(n, pl.split * per);
    pl.j1 = min(n, pl.j0 + per);
    pl.tbl_lo = 0;
    pl.tbl_n = 0;
    const int pj1 = min(pl.j1, pl.np_tiles);
    if (pl.j0 < pj1) {
        const int k_lo = pl.kbeg + pl.j0 * BN;
        const int k_hi = min(pl.kbeg + pj1 * BN, pl.sk.n_prefix);
        if (k_hi > k_lo) {
            const int bt = a.pool.block_tokens;
            pl.tbl_lo = k_lo / bt;
            pl.tbl_n = (k_hi + bt - 1) / bt - pl.tbl_lo;
        }
    }
    return pl;
}

// K tile base of block-table entry `idx` (head g, this layer), or nullptr for an invalid entry.
template <int TBL>
__device__ __forceinline__ const uint8_t *pair_ptr_of(const AttnArgs &a, const PairPlan &pl,
                                                      const uint8_t *const *sPtr, int idx) {
    const int i = idx - pl.tbl_lo;
    if (pl.tbl_n <= TBL && i >= 0 && i < pl.tbl_n) return sPtr[i];
    const int blk = lookup_block(a.pool, pl.sk.seq, idx);
    return blk < 0 ? nullptr : a.pool.prefix + prefix_tile_index(a.pool, a.layer, blk, 0, pl.g) * a.pool.tile_bytes;
}

// This CTA's part of suffix tile j read straight from the caller's row-major bf16 K/V
// ([n_batch][suffix_len][kv_heads][256]) into the swizzled operand stage: K rows [32r, 32r + 32) of
// the tile (kv = 0), or V columns [128r, 128r + 128) of its 64 rows (kv = 1); rows past suffix_len
// are zero. `nthr` threads (tid < nthr) share the 1024 16-byte units, four loads in flight each;
// TO_F16 converts to the f16 operands of Q8_0 pools.
template <bool TO_F16>
__device__ __forceinline__ void pair_suffix_direct(const AttnArgs &a, const PairPlan &pl, int j, int kv, uint8_t *sDst,
                                                   int tid, int nthr) {
    constexpr int BN = 64, D = 256, KH_ROWS = 32, VH_COLS = 128, W = 128;
    const int s_base = (j - pl.np_tiles) * BN;
    const int upr = kv == 0 ? D / 8 : VH_COLS / 8;
    const int row_base = kv == 0 ? pl.rank * KH_ROWS : 0;
    const int col_base = kv == 0 ? 0 : pl.rank * VH_COLS;
    const int dD = kv == 0 ? D : VH_COLS;
    const int64_t row_stride = (int64_t)a.pool.kv_heads * D;
    const uint16_t *src = (kv ? a.v_sfx : a.k_sfx) + ((int64_t)pl.b * a.suffix_len * a.pool.kv_heads + pl.g) * D +
                          col_base;
    constexpr int UNITS = 1024;  // 32 rows x 32 units (K) = 64 rows x 16 units (V)
#pragma unroll 1
    for (int u0 = tid; u0 < UNITS; u0 += 4 * nthr) {
        uint4 v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int u = u0 + i * nthr;
            const int row = u / upr, dl = (u - row * upr) * 8;
            const int srow = s_base + row_base + row;
            v[i] = make_uint4(0, 0, 0, 0);
            if (u < UNITS && srow < a.suffix_len) v[i] = __ldg((const uint4 *)(src + srow * row_stride + dl));
        }
        bool bad = false;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int u = u0 + i * nthr;
            if (u >= UNITS) break;
            const int row = u / upr, dl = (u - row * upr) * 8;
            uint4 w = v[i];
            if (TO_F16) {
                w = make_uint4(bf16x2_to_f16x2(w.x), bf16x2_to_f16x2(w.y), bf16x2_to_f16x2(w.z), bf16x2_to_f16x2(w.w));
                bad |= f16x8_has_inf(w);
            }
            *(uint4 *)(sDst + tile_elem_off(row, dl, dD, W)) = w;
        }
        if (TO_F16 && bad) report_error(a.pool.status, DEV_ERR_F16_RANGE, 2, pl.b, j);
    }
}

// ---- bf16 feeder. K half (kv = 0): tile rows [32r, 32r + 32), in runs of whole blocks (or of 32
// rows of a larger block), one copy per run into the K stage. V half (kv = 1): the two 1 KB column
// chunks [2r, 2r + 2) of each of the tile's 8 row groups, one 2 KB copy per row group into the V
// stage. One lane per copy; rows without a source are zero-filled by the warp. ----
__device__ __forceinline__ void pair_produce_bf16(const AttnArgs &a, const PairPlan &pl, const uint8_t *const *sPtr,
                                                  int j, int kv, uint8_t *sDst, uint32_t bar_full, int lane) {
    using C = PairCfg<false>;
    constexpr int BN = C::BN, RB = C::D * 2;
    const PoolView &p = a.pool;
    const bool suffix = j >= pl.np_tiles;
    if (suffix && a.k_sfx) {
        // the caller's row-major suffix: loaded and swizzled by the warp, then one plain arrival
        pair_suffix_direct<false>(a, pl, j, kv, sDst, lane, 32);
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_full);
        return;
    }
    const int key0 = suffix ? (j - pl.np_tiles) * BN : pl.kbeg + j * BN;  // tile's first key / suffix row
    // copy `lane`: source row range (8-row groups) and destination offset
    int n_cp;        // copies this part needs
    int rows_cp;     // rows per copy
    if (kv == 0) {
        rows_cp = suffix ? C::KH_ROWS : min(p.block_tokens, C::KH_ROWS);
        n_cp = C::KH_ROWS / rows_cp;
    } else {
        rows_cp = 8;
        n_cp = BN / 8;
    }
    const uint32_t cp_bytes = kv == 0 ? (uint32_t)rows_cp * RB : 2048u;
    const uint32_t dst = (uint32_t)lane * cp_bytes;
    const uint8_t *src = nullptr;
    uint32_t bytes = 0;
    if (lane < n_cp) {
        const int row = (kv == 0 ? pl.rank * C::KH_ROWS : 0) + lane * rows_cp;  // tile-local first row
        const int64_t col_off = kv == 0 ? 0 : (int64_t)pl.rank * 2 * 1024;      // V: chunks 2r, 2r + 1
        if (suffix) {
            const int srow = key0 + row;
            if (srow < p.suffix_rows) {
                const int rows = min(rows_cp, p.suffix_rows - srow);
                const uint8_t *t = p.suffix + suffix_tile_index(p, a.layer, pl.sk.seq, kv, pl.g) * p.suffix_tile_bytes;
                if (kv == 0) {
                    src = t + (int64_t)srow * RB;
                    bytes = (uint32_t)rows * RB;
                } else {
                    src = t + (int64_t)(srow >> 3) * 4096 + col_off;
                    bytes = 2048u;
                }
            }
        } else {
            const int k = key0 + row;
            if (k < pl.sk.n_prefix) {
                int rib;
                const int idx = block_index(p, k, rib);
                const uint8_t *t = pair_ptr_of<C::TBL>(a, pl, sPtr, idx);
                if (t) {
                    t += (int64_t)kv * p.kv_heads * p.tile_bytes;
                    if (kv == 0) {
                        src = t + (int64_t)rib * RB;
                        bytes = cp_bytes;
                    } else {
                        src = t + (int64_t)(rib >> 3) * 4096 + col_off;
                        bytes = 2048u;
                    }
                }
            }
        }
    }
    const uint32_t zlo = dst + bytes, zhi = lane < n_cp ? dst + cp_bytes : zlo;
    const uint32_t need_zero = __ballot_sync(0xffffffffu, zhi > zlo);
    const uint32_t total = __reduce_add_sync(0xffffffffu, src ? bytes : 0u);
    if (need_zero) {
        for (uint32_t m = need_zero; m; m &= m - 1) {
            const int s = __ffs(m) - 1;
            const uint32_t z0 = __shfl_sync(0xffffffffu, zlo, s), z1 = __shfl_sync(0xffffffffu, zhi, s);
            for (uint32_t o = z0 + lane * 16; o < z1; o += 32 * 16) *(uint4 *)(sDst + o) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async();
        __syncwarp();
    }
    if (lane == 0) {
        if (total) mbar_arrive_expect_tx(bar_full, total);
        else mbar_arrive(bar_full);
    }
    __syncwarp();
    if (src) bulk_g2s(smem_addr(sDst + dst), src, bytes, bar_full);
}

// ---- Q8_0 feeders. A raw stage holds, per segment of ks = min(block_tokens, 32) key rows: first the
// K and V parts of this CTA's rows [32r, 32r + 32) of the tile (own = 1), then the V parts of the
// peer's rows (own = 0). Each part is [qs ks x D][fp16 scales ks x D/32] -- exactly a pool tile, so
// a whole block with adjacent K and V tiles (one KV head) is ONE copy of both parts. One lane per
// segment; both feeders arrive on the stage's barrier with their byte counts. ----
__device__ __forceinline__ void pair_produce_q8_raw(const AttnArgs &a, const PairPlan &pl, const uint8_t *const *sPtr,
                                                    int j, int own, uint8_t *raw, uint32_t bar_full, int lane) {
    using C = PairCfg<true>;
    constexpr int BN = C::BN, D = C::D, SCB = D / 16;
    const PoolView &p = a.pool;
    const int bt = p.block_tokens;
    const int ks = min(bt, C::KH_ROWS), n_seg = C::KH_ROWS / ks;
    const int row0 = (own ? pl.rank : 1 - pl.rank) * C::KH_ROWS;
    const uint32_t part = (uint32_t)ks * (D + SCB);
    const uint32_t seg_bytes = own ? 2 * part : part;
    uint8_t *base = raw + (own ? 0 : 2 * C::KH_ROWS * C::RAW_ROWB);
    const uint8_t *tk = nullptr;
    int rib = 0;
    if (lane < n_seg) {
        const int k = pl.kbeg + j * BN + row0 + lane * ks;
        const int idx = block_index(p, k, rib);
        if (k < pl.sk.n_prefix) tk = pair_ptr_of<C::TBL>(a, pl, sPtr, idx);
    }
    const uint32_t segmask = (1u << n_seg) - 1u;
    const uint32_t valid = __ballot_sync(0xffffffffu, tk != nullptr) & segmask;
    const uint32_t missing = ~valid & segmask;
    if (missing) {
        for (uint32_t m = missing; m; m &= m - 1) {
            uint8_t *z = base + (__ffs(m) - 1) * seg_bytes;
            for (uint32_t o = lane * 16; o < seg_bytes; o += 32 * 16) *(uint4 *)(z + o) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async();
        __syncwarp();
    }
    if (lane == 0) mbar_arrive_expect_tx(bar_full, (uint32_t)__popc(valid) * seg_bytes);
    __syncwarp();
    if (!tk) return;
    const int64_t v_off = (int64_t)p.kv_heads * p.tile_bytes;  // V tile of the same head
    uint8_t *dst = base + lane * seg_bytes;
    if (ks == bt) {
        if (own && p.kv_heads == 1) {
            bulk_g2s(smem_addr(dst), tk, 2 * part, bar_full);  // K tile + V tile, contiguous
        } else {
            if (own) bulk_g2s(smem_addr(dst), tk, part, bar_full);
            bulk_g2s(smem_addr(dst + (own ? part : 0)), tk + v_off, part, bar_full);
        }
    } else {  // rows [rib, rib + 32) of a larger block: qs and scale planes separately
        for (int kv = own ? 0 : 1; kv < 2; ++kv) {
            const uint8_t *src = tk + kv * v_off;
            uint8_t *d = dst + (own && kv ? part : 0);
            bulk_g2s(smem_addr(d), src + (int64_t)rib * D, (uint32_t)ks * D, bar_full);
            bulk_g2s(smem_addr(d + ks * D), src + (int64_t)bt * D + (int64_t)rib * SCB, (uint32_t)ks * SCB, bar_full);
        }
    }
}

// ---- Q8_0 dequantisation of this CTA's half of a tile (kDq threads, 2 units of 16 values each)
// from its raw stage (segments of 2^seg_shift rows, laid out as pair_produce_q8_raw describes).
// K: this CTA's 32 rows, all 256 columns; V: all 64 rows, columns [128r, 128r + 128).
// 8 consecutive threads take 8 consecutive rows of one 16-column segment (distinct bank groups for
// the swizzled int8 loads and the swizzled operand stores). ----
struct PairDqUnits {
    uint4 q[2];
    uint32_t d[2];
};

// This thread's two int8 units (and their scales) of part kv of a raw stage.
__device__ __forceinline__ PairDqUnits pair_dq_load(const uint8_t *raw, int kv, int rank, int seg_shift, int dtid) {
    using C = PairCfg<true>;
    constexpr int D = C::D, SCB = D / 16;
    const int segs = kv == 0 ? D / 16 : C::VH_COLS / 16;  // 16 or 8 segments per row
    const int rlow = dtid & 7, seg = (dtid >> 3) % segs, rhigh = (dtid >> 3) / segs;
    const int rpass = kDq / segs;  // rows covered per unit step: 16 (K) or 32 (V)
    const int r0 = rhigh * 8 + rlow;
    const int srows = 1 << seg_shift;
    const uint32_t part = (uint32_t)srows * (D + SCB);
    const int d0 = (kv == 0 ? 0 : rank * C::VH_COLS) + seg * 16;
    PairDqUnits u;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int row = r0 + i * rpass;  // K: local row 0-31; V: tile row 0-63
        const bool own = kv == 0 || (row >> 5) == rank;
        const int lr = row & 31, s = lr >> seg_shift, rib = lr & (srows - 1);
        const uint8_t *t = own ? raw + s * 2 * part + kv * part : raw + 2 * C::KH_ROWS * C::RAW_ROWB + s * part;
        u.q[i] = *(const uint4 *)(t + q8_qs_off(rib, d0, D));
        u.d[i] = *(const uint16_t *)(t + srows * D + rib * SCB + (d0 >> 5) * 2);
    }
    return u;
}

// Dequantise the units into the K half [32 rows x 256] or V half [64 rows x 128] operand tile.
__device__ __forceinline__ void pair_dq_store(const PairDqUnits &u, int kv, uint8_t *sDst, int dtid) {
    using C = PairCfg<true>;
    constexpr int D = C::D;
    const int segs = kv == 0 ? D / 16 : C::VH_COLS / 16;
    const int rlow = dtid & 7, seg = (dtid >> 3) % segs, rhigh = (dtid >> 3) / segs;
    const int rpass = kDq / segs;
    const int r0 = rhigh * 8 + rlow;
    const int dD = kv == 0 ? D : C::VH_COLS;
    const uint32_t off_lo = tile_elem_off(r0, seg * 16, dD, C::W), off_hi = tile_elem_off(r0, seg * 16 + 8, dD, C::W);
    const uint32_t step = (uint32_t)(rpass / 8) * (kv == 0 ? C::K_SBO : C::V_SBO);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        uint4 lo, hi;
        dequant16(u.q[i], u.d[i], lo, hi);
        *(uint4 *)(sDst + off_lo + i * step) = lo;
        *(uint4 *)(sDst + off_hi + i * step) = hi;
    }
}

// bf16 suffix slot -> this CTA's f16 K or V half (Q8_0 pools), 4 units of 8 values per thread
__device__ __forceinline__ void pair_convert_suffix(const AttnArgs &a, const PairPlan &pl, int j, int kv,
                                                    uint8_t *sDst, int dtid) {
    using C = PairCfg<true>;
    constexpr int BN = C::BN, D = C::D;
    if (a.k_sfx) {
        pair_suffix_direct<true>(a, pl, j, kv, sDst, dtid, kDq);
        return;
    }
    const PoolView &p = a.pool;
    const int s_base = (j - pl.np_tiles) * BN;
    const uint8_t *src = p.suffix + suffix_tile_index(p, a.layer, pl.sk.seq, kv, pl.g) * p.suffix_tile_bytes;
    const int upr = kv == 0 ? D / 8 : C::VH_COLS / 8;  // 8-value units per row: 32 or 16
    const int row_base = kv == 0 ? pl.rank * C::KH_ROWS : 0;
    const int col_base = kv == 0 ? 0 : pl.rank * C::VH_COLS;
    const int dD = kv == 0 ? D : C::VH_COLS;
    uint4 v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int u = dtid + i * kDq;
        const int row = u / upr, dl = (u - row * upr) * 8;
        const int srow = s_base + row_base + row;
        v[i] = make_uint4(0, 0, 0, 0);
        if (srow < p.suffix_rows) v[i] = __ldg((const uint4 *)(src + tile_elem_off(srow, col_base + dl, D, C::W)));
    }
    bool bad = false;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int u = dtid + i * kDq;
        const int row = u / upr, dl = (u - row * upr) * 8;
        const uint4 w = make_uint4(bf16x2_to_f16x2(v[i].x), bf16x2_to_f16x2(v[i].y), bf16x2_to_f16x2(v[i].z),
                                   bf16x2_to_f16x2(v[i].w));
        bad |= f16x8_has_inf(w);
        *(uint4 *)(sDst + tile_elem_off(row, dl, dD, C::W)) = w;
    }
    if (bad) report_error(p.status, DEV_ERR_F16_RANGE, 2, pl.b, j);
}

__device__ __forceinline__ void pair_fail(const AttnArgs &a, volatile int *abort, int where) {
    *abort = 1;
    report_error(a.pool.status, DEV_ERR_TIMEOUT, where, blockIdx.x, blockIdx.z);
}

__device__ __forceinline__ bool pair_xsync(uint32_t xbar, int use, volatile int *abort, long long budget) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(xbar);
    return mbar_wait(xbar, (uint32_t)use & 1u, abort, budget);
}

// ---- softmax / epilogue of one CTA (warps 0-7): warp w owns query row (w & 3) * 32 + lane and
// S columns [h * 32, h * 32 + 32), h = w >> 2; the two warps of a lane quarter swap chunk maxima
// per tile. P(j) goes back as 16-bit pairs over the tile's S buffer; "P(j) written" is one arrival
// per warp on rank 0's barrier. ----
template <bool Q8>
__device__ __forceinline__ void pair_softmax(const AttnArgs &a, const PairPlan &pl, uint8_t *smem, uint32_t bar0,
                                             uint32_t pvk0, volatile int *abort, uint32_t tmem, int n, int n_qtiles,
                                             const void *omap, int omode) {
    using C = PairCfg<Q8>;
    constexpr int BN = C::BN, D = C::D, DH = D / 2, NS = C::NSTAGE;
    auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int h = warp >> 2, quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = ((uint32_t)(quarter * 32)) << 16;
    const bool row_ok = r < pl.rows_valid;
    const int t = (pl.qrow0 + r) / a.group;
    const MaskDesc m = mask_desc(a, pl.b);
    const bool prefix_simple = !(a.mask_flags & (EKV_MASK_SPAN_ONLY | EKV_MASK_SPAN_EXCLUDE | EKV_MASK_BLOCK_CAUSAL | kVisWordFlags));
    const bool suffix_simple = !(a.mask_flags & (EKV_MASK_SUFFIX_CAUSAL | EKV_MASK_SUFFIX_PREFIX_LM | kVisWordFlags));
    float *xmax = (float *)(smem + C::OFF_XCH);  // [2 parity][2 half][128 rows]
    float *xl = xmax + 4 * kBM;                   // [2 half][128 rows]
    const uint32_t xbar = bar(PB_XCH + quarter);
    int uses = 0;
    float m_used = -INFINITY, l = 0.0f;
    const float inv_scale_log2 = 1.0f / a.scale_log2;
    bool ok = true;
    for (int jj = 0; jj < n; ++jj) {
        const int sb = jj & 1;
        const int j = pl.j0 + jj;
        if (!(ok = mbar_wait(bar(PB_K_EMPTY + jj % NS), stage_parity(jj, NS), abort, a.wait_budget))) break;
        tc_fence_after();
        if (r == 0 && h == 0 && jj < 50) TRACE(300 + jj);
        const bool suffix = j >= pl.np_tiles;
        const int key0 = (suffix ? (j - pl.np_tiles) * BN : pl.kbeg + j * BN) + h * 32;
        const bool all_vis = suffix ? (suffix_simple && key0 + 32 <= a.suffix_len)
                                    : (prefix_simple && key0 + 32 <= pl.sk.prefix_valid);
        const uint32_t vb = all_vis ? 0xffffffffu
                                    : (row_ok ? vis_word(m, suffix, key0, t, pl.sk.prefix_valid, pl.sk.span_b,
                                                         pl.sk.span_e, a.suffix_len, pl.sk.n_prefix)
                                              : 0u);
        const uint32_t s_buf = tmem + lane_base + C::S_COL + (uint32_t)(sb * BN);
        uint32_t rr[32];
        tmem_load32(s_buf + h * 32, rr);
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        if (all_vis) {
#pragma unroll
            for (int i = 0; i < 32; ++i) mx[i & 3] = fmaxf(mx[i & 3], __uint_as_float(rr[i]));
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) mx[i & 3] = fmaxf(mx[i & 3], ((vb >> i) & 1u) ? __uint_as_float(rr[i]) : -INFINITY);
        }
        const float cm = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
        xmax[((jj & 1) * 2 + h) * kBM + r] = cm;
        if (!(ok = pair_xsync(xbar, uses++, abort, a.wait_budget))) break;
        const float rmax = fmaxf(cm, xmax[((jj & 1) * 2 + (h ^ 1)) * kBM + r]);
        if (__any_sync(0xffffffffu, rmax > (m_used + 8.0f) * inv_scale_log2)) {
            const float m_tile = rmax * a.scale_log2;
            float alpha = 1.0f;
            bool rescale = false;
            if (m_tile > m_used) {
                if (m_used == -INFINITY) {
                    m_used = m_tile;
                } else if (m_tile > m_used + 8.0f) {
                    alpha = ex2(m_used - m_tile);
                    m_used = m_tile;
                    l *= alpha;
                    rescale = true;
                }
            }
            if (__any_sync(0xffffffffu, rescale)) {
                if (!(ok = mbar_wait(bar(PB_V_EMPTY + (jj - 1) % NS), stage_parity(jj - 1, NS), abort,
                                             a.wait_budget)))
                    break;
                tc_fence_after();
#pragma unroll 1
                for (int c0 = h * DH; c0 < (h + 1) * DH; c0 += 16) {
                    uint32_t o16[16];
                    tmem_load16(tmem + lane_base + (uint32_t)(C::O_COL + c0), o16);
#pragma unroll
                    for (int i = 0; i < 16; ++i) o16[i] = __float_as_uint(__uint_as_float(o16[i]) * alpha);
                    tmem_st16(tmem + lane_base + (uint32_t)(C::O_COL + c0), o16);
                }
                tmem_wait_st();
            }
        }
        const float neg_m = -m_used;
        const uint32_t pv_bits = (m_used != -INFINITY) ? vb : 0u;
        float ps[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        uint32_t pw[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            float pr[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int c = 2 * i + e;
                const float x = ex2(fmaf(__uint_as_float(rr[c]), a.scale_log2, neg_m));
                pr[e] = ((pv_bits >> c) & 1u) ? x : 0.0f;
                ps[c & 3] += pr[e];
            }
            if (Q8) {
                const __half2 h2 = __floats2half2_rn(pr[0], pr[1]);
                pw[i] = *(const uint32_t *)&h2;
            } else {
                const __nv_bfloat162 b2 = __floats2bfloat162_rn(pr[0], pr[1]);
                pw[i] = *(const uint32_t *)&b2;
            }
        }
        tmem_st16(s_buf + h * 16, pw);
        l += (ps[0] + ps[1]) + (ps[2] + ps[3]);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(pvk0 + 8u * (uint32_t)(jj % NS));
        if (lane == 0 && jj == 7) TRACE(1016 + warp);
        if (r == 0 && h == 0 && jj < 50) TRACE(350 + jj);
    }
    if (!ok) pair_fail(a, abort, 3);
    if (ok && n > 0) {
        ok = mbar_wait(bar(PB_V_EMPTY + (n - 1) % NS), stage_parity(n - 1, NS), abort, a.wait_budget);
        if (!ok) pair_fail(a, abort, 4);
        tc_fence_after();
    }
    // ---- epilogue: row sum over both halves, then this warp's D/2 columns of O ----
    if (r == 0 && h == 0) TRACE(10);
    xl[h * kBM + r] = l;
    if (ok && !pair_xsync(xbar, uses++, abort, a.wait_budget)) {
        ok = false;
        pair_fail(a, abort, 7);
    }
    if (r == 0 && h == 0) TRACE(13);
    const float l_row = ok ? xl[r] + xl[kBM + r] : 0.0f;
    const bool have_o = ok && n > 0;
    // O -> shared staging row r -> the softmax warps write whole rows with consecutive 16-byte lanes
    // (the K/V stages are idle once the last P.V has landed). Without key splits: O / l as bf16 or
    // f32 into `out`; with splits: the unnormalised f32 row into the workspace (a unit's 128 rows
    // are contiguous there), plus the row's running max and sum.
    const bool split = a.n_splits > 1;
    const float inv = split ? 1.0f : ((have_o && l_row > 0.0f) ? 1.0f / l_row : 0.0f);
    const bool f32 = split || a.out_dtype == EKV_DTYPE_F32;
    int64_t unit = 0;
    if (split) {
        unit = (((int64_t)pl.b * a.pool.kv_heads + pl.g) * n_qtiles + (pl.pair * 2 + pl.rank)) * a.n_splits + pl.split;
        if (row_ok && h == 0) {
            float *wml = a.ws_ml + (unit * kBM + r) * 2;
            wml[0] = have_o ? m_used : -INFINITY;
            wml[1] = have_o ? l_row : 0.0f;
        }
    }
    if (omode != OUT_THREADS) {
        // this warp's columns of its lane quarter -> swizzled boxes -> copy engine
        if (r == 0 && h == 0) TRACE(14);
        epilogue_o_tma(a, pl.qrow0, pl.rows_valid, pl.g, pl.b, omap, omode, smem, quarter, lane,
                       tmem + lane_base + (uint32_t)C::O_COL, h * DH, (h + 1) * DH, have_o, inv, f32, unit, 2 + h);
        if (r == 0 && h == 0) TRACE(15);
        return;
    }
    uint8_t *orow = smem + r * C::OSTR;
#pragma unroll 1
    for (int c0 = h * DH; c0 < (h + 1) * DH; c0 += 32) {
        uint32_t o32[32];
        if (have_o) {
            tmem_load32(tmem + lane_base + (uint32_t)(C::O_COL + c0), o32);
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) o32[i] = 0u;
        }
        if (f32) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
                *(float4 *)(orow + (c0 + i) * 4) =
                    make_float4(__uint_as_float(o32[i]) * inv, __uint_as_float(o32[i + 1]) * inv,
                                __uint_as_float(o32[i + 2]) * inv, __uint_as_float(o32[i + 3]) * inv);
        } else {
#pragma unroll
            for (int i0 = 0; i0 < 32; i0 += 8) {
                uint32_t w[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const __nv_bfloat162 b2 = __floats2bfloat162_rn(__uint_as_float(o32[i0 + 2 * i]) * inv,
                                                                    __uint_as_float(o32[i0 + 2 * i + 1]) * inv);
                    w[i] = *(const uint32_t *)&b2;
                }
                *(uint4 *)(orow + (c0 + i0) * 2) = make_uint4(w[0], w[1], w[2], w[3]);
            }
        }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(C::SMW * 32) : "memory");  // the softmax warps only
    const int row_bytes = D * (f32 ? 4 : 2);
    for (int rw = warp; rw < pl.rows_valid; rw += C::SMW) {
        uint8_t *dst;
        if (split) {
            dst = (uint8_t *)(a.ws_o + (unit * kBM + rw) * D);
        } else {
            const int qrw = pl.qrow0 + rw;
            const int tw = qrw / a.group;
            const int hw = pl.g * a.group + (qrw - tw * a.group);
            dst = (uint8_t *)a.out + ((((int64_t)pl.b * a.q_tokens + tw) * a.q_heads + hw) * D) * (f32 ? 4 : 2);
        }
        const uint8_t *srow = smem + rw * C::OSTR;
        for (int o = lane * 16; o < row_bytes; o += 32 * 16) *(uint4 *)(dst + o) = *(const uint4 *)(srow + o);
    }
}

template <bool Q8>
__global__ void __launch_bounds__(PairCfg<Q8>::THREADS, 1)
    attn_pair_kernel(const AttnArgs a, int n_qtiles, const __grid_constant__ CUtensorMap omap, int omode) {
    using C = PairCfg<Q8>;
    constexpr int BN = C::BN, D = C::D, NS = C::NSTAGE;
    extern __shared__ uint8_t smem_raw[];
    // identical offsets in both CTAs: dynamic shared memory starts at the same window address
    uint8_t *smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    uint8_t *sK = smem + C::OFF_K;
    uint8_t *sV = smem + C::OFF_V;
    uint8_t *sRaw = smem + C::OFF_RAW;
    uint64_t *bars = (uint64_t *)(smem + C::OFF_BAR);
    uint32_t *tmem_holder = (uint32_t *)(bars + PB_N);
    volatile int *abort = (volatile int *)(bars + PB_N + 1);
    const uint8_t **sPtr = (const uint8_t **)(smem + C::OFF_TBL);
    const uint32_t bar0 = smem_addr(bars);
    auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (threadIdx.x == 0) {
        trace_init();
        TRACE(0);
        TRACE_CLK(20);
    }
    const PairPlan pl = make_pair_plan(a);
    if (threadIdx.x == 0) TRACE(1);
    const uint32_t bar0_rank0 = mapa_shared(bar0, 0);  // rank 0's barrier block (cluster window)
    if (threadIdx.x == 0 && !pl.sk.ok) report_error(a.pool.status, DEV_ERR_BAD_SEQ, pl.b, a.seq_ids[pl.b], 3);

    if (threadIdx.x == 0) {
        // producers per CTA: the dequant warps (Q8_0) or the feeder's byte-counted arrival (bf16);
        // rank 0's barriers also count rank 1's
        const uint32_t per_rank = Q8 ? kDq / 32 : 1;
        for (int s = 0; s < 2; ++s) mbar_init(bar(PB_KINIT + s), 2 * per_rank);
        for (int s = 0; s < NS; ++s) {
            mbar_init(bar(PB_K_FULL + s), 1);
            mbar_init(bar(PB_V_FULL + s), 1);
            mbar_init(bar(PB_PVK + s), 4 * per_rank + 2 * C::SMW);
            mbar_init(bar(PB_K_EMPTY + s), 1);
            mbar_init(bar(PB_V_EMPTY + s), 1);
        }
        for (int s = 0; s < 3; ++s) {
            mbar_init(bar(PB_RAW_FULL + s), 2);
            mbar_init(bar(PB_RAW_EMPTY + s), kDq / 32);
        }
        mbar_init(bar(PB_DONE), 1);
        mbar_init(bar(PB_STALL), 1);
        for (int q = 0; q < 4; ++q) mbar_init(bar(PB_XCH + q), 2);
        *abort = 0;
        mbar_init_fence();
    }
    if (warp == C::MMA_WARP) tmem_alloc_pair(smem_addr(tmem_holder), C::TMEM_COLS);
    // Q rows of this CTA -> shared staging (all threads, every load before the first store)
    {
        constexpr int UPR = D / 8, UNITS = kBM * UPR, IT = (UNITS + C::THREADS - 1) / C::THREADS;
        uint4 qv[IT];
#pragma unroll
        for (int i = 0; i < IT; ++i) {
            const int u = threadIdx.x + i * C::THREADS;
            const int rq = u / UPR;
            qv[i] = make_uint4(0, 0, 0, 0);
            if (u < UNITS && rq < pl.rows_valid) {
                const int qr = pl.qrow0 + rq, tq = qr / a.group, hq = pl.g * a.group + (qr - tq * a.group);
                qv[i] = __ldg((const uint4 *)(a.q + (((int64_t)pl.b * a.q_tokens + tq) * a.q_heads + hq) * D +
                                              (u - rq * UPR) * 8));
            }
        }
        if (pl.tbl_n <= C::TBL)
            for (int i = threadIdx.x; i < pl.tbl_n; i += C::THREADS) {
                const int blk = lookup_block(a.pool, pl.sk.seq, pl.tbl_lo + i);
                sPtr[i] = blk < 0 ? nullptr
                                  : a.pool.prefix + prefix_tile_index(a.pool, a.layer, blk, 0, pl.g) * a.pool.tile_bytes;
            }
#pragma unroll
        for (int i = 0; i < IT; ++i) {
            const int u = threadIdx.x + i * C::THREADS;
            if (u < UNITS) {
                const int rq = u / UPR;
                *(uint4 *)(smem + rq * C::QSTR + (u - rq * UPR) * 16) = qv[i];
            }
        }
    }
    if (threadIdx.x == 0) TRACE(2);
    tc_fence_before();
    __syncthreads();
    cluster_sync_relaxed();  // both CTAs' barriers initialised (fenced above) and tensor memory allocated
    tc_fence_after();
    if (threadIdx.x == 0) TRACE(5);
    const uint32_t tmem = *tmem_holder;
    if (warp < C::SMW) {
        // row (warp & 3) * 32 + lane; the two warps of a lane quarter take 8 of the 16 column blocks each
        const int rq = (warp & 3) * 32 + lane, hq = warp >> 2;
        const uint32_t taddr = tmem + (((uint32_t)((warp & 3) * 32)) << 16) + C::Q_COL;
        bool q_bad = false;
#pragma unroll 1
        for (int c = hq * 8; c < hq * 8 + 8; ++c) {
            const uint4 a0 = *(const uint4 *)(smem + rq * C::QSTR + c * 32);
            const uint4 a1 = *(const uint4 *)(smem + rq * C::QSTR + c * 32 + 16);
            uint32_t w[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            if (Q8) {
#pragma unroll
                for (int i = 0; i < 8; ++i) w[i] = bf16x2_to_f16x2(w[i]);
                q_bad |= f16x8_has_inf(make_uint4(w[0], w[1], w[2], w[3])) | f16x8_has_inf(make_uint4(w[4], w[5], w[6], w[7]));
            }
            tmem_st8(taddr + (uint32_t)(c * 8), w);
        }
        if (q_bad) report_error(a.pool.status, DEV_ERR_F16_RANGE, 0, pl.b, pl.qrow0);
        tmem_wait_st();
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 0) TRACE(3);
    const int n = pl.j1 - pl.j0;

    if (warp == C::MMA_WARP) {
        if (pl.rank == 0) {
            // ---- MMA issue for the pair, fixed order S(0), [S(j+1), P.V(j)]; one thread ----
            if (n > 0 && lane == 0) {
                const uint32_t idS = idesc_f16_m(!Q8, false, BN, 256);
                const uint32_t idO = idesc_f16_m(!Q8, true, D, 256);
                const uint32_t k_addr = smem_addr(sK), v_addr = smem_addr(sV);
                auto issue_s = [&](int jj) {  // K(jj) is known to be in place
                    const int st = jj % NS, sb = jj & 1;
                    if (jj < 50) TRACE(850 + jj);
                    const uint32_t d_tmem = tmem + C::S_COL + (uint32_t)(sb * BN);
                    const uint64_t bd0 = sdesc(k_addr + st * C::KH_BYTES, 16, C::K_SBO, C::LAYOUT);
                    // K step kk: A columns Q_COL + 8kk; B = 32-byte step kk % 4 of swizzle chunk kk / 4
                    uint32_t av[D / 16];
                    uint64_t bv[D / 16];
#pragma unroll
                    for (int kk = 0; kk < D / 16; ++kk) {
                        av[kk] = tmem + C::Q_COL + (uint32_t)(kk * 8);
                        bv[kk] = bd0 + (((uint32_t)(kk / 4) * (8 * C::W) + (uint32_t)(kk % 4) * 32u) >> 4);
                    }
#pragma unroll
                    for (int g = 0; g < D / 64; ++g)
                        mma_ts_x4<true>(d_tmem, *reinterpret_cast<const uint32_t(*)[4]>(av + 4 * g),
                                        *reinterpret_cast<const uint64_t(*)[4]>(bv + 4 * g), idS, g > 0 ? 1u : 0u);
                    mma_commit_both(bar(PB_K_EMPTY + st));
                    if (jj < 50) TRACE(200 + jj);
                };
                auto issue_pv = [&](int jj) {
                    const int st = jj % NS, sb = jj & 1;
                    if (!mbar_wait(bar(PB_PVK + st), stage_parity(jj, NS), abort, a.wait_budget)) return false;
                    tc_fence_after();
                    if (jj < 50) TRACE(900 + jj);
                    const uint64_t bd0 = sdesc(v_addr + st * C::VH_BYTES, C::V_LBO, C::V_SBO, C::LAYOUT);
                    static_assert(BN == 64, "one group of four P.V steps");
                    uint32_t av[4];
                    uint64_t bv[4];
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        av[kk] = tmem + C::S_COL + (uint32_t)(sb * BN + kk * 8);
                        bv[kk] = bd0 + ((uint32_t)kk * 2u * C::V_SBO >> 4);
                    }
                    mma_ts_x4<true>(tmem + C::O_COL, av, bv, idO, jj > 0 ? 1u : 0u);
                    mma_commit_both(bar(PB_V_EMPTY + st));
                    if (jj < 50) TRACE(250 + jj);
                    return true;
                };
                // S(0), S(1), then P.V(j) and S(j + 2) for each j: one wait per tile
                bool ok = true;
                // test hook (ekv_debug_expire_wait): a wait on a barrier nothing arrives on
                if (a.debug_stall) ok = mbar_wait(bar(PB_STALL), 0, abort, a.wait_budget);
                for (int jj = 0; ok && jj < 2 && jj < n; ++jj) {
                    ok = mbar_wait(bar(PB_KINIT + jj), 0, abort, a.wait_budget);
                    tc_fence_after();
                    if (ok) issue_s(jj);
                }
                for (int jj = 0; ok && jj < n; ++jj) {
                    ok = issue_pv(jj);
                    if (ok && jj + 2 < n) issue_s(jj + 2);
                }
                if (!ok) pair_fail(a, abort, 1);
                mma_commit_pair(bar(PB_DONE));
                mbar_wait_drain(bar(PB_DONE), 0, a.wait_budget);
            }
        }
        __syncwarp();
    } else if (warp == C::TMA_WARP || warp == C::TMA_WARP + 1) {
        // copy-engine feeders, one warp for K and one for V (a bulk-copy issue stalls its warp)
        const int kv = warp - C::TMA_WARP;
        if constexpr (Q8) {
            // warp TMA_WARP: this CTA's rows (K and V); TMA_WARP + 1: the peer's rows (V)
            constexpr int NR = C::NRAW;
            const int np = min(n, max(0, pl.np_tiles - pl.j0));  // suffix tiles are converted by the dequant warps
            int issued = 0;
            for (int it = 0; it < np; ++it) {
                const int r = it % NR;
                if (it >= NR && !mbar_wait(bar(PB_RAW_EMPTY + r), stage_parity(it - NR, NR), abort, a.wait_budget)) {
                    pair_fail(a, abort, 2);
                    break;
                }
                if (lane == 0 && it < 50) TRACE((kv ? 150 : 450) + it);
                pair_produce_q8_raw(a, pl, (const uint8_t *const *)sPtr, pl.j0 + it, 1 - kv, sRaw + r * C::RAW_BYTES,
                                    bar(PB_RAW_FULL + r), lane);
                issued = it + 1;
            }
            if (lane == 0 && *abort)
                for (int jj = max(0, issued - NR); jj < issued; ++jj)
                    mbar_wait_drain(bar(PB_RAW_FULL + jj % NR), stage_parity(jj, NR), a.wait_budget);
        } else {
            uint8_t *stages = kv ? sV : sK;
            const int sbytes = kv ? C::VH_BYTES : C::KH_BYTES;
            const int b_full = kv ? PB_V_FULL : PB_K_FULL, b_empty = kv ? PB_V_EMPTY : PB_K_EMPTY;
            int issued = 0;
            for (int it = 0; it < n; ++it) {
                const int st = it % NS;
                if (it >= NS && !mbar_wait(bar(b_empty + st), stage_parity(it - NS, NS), abort, a.wait_budget)) {
                    pair_fail(a, abort, 2);
                    break;
                }
                if (lane == 0 && it < 50) TRACE((kv ? 150 : 450) + it);
                pair_produce_bf16(a, pl, (const uint8_t *const *)sPtr, pl.j0 + it, kv, stages + st * sbytes,
                                  bar(b_full + st), lane);
                issued = it + 1;
            }
            if (lane == 0 && *abort)
                for (int jj = max(0, issued - NS); jj < issued; ++jj)
                    mbar_wait_drain(bar(b_full + jj % NS), stage_parity(jj, NS), a.wait_budget);
        }
    } else if (!Q8 && warp == C::RELAY_WARP) {
        // ---- bf16: forward "this CTA's K/V half landed" to rank 0, in the order its MMAs use
        // them: K(0), K(1), then V(j) and K(j + 2) per tile ----
        if (n > 0 && lane == 0) {
            auto relay = [&](uint32_t local, uint32_t parity, int remote) {
                if (!mbar_wait(local, parity, abort, a.wait_budget)) return false;
                mbar_arrive_remote(bar0_rank0 + 8u * (uint32_t)remote);
                return true;
            };
            bool ok = relay(bar(PB_K_FULL), 0u, PB_KINIT);
            if (ok && n > 1) ok = relay(bar(PB_K_FULL + 1), 0u, PB_KINIT + 1);
            for (int jj = 0; ok && jj < n; ++jj) {
                ok = relay(bar(PB_V_FULL + jj % NS), stage_parity(jj, NS), PB_PVK + jj % NS);
                const int t = jj + 2;  // K(t) arrives with P.V(jj); past the end, with no data
                if (ok && t < n) ok = relay(bar(PB_K_FULL + t % NS), stage_parity(t, NS), pair_k_bar(t, NS));
                else if (ok) mbar_arrive_remote(bar0_rank0 + 8u * (uint32_t)pair_k_bar(t, NS));
            }
            if (!ok) pair_fail(a, abort, 8);
        }
    } else if (warp >= C::DQ_WARP0) {
        if constexpr (Q8) {
            const int dtid = threadIdx.x - C::DQ_WARP0 * 32;
            const int bt = a.pool.block_tokens;  // a power of two (checked by the launcher)
            const int seg_shift = 31 - __clz(min(bt, C::KH_ROWS));
            for (int jj = 0; jj < n; ++jj) {
                const int j = pl.j0 + jj, st = jj % NS;
                const bool prefix = j < pl.np_tiles;
                if (dtid == 0 && jj < 50) TRACE(500 + jj);
                const int rs = jj % C::NRAW;
                const uint8_t *raw = sRaw + rs * C::RAW_BYTES;
                uint8_t *kdst = sK + st * C::KH_BYTES, *vdst = sV + st * C::VH_BYTES;
                // both operand stages free (S(j - NS) and P.V(j - NS) done), raw landed
                bool ok = jj < NS || (mbar_wait(bar(PB_K_EMPTY + st), stage_parity(jj - NS, NS), abort, a.wait_budget) &&
                                      mbar_wait(bar(PB_V_EMPTY + st), stage_parity(jj - NS, NS), abort, a.wait_budget));
                if (ok && prefix) ok = mbar_wait(bar(PB_RAW_FULL + rs), stage_parity(jj, C::NRAW), abort, a.wait_budget);
                if (!ok) {
                    pair_fail(a, abort, 6);
                    break;
                }
                if (dtid == 0 && jj < 50) TRACE(550 + jj);
                auto publish = [&](int kv) {
                    fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) {
                        if (prefix && kv == 1) mbar_arrive(bar(PB_RAW_EMPTY + rs));
                        // both ranks: rank 0's barrier of the MMA group that uses this half
                        mbar_arrive_remote(bar0_rank0 + 8u * (uint32_t)(kv ? PB_PVK + st : pair_k_bar(jj, NS)));
                    }
                };
                if (prefix) {
                    // every raw load of both parts in flight before the first conversion
                    const PairDqUnits uk = pair_dq_load(raw, 0, pl.rank, seg_shift, dtid);
                    const PairDqUnits uv = pair_dq_load(raw, 1, pl.rank, seg_shift, dtid);
                    pair_dq_store(uk, 0, kdst, dtid);
                    publish(0);
                    if (dtid == 0 && jj < 50) TRACE(800 + jj);
                    if (lane == 0 && jj == 7) TRACE(1000 + (dtid >> 5));
                    pair_dq_store(uv, 1, vdst, dtid);
                    publish(1);
                    if (lane == 0 && jj == 7) TRACE(1008 + (dtid >> 5));
                } else {
                    pair_convert_suffix(a, pl, j, 0, kdst, dtid);
                    publish(0);
                    pair_convert_suffix(a, pl, j, 1, vdst, dtid);
                    publish(1);
                }
                if (dtid == 0 && jj < 50) TRACE(100 + jj);
            }
            // K of the (up to two) tiles past the end still arrives, so the last PVK phases complete
            if (lane == 0 && !*abort)
                for (int t = max(n, 2); t < n + 2; ++t) mbar_arrive_remote(bar0_rank0 + 8u * (uint32_t)pair_k_bar(t, NS));
        }
    } else {
        pair_softmax<Q8>(a, pl, smem, bar0, bar0_rank0 + 8u * PB_PVK, abort, tmem, n, n_qtiles, &omap, omode);
    }
    if (threadIdx.x == 0) {
        TRACE(11);
        TRACE_CLK(21);
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    cluster_sync_relaxed();  // rank 0's MMAs are finished; neither CTA releases memory the other still uses
    tc_fence_after();
    if (warp == C::MMA_WARP) tmem_dealloc_pair(tmem, C::TMEM_COLS);
    if (threadIdx.x == 0) TRACE(12);
    __syncthreads();
    trace_flush();
}

}  // namespace

#ifdef EKV_TRACE
int pair_debug_set_trace(unsigned long long *buf) {
    return cudaMemcpyToSymbol(c_trace, &buf, sizeof(buf)) == cudaSuccess ? 0 : -2;
}
#endif

// Split count for `pair_units` CTA pairs on `sms` SMs (two per pair).
int pair_choose_splits(int64_t pair_units, int max_tiles, int sms) {
    return choose_split_count(pair_units, max_tiles, sms / 2);
}

// One launch of the pair kernel (plus the merge when keys are split), head_dim 256.
int launch_attention_pair(AttnArgs a, cudaStream_t s, size_t ws_bytes, int sms) {
    const bool q8 = a.pool.dtype == EKV_DTYPE_Q8_0;
    if (take_debug_stall()) {
        a.debug_stall = 1;
        a.wait_budget = kDebugWaitBudget;
    }
    const int smem_bytes = q8 ? PairCfg<true>::SMEM : PairCfg<false>::SMEM;
    const int threads = q8 ? PairCfg<true>::THREADS : PairCfg<false>::THREADS;
    static int attr_done[64][2] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr_done[dev][q8]) {
        const cudaError_t e =
            q8 ? cudaFuncSetAttribute(attn_pair_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes)
               : cudaFuncSetAttribute(attn_pair_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
        if (e != cudaSuccess) return EKV_ERR_CUDA;
        attr_done[dev][q8] = 1;
    }
    const int bt = a.pool.block_tokens;
    if (64 % bt != 0 && bt % 64 != 0) return EKV_ERR_UNSUPPORTED;
    const int rows = a.q_tokens * a.group;
    const int n_pairs = (rows + 2 * kBM - 1) / (2 * kBM);
    const int n_qtiles = 2 * n_pairs;  // 128-row tiles, as the merge kernel indexes them
    const int64_t units = (int64_t)a.n_batch * a.pool.kv_heads * n_pairs;
    if (a.n_splits == 0) {
        const int max_prefix = a.pool.max_blocks_per_seq * a.pool.block_tokens;
        const int max_tiles = (max_prefix + 63) / 64 + (a.suffix_len + 63) / 64;
        int sp = pair_choose_splits(units, max_tiles, sms);
        const size_t per_split = (size_t)a.n_batch * a.pool.kv_heads * n_qtiles * kBM * (256 + 2) * sizeof(float);
        while (sp > 1 && per_split * sp > ws_bytes) --sp;
        a.n_splits = sp;
        a.ws_ml = a.ws_o + (size_t)a.n_batch * a.pool.kv_heads * n_qtiles * sp * kBM * 256;
    }
    if (a.n_splits < 1) a.n_splits = 1;
    if ((int64_t)2 * n_pairs * a.n_splits > 0x7fffffff || a.pool.kv_heads > 65535 || a.n_batch > 65535)
        return EKV_ERR_INVALID_ARG;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(2 * n_pairs * a.n_splits), (unsigned)a.pool.kv_heads, (unsigned)a.n_batch);
    cfg.blockDim = dim3((unsigned)threads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)smem_bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CUtensorMap omap;
    const int omode = make_out_map(a, 256, (int64_t)a.n_batch * a.pool.kv_heads * n_qtiles, &omap);
    const cudaError_t e = q8 ? cudaLaunchKernelEx(&cfg, attn_pair_kernel<true>, a, n_qtiles, omap, omode)
                             : cudaLaunchKernelEx(&cfg, attn_pair_kernel<false>, a, n_qtiles, omap, omode);
    if (e != cudaSuccess) return EKV_ERR_CUDA;
    note_launches(1);
    if (a.n_splits > 1) return launch_merge_splits(a, n_qtiles, s);
    return EKV_OK;
}

}  // namespace ekv
