// ekv_attn_pair128.cu -- masked attention over the paged KV pool on CTA pairs with 128-key tiles,
// head_dim 256 (the pi0.5 action expert: 8 query heads over 1 KV head, models/pi05.cpp:406-421).
//
// A cluster of two CTAs (ranks 0, 1) takes 256 query rows of one (request, KV head), rank r owning
// rows [256p + 128r, +128); rank 0 issues every MMA for both with tcgen05 cta_group::2, M = 256:
//
//   S = Q K^T   N = 128 keys, K = 256: A = Q (this CTA's 128 rows, shared memory), B = K rows
//               [64r, 64r + 64) of the tile in each CTA's shared memory
//   O += P V    N = 256, K = 128 keys: A = P (tensor memory), B = V columns [128r, 128r + 128)
//
// Tensor memory (512 columns per CTA): two S buffers of 128 f32 columns (P is written back as
// 16-bit pairs over the first 64 columns of its own buffer) and O (256 f32 columns). Q lives in
// shared memory, loaded once by the copy engine through a 5-D tensor map of the caller's q (rows
// past the call's tokens read as zeros), so that S can be computed 128 keys per MMA (an N = 128
// MMA runs at the tensor pipe's full rate where N = 64 does not) with one barrier wait per 128
// keys in the MMA-issuing thread.
//
// Shared memory per CTA: Q 64 KB | K stages 2 x 32 KB | V stages 2 x 32 KB | barriers, exchange,
// block-pointer table. Q8_0 pools: eight dequantising warps read the int8 and fp16-scale planes
// of their half of each tile straight from the pool into registers one tile ahead
// (ld.global.nc, no staging copy), convert exactly to f16 (0x6480 magic, one f16 multiply by the
// scale) and store the swizzled operand; Q is converted to f16 in place once it has landed, and
// the MMAs run in f16 (11 mantissa bits of q * d). bf16 pools: two copy-engine feeder warps move
// whole pool blocks (pre-swizzled tiles) into the stages and the MMAs run in bf16. Accumulation
// is f32. Warps: 0-15 softmax and epilogue (four per TMEM lane quarter, 32 columns each), 16 MMA
// issue (rank 0) and TMEM allocation, 17 Q load and bf16 K feeder, 18 bf16 V feeder, 19 bf16
// relay of the copies' completion to rank 0, 20-27 Q8_0 dequantisation.
//
// Every wait is bounded; on expiry the CTA records DEV_ERR_TIMEOUT and unwinds through the closing
// cluster barrier after rank 0's MMAs have finished.
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
struct P2Cfg {
    static constexpr int D = 256, BN = 128;
    static constexpr uint32_t LAYOUT = 2u;             // 128-byte swizzle
    static constexpr int KROWS = BN / 2;               // K rows per CTA
    static constexpr int VCOLS = D / 2;                // V columns per CTA
    static constexpr int Q_BYTES = kBM * D * 2;        // 64 KB: 4 chunks of [128 rows][128 B]
    static constexpr int K_BYTES = KROWS * D * 2;      // 32 KB: [8 row groups][4 chunks][8][128 B]
    static constexpr int V_BYTES = BN * VCOLS * 2;     // 32 KB: [16 key groups][2 chunks][8][128 B]
    static constexpr uint32_t Q_CHUNK = kBM * 128;     // bytes per 64-column chunk of Q
    static constexpr uint32_t Q_SBO = 1024;            // 8-row atoms of the TMA-swizzled Q
    static constexpr uint32_t K_SBO = 4096, V_LBO = 1024, V_SBO = 2048;
    static constexpr int NS = 2;                       // K and V operand stages
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = OFF_Q + Q_BYTES;
    static constexpr int OFF_V = OFF_K + NS * K_BYTES;
    static constexpr int OFF_BAR = OFF_V + NS * V_BYTES;
    static constexpr int BAR_BYTES = 256;
    static constexpr int SMH = 4;                      // softmax warps per TMEM lane quarter
    static constexpr int OFF_XCH = OFF_BAR + BAR_BYTES;  // max exchange [2 parity][SMH][128] + sums [SMH][128]
    static constexpr int OFF_TBL = OFF_XCH + 3 * SMH * kBM * 4;
    // block-table cache of the split: tile pointers (8 B) and physical block ids (4 B)
    static constexpr int TBL_ROOM = (232448 - 1024 - OFF_TBL) / 12;
    static constexpr int TBL = TBL_ROOM > 512 ? 512 : TBL_ROOM;
    static constexpr int OFF_BLK = OFF_TBL + TBL * 8;
    static constexpr int SMEM = OFF_BLK + TBL * 4 + 1024;
    // Q8_0: the raw int8 / fp16-scale bytes of a tile land in the upper part of its own operand stage
    // (copy engine) and are converted in place: K -- this CTA's 64 rows as segments of
    // min(block, 64) rows, [qs rows x 256 B][scales rows x 16 B]; V -- this CTA's 128 columns of all
    // 128 rows as segments of min(block, 128) rows, [qs rows x 128 B][scales rows x 16 B]
    static constexpr int RAWK_BYTES = KROWS * (D + D / 16);
    static constexpr int RAWV_BYTES = BN * (VCOLS + D / 16);
    static constexpr int RAWK_OFF = K_BYTES - RAWK_BYTES;
    static constexpr int RAWV_OFF = V_BYTES - RAWV_BYTES;
    static_assert(RAWK_OFF >= 0 && RAWV_OFF >= 0 && RAWK_OFF % 16 == 0 && RAWV_OFF % 128 == 0, "raw staging");
    static constexpr int SMW = 4 * SMH;                // softmax warps
    static constexpr int MMA_WARP = SMW, KF_WARP = SMW + 1, VF_WARP = SMW + 2, RELAY_WARP = SMW + 3,
                         DQ_WARP0 = SMW + 4;
    static constexpr int NDQ = 256;                    // dequantising threads (Q8_0)
    static constexpr int THREADS = Q8 ? (DQ_WARP0 * 32 + NDQ) : (RELAY_WARP + 1) * 32;
    static constexpr int TMEM_COLS = 512;
    static constexpr int S_COL = 0, O_COL = 2 * BN;
    static_assert(O_COL + D == TMEM_COLS, "TMEM budget");
    static_assert(SMEM <= 232448, "shared-memory budget");
    static_assert(TBL >= 64, "block-table cache");
    static_assert((D / 32) * 4 * kOutBox <= OFF_BAR, "epilogue boxes (f32) fit below the barriers");
};

enum {
    P2_QFULL = 0,       // local: Q landed (copy engine)
    P2_KINIT = 1,       // [2] rank 0: Q of both CTAs (K(0) only) and K(0) / K(1) of both CTAs
    P2_SFULL = 3,       // [2] both CTAs: S(j) done -- S readable, K stage j % 2 free
    P2_PVDONE = 5,      // [2] both CTAs: P.V(j) done -- V stage j % 2 free, P(j) consumed, O updated
    P2_PVK = 7,         // [2] rank 0: V(j), P(j) and K(j + 2) of both CTAs
    P2_KFULL = 9,       // [2] local (bf16): this CTA's K half landed
    P2_VFULL = 11,      // [2] local (bf16): this CTA's V half landed
    P2_DONE = 13,       // rank 0: all MMAs finished
    P2_XCH = 14,        // [4] softmax row-maximum exchange, one per TMEM lane quarter
    P2_RAWK = 18,       // [2] local (Q8_0): raw K part of tile j landed in K stage j % 2
    P2_RAWV = 20,       // [2] local (Q8_0): raw V part of tile j landed in V stage j % 2
    P2_TEAM = 22,       // [2] local (Q8_0): the K (V) dequantising team has read the raw part
    P2_N = 24
};
static_assert(P2_N * 8 + 16 <= 256, "barrier block");

// Barrier of rank 0 that the producers of K(t) arrive on: K(0), K(1) on KINIT, later tiles on the
// barrier of the P.V two tiles earlier, so that the MMA thread waits once per tile. A tile past the
// end still arrives there (no data), so every phase completes.
__device__ __forceinline__ int p2_k_bar(int t) { return t < 2 ? P2_KINIT + t : P2_PVK + (t & 1); }
__device__ __forceinline__ uint32_t par2(int j) { return (uint32_t)(j >> 1) & 1u; }

// Key-tile schedule of one CTA (both CTAs of a pair derive the same key range).
struct P2Plan {
    int b, g, pair, split, rank;
    int qrow0, rows_valid;
    SeqKeys sk;
    int kbeg, np_tiles, ns_tiles, j0, j1, tbl_lo, tbl_n;
};

__device__ __forceinline__ P2Plan make_p2_plan(const AttnArgs &a) {
    constexpr int BN = 128;
    P2Plan pl;
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
__device__ __forceinline__ const uint8_t *p2_ptr_of(const AttnArgs &a, const P2Plan &pl, const uint8_t *const *sPtr,
                                                    int idx) {
    const int i = idx - pl.tbl_lo;
    if (pl.tbl_n <= TBL && i >= 0 && i < pl.tbl_n) return sPtr[i];
    const int blk = lookup_block(a.pool, pl.sk.seq, idx);
    return blk < 0 ? nullptr : a.pool.prefix + prefix_tile_index(a.pool, a.layer, blk, 0, pl.g) * a.pool.tile_bytes;
}

__device__ __forceinline__ void p2_fail(const AttnArgs &a, volatile int *abort, int where) {
    *abort = 1;
    report_error(a.pool.status, DEV_ERR_TIMEOUT, where, blockIdx.x, blockIdx.z);
}

// ---- suffix tile j (keys [128 (j - np_tiles), +128) of the suffix) -> this CTA's K half (rows
// [64r, 64r + 64), kv = 0) or V half (columns [128r, 128r + 128) of all 128 rows, kv = 1) of an
// operand stage, from the caller's row-major bf16 buffers (a.k_sfx / a.v_sfx: [n_batch][suffix_len]
// [kv_heads][256]) or the pool's suffix slot; rows past suffix_len are zero. `nthr` threads (tid <
// nthr) share the 2048 16-byte units; TO_F16 converts to the f16 operands of Q8_0 pools. ----
template <bool TO_F16>
__device__ __forceinline__ void p2_suffix_stage(const AttnArgs &a, const P2Plan &pl, int j, int kv, uint8_t *sDst,
                                                int tid, int nthr, volatile int *abort) {
    constexpr int BN = 128, D = 256, KROWS = 64, VCOLS = 128, W = 128;
    const PoolView &p = a.pool;
    const int s_base = (j - pl.np_tiles) * BN;
    const int upr = kv == 0 ? D / 8 : VCOLS / 8;  // 16-byte units per stage row: 32 (K) or 16 (V)
    const int row_base = kv == 0 ? pl.rank * KROWS : 0;
    const int col_base = kv == 0 ? 0 : pl.rank * VCOLS;
    const int dD = kv == 0 ? D : VCOLS;
    const bool direct = a.k_sfx != nullptr;
    const int64_t row_stride = (int64_t)p.kv_heads * D;
    const uint16_t *src = direct ? (kv ? a.v_sfx : a.k_sfx) + ((int64_t)pl.b * a.suffix_len * p.kv_heads + pl.g) * D
                                 : nullptr;
    const uint8_t *slot = direct ? nullptr
                                 : p.suffix + suffix_tile_index(p, a.layer, pl.sk.seq, kv, pl.g) * p.suffix_tile_bytes;
    constexpr int UNITS = 2048;  // 64 rows x 32 units (K) = 128 rows x 16 units (V)
    bool bad = false;
#pragma unroll 1
    for (int u0 = tid; u0 < UNITS; u0 += 4 * nthr) {
        uint4 v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int u = u0 + i * nthr;
            const int row = u / upr, dl = (u - row * upr) * 8;
            const int srow = s_base + row_base + row;
            v[i] = make_uint4(0, 0, 0, 0);
            if (u < UNITS && srow < a.suffix_len) {
                if (direct) v[i] = __ldg((const uint4 *)(src + srow * row_stride + col_base + dl));
                else v[i] = __ldg((const uint4 *)(slot + tile_elem_off(srow, col_base + dl, D, W)));
            }
        }
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
    }
    if (TO_F16 && bad) report_error(a.pool.status, DEV_ERR_F16_RANGE, 1, pl.b, j);
    (void)abort;
}

// ---- Q8_0 raw staging (copy engine) and in-place dequantisation. The K feeder copies this CTA's
// 64 K rows (whole blocks: qs plane then scales, contiguous in the pool), the V feeder this CTA's
// 128 columns of the tile's 128 V rows (a tensor-map load of the qs half of each block, a bulk copy
// of its scale plane), into the upper part of the tile's own operand stage once the stage is free.
// Warps DQ_WARP0 .. +3 then convert K, the next four V: each thread reads its eight units (16 int8
// values and the fp16 scale of their 32-group) from the raw bytes, the team meets at a bounded
// barrier (every raw byte read before any f16 store overwrites the stage), and the thread stores
// its units as f16. Eight consecutive lanes take eight consecutive rows of one 16-column segment:
// the pool's row swizzle of the int8 units (unit ^ (row & 7)) makes their raw loads, and the
// operand layout's swizzle their stores, hit eight distinct bank groups. ----
constexpr int kDqUnits = 8;

// Row (of this CTA's K rows or of the tile's V rows) and logical 16-column segment (of the row, or
// of this CTA's V half) of unit i of team thread ptid.
__device__ __forceinline__ void p2_dq_coords(int ptid, int i, int kv, int &row, int &seg) {
    if (kv == 0) {
        row = 8 * i + (ptid & 7);
        seg = ptid >> 3;            // 0-15
    } else {
        row = 16 * i + 8 * (ptid >> 6) + (ptid & 7);
        seg = (ptid >> 3) & 7;      // 0-7 within this CTA's half
    }
}

template <bool Q8>
__device__ __forceinline__ void p2_dequant_part(const uint8_t *raw, int kv, int rank, int bt, uint8_t *sDst, int ptid,
                                                uint32_t team_bar, int team_use, volatile int *abort, bool &bad,
                                                bool &ok) {
    constexpr int D = 256, VCOLS = 128, W = 128;
    const int ks = kv == 0 ? min(bt, 64) : min(bt, 128);
    const int rowb = kv == 0 ? D : VCOLS;                 // raw qs bytes per row
    const int segb = ks * (rowb + D / 16);                // raw bytes per segment
    uint4 q[kDqUnits];
    uint32_t d[kDqUnits];
#pragma unroll
    for (int i = 0; i < kDqUnits; ++i) {
        int row, seg;
        p2_dq_coords(ptid, i, kv, row, seg);
        const int sg = row / ks, rr = row - sg * ks;
        const uint8_t *base = raw + sg * segb;
        const int pu = seg ^ (row & 7);                  // physical unit (of the row, or of its half)
        const int gs = kv == 0 ? seg : seg + 8 * rank;   // logical segment of the full row
        q[i] = *(const uint4 *)(base + rr * rowb + pu * 16);
        d[i] = *(const uint16_t *)(base + ks * rowb + rr * (D / 16) + (gs >> 1) * 2);
    }
    // every thread of the team has read its raw units before any stores over them
    __syncwarp();
    if (ptid == 0 && kv == 0 && team_use < 30) TRACE(960 + team_use);
    if ((threadIdx.x & 31) == 0) mbar_arrive(team_bar);
    if (!mbar_wait(team_bar, (uint32_t)team_use & 1u, abort, kWaitBudget)) {
        ok = false;
        return;
    }
    if (ptid == 0 && kv == 0 && team_use < 30) TRACE(990 + team_use);
#pragma unroll
    for (int i = 0; i < kDqUnits; ++i) {
        int row, seg;
        p2_dq_coords(ptid, i, kv, row, seg);
        uint4 lo, hi;
        dequant16(q[i], d[i], lo, hi);
        bad |= f16x8_has_inf(lo) | f16x8_has_inf(hi);
        const int dD = kv == 0 ? D : VCOLS;
        *(uint4 *)(sDst + tile_elem_off(row, 16 * seg, dD, W)) = lo;
        *(uint4 *)(sDst + tile_elem_off(row, 16 * seg + 8, dD, W)) = hi;
    }
}

// Raw staging of part kv of prefix tile j into the upper part of the operand stage (one lane per
// segment), with an L2 prefetch of the blocks of tile j + 2 this part will need. Segments past the
// prefix, or of an invalid block, are zero-filled by the warp.
__device__ __forceinline__ void p2_stage_raw(const AttnArgs &a, const P2Plan &pl, const uint8_t *const *sPtr,
                                             const int32_t *sBlk, const void *vmap, int j, int kv, uint8_t *raw,
                                             uint32_t bar_raw, int lane) {
    constexpr int D = 256, BN = 128, KROWS = 64, VCOLS = 128;
    const PoolView &p = a.pool;
    const int bt = p.block_tokens;
    const int ks = kv == 0 ? min(bt, KROWS) : min(bt, BN);
    const int n_seg = (kv == 0 ? KROWS : BN) / ks;
    const int rowb = kv == 0 ? D : VCOLS;
    const uint32_t segb = (uint32_t)ks * (rowb + D / 16);
    const int key_base = pl.kbeg + j * BN + (kv == 0 ? pl.rank * KROWS : 0);
    const int rel0 = pl.tbl_lo << p.bt_shift;
    const uint8_t *t = nullptr;
    int blk = -1, rib = 0;
    if (lane < n_seg) {
        const int key = key_base + lane * ks;
        if (key < pl.sk.n_prefix) {
            const int rel = key - rel0;
            t = sPtr[rel >> p.bt_shift];
            blk = sBlk[rel >> p.bt_shift];
            rib = rel & (bt - 1);
        }
    }
    const uint32_t segmask = n_seg >= 32 ? 0xffffffffu : ((1u << n_seg) - 1u);
    const uint32_t valid = __ballot_sync(0xffffffffu, t != nullptr) & segmask;
    const uint32_t missing = ~valid & segmask;
    if (missing) {
        for (uint32_t m = missing; m; m &= m - 1) {
            uint8_t *z = raw + (__ffs(m) - 1) * segb;
            for (uint32_t o = lane * 16; o < segb; o += 32 * 16) *(uint4 *)(z + o) = make_uint4(0, 0, 0, 0);
        }
        __syncwarp();
    }
    if (lane == 0) mbar_arrive_expect_tx(bar_raw, (uint32_t)__popc(valid) * segb);
    __syncwarp();
    if (t) {
        uint8_t *dst = raw + lane * segb;
        if (kv == 0) {
            if (ks == bt) {
                bulk_g2s(smem_addr(dst), t, segb, bar_raw);  // the whole K tile: qs plane, then scales
            } else {
                bulk_g2s(smem_addr(dst), t + (int64_t)rib * D, (uint32_t)ks * D, bar_raw);
                bulk_g2s(smem_addr(dst + ks * D), t + (int64_t)bt * D + rib * (D / 16), (uint32_t)ks * (D / 16), bar_raw);
            }
        } else {
            const uint8_t *tv = t + (int64_t)p.kv_heads * p.tile_bytes;
            tma_load_4d(smem_addr(dst), vmap, pl.rank * VCOLS, rib, pl.g, a.layer * p.n_blocks + blk, bar_raw);
            bulk_g2s(smem_addr(dst + ks * VCOLS), tv + (int64_t)bt * D + rib * (D / 16), (uint32_t)ks * (D / 16), bar_raw);
        }
    }
    // the blocks of tile j + 2 (this CTA's K rows: K and V tiles; the peer prefetches the rest)
    if (kv == 0 && j + 2 < pl.np_tiles && lane < n_seg) {
        const int key = key_base + 2 * BN + lane * ks;
        const int rel = key - rel0;
        if (key < pl.sk.n_prefix && (rel >> p.bt_shift) < pl.tbl_n) {
            const uint8_t *tp = sPtr[rel >> p.bt_shift];
            if (tp) {
                const uint32_t tb = (uint32_t)p.tile_bytes;
                if (p.kv_heads == 1) bulk_prefetch_l2(tp, 2 * tb);
                else {
                    bulk_prefetch_l2(tp, tb);
                    bulk_prefetch_l2(tp + (int64_t)p.kv_heads * p.tile_bytes, tb);
                }
            }
        }
    }
}

// ---- bf16 feeder: this CTA's K half (kv = 0: tile rows [64r, 64r + 64), one copy per run of whole
// blocks, or of 64 rows of a larger block) or V half (kv = 1: the two 1 KB column chunks [2r, 2r + 2)
// of each of the tile's 16 row groups, one 2 KB copy each) of prefix tile j. Lanes copy; rows
// without a source are zero-filled by the warp. ----
template <int TBL>
__device__ __forceinline__ void p2_produce_bf16(const AttnArgs &a, const P2Plan &pl, const uint8_t *const *sPtr, int j,
                                                int kv, uint8_t *sDst, uint32_t bar_full, int lane) {
    constexpr int BN = 128, KROWS = 64, RB = 512;
    const PoolView &p = a.pool;
    const int key0 = pl.kbeg + j * BN;
    int n_cp, rows_cp;
    if (kv == 0) {
        rows_cp = min(p.block_tokens, KROWS);
        n_cp = KROWS / rows_cp;
    } else {
        rows_cp = 8;
        n_cp = BN / 8;
    }
    const uint32_t cp_bytes = kv == 0 ? (uint32_t)rows_cp * RB : 2048u;
    const uint32_t dst = (uint32_t)lane * cp_bytes;
    const uint8_t *src = nullptr;
    uint32_t bytes = 0;
    if (lane < n_cp) {
        const int row = (kv == 0 ? pl.rank * KROWS : 0) + lane * rows_cp;
        const int k = key0 + row;
        if (k < pl.sk.n_prefix) {
            int rib;
            const int idx = block_index(p, k, rib);
            const uint8_t *t = p2_ptr_of<TBL>(a, pl, sPtr, idx);
            if (t) {
                t += (int64_t)kv * p.kv_heads * p.tile_bytes;
                if (kv == 0) {
                    src = t + (int64_t)rib * RB;
                } else {
                    src = t + (int64_t)(rib >> 3) * 4096 + (int64_t)pl.rank * 2048;
                }
                bytes = cp_bytes;
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

// ---- bf16 suffix tile j into this CTA's K half (kv = 0) or V half (kv = 1). From the pool's suffix
// slot (pre-swizzled rows, as the prefix blocks): one copy of up to 64 K rows, or one 2 KB copy per
// 8-row group of V, zero-filling rows past the slot. From the caller's row-major buffers: tensor-map
// loads of 64-column boxes (K: 4 boxes of 64 rows; V: this CTA's 2 boxes of 128 rows), 128-byte
// swizzled, rows past suffix_len read as zeros; these land chunk-major ([64-column chunk][rows]
// [128 B]), which the MMA reads with its own descriptors (sfx_desc). ----
__device__ __forceinline__ void p2_produce_bf16_suffix(const AttnArgs &a, const P2Plan &pl, int j, int kv,
                                                       uint8_t *sDst, uint32_t bar_full, const void *ksmap,
                                                       const void *vsmap, int lane) {
    constexpr int BN = 128, KROWS = 64, RB = 512;
    const PoolView &p = a.pool;
    const int s_base = (j - pl.np_tiles) * BN;
    if (a.k_sfx) {
        if (lane == 0) {
            mbar_arrive_expect_tx(bar_full, 32768u);
            if (kv == 0) {
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    tma_load_4d(smem_addr(sDst + c * 8192), ksmap, 64 * c, pl.g, s_base + pl.rank * KROWS, pl.b, bar_full);
            } else {
#pragma unroll
                for (int c = 0; c < 2; ++c)
                    tma_load_4d(smem_addr(sDst + c * 16384), vsmap, pl.rank * 128 + 64 * c, pl.g, s_base, pl.b, bar_full);
            }
        }
        __syncwarp();
        return;
    }
    const uint8_t *slot = p.suffix + suffix_tile_index(p, a.layer, pl.sk.seq, kv, pl.g) * p.suffix_tile_bytes;
    const int n_cp = kv == 0 ? 1 : BN / 8;
    const uint32_t cp_full = kv == 0 ? (uint32_t)KROWS * RB : 2048u;
    const uint8_t *src = nullptr;
    uint32_t bytes = 0;
    if (lane < n_cp) {
        const int srow = s_base + (kv == 0 ? pl.rank * KROWS : lane * 8);
        if (srow < p.suffix_rows) {
            const int rows = kv == 0 ? min(KROWS, p.suffix_rows - srow) : 8;
            src = kv == 0 ? slot + (int64_t)srow * RB : slot + (int64_t)(srow >> 3) * 4096 + (int64_t)pl.rank * 2048;
            bytes = kv == 0 ? (uint32_t)rows * RB : 2048u;
        }
    }
    const uint32_t dst = (uint32_t)lane * cp_full;
    const uint32_t zlo = dst + bytes, zhi = lane < n_cp ? dst + cp_full : zlo;
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

__device__ __forceinline__ bool p2_xsync(uint32_t xbar, int use, volatile int *abort) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(xbar);
    return mbar_wait(xbar, (uint32_t)use & 1u, abort, kWaitBudget);
}

// 2^x on the FMA pipe, for part of the softmax's exponentials (the MUFU unit delivers 16 ex2 per
// clock per SM, the FMA pipe 128 operations): x = n + f with n the nearest integer (the
// 1.5 * 2^23 rounding constant) and f in [-0.5, 0.5]; 2^f by a degree-3 polynomial fitted here
// for minimum maximum relative error on that interval (Lawson-weighted least squares over
// Chebyshev nodes; max relative error 7.5e-5, below half an f16 ulp); 2^n added to the exponent
// field. x is clamped at -125 so that the exponent stays normal; the result there is about 2e-38.
__device__ __forceinline__ float exp2_fma(float x) {
    x = fmaxf(x, -125.0f);
    const float t = x + 12582912.0f;
    const float f = x - (t - 12582912.0f);
    const float p = fmaf(fmaf(fmaf(0.0551716648f, f, 0.242611125f), f, 0.693260968f), f, 0.999928057f);
    return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// ---- softmax / epilogue (warps 0-15): warp w owns query row (w & 3) * 32 + lane and S columns
// [32h, 32h + 32), h = w >> 2; the four warps of a lane quarter swap row maxima per tile. P(j) goes
// back as 16-bit pairs over columns [16h, 16h + 16) of the tile's S buffer; "P(j) written" is one
// arrival per warp on rank 0's PVK barrier. ----
template <bool Q8>
__device__ __forceinline__ void p2_softmax(const AttnArgs &a, const P2Plan &pl, uint8_t *smem, uint32_t bar0,
                                           uint32_t bar0_r0, volatile int *abort, uint32_t tmem, int n, int n_qtiles,
                                           const void *omap, int omode) {
    using C = P2Cfg<Q8>;
    constexpr int BN = C::BN, D = C::D, SMH = C::SMH, DH = D / SMH;
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
    float *xmax = (float *)(smem + C::OFF_XCH);  // [2 parity][SMH][128 rows]
    float *xl = xmax + 2 * SMH * kBM;             // [SMH][128 rows]
    const uint32_t xbar = bar(P2_XCH + quarter);
    int uses = 0;
    float m_used = -INFINITY, l = 0.0f;
    const float inv_scale_log2 = 1.0f / a.scale_log2;
    bool ok = true;

    // Q landed: Q8_0 pools convert this warp's share of it to f16 in place; then Q is announced
    // to rank 0 (K(0)'s barrier also counts the softmax warps of each CTA)
    ok = mbar_wait(bar(P2_QFULL), 0u, abort, kWaitBudget);
    if (!ok) p2_fail(a, abort, 20);
    if (threadIdx.x == 0) TRACE(2);
    if (ok && Q8) {
        bool bad = false;
        uint8_t *q = smem + C::OFF_Q;
        const int tid = threadIdx.x;  // 0 .. 32 * SMW - 1
#pragma unroll 4
        for (int i = 0; i < C::Q_BYTES / 16 / (32 * C::SMW); ++i) {
            uint4 *pu = (uint4 *)(q + (size_t)(i * 32 * C::SMW + tid) * 16);
            uint4 w = *pu;
            w = make_uint4(bf16x2_to_f16x2(w.x), bf16x2_to_f16x2(w.y), bf16x2_to_f16x2(w.z), bf16x2_to_f16x2(w.w));
            bad |= f16x8_has_inf(w);
            *pu = w;
        }
        if (bad) report_error(a.pool.status, DEV_ERR_F16_RANGE, 0, pl.b, pl.qrow0);
        fence_proxy_async();
    }
    __syncwarp();
    if (lane == 0) mbar_arrive_remote(bar0_r0 + 8u * P2_KINIT);

    for (int jj = 0; ok && jj < n; ++jj) {
        const int sb = jj & 1;
        const int j = pl.j0 + jj;
        if (!(ok = mbar_wait(bar(P2_SFULL + sb), par2(jj), abort, kWaitBudget))) break;
        tc_fence_after();
        if (r == 0 && h == 0 && jj < 64) TRACE(400 + jj);
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
        float *xm = xmax + (jj & 1) * SMH * kBM;
        xm[h * kBM + r] = cm;
        if (!(ok = p2_xsync(xbar, uses++, abort))) break;
        float rmax = cm;
#pragma unroll
        for (int o = 1; o < SMH; ++o) rmax = fmaxf(rmax, xm[((h + o) & (SMH - 1)) * kBM + r]);
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
                // O holds P.V(jj - 1) once that group has finished
                if (!(ok = mbar_wait(bar(P2_PVDONE + ((jj - 1) & 1)), par2(jj - 1), abort, kWaitBudget))) break;
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
                const float xa = fmaf(__uint_as_float(rr[c]), a.scale_log2, neg_m);
                // one exponential in four on the FMA pipe, the rest on the MUFU unit
                const float x = (c & 3) == 3 ? exp2_fma(xa) : ex2(xa);
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
        if (lane == 0) mbar_arrive_remote(bar0_r0 + 8u * (uint32_t)(P2_PVK + (jj & 1)));
        if (r == 0 && h == 0 && jj < 64) TRACE(500 + jj);
    }
    if (!ok) p2_fail(a, abort, 3);
    if (ok && n > 0) {
        ok = mbar_wait(bar(P2_PVDONE + ((n - 1) & 1)), par2(n - 1), abort, kWaitBudget);
        if (!ok) p2_fail(a, abort, 4);
        tc_fence_after();
    }
    if (r == 0 && h == 0) TRACE(3);
    // ---- epilogue: row sum over the four column groups, then this warp's 64 columns of O ----
    xl[h * kBM + r] = l;
    if (ok && !p2_xsync(xbar, uses++, abort)) {
        ok = false;
        p2_fail(a, abort, 7);
    }
    float l_row = 0.0f;
    if (ok)
#pragma unroll
        for (int o = 0; o < SMH; ++o) l_row += xl[o * kBM + r];
    const bool have_o = ok && n > 0;
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
    // the Q area and the K stages are free once the last P.V has finished: they stage the boxes.
    // This warp's 64 columns, 32 at a time (one tensor-memory load in flight keeps the registers
    // within the softmax budget), staged as the 32-row boxes of epilogue_o_tma; the four warps of
    // the column range meet at named barrier 2 + h and one lane stores each 128-row box.
    {
        const int boxc = f32 ? 32 : 64;
        const uint32_t o_taddr = tmem + lane_base + (uint32_t)C::O_COL;
#pragma unroll 1
        for (int c0 = h * DH; c0 < (h + 1) * DH; c0 += 32) {
            uint32_t o32[32];
            if (have_o) {
                tmem_load32(o_taddr + (uint32_t)c0, o32);
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) o32[i] = 0u;
            }
            stage_o_box<32>(smem, quarter, lane, c0, o32, inv, f32);
        }
        fence_proxy_async();
        asm volatile("bar.sync %0, 128;" ::"r"(2 + h) : "memory");
        bool issued = false;
        const int c0 = h * DH;
        const int cb = c0 / boxc + quarter;
        if (lane == 0 && pl.rows_valid > 0 && cb < (c0 + DH) / boxc) {
            const uint32_t src = smem_addr(smem + cb * 4 * kOutBox);
            if (omode == OUT_TMA_ROWS)
                tma_store_5d(omap, src, cb * boxc, pl.qrow0 % a.group, pl.g, pl.qrow0 / a.group, pl.b);
            else
                tma_store_2d(omap, src, cb * boxc, (int)(unit * kBM));
            issued = true;
        }
        if (issued) {
            bulk_commit_group();
            bulk_wait_group_read0();
        }
        __syncwarp();
    }
    if (r == 0 && h == 0) TRACE(4);
}

template <bool Q8>
__global__ void __launch_bounds__(P2Cfg<Q8>::THREADS, 1)
    attn_pair128_kernel(const AttnArgs a, int n_qtiles, const __grid_constant__ CUtensorMap qmap,
                        const __grid_constant__ CUtensorMap omap, int omode, const __grid_constant__ CUtensorMap vmap,
                        const __grid_constant__ CUtensorMap ksmap, const __grid_constant__ CUtensorMap vsmap) {
    using C = P2Cfg<Q8>;
    constexpr int D = C::D;
    extern __shared__ uint8_t smem_raw[];
    // identical offsets in both CTAs: dynamic shared memory starts at the same window address
    uint8_t *smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    uint8_t *sQ = smem + C::OFF_Q;
    uint8_t *sK = smem + C::OFF_K;
    uint8_t *sV = smem + C::OFF_V;
    uint64_t *bars = (uint64_t *)(smem + C::OFF_BAR);
    uint32_t *tmem_holder = (uint32_t *)(bars + P2_N);
    volatile int *abort = (volatile int *)(bars + P2_N + 1);
    const uint8_t **sPtr = (const uint8_t **)(smem + C::OFF_TBL);
    int32_t *sBlk = (int32_t *)(smem + C::OFF_BLK);
    const uint32_t bar0 = smem_addr(bars);
    auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (threadIdx.x == 0) {
        trace_init();
        TRACE(0);
    }
    const P2Plan pl = make_p2_plan(a);
    const uint32_t bar0_r0 = mapa_shared(bar0, 0);  // rank 0's barrier block (cluster window)
    if (threadIdx.x == 0 && !pl.sk.ok) report_error(a.pool.status, DEV_ERR_BAD_SEQ, pl.b, a.seq_ids[pl.b], 3);

    if (threadIdx.x == 0) {
        // producers per CTA of K or of V: four dequantising warps each (Q8_0) or the relay warp (bf16)
        constexpr uint32_t per_rank = Q8 ? C::NDQ / 64 : 1;
        mbar_init(bar(P2_QFULL), 1);
        mbar_init(bar(P2_KINIT), 2 * per_rank + 2 * C::SMW);
        mbar_init(bar(P2_KINIT + 1), 2 * per_rank);
        for (int s = 0; s < 2; ++s) {
            mbar_init(bar(P2_SFULL + s), 1);
            mbar_init(bar(P2_PVDONE + s), 1);
            mbar_init(bar(P2_PVK + s), 4 * per_rank + 2 * C::SMW);
            mbar_init(bar(P2_KFULL + s), 1);
            mbar_init(bar(P2_VFULL + s), 1);
        }
        mbar_init(bar(P2_DONE), 1);
        for (int q = 0; q < 4; ++q) mbar_init(bar(P2_XCH + q), C::SMH);
        for (int s2 = 0; s2 < 2; ++s2) {
            mbar_init(bar(P2_RAWK + s2), 1);
            mbar_init(bar(P2_RAWV + s2), 1);
            mbar_init(bar(P2_TEAM + s2), C::NDQ / 64);  // the four warps of a team
        }
        *abort = 0;
        mbar_init_fence();
    }
    if (warp == C::MMA_WARP) tmem_alloc_pair(smem_addr(tmem_holder), C::TMEM_COLS);
    if (pl.tbl_n <= C::TBL)
        for (int i = threadIdx.x; i < pl.tbl_n; i += C::THREADS) {
            const int blk = lookup_block(a.pool, pl.sk.seq, pl.tbl_lo + i);
            sPtr[i] = blk < 0 ? nullptr : a.pool.prefix + prefix_tile_index(a.pool, a.layer, blk, 0, pl.g) * a.pool.tile_bytes;
            sBlk[i] = blk;
        }
    tc_fence_before();
    __syncthreads();
    cluster_sync_relaxed();  // both CTAs' barriers initialised (fenced above) and tensor memory allocated
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    const int n = pl.j1 - pl.j0;
    if (threadIdx.x == 0) TRACE(1);
    // Q8_0: 896 threads launch at 72 registers (64,512); each warpgroup sets its own budget as it
    // enters its role -- softmax 64, MMA / feeders 72, dequantisers 88: 512 x 64 + 128 x 72 + 256 x 88
    // = 64,512 (the decreases release exactly what the increase takes)
    static_assert(!Q8 || (C::THREADS == 896 && C::SMW == 16 && C::DQ_WARP0 == 20), "warpgroup register split");
    const int wg = warp >> 2;
    if (wg == C::SMW / 4) {
    if constexpr (Q8) warpgroup_reg_dealloc<72>();
    if (warp == C::MMA_WARP) {
        if (pl.rank == 0 && n > 0 && lane == 0) {
            // ---- MMA issue for the pair: S(0), S(1), then P.V(j) and S(j + 2) per tile, one wait ----
            const uint32_t idS = idesc_f16_m(!Q8, false, C::BN, 256);
            const uint32_t idO = idesc_f16_m(!Q8, true, D, 256);
            const uint32_t q_addr = smem_addr(sQ), k_addr = smem_addr(sK), v_addr = smem_addr(sV);
            const uint64_t qd0 = sdesc(q_addr, 16, C::Q_SBO, C::LAYOUT);
            // bf16 suffix tiles read from the caller's buffers land chunk-major (tensor-map boxes of
            // 64 columns): K 8-row groups 1 KB apart and 64-column chunks 8 KB apart; V 8-key groups
            // 1 KB apart and 64-column chunks 16 KB apart
            const bool sfx_tma = !Q8 && a.k_sfx != nullptr;
            auto issue_s = [&](int jj) {
                const int st = jj & 1;
                const uint32_t d_tmem = tmem + C::S_COL + (uint32_t)(st * C::BN);
                const bool chunk_major = sfx_tma && pl.j0 + jj >= pl.np_tiles;
                const uint64_t kd0 = sdesc(k_addr + st * C::K_BYTES, 16, chunk_major ? 1024u : C::K_SBO, C::LAYOUT);
                const uint32_t kstep = chunk_major ? 8192u : 1024u;
#pragma unroll
                for (int g = 0; g < D / 64; ++g) {
                    uint64_t av[4], bv[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        av[i] = qd0 + (((uint32_t)g * C::Q_CHUNK + (uint32_t)i * 32u) >> 4);
                        bv[i] = kd0 + (((uint32_t)g * kstep + (uint32_t)i * 32u) >> 4);
                    }
                    mma_ss_x4<true>(d_tmem, av, bv, idS, g > 0 ? 1u : 0u);
                }
                mma_commit_both(bar(P2_SFULL + st));
                if (jj < 64) TRACE(300 + jj);
            };
            auto issue_pv = [&](int jj) {
                const int st = jj & 1;
                if (jj < 64) TRACE(100 + jj);
                if (!mbar_wait(bar(P2_PVK + st), par2(jj), abort, kWaitBudget)) return false;
                tc_fence_after();
                if (jj < 64) TRACE(200 + jj);
                const bool chunk_major = sfx_tma && pl.j0 + jj >= pl.np_tiles;
                const uint32_t vsbo = chunk_major ? 1024u : C::V_SBO;
                const uint64_t vd0 = sdesc(v_addr + st * C::V_BYTES, chunk_major ? 16384u : C::V_LBO, vsbo, C::LAYOUT);
#pragma unroll
                for (int g = 0; g < 2; ++g) {
                    uint32_t av[4];
                    uint64_t bv[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int kk = g * 4 + i;
                        av[i] = tmem + C::S_COL + (uint32_t)(st * C::BN + kk * 8);
                        bv[i] = vd0 + (((uint32_t)kk * 2u * vsbo) >> 4);
                    }
                    mma_ts_x4<true>(tmem + C::O_COL, av, bv, idO, (jj > 0 || g > 0) ? 1u : 0u);
                }
                mma_commit_both(bar(P2_PVDONE + st));
                return true;
            };
            bool ok = true;
            for (int jj = 0; ok && jj < 2 && jj < n; ++jj) {
                ok = mbar_wait(bar(P2_KINIT + jj), 0u, abort, kWaitBudget);
                tc_fence_after();
                if (ok) issue_s(jj);
            }
            for (int jj = 0; ok && jj < n; ++jj) {
                ok = issue_pv(jj);
                if (ok && jj + 2 < n) issue_s(jj + 2);
            }
            if (!ok) p2_fail(a, abort, 1);
            mma_commit_pair(bar(P2_DONE));
            mbar_wait(bar(P2_DONE), 0u, abort, kWaitBudget);
        }
        __syncwarp();
    } else if (warp == C::KF_WARP || warp == C::VF_WARP) {
        const int kv = warp - C::KF_WARP;
        if (kv == 0 && lane == 0) {
            // Q of this CTA's 128 rows: four 64-column boxes of (64 columns, group heads, 1 KV head,
            // 128 / group tokens, 1 request), 128-byte swizzled
            mbar_arrive_expect_tx(bar(P2_QFULL), (uint32_t)C::Q_BYTES);
            const int t0 = pl.qrow0 / a.group;
#pragma unroll
            for (int c = 0; c < D / 64; ++c)
                tma_load_5d(smem_addr(sQ + c * C::Q_CHUNK), &qmap, 64 * c, 0, pl.g, t0, pl.b, bar(P2_QFULL));
        }
        __syncwarp();
        if constexpr (Q8) {
            // raw Q8_0 bytes of each prefix tile into the upper part of its stage, once the stage is
            // free: S(j - 2) (K) or P.V(j - 2) (V) done
            const int np = min(n, max(0, pl.np_tiles - pl.j0));
            const int b_free = kv ? P2_PVDONE : P2_SFULL;
            int issued = 0;
            for (int it = 0; it < np; ++it) {
                const int st = it & 1;
                if (it >= 2 && !mbar_wait(bar(b_free + st), par2(it - 2), abort, kWaitBudget)) {
                    p2_fail(a, abort, 2);
                    break;
                }
                uint8_t *raw = kv ? sV + st * C::V_BYTES + C::RAWV_OFF : sK + st * C::K_BYTES + C::RAWK_OFF;
                p2_stage_raw(a, pl, (const uint8_t *const *)sPtr, sBlk, &vmap, pl.j0 + it, kv, raw,
                             bar((kv ? P2_RAWV : P2_RAWK) + st), lane);
                issued = it + 1;
            }
            if (lane == 0 && *abort)
                for (int jj = max(0, issued - 2); jj < issued; ++jj)
                    mbar_wait(bar((kv ? P2_RAWV : P2_RAWK) + (jj & 1)), par2(jj), abort, kWaitBudget / 4);
        } else {
            uint8_t *stages = kv ? sV : sK;
            const int sbytes = kv ? C::V_BYTES : C::K_BYTES;
            const int b_full = kv ? P2_VFULL : P2_KFULL;
            const int b_free = kv ? P2_PVDONE : P2_SFULL;  // stage j % 2 free: S(j - 2) / P.V(j - 2) done
            int issued = 0;
            for (int it = 0; it < n; ++it) {
                const int st = it & 1;
                if (it >= 2 && !mbar_wait(bar(b_free + st), par2(it - 2), abort, kWaitBudget)) {
                    p2_fail(a, abort, 2);
                    break;
                }
                const int j = pl.j0 + it;
                if (j >= pl.np_tiles) {
                    p2_produce_bf16_suffix(a, pl, j, kv, stages + st * sbytes, bar(b_full + st), &ksmap, &vsmap, lane);
                } else {
                    p2_produce_bf16<C::TBL>(a, pl, (const uint8_t *const *)sPtr, j, kv, stages + st * sbytes,
                                            bar(b_full + st), lane);
                }
                issued = it + 1;
            }
            if (lane == 0 && *abort)
                for (int jj = max(0, issued - 2); jj < issued; ++jj)
                    mbar_wait(bar(b_full + (jj & 1)), par2(jj), abort, kWaitBudget / 4);
        }
    } else if (warp == C::RELAY_WARP) {
        if constexpr (!Q8) {
            // ---- bf16: forward "this CTA's K/V half landed" to rank 0, in the order its MMAs use
            // them: K(0), K(1), then V(j) and K(j + 2) per tile ----
            if (n > 0 && lane == 0) {
                auto relay = [&](uint32_t local, uint32_t parity, int remote) {
                    if (!mbar_wait(local, parity, abort, kWaitBudget)) return false;
                    mbar_arrive_remote(bar0_r0 + 8u * (uint32_t)remote);
                    return true;
                };
                bool ok = relay(bar(P2_KFULL), 0u, P2_KINIT);
                if (ok && n > 1) ok = relay(bar(P2_KFULL + 1), 0u, P2_KINIT + 1);
                for (int jj = 0; ok && jj < n; ++jj) {
                    ok = relay(bar(P2_VFULL + (jj & 1)), par2(jj), P2_PVK + (jj & 1));
                    const int t = jj + 2;
                    if (ok && t < n) ok = relay(bar(P2_KFULL + (t & 1)), par2(t), p2_k_bar(t));
                    else if (ok) mbar_arrive_remote(bar0_r0 + 8u * (uint32_t)p2_k_bar(t));
                }
                if (!ok) p2_fail(a, abort, 8);
            }
        }
    }
    } else if (warp >= C::DQ_WARP0) {
        if constexpr (Q8) {
            warpgroup_reg_alloc<88>();
            const int dtid = threadIdx.x - C::DQ_WARP0 * 32;
            const int kv = dtid >> 7;          // team: 0 = K (warps 0-3), 1 = V (warps 4-7)
            const int ptid = dtid & 127;
            const int np = min(n, max(0, pl.np_tiles - pl.j0));  // prefix tiles of this split
            const uint32_t team_bar = bar(P2_TEAM + kv);
            bool bad = false;
            bool ok = true;
            for (int jj = 0; jj < n; ++jj) {
                const int j = pl.j0 + jj, st = jj & 1;
                uint8_t *dst = kv == 0 ? sK + st * C::K_BYTES : sV + st * C::V_BYTES;
                if (jj < np) {
                    // the raw part landed (its feeder waited for the stage to be free)
                    if (!(ok = mbar_wait(bar((kv ? P2_RAWV : P2_RAWK) + st), par2(jj), abort, kWaitBudget))) break;
                    if (ptid == 0 && kv == 0 && jj < 64) TRACE(800 + jj);
                    p2_dequant_part<Q8>(dst + (kv ? C::RAWV_OFF : C::RAWK_OFF), kv, pl.rank, a.pool.block_tokens, dst,
                                        ptid, team_bar, jj, abort, bad, ok);
                    if (!ok) break;
                } else {
                    // suffix tile: K stage j % 2 free once S(j - 2) is done, V stage once P.V(j - 2) is
                    if (jj >= 2 && !(ok = mbar_wait(bar((kv == 0 ? P2_SFULL : P2_PVDONE) + st), par2(jj - 2), abort,
                                                    kWaitBudget)))
                        break;
                    p2_suffix_stage<true>(a, pl, j, kv, dst, ptid, C::NDQ / 2, abort);
                }
                if (ptid == 0 && kv == 0 && jj < 64) TRACE(900 + jj);
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) mbar_arrive_remote(bar0_r0 + 8u * (uint32_t)(kv == 0 ? p2_k_bar(jj) : P2_PVK + st));
                if (ptid == 0 && jj < 64) TRACE((kv == 0 ? 600 : 700) + jj);
            }
            if (!ok) p2_fail(a, abort, 6);
            if (bad) report_error(a.pool.status, DEV_ERR_F16_RANGE, 2, pl.b, pl.j0);
            // K of the (up to two) tiles past the end still arrives, so the last PVK phases complete;
            // like a real K(t), only once S(t - 2) is done: that is when the phase of PVK((t - 2) % 2)
            // it belongs to has begun (PVK(t - 4) completed before S(t - 2) was issued)
            if (ok && kv == 0)
                for (int t = max(n, 2); t < n + 2; ++t) {
                    if (!(ok = mbar_wait(bar(P2_SFULL + (t & 1)), par2(t - 2), abort, kWaitBudget))) break;
                    if (lane == 0) mbar_arrive_remote(bar0_r0 + 8u * (uint32_t)p2_k_bar(t));
                }
            if (!ok) p2_fail(a, abort, 9);
        }
    } else {
        if constexpr (Q8) warpgroup_reg_dealloc<64>();
        p2_softmax<Q8>(a, pl, smem, bar0, bar0_r0, abort, tmem, n, n_qtiles, &omap, omode);
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    cluster_sync_relaxed();  // rank 0's MMAs are finished; neither CTA releases memory the other still uses
    tc_fence_after();
    if (warp == C::MMA_WARP) tmem_dealloc_pair(tmem, C::TMEM_COLS);
    if (threadIdx.x == 0) TRACE(5);
    __syncthreads();
    trace_flush();
}

// The Q tensor map: q [B][Tq][Hq][256] bf16 as (head_dim, head in group, KV head, token, request)
// with boxes of 64 columns x 128 query rows (group heads x 128 / group tokens), 128-byte swizzled;
// rows past the call's tokens fall outside the map and read as zeros. Needs a group dividing 128.
bool make_q_map(const AttnArgs &a, CUtensorMap *map) {
    std::memset(map, 0, sizeof(*map));
    const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc || a.group <= 0 || kBM % a.group || ((uintptr_t)a.q & 15)) return false;
    constexpr int D = 256, es = 2;
    const cuuint64_t dims[5] = {(cuuint64_t)D, (cuuint64_t)a.group, (cuuint64_t)a.pool.kv_heads, (cuuint64_t)a.q_tokens,
                                (cuuint64_t)a.n_batch};
    const cuuint64_t strides[4] = {(cuuint64_t)D * es, (cuuint64_t)a.group * D * es, (cuuint64_t)a.q_heads * D * es,
                                   (cuuint64_t)a.q_tokens * a.q_heads * D * es};
    const cuuint32_t box[5] = {64, (cuuint32_t)a.group, 1, (cuuint32_t)(kBM / a.group), 1};
    const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, (void *)a.q, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Tensor maps of the caller's bf16 suffix K or V ([n_batch][suffix_len][kv_heads][256]) as (column,
// KV head, row, request), boxes of 64 columns x `rows` rows, 128-byte swizzled.
bool make_suffix_map(const AttnArgs &a, const void *base, int rows, CUtensorMap *map) {
    std::memset(map, 0, sizeof(*map));
    const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc || !base || ((uintptr_t)base & 15) || a.suffix_len <= 0) return false;
    constexpr int D = 256, es = 2;
    const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)a.pool.kv_heads, (cuuint64_t)a.suffix_len,
                                (cuuint64_t)a.n_batch};
    const cuuint64_t strides[3] = {(cuuint64_t)D * es, (cuuint64_t)a.pool.kv_heads * D * es,
                                   (cuuint64_t)a.suffix_len * a.pool.kv_heads * D * es};
    const cuuint32_t box[4] = {64, 1, (cuuint32_t)rows, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, (void *)base, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The tensor map of the Q8_0 pool's V int8 planes, for copying one CTA's half of the columns of a
// block's rows: (256 bytes of a row, block rows, KV head, layer * n_blocks + block) over the V tiles
// of the prefix arena, boxes of 128 bytes x min(block, 128) rows.
bool make_vraw_map(const AttnArgs &a, CUtensorMap *map) {
    std::memset(map, 0, sizeof(*map));
    const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    const PoolView &p = a.pool;
    if (!enc) return false;
    const int64_t blocks = (int64_t)p.n_layers * p.n_blocks;
    if (blocks > 0x7fffffff) return false;
    const cuuint64_t dims[4] = {256, (cuuint64_t)p.block_tokens, (cuuint64_t)p.kv_heads, (cuuint64_t)blocks};
    const cuuint64_t strides[3] = {256, (cuuint64_t)p.tile_bytes, (cuuint64_t)(2 * p.kv_heads * p.tile_bytes)};
    const cuuint32_t box[4] = {128, (cuuint32_t)std::min(p.block_tokens, 128), 1, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    void *base = p.prefix + (int64_t)p.kv_heads * p.tile_bytes;  // V tile of block 0, head 0, layer 0
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

#ifdef EKV_TRACE
int pair128_debug_set_trace(unsigned long long *buf) {
    return cudaMemcpyToSymbol(c_trace, &buf, sizeof(buf)) == cudaSuccess ? 0 : -2;
}
#endif

// Key-split count of the 128-key pair kernel for `pair_units` CTA pairs on `sms` SMs: a unit's
// set-up and epilogue take about four 128-key tile-times.
int pair128_choose_splits(int64_t pair_units, int max_tiles, int sms) {
    return choose_split_count_cost(pair_units, max_tiles, sms / 2, 4.0, 1.5);
}

bool pair128_supported(const AttnArgs &a) {
    const int bt = a.pool.block_tokens;
    // power-of-two blocks of at least 8 rows; every block of a split fits the shared pointer table
    return a.pool.head_dim == 256 && a.group > 0 && kBM % a.group == 0 && (bt & (bt - 1)) == 0 && bt >= 8 &&
           a.pool.max_blocks_per_seq <= P2Cfg<true>::TBL && a.pool.max_blocks_per_seq <= P2Cfg<false>::TBL &&
           !((uintptr_t)a.q & 15) && !((uintptr_t)a.out & 15);
}

// One launch of the 128-key pair kernel (plus the merge when keys are split), head_dim 256.
// Returns EKV_ERR_UNSUPPORTED (nothing enqueued) where the shape needs the 64-key pair kernel.
int launch_attention_pair128(AttnArgs a, cudaStream_t s, size_t ws_bytes, int sms) {
    if (!pair128_supported(a)) return EKV_ERR_UNSUPPORTED;
    const bool q8 = a.pool.dtype == EKV_DTYPE_Q8_0;
    CUtensorMap qmap;
    if (!make_q_map(a, &qmap)) return EKV_ERR_UNSUPPORTED;
    const int smem_bytes = q8 ? P2Cfg<true>::SMEM : P2Cfg<false>::SMEM;
    const int threads = q8 ? P2Cfg<true>::THREADS : P2Cfg<false>::THREADS;
    static int attr_done[64][2] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr_done[dev][q8]) {
        const cudaError_t e =
            q8 ? cudaFuncSetAttribute(attn_pair128_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes)
               : cudaFuncSetAttribute(attn_pair128_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
        if (e != cudaSuccess) return EKV_ERR_CUDA;
        attr_done[dev][q8] = 1;
    }
    const int rows = a.q_tokens * a.group;
    const int n_pairs = (rows + 2 * kBM - 1) / (2 * kBM);
    const int n_qtiles = 2 * n_pairs;  // 128-row tiles, as the merge kernel indexes them
    const int64_t units = (int64_t)a.n_batch * a.pool.kv_heads * n_pairs;
    if (a.n_splits == 0) {
        const int max_prefix = a.pool.max_blocks_per_seq * a.pool.block_tokens;
        const int max_tiles = (max_prefix + 127) / 128 + (a.suffix_len + 127) / 128;
        int sp = pair128_choose_splits(units, max_tiles, sms);
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
    CUtensorMap omap, vmap;
    const int omode = make_out_map(a, 256, (int64_t)a.n_batch * a.pool.kv_heads * n_qtiles, &omap);
    if (omode == OUT_THREADS) return EKV_ERR_UNSUPPORTED;
    std::memset(&vmap, 0, sizeof(vmap));
    if (q8 && !make_vraw_map(a, &vmap)) return EKV_ERR_UNSUPPORTED;
    CUtensorMap ksmap, vsmap;
    std::memset(&ksmap, 0, sizeof(ksmap));
    std::memset(&vsmap, 0, sizeof(vsmap));
    if (!q8 && a.k_sfx && a.suffix_len > 0 &&
        (!make_suffix_map(a, a.k_sfx, 64, &ksmap) || !make_suffix_map(a, a.v_sfx, 128, &vsmap)))
        return EKV_ERR_UNSUPPORTED;
    const cudaError_t e =
        q8 ? cudaLaunchKernelEx(&cfg, attn_pair128_kernel<true>, a, n_qtiles, qmap, omap, omode, vmap, ksmap, vsmap)
           : cudaLaunchKernelEx(&cfg, attn_pair128_kernel<false>, a, n_qtiles, qmap, omap, omode, vmap, ksmap, vsmap);
    if (e != cudaSuccess) return EKV_ERR_CUDA;
    note_launches(1);
    if (a.n_splits > 1) return launch_merge_splits(a, n_qtiles, s);
    return EKV_OK;
}

}  // namespace ekv
