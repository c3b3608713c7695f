// ekv_attn_tc.cu -- masked attention over the paged KV pool on tcgen05 tensor cores (sm_100a).
//
// Replaces the reference's per-layer-step concat/permute copies + mul_mat(K,Q) +
// soft_max_ext + mul_mat(V,attn) (models/pi05.cpp:406-421) and ggml_flash_attn_ext
// (models/hy_vla.cpp:1075) with one fused kernel per call.
//
// Work unit (one CTA): 128 query rows that share one KV head (rows = (token, head-in-group),
// so for MQA all 8 heads of 16 tokens share the K/V tiles) x a range of key tiles.
//
// Tensor memory (512 columns): two S buffers of BN f32 columns (P, 16-bit, is written back
// over the first BN/2 columns of its own S buffer), O (head_dim f32 columns) and Q (head_dim/2
// columns of packed 16-bit pairs). Both MMAs take A from tensor memory:
//   S = Q K^T   (M=128, N=BN, K=head_dim; A = Q in TMEM, B = K tile in shared memory)
//   O += P V    (M=128, N=head_dim, K=BN; A = P in TMEM, B = V tile, MN-major)
// so shared memory holds only K/V operand stages (and, for Q8_0, a raw staging ring).
//
// Warp roles:
//   warps 0-3  softmax: thread = query row = TMEM lane. Reads S in 32-column halves, masks
//              (closed-form key ranges), online max/sum in the exp2 domain, writes P into TMEM,
//              rescales O in TMEM only when the running max grows by more than 2^8 (exact after
//              the final division); epilogue O/l -> bf16/f32 (or split partials).
//   warp 4     TMEM allocation; one thread issues tcgen05.mma, polling the K-ready and P-ready
//              barriers so whichever of S(j+1) / PV(j) is ready goes first.
//   warp 5     copy engine feeder: bf16 pools -> one cp.async.bulk per (block, swizzle chunk)
//              straight into a K/V stage (pool tiles are stored pre-swizzled); Q8_0 pools ->
//              bulk copies of the int8 and fp16-scale planes into a raw staging ring.
//   warps 6-9  (Q8_0) dequantise raw -> f16 operand in shared memory: exact int8 -> f16 via the
//              0x6400 magic, one f16 multiply by the scale; the bf16 suffix is converted to f16.
// Q8_0 pools run the MMA in f16, bf16 pools in bf16; accumulation is f32.
//
// Every mbarrier wait is bounded (clock64 budget); on expiry the kernel records
// DEV_ERR_TIMEOUT in the pool status word, raises a CTA-local abort flag and unwinds, waiting
// for its own in-flight copies and MMAs before releasing tensor memory.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <climits>
#include <cstring>

#include "ekv_device.cuh"
#include "ekv_internal.h"
#include "ekv_sm100.cuh"
#include "ekv_attn_common.cuh"

namespace ekv {
namespace {

using namespace sm100;




template <int D, bool Q8>
struct TcCfg {
    static constexpr int BM = kBM;
    static constexpr int BN = D > 128 ? 64 : 128;
    static constexpr int W = (D * 2) % 128 == 0 ? 128 : ((D * 2) % 64 == 0 ? 64 : 32);
    static constexpr uint32_t LAYOUT = W == 128 ? 2u : (W == 64 ? 4u : 6u);
    static constexpr uint32_t SBO = (D * 2 / W) * 8 * W;  // bytes between 8-row groups (= 16 * D)
    static constexpr int NSTAGE = Q8 ? 2 : 3;  // K/V operand stages
    // raw Q8_0 staging: separate K and V rings; K is dequantised first, so its stage frees half a
    // tile earlier and its ring runs one tile deeper
    static constexpr int NRAW_K = Q8 ? 3 : 0;
    static constexpr int NRAW_V = Q8 ? 2 : 0;
    static constexpr int KV_BYTES = BN * D * 2;
    static constexpr int RAW_HALF = BN * (D + D / 16);  // K (or V) of one tile: int8 + fp16 scales
    static constexpr int OFF_K = 0;
    static constexpr int OFF_V = NSTAGE * KV_BYTES;
    static constexpr int OFF_RAW = 2 * NSTAGE * KV_BYTES;
    static constexpr int OFF_RAW_V = OFF_RAW + NRAW_K * RAW_HALF;
    static constexpr int OFF_BAR = OFF_RAW_V + NRAW_V * RAW_HALF;
    // softmax warps per TMEM lane quarter, each owning 32 columns of a tile (1: one thread per row,
    // all BN columns; Q8_0 at BN = 128 keeps that form, its dequantisers use the threads)
    static constexpr int SPLIT_H = BN == 64 ? 2 : (Q8 ? 1 : 4);
    static constexpr int OFF_XCH = OFF_BAR + 256;  // softmax exchange: row maxima [2][H][128], sums [H][128]
    static constexpr int OFF_TBL = OFF_XCH + 3 * (SPLIT_H > 2 ? SPLIT_H : 2) * kBM * 4;
    // tile base pointers of the split's block-table entries (whatever fits, at most 512)
    static constexpr int TBL_ROOM = (232448 - 1024 - OFF_TBL) / 8;
    static constexpr int TBL = TBL_ROOM > 512 ? 512 : TBL_ROOM;
    static constexpr int SMEM = OFF_TBL + TBL * 8 + 1024;  // + 1 KB alignment slack
    // Q staging: rows of D*2 bytes whose 16-byte units are XOR-swizzled by the row (q_stage_off), so
    // both the row-major stores and the per-row reads of a warp hit distinct bank groups
    static constexpr int QSTR = D * 2;
    static constexpr bool SPLIT = SPLIT_H > 1;
    static constexpr int SMW = 4 * SPLIT_H;  // softmax warps
    static constexpr int MMA_WARP = SMW;
    static constexpr int TMA_WARP = SMW + 1;  // K feeder; TMA_WARP + 1 feeds V
    static constexpr int DQ_WARP0 = SMW + 3;
    static constexpr int THREADS = (SMW + 3) * 32 + (Q8 ? kDq : 0);
    static constexpr int TMEM_COLS = 512;
    static constexpr int S_COL = 0;
    static constexpr int O_COL = 2 * BN;
    static constexpr int Q_COL = 512 - D / 2;
    static_assert(O_COL + D <= Q_COL, "TMEM budget");
    static_assert(Q_COL % 8 == 0, "TMEM alignment");
    static_assert(SMEM <= 232448, "shared-memory budget");
    static_assert(TBL >= 64, "block-table cache");
    static_assert(BM * QSTR <= NSTAGE * KV_BYTES, "Q staging fits in the V stages");
    static constexpr int OSTR = D * 4 + 16;  // epilogue staging row stride (f32 worst case)
    static_assert(BM * OSTR <= OFF_BAR, "epilogue staging fits below the barriers");
    static_assert(((D + 31) / 32) * 4 * 4096 <= OFF_BAR, "epilogue boxes (f32) fit below the barriers");
    static_assert(D % 16 == 0, "head_dim must be a multiple of 16");
};

// K and V operand stages are separate rings: a K stage is free again once S(j) has been
// computed, long before P.V(j) releases the V stage.
enum {
    BAR_K_FULL = 0,      // [3] K operand stage filled
    BAR_K_EMPTY = 3,     // [3] K operand stage consumed (S done)
    BAR_V_FULL = 6,      // [3] V operand stage filled
    BAR_V_EMPTY = 9,     // [3] V operand stage consumed (P.V done)
    BAR_RAW_K_FULL = 12,   // [3] raw Q8_0 K stage landed
    BAR_RAW_K_EMPTY = 15,  // [3] raw Q8_0 K stage read
    BAR_RAW_V_FULL = 18,   // [2] raw Q8_0 V stage landed
    BAR_RAW_V_EMPTY = 20,  // [2] raw Q8_0 V stage read
    BAR_P_FULL = 22,       // [2] P(j) in TMEM
    BAR_DONE = 24,
    BAR_XCH = 25,          // [4] softmax pair exchange (one per TMEM lane quarter; SPLIT only)
    BAR_Q_READY = 29,      // Q in TMEM and its shared staging (in the V stages) read
    N_BARS = 30
};
// One commit per MMA group: "S(j) done" is the completion of K stage j % NS and "P.V(j) done"
// that of V stage j % NS. A waiter for S(j) or P.V(j - 1) in the softmax cannot be overtaken by a
// later phase of the same barrier: S(j + NS) needs P(j + NS - 2) and P.V(j - 1 + NS) needs
// P(j - 1 + NS), both produced by the softmax after tile j.
__device__ __forceinline__ uint32_t s_done_parity(int j, int ns) { return (uint32_t)(j / ns) & 1u; }
static_assert(N_BARS * 8 + 16 <= 256, "barrier block");

// Key-tile schedule of one CTA, computed identically by every thread.
struct Plan {
    int b, g, qt, split;
    int qrow0, rows_valid;
    SeqKeys sk;
    int kbeg;       // first key of prefix tile 0 (multiple of BN)
    int np_tiles;   // prefix tiles
    int ns_tiles;   // suffix tiles
    int j0, j1;     // this split's tile range [j0, j1)
    int tbl_lo;     // first block-table index cached in shared memory
    int tbl_n;      // entries cached (table indices [tbl_lo, tbl_lo + tbl_n))
};

// Plan of query tile qt (split `split` of n_splits) of request b, KV head g.
template <int BN>
__device__ __forceinline__ Plan make_plan_at(const AttnArgs &a, int b, int g, int qt, int split, int n_splits) {
    Plan pl;
    pl.qt = qt;
    pl.split = split;
    pl.g = g;
    pl.b = b;
    pl.qrow0 = pl.qt * kBM;
    const int rows_total = a.q_tokens * a.group;
    pl.rows_valid = min(kBM, rows_total - pl.qrow0);
    pl.sk = resolve_seq(a.pool, a.use_prefix, a.seq_ids, a.prefix_len, a.prefix_valid, a.span_begin, a.span_end,
                        pl.b);
    pl.kbeg = 0;
    pl.np_tiles = 0;
    pl.ns_tiles = 0;
    if (pl.sk.ok) {
        int kb = 0, ke = pl.sk.prefix_valid;  // padding keys are never visible
        if (a.mask_flags & EKV_MASK_SPAN_ONLY) {
            kb = max(kb, pl.sk.span_b);
            ke = min(ke, pl.sk.span_e);
        }
        if (a.mask_flags & EKV_MASK_BLOCK_CAUSAL) {
            const int t_lo = pl.qrow0 / a.group;
            const int t_hi = (pl.qrow0 + pl.rows_valid - 1) / a.group;
            const int qc_lo = a.q_chunk0 + t_lo / a.chunk_tokens;
            const int qc_hi = a.q_chunk0 + t_hi / a.chunk_tokens;
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
    // prefix keys this split reads: tiles [j0, min(j1, np_tiles)), clipped to the sequence
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

template <int BN>
__device__ __forceinline__ Plan make_plan(const AttnArgs &a, int n_qtiles) {
    const int n_splits = a.n_splits > 1 ? a.n_splits : 1;
    const int qt = blockIdx.x / n_splits;
    (void)n_qtiles;
    return make_plan_at<BN>(a, blockIdx.z, blockIdx.y, qt, blockIdx.x - qt * n_splits, n_splits);
}

// ---- packed units (a.pack > 0): CTA x holds the units u = x * pack + s, s < pack, unit u being
// request u / kv_heads, KV head u % kv_heads, all its rows_per_unit = q_tokens * group query rows
// (CTA rows [s * rpu, (s + 1) * rpu)). Its key tiles are unit 0's, then unit 1's, ...; a row sees
// only its own unit's tiles. The per-unit plans and the first tile of each unit live in shared
// memory (the block-table cache is not used: tbl_n = 0). ----
constexpr int kMaxPack = 8;
struct PackTable {
    Plan unit[kMaxPack];
};



// K tile base (head g, this layer) of block-table entry `idx`: shared-memory copy when cached,
// otherwise from the global table; nullptr for an invalid entry (reported by lookup_block).
template <int TBL>
__device__ __forceinline__ const uint8_t *ptr_of(const AttnArgs &a, const Plan &pl, const uint8_t *const *sPtr,
                                                 int idx) {
    const int i = idx - pl.tbl_lo;
    if (pl.tbl_n <= TBL && i >= 0 && i < pl.tbl_n) return sPtr[i];
    const int blk = lookup_block(a.pool, pl.sk.seq, idx);
    return blk < 0 ? nullptr
                   : a.pool.prefix + prefix_tile_index(a.pool, a.layer, blk, 0, pl.g) * a.pool.tile_bytes;
}


// ---- Q: bf16 [B][Tq][Hq][D] rows -> shared staging (all threads, every load in flight before
// the first store) -> TMEM Q columns (softmax warps, one row per thread; f16 for Q8_0 pools) ----
template <int D, bool Q8>
struct QStage {
    static constexpr int UPR = D / 8;  // 16-byte units per row
    static constexpr int UNITS = kBM * UPR;
    static constexpr int ITERS = (UNITS + TcCfg<D, Q8>::THREADS - 1) / TcCfg<D, Q8>::THREADS;
    uint4 val[ITERS];
};

template <int D, bool Q8>
__device__ __forceinline__ void stage_q_load(const AttnArgs &a, const Plan &pl, QStage<D, Q8> &qs) {
    using Q = QStage<D, Q8>;
#pragma unroll
    for (int i = 0; i < Q::ITERS; ++i) {
        const int u = threadIdx.x + i * TcCfg<D, Q8>::THREADS;
        const int r = u / Q::UPR;
        qs.val[i] = make_uint4(0, 0, 0, 0);
        int b = pl.b, g = pl.g, qr = pl.qrow0 + r;
        bool ok = r < pl.rows_valid;
        if (a.pack) {  // packed units: row r is row r % rpu of unit r / rpu
            const int rpu = a.q_tokens * a.group, s = r / rpu;
            const int unit = blockIdx.x * a.pack + s;
            b = unit / a.pool.kv_heads;
            g = unit - b * a.pool.kv_heads;
            qr = r - s * rpu;
            ok = s < a.pack && b < a.n_batch;
        }
        if (u < Q::UNITS && ok) {
            const int d0 = (u - r * Q::UPR) * 8;
            const int t = qr / a.group;
            const int h = g * a.group + (qr - t * a.group);
            qs.val[i] = __ldg((const uint4 *)(a.q + (((int64_t)b * a.q_tokens + t) * a.q_heads + h) * D + d0));
        }
    }
}

template <int D, bool Q8>
__device__ __forceinline__ void stage_q_store(const QStage<D, Q8> &qs, uint8_t *stg) {
    using Q = QStage<D, Q8>;
#pragma unroll
    for (int i = 0; i < Q::ITERS; ++i) {
        const int u = threadIdx.x + i * TcCfg<D, Q8>::THREADS;
        if (u >= Q::UNITS) break;
        const int r = u / Q::UPR;
        *(uint4 *)(stg + q_stage_off(r, u - r * Q::UPR, TcCfg<D, Q8>::QSTR)) = qs.val[i];
    }
}

// Q row r (staged bf16) -> tensor memory; Q8_0 pools convert to f16, and the return value says whether
// a value became inf (beyond the f16 range).
template <int D, bool Q8>
__device__ __forceinline__ bool q_to_tmem(const uint8_t *stg, int r, uint32_t taddr, int c_lo, int c_hi) {
    using C = TcCfg<D, Q8>;
    bool bad = false;
#pragma unroll 1
    for (int c = c_lo; c < c_hi; ++c) {  // 16 elements = 8 columns per store
        const uint4 a0 = *(const uint4 *)(stg + q_stage_off(r, 2 * c, C::QSTR));
        const uint4 a1 = *(const uint4 *)(stg + q_stage_off(r, 2 * c + 1, C::QSTR));
        uint32_t w[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        if (Q8) {
#pragma unroll
            for (int i = 0; i < 8; ++i) w[i] = bf16x2_to_f16x2(w[i]);
            bad |= f16x8_has_inf(make_uint4(w[0], w[1], w[2], w[3])) | f16x8_has_inf(make_uint4(w[4], w[5], w[6], w[7]));
        }
        tmem_st8(taddr + (uint32_t)(c * 8), w);
    }
    return bad;
}

// ---- bf16 feeder: one warp, one lane per segment (a block, or the suffix rows of the tile).
// Copies the K (kv = 0) or V (kv = 1) rows of tile j into one operand stage: source and
// destination are runs of whole 8-row groups, one contiguous copy per segment; rows without a
// source are zero-filled by the whole warp ----
template <int D>
__device__ __forceinline__ void produce_bf16_part(const AttnArgs &a, const Plan &pl, const uint8_t *const *sPtr,
                                                  int j, int kv, uint8_t *sDst, uint32_t bar_full, int lane) {
    using C = TcCfg<D, false>;
    constexpr int BN = C::BN, RB = D * 2;
    const PoolView &p = a.pool;
    const bool suffix = j >= pl.np_tiles;
    const int seg = suffix ? BN : min(p.block_tokens, BN);
    const int n_seg = BN / seg;
    const uint8_t *src = nullptr;
    uint32_t bytes = 0;
    const uint32_t dst = (uint32_t)lane * seg * RB;
    if (lane < n_seg) {
        if (suffix) {
            const int s0 = (j - pl.np_tiles) * BN;
            if (s0 < p.suffix_rows) {
                bytes = (uint32_t)min(BN, p.suffix_rows - s0) * RB;
                src = p.suffix + suffix_tile_index(p, a.layer, pl.sk.seq, kv, pl.g) * p.suffix_tile_bytes +
                      (int64_t)s0 * RB;
            }
        } else {
            const int k = pl.kbeg + j * BN + lane * seg;
            int rib;
            const int idx = block_index(p, k, rib);
            if (k < pl.sk.n_prefix) {
                src = ptr_of<C::TBL>(a, pl, sPtr, idx);
                if (src) {
                    src += (int64_t)kv * p.kv_heads * p.tile_bytes + (int64_t)rib * RB;
                    bytes = (uint32_t)seg * RB;
                }
            }
        }
    }
    const uint32_t zlo = dst + bytes, zhi = lane < n_seg ? dst + (uint32_t)seg * RB : zlo;
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

// ---- Q8_0 feeder: one raw stage holds the K (kv = 0) or V (kv = 1) part of a tile: per segment of
// vbt = min(block_tokens, BN) rows, [qs vbt x D][fp16 scales vbt x D/32] -- exactly the pool's
// Q8_0 tile, so a whole block is ONE copy and a partial block one per plane. One lane per
// segment. ----
template <int D>
__device__ __forceinline__ void produce_q8_raw(const AttnArgs &a, const Plan &pl, const uint8_t *const *sPtr, int j,
                                               int kv, uint8_t *raw, uint32_t bar_full, int lane) {
    using C = TcCfg<D, true>;
    constexpr int BN = C::BN, SCB = D / 16;  // scale bytes per row
    const PoolView &p = a.pool;
    const int bt = p.block_tokens;
    const int vbt = min(bt, BN), n_seg = BN / vbt;
    const uint32_t vtile = (uint32_t)vbt * (D + SCB);
    const uint8_t *tk = nullptr;
    int rib = 0;
    if (lane < n_seg) {
        const int k = pl.kbeg + j * BN + lane * vbt;
        const int idx = block_index(p, k, rib);
        if (k < pl.sk.n_prefix) tk = ptr_of<C::TBL>(a, pl, sPtr, idx);
    }
    const uint32_t segmask = n_seg >= 32 ? 0xffffffffu : ((1u << n_seg) - 1u);
    const uint32_t valid = __ballot_sync(0xffffffffu, tk != nullptr) & segmask;
    const uint32_t missing = ~valid & segmask;
    if (missing) {
        for (uint32_t m = missing; m; m &= m - 1) {
            uint8_t *z = raw + (__ffs(m) - 1) * vtile;
            for (uint32_t o = lane * 16; o < vtile; o += 32 * 16) *(uint4 *)(z + o) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async();
        __syncwarp();
    }
    if (lane == 0) {
        if (valid) mbar_arrive_expect_tx(bar_full, (uint32_t)__popc(valid) * vtile);
        else mbar_arrive(bar_full);
    }
    __syncwarp();
    if (!tk) return;
    const uint8_t *src = tk + (int64_t)kv * p.kv_heads * p.tile_bytes;  // K or V tile of this head
    uint8_t *dst = raw + lane * vtile;
    if (vbt == bt) {
        bulk_g2s(smem_addr(dst), src, vtile, bar_full);
    } else {  // rows [rib, rib + BN) of a larger block: qs and scale planes separately
        bulk_g2s(smem_addr(dst), src + (int64_t)rib * D, (uint32_t)BN * D, bar_full);
        bulk_g2s(smem_addr(dst + BN * D), src + (int64_t)bt * D + (int64_t)rib * SCB, (uint32_t)BN * SCB, bar_full);
    }
}

// raw K or V stage -> the matching f16 operand stage (kDq threads; every raw load before the
// first store). Thread mapping: 8 consecutive threads take 8 consecutive rows of one 16-column
// segment, so both the swizzled int8 loads and the swizzled operand stores of a thread-phase hit 8
// distinct bank groups; each thread keeps one segment and one row-in-group, so its operand offsets
// are one base plus a constant stride per unit.
template <int D>
__device__ __forceinline__ void dequant_part(const uint8_t *raw, uint8_t *sDst, int vbt_shift, int dtid) {
    using C = TcCfg<D, true>;
    constexpr int BN = C::BN, W = C::W, UPR = D / 16, RS = kDq / UPR, PER = BN / RS, SCB = D / 16;
    static_assert(kDq % (8 * UPR) == 0 && BN % RS == 0, "dequant thread mapping");
    const int rlow = dtid & 7, seg = (dtid >> 3) % UPR, rhigh = (dtid >> 3) / UPR;
    const int r0 = rhigh * 8 + rlow;
    const int vbt = 1 << vbt_shift;
    const uint32_t vtile = (uint32_t)vbt * (D + SCB);
    uint4 q[PER];
    uint32_t d[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int row = r0 + i * RS;
        const int s = row >> vbt_shift, rib = row & (vbt - 1);
        const uint8_t *t = raw + s * vtile;
        q[i] = *(const uint4 *)(t + q8_qs_off(rib, seg * 16, D));
        d[i] = *(const uint16_t *)(t + vbt * D + rib * SCB + (seg >> 1) * 2);
    }
    const uint32_t off_lo = tile_elem_off(r0, seg * 16, D, W), off_hi = tile_elem_off(r0, seg * 16 + 8, D, W);
    constexpr uint32_t STEP = (RS / 8) * C::SBO;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        uint4 lo, hi;
        dequant16(q[i], d[i], lo, hi);
        *(uint4 *)(sDst + off_lo + i * STEP) = lo;
        *(uint4 *)(sDst + off_hi + i * STEP) = hi;
    }
}

// bf16 suffix slot -> the K or V f16 operand stage (Q8_0 pools), 4 units in flight per thread
template <int D>
__device__ __forceinline__ void convert_suffix_part(const AttnArgs &a, const Plan &pl, int j, int kv, uint8_t *sDst,
                                                    int dtid) {
    using C = TcCfg<D, true>;
    constexpr int BN = C::BN, W = C::W, UPR = D / 8, UNITS = BN * UPR;
    const PoolView &p = a.pool;
    const int s_base = (j - pl.np_tiles) * BN;
    const uint8_t *src = p.suffix + suffix_tile_index(p, a.layer, pl.sk.seq, kv, pl.g) * p.suffix_tile_bytes;
#pragma unroll 1
    for (int u0 = 0; u0 < UNITS; u0 += 4 * kDq) {
        uint4 v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int u = u0 + dtid + i * kDq;
            const int row = u / UPR, d0 = (u - row * UPR) * 8, srow = s_base + row;
            v[i] = make_uint4(0, 0, 0, 0);
            if (u < UNITS && srow < p.suffix_rows) v[i] = __ldg((const uint4 *)(src + tile_elem_off(srow, d0, D, W)));
        }
        bool bad = false;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int u = u0 + dtid + i * kDq;
            if (u >= UNITS) break;
            const int row = u / UPR, d0 = (u - row * UPR) * 8;
            const uint4 w = make_uint4(bf16x2_to_f16x2(v[i].x), bf16x2_to_f16x2(v[i].y), bf16x2_to_f16x2(v[i].z),
                                       bf16x2_to_f16x2(v[i].w));
            bad |= f16x8_has_inf(w);
            *(uint4 *)(sDst + tile_elem_off(row, d0, D, W)) = w;
        }
        if (bad) report_error(p.status, DEV_ERR_F16_RANGE, 2, pl.b, j);
    }
}

// One pass over a tile's S row (thread = row): per 32-column chunk, the masked chunk maximum is
// checked against the running maximum; while no visible score exceeds it by more than 2^8
// (raw-score threshold `thr`), P = 2^(s * scale_log2 - m_used) is written straight back over the
// consumed S columns and the running sum is not rescaled. Returns false (warp-uniform) as soon as
// any row of the warp needs a new maximum; the caller then redoes the tile on the two-pass path,
// which rewrites every P column of the tile. Maxima and sums use four independent accumulators.
template <int BN, bool MASKED, bool F16P>
__device__ __forceinline__ bool softmax_tile_1pass(uint32_t s_col, const uint32_t (&vis_bits)[BN / 32],
                                                   float scale_log2, float m_used, float thr, float &l) {
    const float neg_m = -m_used;
    float ps[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int h32 = 0; h32 < BN / 32; ++h32) {
        uint32_t rr[32];
        tmem_load32(s_col + h32 * 32, rr);
        const uint32_t vb = MASKED ? vis_bits[h32] : 0xffffffffu;
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const float v = __uint_as_float(rr[i]);
            mx[i & 3] = fmaxf(mx[i & 3], (!MASKED || ((vb >> i) & 1u)) ? v : -INFINITY);
        }
        const float cm = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
        if (__any_sync(0xffffffffu, cm > thr)) return false;
        uint32_t pw[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            float pr[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int c = 2 * i + e;
                const float x = ex2(fmaf(__uint_as_float(rr[c]), scale_log2, neg_m));
                pr[e] = (!MASKED || ((vb >> c) & 1u)) ? x : 0.0f;
                ps[c & 3] += pr[e];
            }
            if (F16P) {
                const __half2 h2 = __floats2half2_rn(pr[0], pr[1]);
                pw[i] = *(const uint32_t *)&h2;
            } else {
                const __nv_bfloat162 b2 = __floats2bfloat162_rn(pr[0], pr[1]);
                pw[i] = *(const uint32_t *)&b2;
            }
        }
        tmem_st16(s_col + h32 * 16, pw);
    }
    l += (ps[0] + ps[1]) + (ps[2] + ps[3]);
    return true;
}

__device__ __forceinline__ void fail_timeout(const AttnArgs &a, volatile int *abort, int where) {
    *abort = 1;
    report_error(a.pool.status, DEV_ERR_TIMEOUT, where, blockIdx.x, blockIdx.z);
}

// Bounded wait on this warp's pair-exchange barrier (both warps of a TMEM lane quarter arrive
// once per use, lane 0 after a warp sync, so the lanes' shared-memory writes are released).
__device__ __forceinline__ bool pair_sync(uint32_t xbar, int use, volatile int *abort) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(xbar);
    return mbar_wait(xbar, (uint32_t)use & 1u, abort, kWaitBudget);
}

// ---- softmax / epilogue with H = BN / 32 warps per TMEM lane quarter (2 at BN = 64, 4 at BN = 128):
// warp w owns query row (w & 3) * 32 + lane and S columns [h * 32, h * 32 + 32) of every tile,
// h = w >> 2. Per tile the H warps of a quarter swap their masked chunk maxima through shared memory;
// P for the 32 keys goes back as 16 packed columns [h * 16, h * 16 + 16) of the tile's S buffer (all
// H warps have read S by then). The O rescale and the epilogue split O's columns among them. ----
template <int D, bool Q8, bool PACK>
__device__ __forceinline__ void softmax_split_role(const AttnArgs &a, const Plan &pl, uint8_t *smem, uint32_t bar0,
                                                   volatile int *abort, uint32_t tmem, uint32_t lane_base, int n,
                                                   int n_qtiles, const void *omap, int omode) {
    using C = TcCfg<D, Q8>;
    constexpr int BN = C::BN, H = C::SPLIT_H;
    static_assert(BN == 32 * H, "split softmax: 32 columns per warp");
    auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int h = warp >> 2, quarter = warp & 3;
    const int r = quarter * 32 + lane;
    // packed units: row r belongs to unit r / rpu and sees only that unit's tiles
    const PackTable *pt = (const PackTable *)(smem + C::OFF_TBL);
    const int rpu = a.q_tokens * a.group;
    const int s_row = PACK ? r / rpu : 0;
    const bool row_ok = PACK ? (s_row < a.pack && pt->unit[s_row].rows_valid > 0) : r < pl.rows_valid;
    const int t = PACK ? (r - s_row * rpu) / a.group : (pl.qrow0 + r) / a.group;
    int s_tile = 0, first_tile = 0;  // unit of the current tile, and that unit's first CTA tile
    const MaskDesc m = mask_desc(a, pl.b);  // packed units never carry FLEX masks (the launcher checks)
    const bool prefix_simple = !(a.mask_flags & (EKV_MASK_SPAN_ONLY | EKV_MASK_SPAN_EXCLUDE | EKV_MASK_BLOCK_CAUSAL | kVisWordFlags));
    const bool suffix_simple = !(a.mask_flags & (EKV_MASK_SUFFIX_CAUSAL | EKV_MASK_SUFFIX_PREFIX_LM | kVisWordFlags));
    float *xmax = (float *)(smem + C::OFF_XCH);  // [2 parity][H][128 rows]
    float *xl = xmax + 2 * H * kBM;               // [H][128 rows]
    const uint32_t xbar = bar(BAR_XCH + quarter);
    int uses = 0;
    float m_used = -INFINITY, l = 0.0f;
    const float inv_scale_log2 = 1.0f / a.scale_log2;
    bool ok = true;
    for (int jj = 0; jj < n; ++jj) {
        const int sb = jj & 1;
        const int j = pl.j0 + jj;
        if (!(ok = mbar_wait(bar(BAR_K_EMPTY + jj % C::NSTAGE), s_done_parity(jj, C::NSTAGE), abort, kWaitBudget))) break;
        tc_fence_after();
        if (r == 0 && h == 0 && jj < 50) TRACE(300 + jj);
        uint32_t vb;
        bool all_vis = false;
        if constexpr (PACK) {
            // the tile's unit (tiles run unit by unit); rows of other units see none of its keys
            while (s_tile + 1 < a.pack && jj >= first_tile + (pt->unit[s_tile].j1 - pt->unit[s_tile].j0)) {
                first_tile += pt->unit[s_tile].j1 - pt->unit[s_tile].j0;
                ++s_tile;
            }
            const int jt = jj - first_tile;
            const Plan &up = pt->unit[s_tile];
            const bool suffix = jt >= up.np_tiles;
            const int key0 = (suffix ? (jt - up.np_tiles) * BN : up.kbeg + jt * BN) + h * 32;
            vb = (row_ok && s_row == s_tile)
                     ? vis_word(m, suffix, key0, t, up.sk.prefix_valid, up.sk.span_b, up.sk.span_e, a.suffix_len)
                     : 0u;
        } else {
            const bool suffix = j >= pl.np_tiles;
            const int key0 = (suffix ? (j - pl.np_tiles) * BN : pl.kbeg + j * BN) + h * 32;  // this warp's 32 keys
            // all 32 keys visible to every row (uniform over the CTA; rows past rows_valid score zero
            // queries and are never written)
            all_vis = suffix ? (suffix_simple && key0 + 32 <= a.suffix_len)
                             : (prefix_simple && key0 + 32 <= pl.sk.prefix_valid);
            vb = all_vis ? 0xffffffffu
                         : (row_ok ? vis_word(m, suffix, key0, t, pl.sk.prefix_valid, pl.sk.span_b, pl.sk.span_e,
                                              a.suffix_len, pl.sk.n_prefix)
                                   : 0u);
        }
        const uint32_t s_buf = tmem + lane_base + C::S_COL + (uint32_t)(sb * BN);
        if constexpr (PACK) {
            // No row of this lane quarter belongs to the tile's unit (a 17-row unit touches one or two
            // quarters): its P is zero and its scores need not be read. The four warps of the quarter
            // decide alike, so they skip the maxima exchange together.
            const int lo = s_tile * rpu;
            if (!(lo < quarter * 32 + 32 && lo + rpu > quarter * 32)) {
                uint32_t pz[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) pz[i] = 0u;
                tmem_st16(s_buf + h * 16, pz);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(BAR_P_FULL + sb));
                continue;
            }
        }
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
        // exchange slots alternate by use (a slot is rewritten only after the next exchange, which
        // every warp of the quarter reaches after reading this one)
        const int xp = uses & 1;
        xmax[(xp * H + h) * kBM + r] = cm;
        if (!(ok = pair_sync(xbar, uses++, abort))) break;
        float rmax = cm;  // raw scores (scale > 0)
#pragma unroll
        for (int o = 0; o < H; ++o)
            if (o != h) rmax = fmaxf(rmax, xmax[(xp * H + o) * kBM + r]);
        // a new maximum more than 2^8 above the one in use: rescale l and O (the H warps of a
        // quarter see the same row maxima, so they take this branch together)
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
                // O may only be touched once the previous P.V has landed in TMEM.
                if (!(ok = mbar_wait(bar(BAR_V_EMPTY + (jj - 1) % C::NSTAGE), s_done_parity(jj - 1, C::NSTAGE), abort, kWaitBudget)))
                    break;
                tc_fence_after();
#pragma unroll 1
                for (int c0 = h * 16; c0 < D; c0 += 16 * H) {
                    uint32_t o16[16];
                    tmem_load16(tmem + lane_base + (uint32_t)(C::O_COL + c0), o16);
#pragma unroll
                    for (int i = 0; i < 16; ++i) o16[i] = __float_as_uint(__uint_as_float(o16[i]) * alpha);
                    tmem_st16(tmem + lane_base + (uint32_t)(C::O_COL + c0), o16);
                }
                tmem_wait_st();
            }
        }
        // P = 2^(s * scale_log2 - m_used), masked keys 0
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
        if (lane == 0) mbar_arrive(bar(BAR_P_FULL + sb));
        if (r == 0 && h == 0 && jj < 50) TRACE(350 + jj);
    }
    if (!ok) fail_timeout(a, abort, 3);
    if (ok && n > 0) {
        ok = mbar_wait(bar(BAR_V_EMPTY + (n - 1) % C::NSTAGE), s_done_parity(n - 1, C::NSTAGE), abort, kWaitBudget);
        if (!ok) fail_timeout(a, abort, 4);
        tc_fence_after();
    }
    // ---- epilogue: row sum over the H warps, then this warp's columns of O ----
    if (r == 0 && h == 0) TRACE(10);
    xl[h * kBM + r] = l;
    if (ok && !pair_sync(xbar, uses++, abort)) {
        ok = false;
        fail_timeout(a, abort, 7);
    }
    float l_row = 0.0f;  // same order in every warp
    if (ok) {
#pragma unroll
        for (int o = 0; o < H; ++o) l_row += xl[o * kBM + r];
    }
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
        unit = (((int64_t)pl.b * a.pool.kv_heads + pl.g) * n_qtiles + pl.qt) * a.n_splits + pl.split;
        if (row_ok && h == 0) {
            float *wml = a.ws_ml + (unit * kBM + r) * 2;
            wml[0] = have_o ? m_used : -INFINITY;
            wml[1] = have_o ? l_row : 0.0f;
        }
    }
    if (omode != OUT_THREADS) {
        // the host picks a copy-engine route only for head dims that are whole 64-column blocks:
        // EH column ranges of D / EH (a multiple of 64), one per group of four quarter warps
        constexpr int EH = (D % 64 == 0) ? (D / 64 < H ? D / 64 : H) : 1;
        if constexpr (D % 64 == 0) {
            if (h < EH)
                epilogue_o_tma(a, pl.qrow0, pl.rows_valid, pl.g, pl.b, omap, omode, smem + C::OFF_K, quarter, lane,
                               tmem + lane_base + (uint32_t)C::O_COL, h * (D / EH), (h + 1) * (D / EH), have_o, inv,
                               f32, unit, 2 + h);
        }
        return;
    }
    uint8_t *orow = (smem + C::OFF_K) + r * C::OSTR;
    constexpr int EC = (D % 32 == 0) ? 32 : 16;  // columns per TMEM load
#pragma unroll 1
    for (int c0 = h * EC; c0 < D; c0 += EC * H) {
        uint32_t o32[32];
        if (have_o) {
            if constexpr (EC == 32) {
                tmem_load32(tmem + lane_base + (uint32_t)(C::O_COL + c0), o32);
            } else {
                uint32_t (&o16)[16] = *reinterpret_cast<uint32_t (*)[16]>(o32);
                tmem_load16(tmem + lane_base + (uint32_t)(C::O_COL + c0), o16);
            }
        } else {
#pragma unroll
            for (int i = 0; i < EC; ++i) o32[i] = 0u;
        }
        if (f32) {
#pragma unroll
            for (int i = 0; i < EC; i += 4)
                *(float4 *)(orow + (c0 + i) * 4) =
                    make_float4(__uint_as_float(o32[i]) * inv, __uint_as_float(o32[i + 1]) * inv,
                                __uint_as_float(o32[i + 2]) * inv, __uint_as_float(o32[i + 3]) * inv);
        } else {
#pragma unroll
            for (int i0 = 0; i0 < EC; i0 += 8) {
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
        } else if (PACK) {
            const int s = rw / rpu;
            const Plan &up = pt->unit[s];
            if (up.rows_valid == 0) continue;  // past the last unit
            const int qrw = rw - s * rpu;
            const int tw = qrw / a.group;
            const int hw = up.g * a.group + (qrw - tw * a.group);
            dst = (uint8_t *)a.out + ((((int64_t)up.b * a.q_tokens + tw) * a.q_heads + hw) * D) * (f32 ? 4 : 2);
        } else {
            const int qrw = pl.qrow0 + rw;
            const int tw = qrw / a.group;
            const int hw = pl.g * a.group + (qrw - tw * a.group);
            dst = (uint8_t *)a.out + ((((int64_t)pl.b * a.q_tokens + tw) * a.q_heads + hw) * D) * (f32 ? 4 : 2);
        }
        const uint8_t *srow = (smem + C::OFF_K) + rw * C::OSTR;
        for (int o = lane * 16; o < row_bytes; o += 32 * 16) *(uint4 *)(dst + o) = *(const uint4 *)(srow + o);
    }
}

template <int D, bool Q8, bool PACK = false>
__global__ void __launch_bounds__(TcCfg<D, Q8>::THREADS, 1)
    attn_tc_kernel(const AttnArgs a, int n_qtiles, const __grid_constant__ CUtensorMap omap, int omode) {
    using C = TcCfg<D, Q8>;
    constexpr int BN = C::BN, W = C::W, NS = C::NSTAGE;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *sK = smem + C::OFF_K;
    uint8_t *sV = smem + C::OFF_V;
    uint8_t *sRawK = smem + C::OFF_RAW;
    uint8_t *sRawV = smem + C::OFF_RAW_V;
    uint64_t *bars = (uint64_t *)(smem + C::OFF_BAR);
    uint32_t *tmem_holder = (uint32_t *)(bars + N_BARS);
    volatile int *abort = (volatile int *)(bars + N_BARS + 1);
    const uint8_t **sPtr = (const uint8_t **)(smem + C::OFF_TBL);
    const uint32_t bar0 = smem_addr(bars);
    auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (threadIdx.x == 0) {
        trace_init();
        TRACE(0);
        TRACE_CLK(20);
    }
    Plan pl = make_plan<BN>(a, n_qtiles);
    PackTable *pt = (PackTable *)(smem + C::OFF_TBL);  // packed units only (no block-table cache then)
    const int rpu = a.q_tokens * a.group;
    if constexpr (PACK) {
        static_assert(!Q8 && BN == 128, "packed units: bf16 pools at 128-key tiles");
        {
            static_assert(sizeof(PackTable) <= C::TBL * 8, "pack table fits the block-table cache");
            if (threadIdx.x < a.pack) {
                const int unit = blockIdx.x * a.pack + threadIdx.x;
                const int b = unit / a.pool.kv_heads;
                Plan up{};
                if (b < a.n_batch) {
                    up = make_plan_at<BN>(a, b, unit - b * a.pool.kv_heads, 0, 0, 1);
                    if (!up.sk.ok) report_error(a.pool.status, DEV_ERR_BAD_SEQ, b, a.seq_ids[b], 3);
                }
                up.tbl_n = 0;
                pt->unit[threadIdx.x] = up;
            }
        }
        pl.tbl_n = 0;
        pl.qrow0 = 0;
        pl.rows_valid = a.pack * rpu;
    }
    if (threadIdx.x == 0) TRACE(1);
    if (threadIdx.x == 0 && !PACK && !pl.sk.ok) report_error(a.pool.status, DEV_ERR_BAD_SEQ, pl.b, a.seq_ids[pl.b], 3);

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(bar(BAR_K_FULL + s), Q8 ? kDq / 32 : 1);
            mbar_init(bar(BAR_K_EMPTY + s), 1);
            mbar_init(bar(BAR_V_FULL + s), Q8 ? kDq / 32 : 1);
            mbar_init(bar(BAR_V_EMPTY + s), 1);
        }
        for (int s = 0; s < 3; ++s) {
            mbar_init(bar(BAR_RAW_K_FULL + s), 1);
            mbar_init(bar(BAR_RAW_K_EMPTY + s), kDq / 32);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(bar(BAR_RAW_V_FULL + s), 1);
            mbar_init(bar(BAR_RAW_V_EMPTY + s), kDq / 32);
            mbar_init(bar(BAR_P_FULL + s), C::SMW);
        }
        mbar_init(bar(BAR_DONE), 1);
        for (int q = 0; q < 4; ++q) mbar_init(bar(BAR_XCH + q), C::SPLIT_H);
        mbar_init(bar(BAR_Q_READY), C::SMW);
        *abort = 0;
        mbar_init_fence();
    }
    if (warp == C::MMA_WARP) tmem_alloc(smem_addr(tmem_holder), C::TMEM_COLS);
    QStage<D, Q8> qstage;
    stage_q_load<D, Q8>(a, pl, qstage);  // Q loads in flight while the table is read
    // tile base pointers of the split's block-table entries, validated once, in shared memory
    if (pl.tbl_n <= C::TBL)
        for (int i = threadIdx.x; i < pl.tbl_n; i += C::THREADS) {
            const int blk = lookup_block(a.pool, pl.sk.seq, pl.tbl_lo + i);
            sPtr[i] = blk < 0 ? nullptr
                              : a.pool.prefix + prefix_tile_index(a.pool, a.layer, blk, 0, pl.g) * a.pool.tile_bytes;
        }
    // Q is staged in the V stages: the K stages and the raw ring can fill while Q goes to TMEM;
    // the first V write and the first MMA wait for BAR_Q_READY.
    stage_q_store<D, Q8>(qstage, smem + C::OFF_V);
    if (threadIdx.x == 0) TRACE(2);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    const uint32_t lane_base = ((uint32_t)((warp & 3) * 32)) << 16;
    if (warp < C::SMW) {
        // row (warp & 3) * 32 + lane; with SPLIT the H warps of a lane quarter share its column blocks
        const int h = C::SPLIT ? warp >> 2 : 0, nh = C::SPLIT_H;
        if (q_to_tmem<D, Q8>(smem + C::OFF_V, (warp & 3) * 32 + lane, tmem + lane_base + C::Q_COL, h * (D / 16) / nh,
                             (h + 1) * (D / 16) / nh))
            report_error(a.pool.status, DEV_ERR_F16_RANGE, 0, pl.b, pl.qrow0);
        tmem_wait_st();
        fence_proxy_async();  // staging reads (generic) before the copy engine refills the V stages
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(BAR_Q_READY));
    }
    if (threadIdx.x == 0) TRACE(3);
    if constexpr (PACK) {  // the CTA's tiles: every unit's, in unit order (plans published by the barrier above)
        int total = 0;
        for (int s = 0; s < a.pack; ++s) total += pt->unit[s].j1 - pt->unit[s].j0;
        pl.j0 = 0;
        pl.j1 = total;
        pl.np_tiles = total;
    }
    const int n = pl.j1 - pl.j0;

    if (warp == C::MMA_WARP) {
        // One thread issues everything, in the fixed order S(0), [S(j+1), P.V(j)] for j = 0..n-1.
        // tcgen05.mma issue returns about when the previous MMA starts executing, so every cycle
        // this thread spends elsewhere is an idle tensor pipe: straight-line waits (which return at
        // once when the operand is ready), one commit per group. S(j+1) reuses the S buffer of
        // P(j-1), whose P.V was issued before it (the tensor core executes in issue order).
        if (n > 0 && lane == 0) {
            const uint32_t idS = idesc_f16(!Q8, false, BN);
            const uint32_t idO = idesc_f16(!Q8, true, D);
            const uint32_t k_addr = smem_addr(sK), v_addr = smem_addr(sV);
            bool ok = true;
            auto issue_s = [&](int jj) {
                const int st = jj % NS, sb = jj & 1;
                if (!mbar_wait(bar(BAR_K_FULL + st), (jj / NS) & 1, abort, kWaitBudget)) return false;
                tc_fence_after();
                const uint32_t d_tmem = tmem + C::S_COL + (uint32_t)(sb * BN);
                const uint64_t bd0 = sdesc(k_addr + st * C::KV_BYTES, 16, C::SBO, C::LAYOUT);
                constexpr int KS = D / 16, KPC = W / 32;  // K steps; K steps per swizzle chunk
                uint32_t av[KS];
                uint64_t bv[KS];
#pragma unroll
                for (int kk = 0; kk < KS; ++kk) {
                    av[kk] = tmem + C::Q_COL + (uint32_t)(kk * 8);
                    bv[kk] = bd0 + (((uint32_t)(kk / KPC) * (8 * W) + (uint32_t)(kk % KPC) * 32u) >> 4);
                }
                if constexpr (KS % 4 == 0) {
#pragma unroll
                    for (int g = 0; g < KS / 4; ++g)
                        mma_ts_x4<false>(d_tmem, *reinterpret_cast<const uint32_t(*)[4]>(av + 4 * g),
                                         *reinterpret_cast<const uint64_t(*)[4]>(bv + 4 * g), idS, g > 0 ? 1u : 0u);
                } else {
#pragma unroll
                    for (int kk = 0; kk < KS; ++kk) mma_ts(d_tmem, av[kk], bv[kk], idS, kk > 0 ? 1u : 0u);
                }
                mma_commit(bar(BAR_K_EMPTY + st));  // S(j) done: K stage free, S(j) readable
                if (jj < 50) TRACE(200 + jj);
                return true;
            };
            auto issue_pv = [&](int jj) {
                const int st = jj % NS, sb = jj & 1;
                if (!mbar_wait(bar(BAR_P_FULL + sb), (jj >> 1) & 1, abort, kWaitBudget)) return false;
                if (!mbar_wait(bar(BAR_V_FULL + st), (jj / NS) & 1, abort, kWaitBudget)) return false;
                tc_fence_after();
                const uint64_t bd0 = sdesc(v_addr + st * C::KV_BYTES, 8 * W, C::SBO, C::LAYOUT);
                constexpr int PS = BN / 16;  // P.V K steps (4 or 8)
                uint32_t av[PS];
                uint64_t bv[PS];
#pragma unroll
                for (int kk = 0; kk < PS; ++kk) {
                    av[kk] = tmem + C::S_COL + (uint32_t)(sb * BN + kk * 8);
                    bv[kk] = bd0 + ((uint32_t)kk * 2u * C::SBO >> 4);
                }
#pragma unroll
                for (int g = 0; g < PS / 4; ++g)
                    mma_ts_x4<false>(tmem + C::O_COL, *reinterpret_cast<const uint32_t(*)[4]>(av + 4 * g),
                                     *reinterpret_cast<const uint64_t(*)[4]>(bv + 4 * g), idO, (jj > 0 || g > 0) ? 1u : 0u);
                mma_commit(bar(BAR_V_EMPTY + st));  // P.V(j) done: V stage free, P(j) consumed
                if (jj < 50) TRACE(250 + jj);
                return true;
            };
            ok = mbar_wait(bar(BAR_Q_READY), 0, abort, kWaitBudget);
            tc_fence_after();
            if (ok) ok = issue_s(0);
            for (int jj = 0; ok && jj < n; ++jj) {
                if (jj + 1 < n) ok = issue_s(jj + 1);
                if (ok) ok = issue_pv(jj);
            }
            if (!ok) fail_timeout(a, abort, 1);
            // Every MMA this thread issued must have finished before TMEM is released.
            mma_commit(bar(BAR_DONE));
            mbar_wait(bar(BAR_DONE), 0, abort, kWaitBudget);
        }
        __syncwarp();
    } else if (warp == C::TMA_WARP || warp == C::TMA_WARP + 1) {
        // copy-engine feeders, one warp for K and one for V: a bulk-copy issue stalls its warp for a
        // few hundred cycles, so the two rings are fed in parallel
        const int kv = warp - C::TMA_WARP;
        if constexpr (Q8) {
            // raw prefix tiles (suffix tiles are converted by the dequant warps); the K ring is one
            // stage deeper since K is dequantised first
            const int nr = kv ? C::NRAW_V : C::NRAW_K;
            uint8_t *ring = kv ? sRawV : sRawK;
            const int b_full = kv ? BAR_RAW_V_FULL : BAR_RAW_K_FULL, b_empty = kv ? BAR_RAW_V_EMPTY : BAR_RAW_K_EMPTY;
            const int np = min(n, max(0, pl.np_tiles - pl.j0));
            int issued = 0;
            for (int it = 0; it < np; ++it) {
                const int r = it % nr;
                if (it >= nr && !mbar_wait(bar(b_empty + r), ((it - nr) / nr) & 1, abort, kWaitBudget)) {
                    fail_timeout(a, abort, 2);
                    break;
                }
                if (lane == 0 && it < 50) TRACE((kv ? 150 : 450) + it);
                produce_q8_raw<D>(a, pl, (const uint8_t *const *)sPtr, pl.j0 + it, kv, ring + r * C::RAW_HALF,
                                  bar(b_full + r), lane);
                issued = it + 1;
            }
            // Do not leave the CTA with bulk copies still writing shared memory.
            if (lane == 0 && *abort)
                for (int jj = max(0, issued - nr); jj < issued; ++jj)
                    mbar_wait(bar(b_full + jj % nr), (jj / nr) & 1, abort, kWaitBudget / 4);
        } else {
            // K stage it once S(it - NS) is done; V stage it once P.V(it - NS) is done (and, for the
            // first V, once Q's staging in the V stages has been read)
            uint8_t *stages = kv ? sV : sK;
            const int b_full = kv ? BAR_V_FULL : BAR_K_FULL, b_empty = kv ? BAR_V_EMPTY : BAR_K_EMPTY;
            int issued = 0;
            for (int it = 0; it < n; ++it) {
                const int st = it % NS;
                if (kv && it == 0 && !mbar_wait(bar(BAR_Q_READY), 0, abort, kWaitBudget)) {
                    fail_timeout(a, abort, 2);
                    break;
                }
                if (it >= NS && !mbar_wait(bar(b_empty + st), ((it - NS) / NS) & 1, abort, kWaitBudget)) {
                    fail_timeout(a, abort, 2);
                    break;
                }
                if (lane == 0 && it < 50) TRACE((kv ? 150 : 450) + it);
                if constexpr (PACK) {  // tile `it` of the CTA = tile it - first(s) of unit s
                    int s = 0, first = 0;
                    while (s + 1 < a.pack && it >= first + (pt->unit[s].j1 - pt->unit[s].j0)) {
                        first += pt->unit[s].j1 - pt->unit[s].j0;
                        ++s;
                    }
                    produce_bf16_part<D>(a, pt->unit[s], (const uint8_t *const *)sPtr, it - first, kv,
                                         stages + st * C::KV_BYTES, bar(b_full + st), lane);
                } else
                produce_bf16_part<D>(a, pl, (const uint8_t *const *)sPtr, pl.j0 + it, kv, stages + st * C::KV_BYTES,
                                     bar(b_full + st), lane);
                issued = it + 1;
            }
            // Do not leave the CTA with bulk copies still writing shared memory.
            if (lane == 0 && *abort)
                for (int jj = max(0, issued - NS); jj < issued; ++jj)
                    mbar_wait(bar(b_full + jj % NS), (jj / NS) & 1, abort, kWaitBudget / 4);
        }
    } else if (warp >= C::DQ_WARP0) {
        if constexpr (Q8) {
            const int dtid = threadIdx.x - C::DQ_WARP0 * 32;
            const int vbt = min(a.pool.block_tokens, BN);
            const int vbt_shift = 31 - __clz(vbt);  // power of two: checked by the launcher
            for (int jj = 0; jj < n; ++jj) {
                const int j = pl.j0 + jj, st = jj % NS;
                const bool prefix = j < pl.np_tiles;
                if (dtid == 0 && jj < 50) TRACE(500 + jj);
                bool ok = true;
#pragma unroll 1
                for (int kv = 0; kv < 2; ++kv) {
                    const int nr = kv ? C::NRAW_V : C::NRAW_K, rs = jj % nr;
                    const uint8_t *raw = (kv ? sRawV : sRawK) + rs * C::RAW_HALF;
                    const int b_raw = kv ? BAR_RAW_V_FULL : BAR_RAW_K_FULL;
                    const int b_empty = kv ? BAR_V_EMPTY : BAR_K_EMPTY, b_full = kv ? BAR_V_FULL : BAR_K_FULL;
                    uint8_t *dst = (kv ? sV : sK) + st * C::KV_BYTES;
                    if (prefix && !mbar_wait(bar(b_raw + rs), (jj / nr) & 1, abort, kWaitBudget)) {
                        ok = false;
                        break;
                    }
                    if (kv == 1 && jj == 0 && !mbar_wait(bar(BAR_Q_READY), 0, abort, kWaitBudget)) {  // Q staging read
                        ok = false;
                        break;
                    }
                    if (jj >= NS && !mbar_wait(bar(b_empty + st), ((jj - NS) / NS) & 1, abort, kWaitBudget)) {
                        ok = false;
                        break;
                    }
                    if (dtid == 0 && jj < 50) TRACE(550 + 250 * kv + jj);
                    if (prefix) dequant_part<D>(raw, dst, vbt_shift, dtid);
                    else convert_suffix_part<D>(a, pl, j, kv, dst, dtid);
                    fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) {
                        if (prefix) mbar_arrive(bar((kv ? BAR_RAW_V_EMPTY : BAR_RAW_K_EMPTY) + rs));
                        mbar_arrive(bar(b_full + st));
                    }
                }
                if (!ok) {
                    fail_timeout(a, abort, 6);
                    break;
                }
                if (dtid == 0 && jj < 50) TRACE(100 + jj);
            }
        }
    } else if (warp < C::SMW && C::SPLIT) {
        if constexpr (C::SPLIT)
            softmax_split_role<D, Q8, PACK>(a, pl, smem, bar0, abort, tmem, lane_base, n, n_qtiles, &omap, omode);
    } else if (warp < 4) {
        // ---- softmax / epilogue: thread = query row = TMEM lane ----
        const int r = threadIdx.x;
        const bool row_ok = r < pl.rows_valid;
        const int qr = pl.qrow0 + r;
        const int t = qr / a.group;
        const MaskDesc m = mask_desc(a, pl.b);
        const bool prefix_simple = !(a.mask_flags & (EKV_MASK_SPAN_ONLY | EKV_MASK_SPAN_EXCLUDE | EKV_MASK_BLOCK_CAUSAL | kVisWordFlags));
        const bool suffix_simple = !(a.mask_flags & (EKV_MASK_SUFFIX_CAUSAL | EKV_MASK_SUFFIX_PREFIX_LM | kVisWordFlags));
        float m_used = -INFINITY, l = 0.0f;
        const float inv_scale_log2 = 1.0f / a.scale_log2;
        bool ok = true;
        for (int jj = 0; jj < n; ++jj) {
            const int sb = jj & 1;
            const int j = pl.j0 + jj;
            if (!(ok = mbar_wait(bar(BAR_K_EMPTY + jj % C::NSTAGE), s_done_parity(jj, C::NSTAGE), abort, kWaitBudget))) break;
            tc_fence_after();
            if (r == 0 && jj < 50) TRACE(300 + jj);
            const bool suffix = j >= pl.np_tiles;
            const int key0 = suffix ? (j - pl.np_tiles) * BN : pl.kbeg + j * BN;
            // every key of the tile visible to every row (uniform over the CTA): rows past
            // rows_valid score zero queries and are never written, so they take that path too
            const bool tile_vis = suffix ? (suffix_simple && key0 + BN <= a.suffix_len)
                                         : (prefix_simple && key0 + BN <= pl.sk.prefix_valid);
            const bool all_vis = row_ok && tile_vis;
            uint32_t vis_bits[BN / 32];
#pragma unroll
            for (int w = 0; w < BN / 32; ++w)
                vis_bits[w] = all_vis ? 0xffffffffu
                                      : (row_ok ? vis_word(m, suffix, key0 + 32 * w, t, pl.sk.prefix_valid, pl.sk.span_b,
                                                           pl.sk.span_e, a.suffix_len, pl.sk.n_prefix)
                                                : 0u);
            const uint32_t s_col = tmem + lane_base + C::S_COL + (uint32_t)(sb * BN);
            // common case: one pass, no new maximum (see softmax_tile_1pass)
            const float thr = (m_used + 8.0f) * inv_scale_log2;
            const bool one_pass = tile_vis ? softmax_tile_1pass<BN, false, Q8>(s_col, vis_bits, a.scale_log2, m_used, thr, l)
                                           : softmax_tile_1pass<BN, true, Q8>(s_col, vis_bits, a.scale_log2, m_used, thr, l);
            if (!one_pass) {
            // two passes: the S row is read in 32-column halves twice (max, then exponentials):
            // only 32 scores are live at a time; P (16-bit) goes back over the consumed S columns.
            // The max is taken on raw scores and scaled once (scale > 0).
            float s_max = -INFINITY;
#pragma unroll
            for (int h32 = 0; h32 < BN / 32; ++h32) {
                uint32_t rr[32];
                tmem_load32(s_col + h32 * 32, rr);
                if (all_vis) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) s_max = fmaxf(s_max, __uint_as_float(rr[i]));
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if ((vis_bits[h32] >> i) & 1u) s_max = fmaxf(s_max, __uint_as_float(rr[i]));
                }
            }
            const float m_tile = s_max * a.scale_log2;
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
                // O may only be touched once the previous P.V has landed in TMEM.
                if (!(ok = mbar_wait(bar(BAR_V_EMPTY + (jj - 1) % C::NSTAGE), s_done_parity(jj - 1, C::NSTAGE), abort, kWaitBudget)))
                    break;
                tc_fence_after();
#pragma unroll 1
                for (int c0 = 0; c0 < D; c0 += 16) {
                    uint32_t rr[16];
                    tmem_load16(tmem + lane_base + (uint32_t)(C::O_COL + c0), rr);
#pragma unroll
                    for (int i = 0; i < 16; ++i) rr[i] = __float_as_uint(__uint_as_float(rr[i]) * alpha);
                    tmem_st16(tmem + lane_base + (uint32_t)(C::O_COL + c0), rr);
                }
                tmem_wait_st();
            }
            float psum = 0.0f;
            const float neg_m = -m_used;
            const bool any_vis = m_used != -INFINITY;
#pragma unroll
            for (int h32 = 0; h32 < BN / 32; ++h32) {
                uint32_t rr[32];
                tmem_load32(s_col + h32 * 32, rr);
                uint32_t pw[16];
                const uint32_t vb = all_vis ? 0xffffffffu : (any_vis ? vis_bits[h32] : 0u);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    float pr[2];
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int c = 2 * i + e;
                        const float x = ex2(fmaf(__uint_as_float(rr[c]), a.scale_log2, neg_m));
                        pr[e] = ((vb >> c) & 1u) ? x : 0.0f;
                        psum += pr[e];
                    }
                    if (Q8) {
                        const __half2 h2 = __floats2half2_rn(pr[0], pr[1]);
                        pw[i] = *(const uint32_t *)&h2;
                    } else {
                        const __nv_bfloat162 b2 = __floats2bfloat162_rn(pr[0], pr[1]);
                        pw[i] = *(const uint32_t *)&b2;
                    }
                }
                tmem_st16(s_col + h32 * 16, pw);
            }
            l += psum;
            }  // two-pass path
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if ((threadIdx.x & 31) == 0) mbar_arrive(bar(BAR_P_FULL + sb));
            if (r == 0 && jj < 50) TRACE(350 + jj);
        }
        if (!ok) fail_timeout(a, abort, 3);
        if (ok && n > 0) {
            ok = mbar_wait(bar(BAR_V_EMPTY + (n - 1) % C::NSTAGE), s_done_parity(n - 1, C::NSTAGE), abort, kWaitBudget);
            if (!ok) fail_timeout(a, abort, 4);
            tc_fence_after();
        }
        // ---- epilogue ----
        if (r == 0) TRACE(10);
        const bool have_o = ok && n > 0;
        if (omode != OUT_THREADS) {
            // O (or O / l) of this warp's lane quarter -> swizzled boxes -> copy engine
            const bool split = a.n_splits > 1;
            const bool f32 = split || a.out_dtype == EKV_DTYPE_F32;
            const float inv = split ? 1.0f : ((have_o && l > 0.0f) ? 1.0f / l : 0.0f);
            int64_t unit = 0;
            if (split) {
                unit = (((int64_t)pl.b * a.pool.kv_heads + pl.g) * n_qtiles + pl.qt) * a.n_splits + pl.split;
                if (row_ok) {
                    float *wml = a.ws_ml + (unit * kBM + r) * 2;
                    wml[0] = have_o ? m_used : -INFINITY;
                    wml[1] = have_o ? l : 0.0f;
                }
            }
            // the host picks a copy-engine route only for head dims that are whole 64-column blocks
            if constexpr (D % 64 == 0)
                epilogue_o_tma(a, pl.qrow0, pl.rows_valid, pl.g, pl.b, &omap, omode, smem + C::OFF_K, warp, lane,
                               tmem + lane_base + (uint32_t)C::O_COL, 0, D, have_o, inv, f32, unit, 1);
        } else if (a.n_splits > 1) {
            const int64_t unit = (((int64_t)pl.b * a.pool.kv_heads + pl.g) * n_qtiles + pl.qt) * a.n_splits + pl.split;
            float *wo = a.ws_o + (unit * kBM + r) * D;
            float *wml = a.ws_ml + (unit * kBM + r) * 2;
#pragma unroll 1
            for (int c0 = 0; c0 < D; c0 += 16) {
                uint32_t rr[16];
                if (have_o) {
                    tmem_load16(tmem + lane_base + (uint32_t)(C::O_COL + c0), rr);
                } else {
#pragma unroll
                    for (int i = 0; i < 16; ++i) rr[i] = 0u;
                }
                if (row_ok) {
#pragma unroll
                    for (int i = 0; i < 16; i += 4)
                        *(float4 *)(wo + c0 + i) = make_float4(__uint_as_float(rr[i]), __uint_as_float(rr[i + 1]),
                                                               __uint_as_float(rr[i + 2]), __uint_as_float(rr[i + 3]));
                }
            }
            if (row_ok) {
                wml[0] = have_o ? m_used : -INFINITY;
                wml[1] = have_o ? l : 0.0f;
            }
        } else {
            // O/l (bf16 or f32) -> shared staging row r -> each warp writes whole rows with
            // consecutive 16-byte lanes (the K/V stages are idle once the last P.V has landed).
            const float inv = (have_o && l > 0.0f) ? 1.0f / l : 0.0f;
            const bool f32 = a.out_dtype == EKV_DTYPE_F32;
            uint8_t *orow = smem + C::OFF_K + r * C::OSTR;
            constexpr int EC = (D % 32 == 0) ? 32 : 16;  // columns per TMEM load
#pragma unroll 2
            for (int c0 = 0; c0 < D; c0 += EC) {
                uint32_t rr[32];
                if (have_o) {
                    if constexpr (EC == 32) {
                        tmem_load32(tmem + lane_base + (uint32_t)(C::O_COL + c0), rr);
                    } else {
                        uint32_t (&r16)[16] = *reinterpret_cast<uint32_t (*)[16]>(rr);
                        tmem_load16(tmem + lane_base + (uint32_t)(C::O_COL + c0), r16);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < EC; ++i) rr[i] = 0u;
                }
                if (f32) {
#pragma unroll
                    for (int i = 0; i < EC; i += 4)
                        *(float4 *)(orow + (c0 + i) * 4) =
                            make_float4(__uint_as_float(rr[i]) * inv, __uint_as_float(rr[i + 1]) * inv,
                                        __uint_as_float(rr[i + 2]) * inv, __uint_as_float(rr[i + 3]) * inv);
                } else {
#pragma unroll
                    for (int i0 = 0; i0 < EC; i0 += 8) {
                        uint32_t w[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const __nv_bfloat162 b2 = __floats2bfloat162_rn(__uint_as_float(rr[i0 + 2 * i]) * inv,
                                                                            __uint_as_float(rr[i0 + 2 * i + 1]) * inv);
                            w[i] = *(const uint32_t *)&b2;
                        }
                        *(uint4 *)(orow + (c0 + i0) * 2) = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                }
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");  // the 4 softmax warps only
            const int row_bytes = D * (f32 ? 4 : 2);
            for (int rw = warp; rw < pl.rows_valid; rw += 4) {
                const int qrw = pl.qrow0 + rw;
                const int tw = qrw / a.group;
                const int hw = pl.g * a.group + (qrw - tw * a.group);
                uint8_t *dst = (uint8_t *)a.out + ((((int64_t)pl.b * a.q_tokens + tw) * a.q_heads + hw) * D) * (f32 ? 4 : 2);
                const uint8_t *srow = smem + C::OFF_K + rw * C::OSTR;
                for (int o = lane * 16; o < row_bytes; o += 32 * 16) *(uint4 *)(dst + o) = *(const uint4 *)(srow + o);
            }
        }
    }
    if (threadIdx.x == 0) {
        TRACE(11);
        TRACE_CLK(21);
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == C::MMA_WARP) tmem_dealloc(tmem, C::TMEM_COLS);
    if (threadIdx.x == 0) TRACE(12);
    __syncthreads();
    trace_flush();
}

// Combine the per-split partial outputs: O = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s.
// One warp per query row: lane s < n_splits reads split s's (m, l); the row's D floats of every
// split are read as consecutive float4s across the lanes (coalesced), the output written likewise.
constexpr int kMergeWarps = 8;

template <int D>
__global__ void __launch_bounds__(kMergeWarps * 32) merge_splits_kernel(const AttnArgs a, int n_qtiles) {
    static_assert(D % 4 == 0, "float4 columns");
    constexpr int BPT = kBM / kMergeWarps;  // blocks per 128-row tile: every row gets its own warp
    const int qt = blockIdx.x / BPT, g = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int64_t unit0 = (((int64_t)b * a.pool.kv_heads + g) * n_qtiles + qt) * a.n_splits;
    const bool f32 = a.out_dtype == EKV_DTYPE_F32;
    {
        const int r = (blockIdx.x % BPT) * kMergeWarps + warp;
        const int qr = qt * kBM + r;
        if (qr >= a.q_tokens * a.group) return;
        const int t = qr / a.group;
        const int h = g * a.group + (qr - t * a.group);
        float ms = -INFINITY, ls = 0.0f;
        if (lane < a.n_splits) {
            ms = a.ws_ml[((unit0 + lane) * kBM + r) * 2];
            ls = a.ws_ml[((unit0 + lane) * kBM + r) * 2 + 1];
        }
        float mmax = ms;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mmax = fmaxf(mmax, __shfl_xor_sync(0xffffffffu, mmax, o));
        const float wv = (ms == -INFINITY) ? 0.0f : ex2(ms - mmax);
        float wsum = wv * ls;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
        const float inv = wsum > 0.0f ? 1.0f / wsum : 0.0f;
        const int64_t obase = (((int64_t)b * a.q_tokens + t) * a.q_heads + h) * D;
        for (int u = lane; u < D / 4; u += 32) {
            // every split's float4 in flight before the first use
            float4 o[kMaxSplits];
#pragma unroll
            for (int sp = 0; sp < kMaxSplits; ++sp)
                if (sp < a.n_splits) o[sp] = *(const float4 *)(a.ws_o + ((unit0 + sp) * kBM + r) * D + 4 * u);
            float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
            for (int sp = 0; sp < kMaxSplits; ++sp) {
                const float w = __shfl_sync(0xffffffffu, wv, sp);
                if (sp >= a.n_splits || w == 0.0f) continue;
                acc.x += w * o[sp].x;
                acc.y += w * o[sp].y;
                acc.z += w * o[sp].z;
                acc.w += w * o[sp].w;
            }
            acc.x *= inv;
            acc.y *= inv;
            acc.z *= inv;
            acc.w *= inv;
            if (f32) {
                *(float4 *)((float *)a.out + obase + 4 * u) = acc;
            } else {
                uint2 pk;
                pk.x = (uint32_t)f32_to_bf16_bits(acc.x) | ((uint32_t)f32_to_bf16_bits(acc.y) << 16);
                pk.y = (uint32_t)f32_to_bf16_bits(acc.z) | ((uint32_t)f32_to_bf16_bits(acc.w) << 16);
                *(uint2 *)((uint16_t *)a.out + obase + 4 * u) = pk;
            }
        }
    }
}

int sm_count() {
    int dev = 0, n = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

int choose_splits(int64_t units, int max_tiles) { return choose_split_count(units, max_tiles, sm_count()); }

template <int D, bool Q8>
int launch_impl(AttnArgs a, cudaStream_t s, size_t ws_bytes) {
    using C = TcCfg<D, Q8>;
    static int attr_done[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr_done[dev]) {
        if (cudaFuncSetAttribute(attn_tc_kernel<D, Q8>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) !=
            cudaSuccess)
            return EKV_ERR_CUDA;
        attr_done[dev] = 1;
    }
    const int bt = a.pool.block_tokens;
    if (C::BN % bt != 0 && bt % C::BN != 0) return EKV_ERR_UNSUPPORTED;  // blocks must tile key tiles
    if constexpr (!Q8 && C::BN == 128) {
        // Units of at most 64 query rows (GR00T's 17 queries x 1 head): several per CTA, so that a
        // call of thousands of small (request, head) units runs a few CTAs per SM instead of one CTA
        // (and its set-up) per unit. Only when the units outnumber the SMs; no key splits.
        const int rpu = a.q_tokens * a.group;
        const int64_t n_units = (int64_t)a.n_batch * a.pool.kv_heads;
        if (2 * rpu <= kBM && n_units > sm_count() && !(a.mask_flags & kVisWordFlags)) {
            a.pack = std::min(kMaxPack, kBM / rpu);
            a.n_splits = 1;
            const int64_t ctas = (n_units + a.pack - 1) / a.pack;
            if (ctas > 0x7fffffff) return EKV_ERR_INVALID_ARG;
            CUtensorMap omap;
            std::memset(&omap, 0, sizeof(omap));
            static int pack_attr_done[64] = {0};
            if (dev < 64 && !pack_attr_done[dev]) {
                if (cudaFuncSetAttribute(attn_tc_kernel<D, Q8, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::SMEM) != cudaSuccess)
                    return EKV_ERR_CUDA;
                pack_attr_done[dev] = 1;
            }
            attn_tc_kernel<D, Q8, true><<<dim3((unsigned)ctas, 1, 1), C::THREADS, C::SMEM, s>>>(a, 1, omap, OUT_THREADS);
            if (cudaGetLastError() != cudaSuccess) return EKV_ERR_CUDA;
            note_launches(1);
            return EKV_OK;
        }
    }
    const int n_qtiles = (a.q_tokens * a.group + kBM - 1) / kBM;
    const int64_t units = (int64_t)a.n_batch * a.pool.kv_heads * n_qtiles;
    if (a.n_splits == 0) {
        const int max_prefix = a.pool.max_blocks_per_seq * a.pool.block_tokens;
        const int max_tiles = (max_prefix + C::BN - 1) / C::BN + (a.suffix_len + C::BN - 1) / C::BN;
        int sp = choose_splits(units, max_tiles);
        const size_t per_split = (size_t)units * kBM * (D + 2) * sizeof(float);
        while (sp > 1 && per_split * sp > ws_bytes) --sp;
        float *ws = a.ws_o;
        a.n_splits = sp;
        a.ws_o = ws;
        a.ws_ml = ws + (size_t)units * sp * kBM * D;
    }
    if (a.n_splits < 1) a.n_splits = 1;
    if ((int64_t)n_qtiles * a.n_splits > 0x7fffffff || a.pool.kv_heads > 65535 || a.n_batch > 65535)
        return EKV_ERR_INVALID_ARG;
    dim3 grid((unsigned)(n_qtiles * a.n_splits), (unsigned)a.pool.kv_heads, (unsigned)a.n_batch);
    CUtensorMap omap;
    const int omode = make_out_map(a, D, units, &omap);
    attn_tc_kernel<D, Q8><<<grid, C::THREADS, C::SMEM, s>>>(a, n_qtiles, omap, omode);
    if (cudaGetLastError() != cudaSuccess) return EKV_ERR_CUDA;
    note_launches(1);
    if (a.n_splits > 1) {
        merge_splits_kernel<D><<<dim3(n_qtiles * (kBM / kMergeWarps), a.pool.kv_heads, a.n_batch), kMergeWarps * 32, 0, s>>>(
            a, n_qtiles);
        if (cudaGetLastError() != cudaSuccess) return EKV_ERR_CUDA;
        note_launches(1);
    }
    return EKV_OK;
}

template <bool Q8>
int dispatch(const AttnArgs &a, cudaStream_t s, size_t ws) {
    switch (a.pool.head_dim) {
        case 64: return launch_impl<64, Q8>(a, s, ws);
        case 128: return launch_impl<128, Q8>(a, s, ws);
        case 256: return launch_impl<256, Q8>(a, s, ws);
        default: break;
    }
    if (!Q8 && a.pool.head_dim == 48) return launch_impl<48, false>(a, s, ws);
    return EKV_ERR_UNSUPPORTED;
}

}  // namespace

#ifdef EKV_TRACE
}  // namespace ekv
extern "C" int ekv_debug_set_trace(unsigned long long *buf) {
    if (cudaMemcpyToSymbol(ekv::c_trace, &buf, sizeof(buf)) != cudaSuccess) return -2;
    if (ekv::pair_debug_set_trace(buf)) return -2;
    if (ekv::pair128_debug_set_trace(buf)) return -2;
    if (ekv::heads_debug_set_trace(buf)) return -2;
    return ekv::project_debug_set_trace(buf);
}
namespace ekv {
#endif

size_t attention_tc_workspace(const PoolView &p, const ekv_attn_params &prm, int max_prefix, int sms) {
    if (prm.q_heads <= 0 || p.kv_heads <= 0 || prm.q_heads % p.kv_heads) return 0;
    const int group = prm.q_heads / p.kv_heads;
    const int bn = p.head_dim > 128 ? 64 : 128;
    const int n_qtiles = (prm.q_tokens * group + kBM - 1) / kBM;
    const int64_t units = (int64_t)prm.n_batch * p.kv_heads * n_qtiles;
    const int max_tiles = (max_prefix + bn - 1) / bn + (prm.suffix_len + bn - 1) / bn;
    const int sp = choose_split_count(units, max_tiles, sms);
    size_t need = sp <= 1 ? 0 : (size_t)units * sp * kBM * (p.head_dim + 2) * sizeof(float);
    if (p.head_dim == 256) {  // the CTA-pair kernel's choice (pairs of 128-row tiles)
        const int n_pairs = (prm.q_tokens * group + 2 * kBM - 1) / (2 * kBM);
        const int64_t pair_units = (int64_t)prm.n_batch * p.kv_heads * n_pairs;
        const int psp = pair_choose_splits(pair_units, max_tiles, sms);
        if (psp > 1) need = std::max(need, (size_t)pair_units * 2 * psp * kBM * (p.head_dim + 2) * sizeof(float));
        // the 128-key pair kernel's choice
        const int max_tiles128 = (max_prefix + 127) / 128 + (prm.suffix_len + 127) / 128;
        const int psp128 = pair128_choose_splits(pair_units, max_tiles128, sms);
        if (psp128 > 1)
            need = std::max(need, (size_t)pair_units * 2 * psp128 * kBM * (p.head_dim + 2) * sizeof(float));
    }
    return need;
}

int launch_merge_splits(const AttnArgs &a, int n_qtiles, cudaStream_t s) {
    const dim3 grid((unsigned)(n_qtiles * (kBM / kMergeWarps)), (unsigned)a.pool.kv_heads, (unsigned)a.n_batch);
    switch (a.pool.head_dim) {
        case 48: merge_splits_kernel<48><<<grid, kMergeWarps * 32, 0, s>>>(a, n_qtiles); break;
        case 64: merge_splits_kernel<64><<<grid, kMergeWarps * 32, 0, s>>>(a, n_qtiles); break;
        case 128: merge_splits_kernel<128><<<grid, kMergeWarps * 32, 0, s>>>(a, n_qtiles); break;
        case 256: merge_splits_kernel<256><<<grid, kMergeWarps * 32, 0, s>>>(a, n_qtiles); break;
        default: return EKV_ERR_UNSUPPORTED;
    }
    if (cudaGetLastError() != cudaSuccess) return EKV_ERR_CUDA;
    note_launches(1);
    return EKV_OK;
}

int launch_attention_tc(const AttnArgs &a, cudaStream_t s, TcKernel k) {
    // a.n_splits == 0 means: a workspace was given at a.ws_o, choose the split count.
    size_t ws = 0;
    if (a.n_splits == 0) ws = (size_t)-1;  // the C-ABI checked the size against the maximum need
    // head_dim 256: each SM of a pair copies (bf16) or dequantises (Q8_0) half of every tile, and
    // each K/V byte crosses L2 -> SM twice per request instead of four times
    if (k == TcKernel::Heads) return launch_attention_heads(a, s, sm_count());
    if (k == TcKernel::Auto && heads_fits(a) && heads_units(a) * 4 >= sm_count()) {
        const int rc = launch_attention_heads(a, s, sm_count());
        if (rc != EKV_ERR_UNSUPPORTED) return rc;  // else nothing was enqueued: the kernels below
    }
    const bool pair = a.pool.head_dim == 256 && k != TcKernel::OneCta;
    if (pair && k == TcKernel::Pair) return launch_attention_pair128(a, s, ws, sm_count());
    // bf16 pools: the 128-key pair kernel for calls of at most 8 (request, 256-row tile) pair units, where
    // its fewer, larger MMA groups shorten a latency-bound call (batch 1: 14.8 against 15.3 us); from 16
    // units on the 64-key kernel is ahead (2-4% at batch 16-256). Q8_0 pools keep the 64-key pair kernel:
    // with Q in shared memory, the N = 128 MMAs' operand reads leave too little shared-memory bandwidth
    // for the in-place dequantisation of every tile.
    const int64_t pair_units = (int64_t)a.n_batch * a.pool.kv_heads * ((a.q_tokens * a.group + 255) / 256);
    if (pair && k == TcKernel::Auto && a.pool.dtype == EKV_DTYPE_BF16 && pair_units <= 8) {
        const int rc = launch_attention_pair128(a, s, ws, sm_count());
        if (rc != EKV_ERR_UNSUPPORTED) return rc;
    }
    if (pair) return launch_attention_pair(a, s, ws, sm_count());
    return a.pool.dtype == EKV_DTYPE_Q8_0 ? dispatch<true>(a, s, ws) : dispatch<false>(a, s, ws);
}

}  // namespace ekv
