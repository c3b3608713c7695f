// ekv_attn_heads.cu -- masked attention over the paged bf16 pool for multi-head calls with few query
// tokens per head: GR00T-N1.7's DiT action head, 17 queries x 32 heads of 48 dims cross-attending a
// cached 300-token backbone and self-attending among the 17 (models/groot_n1.cpp:328-364, masks
// :708-718), on tcgen05 tensor cores.
//
// Such a call is a stream of K/V bytes with little arithmetic per byte: each (request, head) has only
// 17 query rows, so one 128-row query tile per head would leave the MMA 13% full and pay a CTA's
// set-up for a handful of key tiles, and a pool block holds only bt x 96 bytes per head, far below
// the size at which the copy engine reaches its bandwidth. This kernel therefore works on units of
// four heads of one request, one head per TMEM lane quarter (query token t of head h is row
// 32h + t, so a unit needs q_tokens <= 32 and an MHA call), and copies the four heads' K (or V)
// rows of a block with ONE bulk copy: in the pool the tiles of consecutive heads of one (layer,
// block, K|V) are adjacent. A K stage then holds 256 rows -- for each block run r of the tile and
// head h, bt rows -- in one uniform K-major layout, so per 64-key tile:
//
//   S = Q K_stage^T   M = 128 (the four heads' query rows), N = 256 stage rows, K = D: D/16 MMAs
//                     for all four heads; column c of S is stage row c, and head h reads only the
//                     columns of its own rows in its own lane quarter
//   O += P_h V_h      per head h: M = 128, N = D, K = 64 keys (four MMAs of 16 keys); A = P_h in
//                     tensor memory, B = head h's V rows of the stage
//
// P_h has its own 32 columns of tensor memory, written by head h's softmax warps in quarter h and zero
// in the other quarters (written once at start), so one O accumulator collects every head's P_h V_h
// in the head's own rows. An MMA issue waits for the previous MMA to start, so every MMA group is
// issued back to back with precomputed descriptors, and S uses N = 256 (about 128 cycles per MMA,
// against about 150 cycles of issue cost for any small MMA).
//
// Tensor memory (512 columns): S [256] | P [4 heads][32 columns of bf16 pairs] | O [2][64]
// (double-buffered across units). Shared memory: Q [2 units][128 rows][D] | K stages [NS][256 rows] |
// V stages | barriers | exchange | unit plans [4].
//
// The kernel is persistent: min(units, SMs) CTAs each walk units blockIdx.x, blockIdx.x + gridDim.x,
// ...; every role iterates the same units, so the copy engine streams the next unit's K/V while the
// current unit's softmax and epilogue run. Warps: 0 TMEM allocation and MMA issue (one thread), 1 K
// feeder, 2 V feeder, 3 planner (per unit: sequence, visible key range, block ids -> shared memory) and
// Q loader, 4-11 softmax (warp w: head w & 3 of the unit, keys [32 ((w - 4) >> 2), +32) of each tile,
// lane = query token; the two warps of a head swap row maxima per tile), 12-15 epilogue (warp e: head
// e & 3, O / l of a unit once its last P.V is done, while the softmax warps go on to the next unit).
//
// Every wait is bounded; on expiry the CTA records DEV_ERR_TIMEOUT, raises its abort flag and unwinds
// after its copies and MMAs in flight have finished.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cstring>

#include "ekv_attn_common.cuh"
#include "ekv_device.cuh"
#include "ekv_internal.h"
#include "ekv_sm100.cuh"

namespace ekv {
namespace {

using namespace sm100;

constexpr int kHG = 4;         // heads per unit, one per TMEM lane quarter
constexpr int kHBN = 64;       // keys per tile
constexpr int kHMaxBlk = 64;   // block ids cached per unit plan (further ones are looked up directly)

template <int D>
struct HCfg {
    static constexpr int G = kHG, BN = kHBN, ROWS = G * BN;  // stage rows: 4 heads x 64 keys
    static constexpr int W = (D * 2) % 128 == 0 ? 128 : ((D * 2) % 64 == 0 ? 64 : 32);
    static constexpr uint32_t LAYOUT = W == 128 ? 2u : (W == 64 ? 4u : 6u);
    static constexpr int ROWB = 2 * D;                 // bytes per bf16 row
    static constexpr uint32_t SBO = 16u * D;           // bytes per 8-row group of a tile
    static constexpr int STAGE = ROWS * ROWB;          // one K (or V) stage
    static constexpr int Q_BYTES0 = kBM * ROWB;
    // K/V stages that fit beside two Q buffers, barriers, exchange and plans (at most 4)
    static constexpr int NS_FIT = (232448 - 1024 - 512 - 8 * kBM * 4 - 4 * (64 + kHMaxBlk * 4) - 2 * Q_BYTES0) / (2 * STAGE);
    static constexpr int NS = NS_FIT > 4 ? 4 : NS_FIT;
    static_assert(NS >= 2, "stage ring");
    static constexpr int Q_BYTES = kBM * ROWB;
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = 2 * Q_BYTES;
    static constexpr int OFF_V = OFF_K + NS * STAGE;
    static constexpr int OFF_BAR = OFF_V + NS * STAGE;
    static constexpr int BAR_BYTES = 512;
    static constexpr int OFF_XCH = OFF_BAR + BAR_BYTES;  // row maxima [2 parity][2 halves][128], sums [2 units][2][128]
    static constexpr int OFF_PLAN = OFF_XCH + 8 * kBM * 4;
    static constexpr int SMEM = OFF_PLAN + 4 * (64 + kHMaxBlk * 4) + 1024;  // + alignment slack
    static constexpr int SMW = 8;                       // softmax warps
    // The MMA-issuing warp is warp 0: a sub-partition issues from its lowest-numbered ready warp first,
    // and the issuing thread must not wait behind the softmax warps' long arithmetic runs.
    static constexpr int MMA_WARP = 0, KF_WARP = 1, VF_WARP = 2, Q_WARP = 3, SM_WARP0 = 4, EPI_WARP0 = 12;
    static constexpr int EPW = 4;                       // epilogue warps, one per TMEM lane quarter
    static constexpr int THREADS = (EPI_WARP0 + EPW) * 32;
    static constexpr int S_COL = 0, P_COL = ROWS, O_COL = P_COL + G * BN / 2, O_STRIDE = 64;
    static constexpr int KS = D / 16;                   // K steps of S
    static_assert(O_COL + 2 * O_STRIDE <= 512, "TMEM budget");
    static_assert(D % 16 == 0 && D <= O_STRIDE, "head_dim");
    static_assert(SMEM <= 232448, "shared-memory budget");
    static constexpr int NCH = D * 2 / W;               // swizzle chunks per row
    // byte offset of K step kk (16 elements) in the Q buffer [chunk][128 rows][W]
    __device__ static constexpr uint32_t qstep(int kk) {
        return (uint32_t)((kk * 32) / W) * (uint32_t)(kBM * W) + (uint32_t)((kk * 32) % W);
    }
    // byte offset of K step kk (16 elements) in a K-major swizzled tile row
    __device__ static constexpr uint32_t kstep(int kk) {
        return (uint32_t)((kk * 32) / W) * (8u * W) + (uint32_t)((kk * 32) % W);
    }
};

enum {
    HB_KF = 0,     // [4] K stage landed (feeder: expected bytes)
    HB_VF = 4,     // [4] V stage landed
    HB_KE = 8,     // [4] S(t) done: K stage free, S readable (commit)
    HB_VE = 12,    // [4] P.V(t) done: V stage free, P buffers free, O updated (commit)
    HB_SE = 16,    // the softmax warps have read S(t): the S columns may be overwritten
    HB_PF = 17,    // the softmax warps have written P(t)
    HB_QF = 18,    // [2] Q of a unit staged
    HB_QE = 20,    // [2] the last S of the unit that used a Q buffer is done (commit)
    HB_OE = 22,    // [2] the epilogue warps have read an O buffer and its row sums
    HB_LF = 24,    // [4] unit plan written
    HB_LE = 28,    // [4] unit plan released by its readers
    HB_DONE = 32,  // every MMA of the CTA finished
    HB_XCH = 33,   // [4] the two softmax warps of a head swap row maxima
    HB_LR = 37,    // [2] the softmax warps have written a unit's row sums
    HB_OF = 39,    // [2] a unit's last P.V is done (commit), or the unit has no tiles
    HB_N = 41
};
static_assert(HB_N * 8 + 16 <= 512, "barrier block");
constexpr int kPlanReaders = 15;  // K feeder, V feeder, MMA thread, 8 softmax warps, 4 epilogue warps

// Per-unit schedule written by the planner warp (shared memory, 4 slots).
struct HPlan {
    int32_t b, hg, seq, n_prefix, prefix_valid, span_b, span_e, kbeg;
    int32_t np, ns, blk0, nblk, pad[4];
    int32_t blk[kHMaxBlk];
};
static_assert(sizeof(HPlan) == 64 + kHMaxBlk * 4, "plan slot");

// Stage row (= S column) of key k (0..63 of the tile) of head h: prefix tiles hold, for each run of
// bt keys, the four heads' bt rows; suffix tiles the four heads' slot tiles of suffix_rows rows.
__device__ __forceinline__ int heads_row(bool suffix, int h, int k, int bt_shift, int suffix_rows) {
    return suffix ? h * suffix_rows + k
                  : ((k >> bt_shift) * kHG + h) * (1 << bt_shift) + (k & ((1 << bt_shift) - 1));
}

__device__ __forceinline__ void heads_fail(const AttnArgs &a, volatile int *abort, int where) {
    *abort = 1;
    report_error(a.pool.status, DEV_ERR_TIMEOUT, where, blockIdx.x, 0);
}

// ---- planner: unit u of this CTA (global unit blockIdx.x + u * gridDim.x) ----
__device__ __forceinline__ void heads_plan(const AttnArgs &a, HPlan *pl, int gu, int n_hg, int lane) {
    const PoolView &p = a.pool;
    const int b = gu / n_hg, hg = gu - b * n_hg;
    const SeqKeys sk = resolve_seq(p, a.use_prefix, a.seq_ids, a.prefix_len, a.prefix_valid, a.span_begin, a.span_end, b);
    if (lane == 0 && !sk.ok) report_error(p.status, DEV_ERR_BAD_SEQ, b, a.seq_ids[b], 5);
    int kb = 0, ke = sk.prefix_valid, kbeg = 0, np = 0;
    if (a.mask_flags & EKV_MASK_SPAN_ONLY) {
        kb = max(kb, sk.span_b);
        ke = min(ke, sk.span_e);
    }
    if (a.mask_flags & EKV_MASK_SPAN_EXCLUDE) {  // a span at either end of the range removes it
        if (sk.span_b <= kb) kb = max(kb, sk.span_e);
        if (sk.span_e >= ke) ke = min(ke, sk.span_b);
    }
    if (a.mask_flags & EKV_MASK_BLOCK_CAUSAL) {
        const int qc_lo = a.q_chunk0, qc_hi = a.q_chunk0 + (a.q_tokens - 1) / a.chunk_tokens;
        kb = max(kb, (qc_lo - a.window_chunks + 1) * a.chunk_stride);
        ke = min(ke, (qc_hi + 1) * a.chunk_stride);
    }
    if (sk.ok && ke > kb) {
        kbeg = kb / kHBN * kHBN;
        np = (ke - kbeg + kHBN - 1) / kHBN;
    }
    const int ns = (sk.ok && a.suffix_len > 0) ? 1 : 0;
    const int bt = p.block_tokens;
    const int blk0 = kbeg / bt;
    const int k_end = min(kbeg + np * kHBN, sk.n_prefix);
    const int nblk = np > 0 && k_end > kbeg ? min(kHMaxBlk, (k_end + bt - 1) / bt - blk0) : 0;
    for (int i = lane; i < nblk; i += 32) pl->blk[i] = lookup_block(p, sk.seq, blk0 + i);
    if (lane == 0) {
        pl->b = b;
        pl->hg = hg;
        pl->seq = sk.seq;
        pl->n_prefix = sk.n_prefix;
        pl->prefix_valid = sk.prefix_valid;
        pl->span_b = sk.span_b;
        pl->span_e = sk.span_e;
        pl->kbeg = kbeg;
        pl->np = np;
        pl->ns = ns;
        pl->blk0 = blk0;
        pl->nblk = nblk;
    }
}

// ---- feeder: tile j of a unit, K (kv = 0) or V (kv = 1) of its four heads into one stage. Prefix
// tile: one copy per block run of bt keys (the four heads' tiles of that block, adjacent in the
// pool) to stage row run * 4 * bt; a run past the sequence is zero-filled. Suffix tile: the four
// heads' slot tiles in one copy. ----
template <int D>
__device__ __forceinline__ void heads_produce(const AttnArgs &a, const HPlan &pl, int j, int kv, uint8_t *stage,
                                              uint32_t bar_full, int lane) {
    using C = HCfg<D>;
    const PoolView &p = a.pool;
    const uint8_t *src = nullptr;
    uint32_t bytes = 0, dst = 0, zlo = 0, zhi = 0;
    if (j < pl.np) {
        const int bt = p.block_tokens, nrun = C::BN / bt;
        const uint32_t run_bytes = (uint32_t)(C::G * bt * C::ROWB);
        if (lane < nrun) {
            const int kr = pl.kbeg + j * C::BN + lane * bt;
            dst = (uint32_t)lane * run_bytes;
            int blk = -1;
            if (kr < pl.n_prefix) {
                const int idx = kr >> p.bt_shift;
                const int ci = idx - pl.blk0;
                blk = (ci >= 0 && ci < pl.nblk) ? pl.blk[ci] : lookup_block(p, pl.seq, idx);
            }
            if (blk >= 0) {
                src = p.prefix + prefix_tile_index(p, a.layer, blk, kv, pl.hg * C::G) * p.tile_bytes;
                bytes = run_bytes;
            } else {
                zlo = dst;
                zhi = dst + run_bytes;
            }
        }
    } else if (lane == 0) {
        src = p.suffix + suffix_tile_index(p, a.layer, pl.seq, kv, pl.hg * C::G) * p.suffix_tile_bytes;
        bytes = (uint32_t)(C::G * p.suffix_tile_bytes);
    }
    const uint32_t need_zero = __ballot_sync(0xffffffffu, zhi > zlo);
    if (need_zero) {
        for (uint32_t m = need_zero; m; m &= m - 1) {
            const int s = __ffs(m) - 1;
            const uint32_t z0 = __shfl_sync(0xffffffffu, zlo, s), z1 = __shfl_sync(0xffffffffu, zhi, s);
            for (uint32_t o = z0 + lane * 16; o < z1; o += 32 * 16) *(uint4 *)(stage + o) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async();
    }
    __syncwarp();
    const uint32_t total = __reduce_add_sync(0xffffffffu, src ? bytes : 0u);
    if (lane == 0) {
        if (total) mbar_arrive_expect_tx(bar_full, total);
        else mbar_arrive(bar_full);
    }
    __syncwarp();
    if (src) bulk_g2s(smem_addr(stage + dst), src, bytes, bar_full);
}

__device__ __forceinline__ bool heads_xsync(uint32_t xbar, int use, volatile int *abort, long long budget) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(xbar);
    return mbar_wait(xbar, (uint32_t)use & 1u, abort, budget);
}

template <int D>
__global__ void __launch_bounds__(HCfg<D>::THREADS, 1)
    attn_heads_kernel(const AttnArgs a, int n_units, const __grid_constant__ CUtensorMap qmap) {
    using C = HCfg<D>;
    constexpr int NS = C::NS, G = C::G, BN = C::BN;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    uint8_t *sQ = smem + C::OFF_Q;
    uint8_t *sK = smem + C::OFF_K;
    uint8_t *sV = smem + C::OFF_V;
    uint64_t *bars = (uint64_t *)(smem + C::OFF_BAR);
    uint32_t *tmem_holder = (uint32_t *)(bars + HB_N);
    volatile int *abort = (volatile int *)(bars + HB_N + 1);
    HPlan *plans = (HPlan *)(smem + C::OFF_PLAN);
    const uint32_t bar0 = smem_addr(bars);
    auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const long long budget = a.wait_budget;
    const int n_hg = a.pool.kv_heads / G;
    const int U = ((int)blockIdx.x < n_units) ? (n_units - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;

    if (threadIdx.x == 0) {
        trace_init();
        TRACE(0);
        for (int s = 0; s < 4; ++s) {
            mbar_init(bar(HB_KF + s), 1);
            mbar_init(bar(HB_VF + s), 1);
            mbar_init(bar(HB_KE + s), 1);
            mbar_init(bar(HB_VE + s), 1);
            mbar_init(bar(HB_LF + s), 1);
            mbar_init(bar(HB_LE + s), kPlanReaders);
            mbar_init(bar(HB_XCH + s), 2);
        }
        mbar_init(bar(HB_SE), C::SMW);
        mbar_init(bar(HB_PF), C::SMW);
        for (int s = 0; s < 2; ++s) {
            mbar_init(bar(HB_QF + s), 1);
            mbar_init(bar(HB_QE + s), 1);
            mbar_init(bar(HB_OE + s), C::EPW);
            mbar_init(bar(HB_LR + s), C::SMW);
            mbar_init(bar(HB_OF + s), 1);
        }
        mbar_init(bar(HB_DONE), 1);
        *abort = 0;
        mbar_init_fence();
    }
    if (warp == C::MMA_WARP) tmem_alloc(smem_addr(tmem_holder), 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    if (threadIdx.x == 0) TRACE(1);

    if (warp == C::Q_WARP) {
        // ---- per unit: the plan (sequence, visible key range, block ids), then Q by the copy engine: row
        // 32h + t of swizzle chunk c = token t of head 4 hg + h (zero past q_tokens), the MMA's K-major
        // A operand laid out [chunk][128 rows][W bytes] ----
        for (int u = 0; u < U; ++u) {
            const int slot = u & 3;
            if (u >= 4 && !mbar_wait_backoff(bar(HB_LE + slot), (uint32_t)((u >> 2) - 1) & 1u, abort, budget)) {
                if (lane == 0) heads_fail(a, abort, 10);
                break;
            }
            const int gu = (int)blockIdx.x + u * (int)gridDim.x;
            heads_plan(a, plans + slot, gu, n_hg, lane);
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(HB_LF + slot));
            if (lane == 0 && u < 20) TRACE(480 + u);
            if (u >= 2 && !mbar_wait_backoff(bar(HB_QE + (u & 1)), (uint32_t)((u - 2) >> 1) & 1u, abort, budget)) {
                if (lane == 0) heads_fail(a, abort, 11);
                break;
            }
            const int b = gu / n_hg, hg = gu - b * n_hg;
            if (lane == 0) {  // four heads x the row's swizzle chunks, one tensor-map box of 32 tokens each
                const uint32_t qb = smem_addr(sQ + (u & 1) * C::Q_BYTES), qf = bar(HB_QF + (u & 1));
                mbar_arrive_expect_tx(qf, (uint32_t)C::Q_BYTES);
                for (int c = 0; c < C::NCH; ++c)
                    for (int h = 0; h < G; ++h)
                        tma_load_4d(qb + (uint32_t)(c * kBM * C::W + h * 32 * C::W), &qmap, c * (C::W / 2), hg * G + h, 0, b,
                                    qf);
            }
            __syncwarp();
            if (lane == 0 && u < 20) TRACE(450 + u);
        }
    } else if (warp == C::KF_WARP || warp == C::VF_WARP) {
        const int kv = warp - C::KF_WARP;
        uint8_t *stages = kv ? sV : sK;
        const int b_full = kv ? HB_VF : HB_KF, b_empty = kv ? HB_VE : HB_KE;
        int t = 0, issued = 0;
        bool ok = true;
        for (int u = 0; ok && u < U; ++u) {
            const int slot = u & 3;
            if (!mbar_wait_backoff(bar(HB_LF + slot), (uint32_t)(u >> 2) & 1u, abort, budget)) {
                ok = false;
                break;
            }
            const HPlan &pl = plans[slot];
            const int n = pl.np + pl.ns;
            for (int j = 0; j < n; ++j, ++t) {
                const int s = t % NS;
                if (t >= NS && !mbar_wait_backoff(bar(b_empty + s), (uint32_t)(t / NS - 1) & 1u, abort, budget)) {
                    ok = false;
                    break;
                }
                heads_produce<D>(a, pl, j, kv, stages + s * C::STAGE, bar(b_full + s), lane);
                if (lane == 0 && t < 50) TRACE((kv ? 500 : 100) + t);
                issued = t + 1;
            }
            __syncwarp();
            if (ok && lane == 0) mbar_arrive(bar(HB_LE + slot));
        }
        if (!ok && lane == 0) heads_fail(a, abort, 12 + kv);
        if (lane == 0 && *abort)
            for (int tt = max(0, issued - NS); tt < issued; ++tt)
                mbar_wait_drain(bar(b_full + tt % NS), (uint32_t)(tt / NS) & 1u, budget);
    } else if (warp == C::MMA_WARP) {
        if (lane == 0) {
            const PoolView &p = a.pool;
            const int srows = p.suffix_rows;
            const uint32_t idO = idesc_f16(true, true, D);
            // P.V operands of head h, key step kk (index 4h + kk): A in tensor memory; B at a fixed offset in
            // the V stage (prefix and suffix tiles), in 16-byte units of the descriptor's address field
            uint32_t pv_a[G * 4], pv_bp[G * 4], pv_bs[G * 4];
#pragma unroll
            for (int h = 0; h < G; ++h)
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    pv_a[4 * h + kk] = tmem + (uint32_t)(C::P_COL + h * (BN / 2) + kk * 8);
                    pv_bp[4 * h + kk] = (uint32_t)(heads_row(false, h, 16 * kk, p.bt_shift, srows) / 8) * (C::SBO >> 4);
                    pv_bs[4 * h + kk] = (uint32_t)(heads_row(true, h, 16 * kk, p.bt_shift, srows) / 8) * (C::SBO >> 4);
                }
            const uint32_t idSp = idesc_f16(true, false, C::ROWS);
            const uint32_t idSs = idesc_f16(true, false, srows > 0 ? G * srows : 16);
            const int nks = (a.suffix_len + 15) / 16;  // P.V key steps of a suffix tile, per head
            bool ok = true;
            // S cursor: unit su, tile sj, global tile st (the next S to issue)
            int su = 0, sj = 0, st = 0;
            // Move the S cursor onto the next tile in a unit <= limit; units without tiles are passed (their Q
            // buffer released at once). 1: on a tile; 0: none up to limit; -1: timeout.
            auto s_find = [&](int limit) -> int {
                while (su < U && su <= limit) {
                    if (!mbar_wait(bar(HB_LF + (su & 3)), (uint32_t)(su >> 2) & 1u, abort, budget)) return -1;
                    const HPlan &pl = plans[su & 3];
                    if (sj < pl.np + pl.ns) return 1;
                    if (pl.np + pl.ns == 0) mbar_arrive(bar(HB_QE + (su & 1)));
                    ++su;
                    sj = 0;
                }
                return 0;
            };
            // S for all four heads: one MMA per K step, N = the stage's rows
            auto issue_s = [&]() -> bool {
                const HPlan &pl = plans[su & 3];
                const int s = st % NS, n = pl.np + pl.ns;
                if (st < 50) TRACE(750 + st);
                if (!mbar_wait(bar(HB_KF + s), (uint32_t)(st / NS) & 1u, abort, budget)) return false;
                if (st >= 1 && !mbar_wait(bar(HB_SE), (uint32_t)(st - 1) & 1u, abort, budget)) return false;
                if (sj == 0 && !mbar_wait(bar(HB_QF + (su & 1)), (uint32_t)(su >> 1) & 1u, abort, budget)) return false;
                tc_fence_after();
                if (st < 50) TRACE(200 + st);
                const uint64_t qd = sdesc(smem_addr(sQ + (su & 1) * C::Q_BYTES), 16, 8u * C::W, C::LAYOUT);
                const uint64_t kd = sdesc(smem_addr(sK + s * C::STAGE), 16, C::SBO, C::LAYOUT);
                const uint32_t idS = sj < pl.np ? idSp : idSs;
                uint64_t ad[C::KS], bd[C::KS];
#pragma unroll
                for (int kk = 0; kk < C::KS; ++kk) {
                    ad[kk] = qd + (C::qstep(kk) >> 4);
                    bd[kk] = kd + (C::kstep(kk) >> 4);
                }
#pragma unroll
                for (int kk = 0; kk < C::KS; ++kk) mma_ss(tmem + C::S_COL, ad[kk], bd[kk], idS, kk > 0 ? 1u : 0u);
                mma_commit(bar(HB_KE + s));                          // S(st) done, K stage free
                if (sj == n - 1) mma_commit(bar(HB_QE + (su & 1)));  // the unit's Q buffer is free
                ++sj;
                ++st;
                return true;
            };
            // P.V for each head, issued in blocks of four MMAs
            auto issue_pv = [&](int u, int j, int t, const HPlan &pl) -> bool {
                const int s = t % NS;
                if (t < 50) TRACE(800 + t);
                if (!mbar_wait(bar(HB_PF), (uint32_t)t & 1u, abort, budget)) return false;
                if (!mbar_wait(bar(HB_VF + s), (uint32_t)(t / NS) & 1u, abort, budget)) return false;
                if (j == 0 && u >= 2 && !mbar_wait(bar(HB_OE + (u & 1)), (uint32_t)((u - 2) >> 1) & 1u, abort, budget))
                    return false;
                tc_fence_after();
                if (t < 50) TRACE(250 + t);
                const uint64_t vd = sdesc(smem_addr(sV + s * C::STAGE), 8 * C::W, C::SBO, C::LAYOUT);
                const uint32_t od = tmem + (uint32_t)(C::O_COL + (u & 1) * C::O_STRIDE);
                const bool suffix = j >= pl.np;
                const int nk = suffix ? nks : BN / 16;
                uint64_t bv[G * 4];
#pragma unroll
                for (int i = 0; i < G * 4; ++i) bv[i] = vd + (suffix ? pv_bs[i] : pv_bp[i]);
                if (nk == 4) {
#pragma unroll
                    for (int h = 0; h < G; ++h)
                        mma_ts_x4<false>(od, *reinterpret_cast<const uint32_t(*)[4]>(pv_a + 4 * h),
                                         *reinterpret_cast<const uint64_t(*)[4]>(bv + 4 * h), idO,
                                         (j > 0 || h > 0) ? 1u : 0u);
                } else {  // a suffix tile of at most 48 keys: nk key steps per head, all heads back to back
                    static_assert(G == 4, "four heads per unit");
                    const uint32_t acc0 = j > 0 ? 1u : 0u;
                    if (nk == 1) {
                        const uint32_t a4[4] = {pv_a[0], pv_a[4], pv_a[8], pv_a[12]};
                        const uint64_t b4[4] = {bv[0], bv[4], bv[8], bv[12]};
                        mma_ts_x4<false>(od, a4, b4, idO, acc0);
                    } else if (nk == 2) {
                        const uint32_t a8[8] = {pv_a[0], pv_a[1], pv_a[4], pv_a[5], pv_a[8], pv_a[9], pv_a[12], pv_a[13]};
                        const uint64_t b8[8] = {bv[0], bv[1], bv[4], bv[5], bv[8], bv[9], bv[12], bv[13]};
                        mma_ts_x8(od, a8, b8, idO, acc0);
                    } else {
                        const uint32_t a4[4] = {pv_a[0], pv_a[1], pv_a[2], pv_a[4]};
                        const uint64_t b4[4] = {bv[0], bv[1], bv[2], bv[4]};
                        const uint32_t a8[8] = {pv_a[5], pv_a[6], pv_a[8], pv_a[9], pv_a[10], pv_a[12], pv_a[13], pv_a[14]};
                        const uint64_t b8[8] = {bv[5], bv[6], bv[8], bv[9], bv[10], bv[12], bv[13], bv[14]};
                        mma_ts_x4<false>(od, a4, b4, idO, acc0);
                        mma_ts_x8(od, a8, b8, idO, 1u);
                    }
                }
                mma_commit(bar(HB_VE + s));  // P.V(t) done: V stage and P buffers free, O updated
                if (t < 50) TRACE(150 + t);
                return true;
            };
            int t = 0;
            for (int u = 0; ok && u < U; ++u) {
                if (!mbar_wait(bar(HB_LF + (u & 3)), (uint32_t)(u >> 2) & 1u, abort, budget)) {
                    ok = false;
                    break;
                }
                if (u < 50) TRACE(550 + u);
                const HPlan &pl = plans[u & 3];
                const int n = pl.np + pl.ns;
                if (n == 0) {  // no tiles: the epilogue writes zeros once the unit's O buffer is free
                    if (u >= 2 && !mbar_wait(bar(HB_OE + (u & 1)), (uint32_t)((u - 2) >> 1) & 1u, abort, budget)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive(bar(HB_OF + (u & 1)));
                }
                for (int j = 0; ok && j < n; ++j, ++t) {
                    while (ok && st <= t) {  // S(t) first (its unit's plan is held)
                        ok = s_find(u) == 1;
                        if (ok) ok = issue_s();
                    }
                    if (ok && st == t + 1) {  // then S(t + 1) ahead of P.V(t), if its unit is near
                        const int r = s_find(u + 3);
                        if (r < 0) ok = false;
                        else if (r == 1) ok = issue_s();
                    }
                    if (ok) ok = issue_pv(u, j, t, pl);
                    if (ok && j == n - 1) mma_commit(bar(HB_OF + (u & 1)));  // the unit's O is complete
                }
                if (ok) mbar_arrive(bar(HB_LE + (u & 3)));
            }
            if (ok) ok = s_find(U) == 0;  // units without tiles at the end release their Q buffers
            if (!ok) heads_fail(a, abort, 14);
            mma_commit(bar(HB_DONE));
            mbar_wait_drain(bar(HB_DONE), 0, budget);
        }
        __syncwarp();
    } else if (warp >= C::EPI_WARP0) {
        // ---- epilogue: warp e = head (e & 3) of each unit (its TMEM lane quarter), lane = query token:
        // O / l -> out[b][t][head][:] once the unit's last P.V is done ----
        const int h = warp & 3;
        const uint32_t lb = ((uint32_t)(32 * h)) << 16;
        const int r = 32 * h + lane;
        const bool row_ok = lane < a.q_tokens;
        const float *lsum = (const float *)(smem + C::OFF_XCH) + 4 * kBM;
        const bool f32 = a.out_dtype == EKV_DTYPE_F32;
        bool ok = true;
        for (int u = 0; ok && u < U; ++u) {
            const int slot = u & 3;
            if (!mbar_wait(bar(HB_LF + slot), (uint32_t)(u >> 2) & 1u, abort, budget)) {
                ok = false;
                break;
            }
            const HPlan &pl = plans[slot];
            const int n = pl.np + pl.ns, b = pl.b, head = pl.hg * G + h;
            if (!mbar_wait(bar(HB_LR + (u & 1)), (uint32_t)(u >> 1) & 1u, abort, budget) ||
                !mbar_wait(bar(HB_OF + (u & 1)), (uint32_t)(u >> 1) & 1u, abort, budget)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const float l_row = lsum[((u & 1) * 2) * kBM + r] + lsum[((u & 1) * 2 + 1) * kBM + r];
            const float inv = (n > 0 && l_row > 0.0f) ? 1.0f / l_row : 0.0f;
            const uint32_t od = tmem + lb + (uint32_t)(C::O_COL + (u & 1) * C::O_STRIDE);
            uint8_t *orow = (uint8_t *)a.out +
                            (((int64_t)b * a.q_tokens + lane) * a.q_heads + head) * (int64_t)D * (f32 ? 4 : 2);
#pragma unroll
            for (int c0 = 0; c0 < D; c0 += 16) {
                uint32_t o16[16];
                if (n > 0) {
                    tmem_load16(od + (uint32_t)c0, o16);
                } else {
#pragma unroll
                    for (int i = 0; i < 16; ++i) o16[i] = 0u;
                }
                if (row_ok) {
                    if (f32) {
#pragma unroll
                        for (int i = 0; i < 16; i += 4)
                            *(float4 *)(orow + (c0 + i) * 4) =
                                make_float4(__uint_as_float(o16[i]) * inv, __uint_as_float(o16[i + 1]) * inv,
                                            __uint_as_float(o16[i + 2]) * inv, __uint_as_float(o16[i + 3]) * inv);
                    } else {
#pragma unroll
                        for (int i0 = 0; i0 < 16; i0 += 8) {
                            uint32_t w[4];
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const __nv_bfloat162 b2 = __floats2bfloat162_rn(__uint_as_float(o16[i0 + 2 * i]) * inv,
                                                                                __uint_as_float(o16[i0 + 2 * i + 1]) * inv);
                                w[i] = *(const uint32_t *)&b2;
                            }
                            *(uint4 *)(orow + (c0 + i0) * 2) = make_uint4(w[0], w[1], w[2], w[3]);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(bar(HB_OE + (u & 1)));
                mbar_arrive(bar(HB_LE + slot));
            }
            if (warp == C::EPI_WARP0 && lane == 0 && u < 20) TRACE(420 + u);
        }
        if (!ok && lane == 0) heads_fail(a, abort, 16);
    } else {
        // ---- softmax: warp w = head (w & 3) of the unit, keys [32 half, +32) of each tile, half = w >> 2;
        // lane = query token ----
        const int h = warp & 3, half = (warp - C::SM_WARP0) >> 2;
        const uint32_t lb = ((uint32_t)(32 * h)) << 16;
        const int r = 32 * h + lane;  // TMEM lane / exchange row
        const bool row_ok = lane < a.q_tokens;
        const int bs = a.pool.bt_shift, srows = a.pool.suffix_rows;
        // S columns of this warp's two 16-key chunks in prefix and suffix tiles
        const int row_p0 = heads_row(false, h, 32 * half, bs, srows), row_p1 = heads_row(false, h, 32 * half + 16, bs, srows);
        const int row_s0 = heads_row(true, h, 32 * half, bs, srows), row_s1 = heads_row(true, h, 32 * half + 16, bs, srows);
        float *xmax = (float *)(smem + C::OFF_XCH);  // [2 parity][2 halves][128 rows]
        float *lsum = xmax + 4 * kBM;                 // [2 units][2 halves][128 rows]
        const uint32_t xbar = bar(HB_XCH + h);
        int uses = 0;
        if (half == 0) {  // the other heads' P columns of this lane quarter stay zero
            uint32_t z[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) z[i] = 0u;
            for (int hh = 0; hh < G; ++hh)
                if (hh != h) tmem_st32(tmem + lb + (uint32_t)(C::P_COL + hh * (BN / 2)), z);
            tmem_wait_st();
        }
        const bool prefix_simple =
            !(a.mask_flags & (EKV_MASK_SPAN_ONLY | EKV_MASK_SPAN_EXCLUDE | EKV_MASK_BLOCK_CAUSAL | kVisWordFlags));
        const bool suffix_simple = !(a.mask_flags & (EKV_MASK_SUFFIX_CAUSAL | EKV_MASK_SUFFIX_PREFIX_LM | kVisWordFlags));
        const float inv_scale_log2 = 1.0f / a.scale_log2;
        int t = 0;
        bool ok = true;
        for (int u = 0; ok && u < U; ++u) {
            const int slot = u & 3;
            if (!mbar_wait(bar(HB_LF + slot), (uint32_t)(u >> 2) & 1u, abort, budget)) {
                ok = false;
                break;
            }
            const HPlan &pl = plans[slot];
            const int n = pl.np + pl.ns, np = pl.np, kbeg = pl.kbeg, b = pl.b;
            const int pvalid = pl.prefix_valid, sb = pl.span_b, se = pl.span_e, n_prefix = pl.n_prefix;
            const MaskDesc m = mask_desc(a, b);
            const uint32_t od = tmem + lb + (uint32_t)(C::O_COL + (u & 1) * C::O_STRIDE);
            float m_used = -INFINITY, l = 0.0f;
            for (int j = 0; j < n; ++j, ++t) {
                if (!mbar_wait(bar(HB_KE + t % NS), (uint32_t)(t / NS) & 1u, abort, budget)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (warp == C::SM_WARP0 && lane == 0 && t < 50) TRACE(300 + t);
                if (warp == C::SM_WARP0 + 3 && lane == 0 && t < 50) TRACE(650 + t);
                const bool suffix = j >= np;
                uint32_t s0[16], s1[16];  // keys [32 half, +16), [32 half + 16, +16)
                tmem_load16x2(tmem + lb + (uint32_t)(C::S_COL + (suffix ? row_s0 : row_p0)),
                              tmem + lb + (uint32_t)(C::S_COL + (suffix ? row_s1 : row_p1)), s0, s1);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(HB_SE));
                if (warp == C::SM_WARP0 && lane == 0 && t < 50) TRACE(850 + t);
                const int w0 = (suffix ? 0 : kbeg + j * BN) + 32 * half;
                // rows past the call's tokens count as fully visible: their Q rows are zero, their
                // scores finite, and their output rows are never stored
                uint32_t vb;
                if (!row_ok) vb = 0xffffffffu;
                else if (suffix ? (suffix_simple && w0 + 32 <= a.suffix_len) : (prefix_simple && w0 + 32 <= pvalid))
                    vb = 0xffffffffu;
                else
                    vb = vis_word(m, suffix, w0, lane, pvalid, sb, se, a.suffix_len, n_prefix);
                const bool all_vis = __all_sync(0xffffffffu, vb == 0xffffffffu);
                // no key of this warp's 32 visible to any of its rows (a short suffix tile, the end of a
                // span): no maximum, and P is zero without exponentials
                const bool none_vis = __all_sync(0xffffffffu, vb == 0u);
                float mx[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) mx[i] = -INFINITY;
                if (none_vis) {
                } else if (all_vis) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        mx[i & 3] = fmaxf(mx[i & 3], __uint_as_float(s0[i]));
                        mx[4 + (i & 3)] = fmaxf(mx[4 + (i & 3)], __uint_as_float(s1[i]));
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        mx[i & 3] = fmaxf(mx[i & 3], ((vb >> i) & 1u) ? __uint_as_float(s0[i]) : -INFINITY);
                        mx[4 + (i & 3)] = fmaxf(mx[4 + (i & 3)], ((vb >> (16 + i)) & 1u) ? __uint_as_float(s1[i]) : -INFINITY);
                    }
                }
                const float cm = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                                       fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
                xmax[((t & 1) * 2 + half) * kBM + r] = cm;
                if (warp == C::SM_WARP0 && lane == 0 && t < 50) TRACE(900 + t);
                if (!(ok = heads_xsync(xbar, uses++, abort, budget))) break;
                if (warp == C::SM_WARP0 && lane == 0 && t < 50) TRACE(950 + t);
                const float rmax = fmaxf(cm, xmax[((t & 1) * 2 + (half ^ 1)) * kBM + r]);
                bool waited = false;
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
                    // both warps of the head take the same decisions; the first rescales O
                    if (__any_sync(0xffffffffu, rescale)) {
                        if (!mbar_wait(bar(HB_VE + (t - 1) % NS), (uint32_t)((t - 1) / NS) & 1u, abort, budget)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        waited = true;
                        if (half == 0) {
#pragma unroll
                            for (int c0 = 0; c0 < D; c0 += 16) {
                                uint32_t o16[16];
                                tmem_load16(od + (uint32_t)c0, o16);
#pragma unroll
                                for (int i = 0; i < 16; ++i) o16[i] = __float_as_uint(__uint_as_float(o16[i]) * alpha);
                                tmem_st16(od + (uint32_t)c0, o16);
                            }
                            tmem_wait_st();
                        }
                    }
                }
                const float neg_m = -m_used;
                const uint32_t pv = m_used != -INFINITY ? vb : 0u;
                const bool all_p = all_vis && __all_sync(0xffffffffu, m_used != -INFINITY);
                float ps[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                uint32_t pw[16];
                if (none_vis) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) pw[i] = 0u;
                } else if (all_p) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float x0 = ex2(fmaf(__uint_as_float(s0[2 * i]), a.scale_log2, neg_m));
                        const float x1 = ex2(fmaf(__uint_as_float(s0[2 * i + 1]), a.scale_log2, neg_m));
                        const float y0 = ex2(fmaf(__uint_as_float(s1[2 * i]), a.scale_log2, neg_m));
                        const float y1 = ex2(fmaf(__uint_as_float(s1[2 * i + 1]), a.scale_log2, neg_m));
                        ps[0] += x0;
                        ps[1] += x1;
                        ps[2] += y0;
                        ps[3] += y1;
                        const __nv_bfloat162 lo = __floats2bfloat162_rn(x0, x1);
                        const __nv_bfloat162 hi = __floats2bfloat162_rn(y0, y1);
                        pw[i] = *(const uint32_t *)&lo;
                        pw[8 + i] = *(const uint32_t *)&hi;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        float pr[4];
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int c = 2 * i + e;
                            const float x0 = ex2(fmaf(__uint_as_float(s0[c]), a.scale_log2, neg_m));
                            const float x1 = ex2(fmaf(__uint_as_float(s1[c]), a.scale_log2, neg_m));
                            pr[e] = ((pv >> c) & 1u) ? x0 : 0.0f;
                            pr[2 + e] = ((pv >> (16 + c)) & 1u) ? x1 : 0.0f;
                            ps[e] += pr[e];
                            ps[2 + e] += pr[2 + e];
                        }
                        const __nv_bfloat162 lo = __floats2bfloat162_rn(pr[0], pr[1]);
                        const __nv_bfloat162 hi = __floats2bfloat162_rn(pr[2], pr[3]);
                        pw[i] = *(const uint32_t *)&lo;
                        pw[8 + i] = *(const uint32_t *)&hi;
                    }
                }
                l += (ps[0] + ps[1]) + (ps[2] + ps[3]);
                if (warp == C::SM_WARP0 && lane == 0 && t < 50) TRACE(600 + t);
                // P(t - 1) has been consumed (P.V(t - 1) done) before P(t) overwrites it
                if (t >= 1 && !waited) {
                    if (!mbar_wait(bar(HB_VE + (t - 1) % NS), (uint32_t)((t - 1) / NS) & 1u, abort, budget)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                }
                tmem_st16(tmem + lb + (uint32_t)(C::P_COL + h * (BN / 2) + half * 16), pw);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(HB_PF));
                if (warp == C::SM_WARP0 && lane == 0 && t < 50) TRACE(350 + t);
                if (warp == C::SM_WARP0 + 3 && lane == 0 && t < 50) TRACE(700 + t);
            }
            if (!ok) break;
            // ---- the unit's row sums to the epilogue warps (this unit's slot is free once the epilogue of
            // unit u - 2 has released the O buffer of the same parity) ----
            if (u >= 2 && !mbar_wait(bar(HB_OE + (u & 1)), (uint32_t)((u - 2) >> 1) & 1u, abort, budget)) {
                ok = false;
                break;
            }
            lsum[((u & 1) * 2 + half) * kBM + r] = l;
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(bar(HB_LR + (u & 1)));
                mbar_arrive(bar(HB_LE + slot));
            }
            if (warp == C::SM_WARP0 && lane == 0 && u < 20) TRACE(400 + u);
        }
        if (!ok && lane == 0) heads_fail(a, abort, 15);
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == C::MMA_WARP) tmem_dealloc(tmem, 512);
    if (threadIdx.x == 0) TRACE(11);
    __syncthreads();
    trace_flush();
}

}  // namespace

#ifdef EKV_TRACE
int heads_debug_set_trace(unsigned long long *buf) {
    return cudaMemcpyToSymbol(c_trace, &buf, sizeof(buf)) == cudaSuccess ? 0 : -2;
}
#endif

// The shapes the kernel takes: bf16 pool, one query head per KV head (MHA), at most 32 query tokens,
// head_dim 48 or 64, KV heads a multiple of 4, blocks of 16, 32 or 64 tokens, at most 64 suffix keys
// in slot tiles of at most 64 rows.
bool heads_fits(const AttnArgs &a) {
    const PoolView &p = a.pool;
    if (p.dtype != EKV_DTYPE_BF16 || a.group != 1 || a.q_tokens < 1 || a.q_tokens > 32) return false;
    if (p.head_dim != 48 && p.head_dim != 64) return false;
    if (p.kv_heads % kHG != 0 || a.k_sfx) return false;
    if (p.block_tokens != 16 && p.block_tokens != 32 && p.block_tokens != 64) return false;
    if (a.suffix_len > 0 && (a.suffix_len > kHBN || p.suffix_rows <= 0 || p.suffix_rows > kHBN || p.suffix_rows % 16))
        return false;
    return (int64_t)a.n_batch * (p.kv_heads / kHG) <= INT_MAX;
}

int heads_units(const AttnArgs &a) { return a.n_batch * (a.pool.kv_heads / kHG); }

// Tensor map of the caller's q [n_batch][q_tokens][q_heads][D] as (dim, head, token, request), boxes of
// one swizzle chunk x 1 head x 32 tokens (tokens past q_tokens read as zeros), swizzled like the pool.
static bool make_heads_q_map(const AttnArgs &a, CUtensorMap *map) {
    std::memset(map, 0, sizeof(*map));
    const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    const int D = a.pool.head_dim, es = 2, W = swizzle_bytes_for(D);
    if (!enc || ((uintptr_t)a.q & 15)) return false;
    const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)a.q_heads, (cuuint64_t)a.q_tokens, (cuuint64_t)a.n_batch};
    const cuuint64_t strides[3] = {(cuuint64_t)D * es, (cuuint64_t)a.q_heads * D * es,
                                   (cuuint64_t)a.q_tokens * a.q_heads * D * es};
    const cuuint32_t box[4] = {(cuuint32_t)(W / es), 1, 32, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUtensorMapSwizzle sw = W == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                  : W == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B;
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, (void *)a.q, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int launch_attention_heads(const AttnArgs &a, cudaStream_t s, int sms) {
    if (!heads_fits(a)) return EKV_ERR_UNSUPPORTED;
    CUtensorMap qmap;
    if (!make_heads_q_map(a, &qmap)) return EKV_ERR_UNSUPPORTED;
    const bool d48 = a.pool.head_dim == 48;
    const int smem_bytes = d48 ? HCfg<48>::SMEM : HCfg<64>::SMEM;
    static int attr_done[64][2] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr_done[dev][d48]) {
        const cudaError_t e =
            d48 ? cudaFuncSetAttribute(attn_heads_kernel<48>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes)
                : cudaFuncSetAttribute(attn_heads_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
        if (e != cudaSuccess) return EKV_ERR_CUDA;
        attr_done[dev][d48] = 1;
    }
    const int n_units = heads_units(a);
    const int grid = std::max(1, std::min(n_units, sms));
    if (d48)
        attn_heads_kernel<48><<<grid, HCfg<48>::THREADS, smem_bytes, s>>>(a, n_units, qmap);
    else
        attn_heads_kernel<64><<<grid, HCfg<64>::THREADS, smem_bytes, s>>>(a, n_units, qmap);
    if (cudaGetLastError() != cudaSuccess) return EKV_ERR_CUDA;
    note_launches(1);
    return EKV_OK;
}

}  // namespace ekv
