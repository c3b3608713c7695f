// ekv_attn_tc.cu -- masked attention over the paged KV pool on tcgen05 tensor cores (sm_100a).
//
// Replaces the reference's per-layer-step concat/permute copies + mul_mat(K,Q) +
// soft_max_ext + mul_mat(V,attn) (models/pi05.cpp:406-421) and ggml_flash_attn_ext
// (models/hy_vla.cpp:1075) with one fused kernel per call.
//
// Work unit (one CTA): 128 query rows that share one KV head (rows = (token, head-in-group),
// so for MQA all 8 heads of 16 tokens share the K/V tiles) x a range of key tiles.
//   warps 0-3  softmax: each thread owns one query row = one TMEM lane; reads S from TMEM,
//              applies the mask, online max/sum in the exp2 domain, writes P (bf16/f16) to
//              shared memory, rescales O in TMEM when the running max grows by > 2^8, and
//              finally normalises O and stores it.
//   warp 4     TMEM allocation + single-thread tcgen05.mma issue: S = Q K^T (M=128, N=BN,
//              K=head_dim) into a double-buffered TMEM S, O += P V (M=128, N=head_dim, K=BN)
//              into TMEM O; tcgen05.commit signals the mbarriers.
//   warps 5+   producers: bf16 pools copy K/V block chunks with cp.async.bulk straight from the
//              pool (tiles are stored pre-swizzled, so one contiguous copy per (block, chunk)
//              lands as a canonical SW128/64/32 operand); Q8_0 pools load int8 + fp16 scales
//              with 16-byte vector loads and dequantise in registers (exact int8 -> f16 via the
//              0x6400 magic, one f16 multiply by the scale) into the same swizzled layout.
// Q8_0 pools run the MMA in f16 (Q and the bf16 suffix converted exactly for normal values),
// bf16 pools in bf16. Accumulation is f32 throughout.
//
// Every mbarrier wait is bounded (clock64 budget); on expiry the kernel records
// DEV_ERR_TIMEOUT in the pool status word, raises a CTA-local abort flag and unwinds.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "ekv_device.cuh"
#include "ekv_internal.h"
#include "ekv_sm100.cuh"

namespace ekv {
namespace {

using namespace sm100;

constexpr long long kWaitBudget = 4000000000LL;  // clock cycles (~2-3 s) before giving up
constexpr int kBM = 128;
constexpr int kMaxSplits = 8;

template <int D, bool Q8>
struct TcCfg {
    static constexpr int BM = kBM;
    static constexpr int BN = D > 128 ? 64 : 128;
    static constexpr int W = (D * 2) % 128 == 0 ? 128 : ((D * 2) % 64 == 0 ? 64 : 32);
    static constexpr uint32_t LAYOUT = W == 128 ? 2u : (W == 64 ? 4u : 6u);
    static constexpr int Q_BYTES = BM * D * 2;
    static constexpr int KV_BYTES = BN * D * 2;
    static constexpr int P_BYTES = BM * BN * 2;
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = OFF_Q + Q_BYTES;
    static constexpr int OFF_V = OFF_K + 2 * KV_BYTES;
    static constexpr int OFF_P = OFF_V + 2 * KV_BYTES;
    static constexpr int OFF_BAR = OFF_P + 2 * P_BYTES;
    static constexpr int SMEM = OFF_BAR + 256 + 1024;  // barriers/flags + 1 KB alignment slack
    static constexpr int MMA_WARP = 4;
    static constexpr int PROD_WARP0 = 5;
    static constexpr int N_PROD = Q8 ? 128 : 32;
    static constexpr int THREADS = 160 + N_PROD;
    static constexpr int TMEM_COLS = 512;
    static constexpr int O_COL = 2 * BN;
    static_assert(O_COL + D <= TMEM_COLS, "TMEM budget");
    static_assert(SMEM <= 232448, "shared-memory budget");
    static_assert(D % 16 == 0, "head_dim must be a multiple of 16");
};

enum { BAR_KV_FULL = 0, BAR_KV_EMPTY = 2, BAR_S_FULL = 4, BAR_P_FULL = 6, BAR_P_EMPTY = 8, BAR_DONE = 10, N_BARS = 11 };

// Key-tile schedule of one CTA, computed identically by every thread.
struct Plan {
    int b, g, qt, split;
    int qrow0, rows_valid;
    SeqKeys sk;
    int kbeg;       // first key of prefix tile 0 (multiple of BN)
    int np_tiles;   // prefix tiles
    int ns_tiles;   // suffix tiles
    int j0, j1;     // this split's tile range [j0, j1)
};

template <int BN>
__device__ __forceinline__ Plan make_plan(const AttnArgs &a, int n_qtiles) {
    Plan pl;
    const int n_splits = a.n_splits > 1 ? a.n_splits : 1;
    pl.qt = blockIdx.x / n_splits;
    pl.split = blockIdx.x - pl.qt * n_splits;
    pl.g = blockIdx.y;
    pl.b = blockIdx.z;
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
    (void)n_qtiles;
    return pl;
}

// ---- Q tile: bf16 [B][Tq][Hq][D] rows -> swizzled K-major A operand (f16 for Q8_0 pools) ----
template <int D, bool Q8>
__device__ __forceinline__ void load_q_tile(const AttnArgs &a, const Plan &pl, uint8_t *sQ) {
    using C = TcCfg<D, Q8>;
    constexpr int UNITS_PER_ROW = D / 8;
    for (int u = threadIdx.x; u < kBM * UNITS_PER_ROW; u += C::THREADS) {
        const int r = u / UNITS_PER_ROW;
        const int d0 = (u - r * UNITS_PER_ROW) * 8;
        uint4 val = make_uint4(0, 0, 0, 0);
        if (r < pl.rows_valid) {
            const int qr = pl.qrow0 + r;
            const int t = qr / a.group;
            const int h = pl.g * a.group + (qr - t * a.group);
            val = *(const uint4 *)(a.q + (((int64_t)pl.b * a.q_tokens + t) * a.q_heads + h) * D + d0);
            if (Q8) {
                uint32_t w[4] = {val.x, val.y, val.z, val.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const __half2 h2 = __floats2half2_rn(__uint_as_float(w[i] << 16),
                                                         __uint_as_float(w[i] & 0xffff0000u));
                    w[i] = *(const uint32_t *)&h2;
                }
                val = make_uint4(w[0], w[1], w[2], w[3]);
            }
        }
        *(uint4 *)(sQ + tile_elem_off(r, d0, kBM, C::W)) = val;
    }
}

// ---- bf16 producer: one warp; zero-fills missing rows, lane 0 issues the bulk copies ----
template <int D>
__device__ __forceinline__ void produce_bf16_tile(const AttnArgs &a, const Plan &pl, int j, uint8_t *sK,
                                                  uint8_t *sV, uint32_t bar_full, int lane) {
    using C = TcCfg<D, false>;
    constexpr int BN = C::BN, W = C::W, NCH = D * 2 / W;
    const PoolView &p = a.pool;
    const bool suffix = j >= pl.np_tiles;
    // Segments of the tile: [row0, row0+len) of the tile come from one block (or the suffix
    // tile); src == nullptr means zero-fill.
    uint32_t total = 0;
    // pass 0: zero-fill (all lanes) and byte count; pass 1: lane 0 issues copies
    for (int pass = 0; pass < 2; ++pass) {
        if (pass == 1) {
            fence_proxy_async();
            __syncwarp();
            if (lane != 0) break;
            if (total) mbar_arrive_expect_tx(bar_full, total);
            else mbar_arrive(bar_full);
        }
        int row = 0;
        while (row < BN) {
            const uint8_t *srcK = nullptr, *srcV = nullptr;
            int len, src_rows = 0, src_row0 = 0;
            if (suffix) {
                const int s0 = (j - pl.np_tiles) * BN + row;
                len = BN - row;
                if (s0 < p.suffix_rows) {
                    len = min(len, p.suffix_rows - s0);
                    srcK = p.suffix + suffix_tile_index(p, a.layer, pl.sk.seq, 0, pl.g) * p.suffix_tile_bytes;
                    srcV = p.suffix + suffix_tile_index(p, a.layer, pl.sk.seq, 1, pl.g) * p.suffix_tile_bytes;
                    src_rows = p.suffix_rows;
                    src_row0 = s0;
                }
            } else {
                const int k = pl.kbeg + j * BN + row;
                const int rib = k % p.block_tokens;
                len = min(BN - row, p.block_tokens - rib);
                if (k < pl.sk.n_prefix) {
                    const int blk = lookup_block(p, pl.sk.seq, k / p.block_tokens);
                    if (blk >= 0) {
                        srcK = p.prefix + prefix_tile_index(p, a.layer, blk, 0, pl.g) * p.tile_bytes;
                        srcV = p.prefix + prefix_tile_index(p, a.layer, blk, 1, pl.g) * p.tile_bytes;
                        src_rows = p.block_tokens;
                        src_row0 = rib;
                    }
                }
            }
            for (int c = 0; c < NCH; ++c) {
                const uint32_t dst_off = (uint32_t)c * (BN * W) + (uint32_t)row * W;
                const uint32_t bytes = (uint32_t)len * W;
                if (srcK) {
                    if (pass == 0) {
                        total += 2 * bytes;
                    } else {
                        const int64_t so = (int64_t)c * src_rows * W + (int64_t)src_row0 * W;
                        bulk_g2s(smem_addr(sK + dst_off), srcK + so, bytes, bar_full);
                        bulk_g2s(smem_addr(sV + dst_off), srcV + so, bytes, bar_full);
                    }
                } else if (pass == 0) {
                    for (uint32_t o = lane * 16; o < bytes; o += 32 * 16) {
                        *(uint4 *)(sK + dst_off + o) = make_uint4(0, 0, 0, 0);
                        *(uint4 *)(sV + dst_off + o) = make_uint4(0, 0, 0, 0);
                    }
                }
            }
            row += len;
        }
    }
}

// ---- Q8_0 producer: 128 threads; int8 + fp16 scale -> f16 in registers ----
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

__device__ __forceinline__ uint4 bf16x8_to_f16x8(uint4 v) {
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2 h2 = __floats2half2_rn(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u));
        w[i] = *(const uint32_t *)&h2;
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

template <int D>
struct Q8Raw {
    static constexpr int BN = TcCfg<D, true>::BN;
    static constexpr int PU = BN * (D / 16) / 128;  // prefix units (16 int8) per thread
    static constexpr int SU = BN * (D / 8) / 128;   // suffix units (8 bf16) per thread
    static constexpr int NU = PU > SU ? PU : SU;
    uint4 k[NU], v[NU];
    uint32_t dk[PU], dv[PU];
};

template <int D>
__device__ __forceinline__ void q8_load_tile(const AttnArgs &a, const Plan &pl, int j, int ptid, Q8Raw<D> &raw) {
    constexpr int BN = TcCfg<D, true>::BN;
    const PoolView &p = a.pool;
    if (j >= pl.np_tiles) {
        const int s_base = (j - pl.np_tiles) * BN;
        const uint8_t *tk = p.suffix + suffix_tile_index(p, a.layer, pl.sk.seq, 0, pl.g) * p.suffix_tile_bytes;
        const uint8_t *tv = p.suffix + suffix_tile_index(p, a.layer, pl.sk.seq, 1, pl.g) * p.suffix_tile_bytes;
#pragma unroll
        for (int i = 0; i < Q8Raw<D>::SU; ++i) {
            const int u = ptid + i * 128;
            const int row = u / (D / 8);
            const int d0 = (u - row * (D / 8)) * 8;
            const int s = s_base + row;
            if (s < p.suffix_rows) {
                const uint32_t off = tile_elem_off(s, d0, p.suffix_rows, p.swz_bytes);
                raw.k[i] = __ldg((const uint4 *)(tk + off));
                raw.v[i] = __ldg((const uint4 *)(tv + off));
            } else {
                raw.k[i] = raw.v[i] = make_uint4(0, 0, 0, 0);
            }
        }
        return;
    }
    const int groups = D / 32;
#pragma unroll
    for (int i = 0; i < Q8Raw<D>::PU; ++i) {
        const int u = ptid + i * 128;
        const int row = u / (D / 16);
        const int seg = u - row * (D / 16);
        const int k = pl.kbeg + j * BN + row;
        raw.k[i] = raw.v[i] = make_uint4(0, 0, 0, 0);
        raw.dk[i] = raw.dv[i] = 0;
        if (k < pl.sk.n_prefix) {
            const int blk = lookup_block(p, pl.sk.seq, k / p.block_tokens);
            if (blk >= 0) {
                const int rib = k % p.block_tokens;
                const uint8_t *tk = p.prefix + prefix_tile_index(p, a.layer, blk, 0, pl.g) * p.tile_bytes;
                const uint8_t *tv = p.prefix + prefix_tile_index(p, a.layer, blk, 1, pl.g) * p.tile_bytes;
                const int64_t qo = (int64_t)rib * D + seg * 16;
                const int64_t so = (int64_t)p.block_tokens * D + ((int64_t)rib * groups + seg / 2) * 2;
                raw.k[i] = __ldg((const uint4 *)(tk + qo));
                raw.v[i] = __ldg((const uint4 *)(tv + qo));
                raw.dk[i] = __ldg((const uint16_t *)(tk + so));
                raw.dv[i] = __ldg((const uint16_t *)(tv + so));
            }
        }
    }
}

template <int D>
__device__ __forceinline__ void q8_store_tile(const Plan &pl, int j, int ptid, const Q8Raw<D> &raw, uint8_t *sK,
                                              uint8_t *sV) {
    using C = TcCfg<D, true>;
    constexpr int BN = C::BN, W = C::W;
    if (j >= pl.np_tiles) {
#pragma unroll
        for (int i = 0; i < Q8Raw<D>::SU; ++i) {
            const int u = ptid + i * 128;
            const int row = u / (D / 8);
            const int d0 = (u - row * (D / 8)) * 8;
            const uint32_t off = tile_elem_off(row, d0, BN, W);
            *(uint4 *)(sK + off) = bf16x8_to_f16x8(raw.k[i]);
            *(uint4 *)(sV + off) = bf16x8_to_f16x8(raw.v[i]);
        }
        return;
    }
#pragma unroll
    for (int i = 0; i < Q8Raw<D>::PU; ++i) {
        const int u = ptid + i * 128;
        const int row = u / (D / 16);
        const int d0 = (u - row * (D / 16)) * 16;
        uint4 lo, hi;
        dequant16(raw.k[i], raw.dk[i], lo, hi);
        *(uint4 *)(sK + tile_elem_off(row, d0, BN, W)) = lo;
        *(uint4 *)(sK + tile_elem_off(row, d0 + 8, BN, W)) = hi;
        dequant16(raw.v[i], raw.dv[i], lo, hi);
        *(uint4 *)(sV + tile_elem_off(row, d0, BN, W)) = lo;
        *(uint4 *)(sV + tile_elem_off(row, d0 + 8, BN, W)) = hi;
    }
}

__device__ __forceinline__ void fail_timeout(const AttnArgs &a, volatile int *abort, int where) {
    *abort = 1;
    report_error(a.pool.status, DEV_ERR_TIMEOUT, where, blockIdx.x, blockIdx.z);
}

template <int D, bool Q8>
__global__ void __launch_bounds__(TcCfg<D, Q8>::THREADS, 1) attn_tc_kernel(const AttnArgs a, int n_qtiles) {
    using C = TcCfg<D, Q8>;
    constexpr int BN = C::BN, W = C::W;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *sQ = smem + C::OFF_Q;
    uint8_t *sK = smem + C::OFF_K;
    uint8_t *sV = smem + C::OFF_V;
    uint8_t *sP = smem + C::OFF_P;
    uint64_t *bars = (uint64_t *)(smem + C::OFF_BAR);
    uint32_t *tmem_holder = (uint32_t *)(bars + N_BARS);
    volatile int *abort = (volatile int *)(bars + N_BARS + 1);
    const uint32_t bar0 = smem_addr(bars);
    auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const Plan pl = make_plan<BN>(a, n_qtiles);
    if (threadIdx.x == 0 && !pl.sk.ok) report_error(a.pool.status, DEV_ERR_BAD_SEQ, pl.b, a.seq_ids[pl.b], 3);

    if (threadIdx.x == 0) {
        for (int s = 0; s < 2; ++s) {
            mbar_init(bar(BAR_KV_FULL + s), Q8 ? 128 : 1);
            mbar_init(bar(BAR_KV_EMPTY + s), 1);
            mbar_init(bar(BAR_S_FULL + s), 1);
            mbar_init(bar(BAR_P_FULL + s), 128);
            mbar_init(bar(BAR_P_EMPTY + s), 1);
        }
        mbar_init(bar(BAR_DONE), 1);
        *abort = 0;
        mbar_init_fence();
    }
    if (warp == C::MMA_WARP) tmem_alloc(smem_addr(tmem_holder), C::TMEM_COLS);
    load_q_tile<D, Q8>(a, pl, sQ);
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    const int n = pl.j1 - pl.j0;

    if (warp == C::MMA_WARP) {
        if (lane == 0 && n > 0) {
            const uint32_t idS = idesc_f16(!Q8, false, BN);
            const uint32_t idO = idesc_f16(!Q8, true, D);
            const uint32_t q_addr = smem_addr(sQ), k_addr = smem_addr(sK), v_addr = smem_addr(sV),
                           p_addr = smem_addr(sP);
            bool ok = true;
            auto issue_s = [&](int jj) {
                const int st = jj & 1;
                if (!mbar_wait(bar(BAR_KV_FULL + st), (jj >> 1) & 1, abort, kWaitBudget)) return false;
                tc_fence_after();
                const uint32_t d_tmem = tmem + (uint32_t)(st * BN);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t byte = (uint32_t)kk * 32u;
                    const uint32_t chunk = byte / W, within = byte % W;
                    const uint64_t ad = sdesc(q_addr + chunk * (kBM * W) + within, 16, 8 * W, C::LAYOUT);
                    const uint64_t bd =
                        sdesc(k_addr + st * C::KV_BYTES + chunk * (BN * W) + within, 16, 8 * W, C::LAYOUT);
                    mma_ss(d_tmem, ad, bd, idS, kk > 0 ? 1u : 0u);
                }
                mma_commit(bar(BAR_S_FULL + st));
                return true;
            };
            ok = issue_s(0);
            for (int jj = 0; ok && jj < n; ++jj) {
                if (jj + 1 < n && !(ok = issue_s(jj + 1))) break;
                const int st = jj & 1;
                if (!(ok = mbar_wait(bar(BAR_P_FULL + st), (jj >> 1) & 1, abort, kWaitBudget))) break;
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < BN / 16; ++kk) {
                    const uint32_t byte = (uint32_t)kk * 32u;
                    const uint64_t ad = sdesc(p_addr + st * C::P_BYTES + (byte / 128) * (kBM * 128) + byte % 128, 16,
                                              1024, 2u);
                    const uint64_t bd = sdesc(v_addr + st * C::KV_BYTES + (uint32_t)kk * 16u * W, BN * W, 8 * W,
                                              C::LAYOUT);
                    mma_ss(tmem + C::O_COL, ad, bd, idO, (jj > 0 || kk > 0) ? 1u : 0u);
                }
                mma_commit(bar(BAR_KV_EMPTY + st));
                mma_commit(bar(BAR_P_EMPTY + st));
            }
            if (!ok) fail_timeout(a, abort, 1);
            // Every MMA this thread issued must have finished before TMEM is released.
            mma_commit(bar(BAR_DONE));
            mbar_wait(bar(BAR_DONE), 0, abort, kWaitBudget);
        }
    } else if (warp >= C::PROD_WARP0) {
        const int ptid = threadIdx.x - C::PROD_WARP0 * 32;
        if constexpr (Q8) {
            Q8Raw<D> raw;
            for (int jj = 0; jj < n; ++jj) {
                const int st = jj & 1;
                q8_load_tile<D>(a, pl, pl.j0 + jj, ptid, raw);
                if (jj >= 2 && !mbar_wait(bar(BAR_KV_EMPTY + st), ((jj - 2) >> 1) & 1, abort, kWaitBudget)) {
                    fail_timeout(a, abort, 2);
                    break;
                }
                q8_store_tile<D>(pl, pl.j0 + jj, ptid, raw, sK + st * C::KV_BYTES, sV + st * C::KV_BYTES);
                fence_proxy_async();
                mbar_arrive(bar(BAR_KV_FULL + st));
            }
        } else {
            for (int jj = 0; jj < n; ++jj) {
                const int st = jj & 1;
                if (jj >= 2 && !mbar_wait(bar(BAR_KV_EMPTY + st), ((jj - 2) >> 1) & 1, abort, kWaitBudget)) {
                    fail_timeout(a, abort, 2);
                    break;
                }
                produce_bf16_tile<D>(a, pl, pl.j0 + jj, sK + st * C::KV_BYTES, sV + st * C::KV_BYTES,
                                     bar(BAR_KV_FULL + st), lane);
            }
            // Do not leave the CTA with bulk copies still writing shared memory.
            if (lane == 0 && n > 0 && *abort) {
                for (int jj = max(0, n - 2); jj < n; ++jj)
                    mbar_wait(bar(BAR_KV_FULL + (jj & 1)), (jj >> 1) & 1, abort, kWaitBudget / 4);
            }
        }
    } else {
        // ---- softmax / epilogue: thread = query row = TMEM lane ----
        const int r = threadIdx.x;
        const bool row_ok = r < pl.rows_valid;
        const int qr = pl.qrow0 + r;
        const int t = qr / a.group;
        const uint32_t lane_base = ((uint32_t)(warp * 32)) << 16;
        const MaskDesc m{a.mask_flags, a.chunk_tokens, a.chunk_stride, a.window_chunks, a.q_chunk0};
        const bool prefix_simple = !(a.mask_flags & (EKV_MASK_SPAN_ONLY | EKV_MASK_SPAN_EXCLUDE | EKV_MASK_BLOCK_CAUSAL));
        const bool suffix_simple = !(a.mask_flags & (EKV_MASK_SUFFIX_CAUSAL | EKV_MASK_SUFFIX_PREFIX_LM));
        float m_used = -INFINITY, l = 0.0f;
        bool ok = true;
        for (int jj = 0; jj < n; ++jj) {
            const int st = jj & 1;
            const int j = pl.j0 + jj;
            if (!(ok = mbar_wait(bar(BAR_S_FULL + st), (jj >> 1) & 1, abort, kWaitBudget))) break;
            tc_fence_after();
            float x[BN];
#pragma unroll
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t rr[32];
                tmem_load32(tmem + lane_base + (uint32_t)(st * BN + c0), rr);
#pragma unroll
                for (int i = 0; i < 32; ++i) x[c0 + i] = __uint_as_float(rr[i]);
            }
            // mask + scale (exp2 domain)
            const bool suffix = j >= pl.np_tiles;
            const int key0 = suffix ? (j - pl.np_tiles) * BN : pl.kbeg + j * BN;
            const bool all_vis = row_ok && (suffix ? (suffix_simple && key0 + BN <= a.suffix_len)
                                                   : (prefix_simple && key0 + BN <= pl.sk.prefix_valid));
            float m_tile = -INFINITY;
#pragma unroll
            for (int c = 0; c < BN; ++c) {
                bool vis = all_vis;
                if (!all_vis && row_ok) {
                    vis = suffix ? suffix_allowed(m, t, key0 + c, a.suffix_len)
                                 : prefix_allowed(m, t, key0 + c, pl.sk.prefix_valid, pl.sk.span_b, pl.sk.span_e);
                }
                x[c] = vis ? x[c] * a.scale_log2 : -INFINITY;
                m_tile = fmaxf(m_tile, x[c]);
            }
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
            float psum = 0.0f;
#pragma unroll
            for (int c = 0; c < BN; ++c) {
                const float pv = (x[c] == -INFINITY) ? 0.0f : ex2(x[c] - m_used);
                x[c] = pv;
                psum += pv;
            }
            l += psum;
            if (__any_sync(0xffffffffu, rescale)) {
                // O may only be touched once the previous P.V has landed in TMEM.
                if (!(ok = mbar_wait(bar(BAR_P_EMPTY + ((jj - 1) & 1)), ((jj - 1) >> 1) & 1, abort, kWaitBudget)))
                    break;
                tc_fence_after();
#pragma unroll
                for (int c0 = 0; c0 < D; c0 += 16) {
                    uint32_t rr[16];
                    tmem_load16(tmem + lane_base + (uint32_t)(C::O_COL + c0), rr);
#pragma unroll
                    for (int i = 0; i < 16; ++i) rr[i] = __float_as_uint(__uint_as_float(rr[i]) * alpha);
                    tmem_st16(tmem + lane_base + (uint32_t)(C::O_COL + c0), rr);
                }
                tmem_wait_st();
            }
            if (jj >= 2 && !(ok = mbar_wait(bar(BAR_P_EMPTY + st), ((jj - 2) >> 1) & 1, abort, kWaitBudget))) break;
            uint8_t *pbuf = sP + st * C::P_BYTES;
#pragma unroll
            for (int c8 = 0; c8 < BN / 8; ++c8) {
                uint32_t w[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float lo = x[c8 * 8 + 2 * i], hi = x[c8 * 8 + 2 * i + 1];
                    if (Q8) {
                        const __half2 h2 = __floats2half2_rn(lo, hi);
                        w[i] = *(const uint32_t *)&h2;
                    } else {
                        const __nv_bfloat162 b2 = __floats2bfloat162_rn(lo, hi);
                        w[i] = *(const uint32_t *)&b2;
                    }
                }
                const uint32_t byte = (uint32_t)c8 * 16u;
                const uint32_t off = (byte / 128) * (kBM * 128) + swz((uint32_t)r * 128u + byte % 128, 7u);
                *(uint4 *)(pbuf + off) = make_uint4(w[0], w[1], w[2], w[3]);
            }
            fence_proxy_async();
            tc_fence_before();
            mbar_arrive(bar(BAR_P_FULL + st));
        }
        if (!ok) fail_timeout(a, abort, 3);
        if (ok && n > 0) {
            ok = mbar_wait(bar(BAR_P_EMPTY + ((n - 1) & 1)), ((n - 1) >> 1) & 1, abort, kWaitBudget);
            if (!ok) fail_timeout(a, abort, 4);
            tc_fence_after();
        }
        // ---- epilogue ----
        const bool have_o = ok && n > 0;
        const int h = pl.g * a.group + (qr - t * a.group);
        if (a.n_splits > 1) {
            const int64_t unit = (((int64_t)pl.b * a.pool.kv_heads + pl.g) * n_qtiles + pl.qt) * a.n_splits + pl.split;
            float *wo = a.ws_o + (unit * kBM + r) * D;
            float *wml = a.ws_ml + (unit * kBM + r) * 2;
#pragma unroll
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
            const float inv = (have_o && l > 0.0f) ? 1.0f / l : 0.0f;
            const int64_t obase = (((int64_t)pl.b * a.q_tokens + t) * a.q_heads + h) * D;
#pragma unroll
            for (int c0 = 0; c0 < D; c0 += 16) {
                uint32_t rr[16];
                if (have_o) {
                    tmem_load16(tmem + lane_base + (uint32_t)(C::O_COL + c0), rr);
                } else {
#pragma unroll
                    for (int i = 0; i < 16; ++i) rr[i] = 0u;
                }
                if (!row_ok) continue;
                if (a.out_dtype == EKV_DTYPE_F32) {
                    float *o = (float *)a.out + obase + c0;
#pragma unroll
                    for (int i = 0; i < 16; i += 4)
                        *(float4 *)(o + i) =
                            make_float4(__uint_as_float(rr[i]) * inv, __uint_as_float(rr[i + 1]) * inv,
                                        __uint_as_float(rr[i + 2]) * inv, __uint_as_float(rr[i + 3]) * inv);
                } else {
                    uint32_t w[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const __nv_bfloat162 b2 = __floats2bfloat162_rn(__uint_as_float(rr[2 * i]) * inv,
                                                                        __uint_as_float(rr[2 * i + 1]) * inv);
                        w[i] = *(const uint32_t *)&b2;
                    }
                    uint4 *o = (uint4 *)((uint16_t *)a.out + obase + c0);
                    o[0] = make_uint4(w[0], w[1], w[2], w[3]);
                    o[1] = make_uint4(w[4], w[5], w[6], w[7]);
                }
            }
        }
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == C::MMA_WARP) tmem_dealloc(tmem, C::TMEM_COLS);
}

// Combine the per-split partial outputs: O = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s.
template <int D>
__global__ void merge_splits_kernel(const AttnArgs a, int n_qtiles) {
    const int qt = blockIdx.x, g = blockIdx.y, b = blockIdx.z, r = threadIdx.x;
    const int qr = qt * kBM + r;
    if (qr >= a.q_tokens * a.group) return;
    const int t = qr / a.group;
    const int h = g * a.group + (qr - t * a.group);
    const int64_t unit0 = (((int64_t)b * a.pool.kv_heads + g) * n_qtiles + qt) * a.n_splits;
    float mmax = -INFINITY;
    for (int s = 0; s < a.n_splits; ++s) mmax = fmaxf(mmax, a.ws_ml[((unit0 + s) * kBM + r) * 2]);
    float wsum = 0.0f, wts[kMaxSplits];
    for (int s = 0; s < a.n_splits; ++s) {
        const float ms = a.ws_ml[((unit0 + s) * kBM + r) * 2];
        const float wv = (ms == -INFINITY) ? 0.0f : ex2(ms - mmax);
        wts[s] = wv;
        wsum += wv * a.ws_ml[((unit0 + s) * kBM + r) * 2 + 1];
    }
    const float inv = wsum > 0.0f ? 1.0f / wsum : 0.0f;
    const int64_t obase = (((int64_t)b * a.q_tokens + t) * a.q_heads + h) * D;
    for (int d = 0; d < D; ++d) {
        float acc = 0.0f;
        for (int s = 0; s < a.n_splits; ++s)
            if (wts[s] != 0.0f) acc += wts[s] * a.ws_o[((unit0 + s) * kBM + r) * D + d];
        acc *= inv;
        if (a.out_dtype == EKV_DTYPE_F32)
            ((float *)a.out)[obase + d] = acc;
        else
            ((uint16_t *)a.out)[obase + d] = f32_to_bf16_bits(acc);
    }
}

int sm_count() {
    int dev = 0, n = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

// Split count that best fills the SMs with one CTA each: minimise waves per split (with a
// small per-split merge cost), keeping at least 4 key tiles per split.
int choose_splits(int64_t units, int max_tiles) {
    const int sms = sm_count();
    int best = 1;
    double best_cost = 1e30;
    for (int s = 1; s <= kMaxSplits; ++s) {
        if (s > 1 && max_tiles / s < 4) break;
        const double waves = (double)((units * s + sms - 1) / sms) / s;
        const double cost = waves * (1.0 + 0.03 * (s - 1));
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = s;
        }
    }
    return best;
}

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
    attn_tc_kernel<D, Q8><<<grid, C::THREADS, C::SMEM, s>>>(a, n_qtiles);
    if (cudaGetLastError() != cudaSuccess) return EKV_ERR_CUDA;
    if (a.n_splits > 1) {
        merge_splits_kernel<D><<<dim3(n_qtiles, a.pool.kv_heads, a.n_batch), kBM, 0, s>>>(a, n_qtiles);
        if (cudaGetLastError() != cudaSuccess) return EKV_ERR_CUDA;
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

size_t attention_tc_workspace(const PoolView &p, const ekv_attn_params &prm, int max_prefix) {
    if (prm.q_heads <= 0 || p.kv_heads <= 0 || prm.q_heads % p.kv_heads) return 0;
    const int group = prm.q_heads / p.kv_heads;
    const int bn = p.head_dim > 128 ? 64 : 128;
    const int n_qtiles = (prm.q_tokens * group + kBM - 1) / kBM;
    const int64_t units = (int64_t)prm.n_batch * p.kv_heads * n_qtiles;
    const int max_tiles = (max_prefix + bn - 1) / bn + (prm.suffix_len + bn - 1) / bn;
    const int sp = choose_splits(units, max_tiles);
    if (sp <= 1) return 0;
    return (size_t)units * sp * kBM * (p.head_dim + 2) * sizeof(float);
}

int launch_attention_tc(const AttnArgs &a, cudaStream_t s) {
    // a.n_splits == 0 means: a workspace was given at a.ws_o, choose the split count.
    size_t ws = 0;
    if (a.n_splits == 0) ws = (size_t)-1;  // the C-ABI checked the size against the maximum need
    return a.pool.dtype == EKV_DTYPE_Q8_0 ? dispatch<true>(a, s, ws) : dispatch<false>(a, s, ws);
}

}  // namespace ekv
