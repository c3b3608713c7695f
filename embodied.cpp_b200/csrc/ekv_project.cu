// ekv_project.cu -- the action expert's Q/K/V projection of one layer-step with RoPE, K and V written
// straight into the pool's suffix slots (or the caller's row-major K/V buffers), on tcgen05 tensor cores.
//
// Replaces, per layer-step of the pi0.5 denoise loop (models/pi05.cpp:391-407):
//   q = mul_mat(Wq, x_norm), k = mul_mat(Wk, x_norm), v = mul_mat(Wv, x_norm)     (:391-393)
//   q_rope, k_rope = rope_ext(.., positions, head_dim, GGML_ROPE_TYPE_NEOX, base)  (:395-402)
//   the concat of k_rope / v onto the cached prefix                            (:406-407)
// so that the attention that follows (ekv_attention over the slot, or ekv_append_suffix_attention over
// the row-major K/V) reads the step's keys without a separate append.
//
// A tile is 256 token rows x one head (D columns) of [q | k | v] = x W^T, held as two 128-row
// accumulators in tensor memory that share every weight stage (so the copy engine moves 32 KB of x and
// D x 128 B of weights per 2 x D/64 x 512 tensor cycles rather than 16 KB + D x 128 B per half of that).
// Persistent CTAs (one per SM) walk the tiles; where tensor memory holds two tiles' accumulators
// (D <= 128) a tile's epilogue runs under the next tile's MMAs. For each tile the copy engine loads
// 256 x 64 tiles of x and D x 64 tiles of the head's weight rows (both K-major, 128-byte swizzled)
// through tensor maps into a ring of stages; one thread issues tcgen05.mma (M = 128 per half, N = D,
// K = 16, bf16, f32 accumulation in tensor memory); sixteen epilogue warps (for each half and TMEM
// lane quarter two, thread = token row, each warp half of the pairs) rotate dimension pairs
// (i, i + D/2) of q and k heads -- the angle in float32, starting at the token's position and
// multiplied by base^(-2/D) after each pair, as ggml's NEOX rope does -- round to bf16 and store: q
// rows to q_out, k / v rows into the swizzled suffix-slot tile of (sequence, layer, KV head) at the
// token's row, or to the caller's row-major buffers.
//
// Every wait is bounded; on expiry the CTA records DEV_ERR_TIMEOUT in the pool's status word.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstring>

#include "../../include/ekv.h"
#include "ekv_attn_common.cuh"
#include "ekv_device.cuh"
#include "ekv_internal.h"
#include "ekv_sm100.cuh"

namespace ekv {
namespace {

using namespace sm100;

constexpr int kPBM = 128, kPBK = 64;

// sin and cos of a RoPE angle x (0 <= x < 65536 * 2 pi): Cody-Waite reduction x = k * 2 pi + r with
// k = rint(x / 2 pi) and 2 pi split into 201 / 32 (8 significant bits, so k * 201/32 is exact for
// k < 2^16) plus the float nearest the remainder 2 pi - 201/32, then the special-function unit's sin
// and cos on r in [-pi, pi] (absolute error about 5e-7, against 2^-9 relative for the bf16 rounding
// that follows).
__device__ __forceinline__ void rope_sincos(float x, float &s, float &c) {
    constexpr float kInv2Pi = 0.159154943091895336f;
    constexpr float kTwoPiHi = 6.28125f;
    constexpr float kTwoPiLo = 1.93530717958647692e-3f;
    const float k = rintf(x * kInv2Pi);
    const float r = fmaf(-k, kTwoPiLo, fmaf(-k, kTwoPiHi, x));
    __sincosf(r, &s, &c);
}

template <int D>
struct PCfg {
    // a tile is MH x 128 token rows: MH accumulators (one per 128 rows) share each weight stage, so the
    // copy engine feeds (MH x 16 KB + D x 128 B) per MH x (D / 64) x 512 tensor cycles
    static constexpr int MH = 2;
    static constexpr int A_BYTES = MH * kPBM * kPBK * 2;  // 32 KB: 256 token rows x 64 hidden
    static constexpr int B_BYTES = D * kPBK * 2;          // D weight rows x 64 hidden
    static constexpr int STAGE = A_BYTES + B_BYTES;
    static constexpr int NS_FIT = (232448 - 2048) / STAGE;
    static constexpr int NS = NS_FIT > 6 ? 6 : NS_FIT;
    static constexpr int OFF_BAR = NS * STAGE;
    static constexpr int SMEM = OFF_BAR + 256 + 1024;  // barriers + alignment slack
    // accumulator buffers (tiles in flight between the MMA and the epilogue) in the 512 TMEM columns
    static constexpr int NB = 2 * MH * D <= 512 ? 2 : 1;
    static constexpr int TMEM_COLS = NB * MH * D;
    // warp 0 copies, warp 1 TMEM + MMA issue, warps 2-17 epilogue: for each 128-row half of a tile and
    // each TMEM lane quarter two warps, each rotating half of the dimension pairs
    static constexpr int EPW = 8 * MH;
    static constexpr int THREADS = (2 + EPW) * 32;
    static_assert(NS >= 3, "stage ring");
    static_assert(TMEM_COLS <= 512 && (TMEM_COLS & (TMEM_COLS - 1)) == 0, "tensor-memory allocation");
    static_assert((2 * NS + 7) * 8 <= 256, "barrier block");
    static_assert(SMEM <= 232448, "shared-memory budget");
};

struct ProjArgs {
    PoolView pool;
    int32_t layer, rows, tokens, q_heads, kv_heads, hidden, to_slot;
    int32_t wide_stores;  // q_out (and row-major k_out / v_out) 32-byte aligned: 32-byte stores
    const int32_t *seq_ids, *positions;
    float theta_scale;
    uint16_t *q_out, *k_out, *v_out;
    long long wait_budget;
};

template <int D>
__global__ void __launch_bounds__(PCfg<D>::THREADS, 1)
    project_qkv_kernel(const ProjArgs a, int m_tiles, const __grid_constant__ CUtensorMap xmap,
                       const __grid_constant__ CUtensorMap wqmap, const __grid_constant__ CUtensorMap wkmap,
                       const __grid_constant__ CUtensorMap wvmap) {
    using C = PCfg<D>;
    constexpr int NS = C::NS;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    uint64_t *bars = (uint64_t *)(smem + C::OFF_BAR);
    uint32_t *tmem_holder = (uint32_t *)(bars + 2 * NS + 5);
    volatile int *abort = (volatile int *)(bars + 2 * NS + 6);
    const uint32_t bar0 = smem_addr(bars);
    // full [0, NS), empty [NS, 2NS), accumulator full 2NS + {0, 1}, accumulator empty 2NS + 2 + {0, 1},
    // every MMA of the CTA finished 2NS + 4
    constexpr int NB = C::NB, MH = C::MH, TROWS = MH * kPBM;
    auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int KT = a.hidden / kPBK;
    const int n_tiles = m_tiles * (a.q_heads + 2 * a.kv_heads);
    // this CTA's tiles: blockIdx.x, blockIdx.x + gridDim.x, ...; tile t = (TROWS token rows m, head hh), m fastest
    const int U = ((int)blockIdx.x < n_tiles) ? (n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;

    trace_init();
    if (threadIdx.x == 0) {
        TRACE(0);
        for (int s = 0; s < NS; ++s) {
            mbar_init(bar(s), 1);
            mbar_init(bar(NS + s), 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(bar(2 * NS + i), 1);
            mbar_init(bar(2 * NS + 2 + i), C::EPW);
        }
        mbar_init(bar(2 * NS + 4), 1);
        *abort = 0;
        mbar_init_fence();
    }
    if (warp == 1) tmem_alloc(smem_addr(tmem_holder), C::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 0) {
        if (lane == 0) {
            int kc = 0;
            bool ok = true;
            for (int i = 0; ok && i < U; ++i) {
                const int tile = (int)blockIdx.x + i * (int)gridDim.x, m0 = (tile % m_tiles) * TROWS, hh = tile / m_tiles;
                const CUtensorMap *wm = hh < a.q_heads ? &wqmap : (hh < a.q_heads + a.kv_heads ? &wkmap : &wvmap);
                const int wrow =
                    (hh < a.q_heads ? hh : (hh < a.q_heads + a.kv_heads ? hh - a.q_heads : hh - a.q_heads - a.kv_heads)) * D;
                for (int k = 0; k < KT; ++k, ++kc) {
                    const int s = kc % NS;
                    if (kc >= NS && !(ok = mbar_wait(bar(NS + s), (uint32_t)(kc / NS - 1) & 1u, abort, a.wait_budget)))
                        break;
                    const uint32_t st = smem_addr(smem + s * C::STAGE);
                    if (kc < 64) TRACE(200 + kc);
                    mbar_arrive_expect_tx(bar(s), (uint32_t)C::STAGE);
                    tma_load_2d(st, &xmap, k * kPBK, m0, bar(s));
                    tma_load_2d(st + C::A_BYTES, wm, k * kPBK, wrow, bar(s));
                }
            }
            if (!ok) {
                *abort = 1;
                report_error(a.pool.status, DEV_ERR_TIMEOUT, 30, blockIdx.x, 0);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = idesc_f16(true, false, D);
            bool ok = true;
            int kc = 0;
            for (int i = 0; ok && i < U; ++i) {
                const int bsel = i % NB;
                const uint32_t acc = tmem + (uint32_t)(bsel * MH * D);
                // the epilogue has read this accumulator buffer's previous tile
                if (i >= NB && !(ok = mbar_wait(bar(2 * NS + 2 + bsel), (uint32_t)(i / NB - 1) & 1u, abort, a.wait_budget)))
                    break;
                tc_fence_after();
                for (int k = 0; k < KT; ++k, ++kc) {
                    const int s = kc % NS;
                    if (!(ok = mbar_wait(bar(s), (uint32_t)(kc / NS) & 1u, abort, a.wait_budget))) break;
                    tc_fence_after();
                    if (kc < 64) TRACE(300 + kc);
                    const uint32_t st = smem_addr(smem + s * C::STAGE);
                    const uint64_t bd = sdesc(st + C::A_BYTES, 16, 1024, 2u);
                    const uint64_t bv[4] = {bd, bd + 2, bd + 4, bd + 6};  // K steps of 32 bytes in the 128-byte rows
#pragma unroll
                    for (int h = 0; h < MH; ++h) {  // rows [128 h, 128 h + 128) of the tile: 16 KB further in the stage
                        const uint64_t ad = sdesc(st + h * kPBM * kPBK * 2, 16, 1024, 2u);
                        const uint64_t av[4] = {ad, ad + 2, ad + 4, ad + 6};
                        mma_ss_x4<false>(acc + (uint32_t)(h * D), av, bv, idesc, k > 0 ? 1u : 0u);
                    }
                    mma_commit(bar(NS + s));
                }
                if (ok) mma_commit(bar(2 * NS + bsel));  // this tile's accumulators are complete
                if (i < 32) TRACE(100 + i);
            }
            if (!ok) {
                *abort = 1;
                report_error(a.pool.status, DEV_ERR_TIMEOUT, 31, blockIdx.x, 0);
            }
            mma_commit(bar(2 * NS + 4));  // every MMA of the CTA finished before teardown
            mbar_wait_drain(bar(2 * NS + 4), 0u, a.wait_budget);
        }
        __syncwarp();
    } else {
        // ---- epilogue: warp e = warp - 2 takes the tile's 128-row half h = e >> 3; thread = token row
        // 128 h + 32 (warp & 3) + lane; dimension pairs [0, D/4) for (e >> 2) even, [D/4, D/2) for odd ----
        const int q4 = warp & 3, part = ((warp - 2) >> 2) & 1, mh = (warp - 2) >> 3;
        const uint32_t lb = ((uint32_t)(32 * q4)) << 16;
        constexpr int W = 128;  // the pool's swizzle width at head_dim 64 / 128 / 256 (checked at launch)
        for (int i = 0; i < U; ++i) {
            const int tile = (int)blockIdx.x + i * (int)gridDim.x, m0 = (tile % m_tiles) * TROWS, hh = tile / m_tiles;
            const int bsel = i % NB;
            // the row's set-up (position, first RoPE angle, destination) reads global memory: done before the
            // accumulator is ready, under the tile's MMAs
            const int grow = m0 + mh * kPBM + 32 * q4 + lane;
            const bool row_ok = grow < a.rows;
            const bool is_q = hh < a.q_heads, is_k = !is_q && hh < a.q_heads + a.kv_heads;
            const bool rope = is_q || is_k;
            const int g = is_q ? 0 : (is_k ? hh - a.q_heads : hh - a.q_heads - a.kv_heads);
            const int b = row_ok ? grow / a.tokens : 0, t = row_ok ? grow - b * a.tokens : 0;
            float theta = row_ok ? (float)a.positions[grow] : 0.0f;
            // the angle of this warp's first pair: ggml's float32 recurrence, advanced over the other part's pairs
            for (int j = 0; j < part * (D / 4); ++j) theta = __fmul_rn(theta, a.theta_scale);
            // destination of this row: q_out row, a suffix-slot tile row (swizzled), or a row-major K / V row
            uint8_t *dst = nullptr;
            bool slot = false;
            if (row_ok) {
                if (is_q) {
                    dst = (uint8_t *)(a.q_out + ((int64_t)grow * a.q_heads + hh) * D);
                } else if (a.to_slot) {
                    const int seq = a.seq_ids[b];
                    if (seq < 0 || seq >= a.pool.max_seqs) {
                        report_error(a.pool.status, DEV_ERR_BAD_SEQ, b, seq, 6);
                    } else {
                        dst = a.pool.suffix + suffix_tile_index(a.pool, a.layer, seq, is_k ? 0 : 1, g) * a.pool.suffix_tile_bytes;
                        slot = true;
                    }
                } else {
                    dst = (uint8_t *)((is_k ? a.k_out : a.v_out) + ((int64_t)grow * a.kv_heads + g) * D);
                }
            }
            const bool done = mbar_wait(bar(2 * NS + bsel), (uint32_t)(i / NB) & 1u, abort, a.wait_budget);
            if (!done) {
                if (lane == 0) report_error(a.pool.status, DEV_ERR_TIMEOUT, 32, blockIdx.x, hh);
                break;
            }
            tc_fence_after();
            if (lane == 0 && i < 16) TRACE(400 + 16 * (warp - 2) + i);
            const uint32_t acc = tmem + lb + (uint32_t)(bsel * MH * D + mh * D);
            // 16 dimension pairs per step; the next step's accumulator columns load while this step rotates
            // and stores
            const int c_beg = part * (D / 4), c_end = c_beg + D / 4;
            const bool wide = a.wide_stores && !slot;  // 32-byte stores into 32-byte aligned rows
            uint32_t lo[16], hi[16];
            tmem_load16x2_nowait(acc + (uint32_t)c_beg, acc + (uint32_t)(c_beg + D / 2), lo, hi);
            tmem_wait_ld16x2(lo, hi);
#pragma unroll 1
            for (int c0 = c_beg; c0 < c_end; c0 += 16) {
                float o0[16], o1[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    o0[j] = __uint_as_float(lo[j]);
                    o1[j] = __uint_as_float(hi[j]);
                }
                const bool more = c0 + 16 < c_end;
                if (more) tmem_load16x2_nowait(acc + (uint32_t)(c0 + 16), acc + (uint32_t)(c0 + 16 + D / 2), lo, hi);
                if (rope) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float x0 = o0[j], x1 = o1[j];
                        float sn, cs;
                        rope_sincos(theta, sn, cs);
                        o0[j] = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
                        o1[j] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
                        theta = __fmul_rn(theta, a.theta_scale);
                    }
                }
                if (dst) {
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        const float *o = half ? o1 : o0;
                        const int c = c0 + half * (D / 2);
                        uint32_t w[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            const __nv_bfloat162 b2 = __floats2bfloat162_rn(o[2 * e], o[2 * e + 1]);
                            w[e] = *(const uint32_t *)&b2;
                        }
                        if (wide) {
                            st_global_32B(dst + (uint32_t)c * 2u, w);
                        } else if (slot) {
                            // the swizzle keeps the two 16-byte units of an aligned 32-byte group together, in
                            // either order: one 32-byte store, halves swapped where the row's swizzle swaps them
                            // (a select, not a branch: odd and even rows of a warp take the same path)
                            const uint32_t off0 = tile_elem_off(t, c, D, W), off1 = tile_elem_off(t, c + 8, D, W);
                            const uint32_t lo_off = min(off0, off1);
                            if (max(off0, off1) == lo_off + 16u && ((uintptr_t)(dst + lo_off) & 31u) == 0u) {
                                const bool sw = off0 > off1;
                                uint32_t x[8];
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    x[e] = sw ? w[4 + e] : w[e];
                                    x[4 + e] = sw ? w[e] : w[4 + e];
                                }
                                st_global_32B(dst + lo_off, x);
                            } else {
                                *(uint4 *)(dst + off0) = make_uint4(w[0], w[1], w[2], w[3]);
                                *(uint4 *)(dst + off1) = make_uint4(w[4], w[5], w[6], w[7]);
                            }
                        } else {
#pragma unroll
                            for (int u = 0; u < 2; ++u)  // 8 values = one 16-byte unit
                                *(uint4 *)(dst + (uint32_t)(c + 8 * u) * 2u) = make_uint4(w[4 * u], w[4 * u + 1], w[4 * u + 2], w[4 * u + 3]);
                        }
                    }
                }
                if (more) tmem_wait_ld16x2(lo, hi);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(2 * NS + 2 + bsel));  // the accumulator buffer may take the next tile
            if (lane == 0 && i < 16) TRACE(700 + 16 * (warp - 2) + i);
        }
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
    if (threadIdx.x == 0) TRACE(11);
    trace_flush();
}

// 2-D tensor map of a row-major bf16 matrix [rows][cols] with boxes of 64 columns x box_rows rows, 128-byte
// swizzled (the K-major operand layout of the MMA).
bool make_rows_map(const void *base, int64_t rows, int64_t cols, int box_rows, CUtensorMap *map) {
    std::memset(map, 0, sizeof(*map));
    const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc || ((uintptr_t)base & 15) || (cols * 2) % 16) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kPBK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void *)base, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int D>
int launch_project(const ProjArgs &a, const void *x, const void *wq, const void *wk, const void *wv, cudaStream_t s) {
    using C = PCfg<D>;
    if (a.pool.swz_bytes != 128) return EKV_ERR_UNSUPPORTED;
    CUtensorMap xm, qm, km, vm;
    if (!make_rows_map(x, a.rows, a.hidden, C::MH * kPBM, &xm) || !make_rows_map(wq, (int64_t)a.q_heads * D, a.hidden, D, &qm) ||
        !make_rows_map(wk, (int64_t)a.kv_heads * D, a.hidden, D, &km) ||
        !make_rows_map(wv, (int64_t)a.kv_heads * D, a.hidden, D, &vm))
        return EKV_ERR_INVALID_ARG;
    static int attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr_done[dev]) {
        if (cudaFuncSetAttribute(project_qkv_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
            return EKV_ERR_CUDA;
        attr_done[dev] = 1;
    }
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int m_tiles = (a.rows + C::MH * kPBM - 1) / (C::MH * kPBM);
    const int n_tiles = m_tiles * (a.q_heads + 2 * a.kv_heads);
    project_qkv_kernel<D><<<std::min(n_tiles, sms), C::THREADS, C::SMEM, s>>>(a, m_tiles, xm, qm, km, vm);
    if (cudaGetLastError() != cudaSuccess) return EKV_ERR_CUDA;
    note_launches(1);
    return EKV_OK;
}

}  // namespace

#ifdef EKV_TRACE
int project_debug_set_trace(unsigned long long *buf) {
    return cudaMemcpyToSymbol(c_trace, &buf, sizeof(buf)) == cudaSuccess ? 0 : -2;
}
#endif

int launch_project_qkv(const PoolView &p, int layer, int n_batch, const int32_t *seq_ids, int tokens, int q_heads,
                       int hidden, const void *x, const void *wq, const void *wk, const void *wv, const int32_t *positions,
                       float rope_base, void *q_out, void *k_out, void *v_out, cudaStream_t s) {
    ProjArgs a{};
    a.pool = p;
    a.layer = layer;
    a.rows = n_batch * tokens;
    a.tokens = tokens;
    a.q_heads = q_heads;
    a.kv_heads = p.kv_heads;
    a.hidden = hidden;
    a.to_slot = k_out == nullptr;
    a.seq_ids = seq_ids;
    a.positions = positions;
    a.theta_scale = powf(rope_base, -2.0f / (float)p.head_dim);
    a.q_out = (uint16_t *)q_out;
    a.k_out = (uint16_t *)k_out;
    a.v_out = (uint16_t *)v_out;
    a.wait_budget = kDefaultWaitBudget;
    a.wide_stores = (((uintptr_t)q_out | (uintptr_t)k_out | (uintptr_t)v_out) & 31) == 0;
    switch (p.head_dim) {
        case 64: return launch_project<64>(a, x, wq, wk, wv, s);
        case 128: return launch_project<128>(a, x, wq, wk, wv, s);
        case 256: return launch_project<256>(a, x, wq, wk, wv, s);
        default: return EKV_ERR_UNSUPPORTED;
    }
}

}  // namespace ekv
