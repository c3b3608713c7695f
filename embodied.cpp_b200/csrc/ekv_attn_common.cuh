// ekv_attn_common.cuh -- device helpers shared by the attention kernels (one-CTA and CTA-pair):
// closed-form key-visibility words, paged-block indexing, Q8_0 -> f16 and bf16 -> f16 conversion.
#pragma once

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

namespace ekv {
namespace {
#ifdef EKV_TRACE
// Diagnostic builds only: CTAs (0, 0, 0) and (1, 0, 0) stamp globaltimer (low 32 bits) into shared memory, flushed
// to the host buffer at the end (a global store per stamp would perturb the roles it times).
__constant__ unsigned long long *c_trace = nullptr;
constexpr int kTraceSlots = 1024;
__shared__ unsigned int s_trace[kTraceSlots];
__device__ __forceinline__ bool trace_cta() { return c_trace && blockIdx.x < 2 && blockIdx.y == 0 && blockIdx.z == 0; }
__device__ __forceinline__ void trace_at(int slot) {
    if (trace_cta()) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        s_trace[slot] = (unsigned int)t;
    }
}
#define TRACE(slot) trace_at(slot)
__device__ __forceinline__ void trace_clock(int slot) {
    if (trace_cta()) s_trace[slot] = (unsigned int)clock64();
}
#define TRACE_CLK(slot) trace_clock(slot)
// every CTA: [start, end, SM id] at 2 * kTraceSlots + 4 * (linear block id)
__device__ __forceinline__ unsigned long long trace_span_slot() {
    return 2ull * kTraceSlots + 4ull * (blockIdx.x + gridDim.x * (blockIdx.y + (unsigned long long)gridDim.y * blockIdx.z));
}
__device__ __forceinline__ void trace_init() {
    if (c_trace) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        c_trace[trace_span_slot()] = t;
    }
    if (trace_cta())
        for (int i = 0; i < kTraceSlots; ++i) s_trace[i] = 0u;
}
__device__ __forceinline__ void trace_flush() {
    if (c_trace && threadIdx.x == 0) {
        unsigned long long t;
        unsigned int smid;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
        c_trace[trace_span_slot() + 1] = t;
        c_trace[trace_span_slot() + 2] = smid;
    }
    if (trace_cta())
        for (int i = threadIdx.x; i < kTraceSlots; i += blockDim.x) c_trace[blockIdx.x * kTraceSlots + i] = s_trace[i];
}
#else
#define TRACE(slot) ((void)0)
#define TRACE_CLK(slot) ((void)0)
__device__ __forceinline__ void trace_init() {}
__device__ __forceinline__ void trace_flush() {}
#endif
}  // namespace

namespace {

constexpr long long kWaitBudget = 4000000000LL;  // clock cycles (~2-3 s) before giving up
constexpr int kBM = 128;                          // query rows per CTA (TMEM lanes)
constexpr int kMaxSplits = 8;
constexpr int kDq = 256;  // dequantising threads (Q8_0): 8 warps, two per SM sub-partition

// Key-split count for `units` work units (one CTA or CTA pair each) over `slots` concurrent units,
// `max_tiles` key tiles per unit: minimises waves x (per-unit fixed cost + tiles per split x tile
// cost) + a merge pass when split. The costs are in tile-times, measured on B200: a unit's set-up
// and epilogue (Q load, table, O write) take about five tile-times, the merge about two.
inline int choose_split_count_cost(int64_t units, int max_tiles, int slots, double kFixed, double kMerge) {
    slots = slots > 0 ? slots : 1;
    int best = 1;
    double best_cost = 1e30;
    for (int s = 1; s <= kMaxSplits; ++s) {
        const int per = (max_tiles + s - 1) / s;
        if (s > 1 && per < 2) break;
        const double waves = (double)((units * s + slots - 1) / slots);
        const double cost = waves * (kFixed + per) + (s > 1 ? kMerge : 0.0);
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = s;
        }
    }
    return best;
}

inline int choose_split_count(int64_t units, int max_tiles, int slots) {
    return choose_split_count_cost(units, max_tiles, slots, 5.0, 2.0);
}

// Bits of the keys [lo, hi) inside the 32-key word starting at key w0.
__device__ __forceinline__ uint32_t range_bits(int lo, int hi, int w0) {
    const int a = max(lo - w0, 0), b = min(hi - w0, 32);
    if (b <= a) return 0u;
    const uint32_t upto_b = b >= 32 ? 0xffffffffu : ((1u << b) - 1u);
    const uint32_t below_a = (1u << a) - 1u;  // a < 32 here
    return upto_b & ~below_a;
}

// FLEX masks: the bits of `bits` (keys key0 + i of the call's key order) that query token t may see;
// one metadata word per candidate key.
__device__ __forceinline__ uint32_t flex_word(const MaskDesc &m, int t, int key0, uint32_t bits) {
    const uint32_t qm = (uint32_t)__ldg(m.flex + m.flex_q0 + t);
    if ((qm >> 24) == 0u) return 0u;
    uint32_t out = 0u;
    for (uint32_t rem = bits; rem; rem &= rem - 1u) {
        const int i = __ffs(rem) - 1;
        const uint32_t km = (uint32_t)__ldg(m.flex + m.flex_k0 + key0 + i);
        if (flex_allowed(m.flags, qm, km, m.flex_window)) out |= 1u << i;
    }
    return out;
}

// Visibility of keys [w0, w0+32) for query token t, from key ranges (no per-key loop except for
// the FLEX masks' metadata): the predicate of prefix_allowed / suffix_allowed in closed form.
// n_prefix places suffix keys in the call's key order (FLEX metadata index).
__device__ __forceinline__ uint32_t vis_word(const MaskDesc &m, bool suffix, int w0, int t, int prefix_valid,
                                             int span_b, int span_e, int suffix_len, int n_prefix = 0) {
    if (suffix) {
        int hi = suffix_len;
        if (m.flags & EKV_MASK_SUFFIX_CAUSAL) hi = min(hi, t + 1);
        if ((m.flags & EKV_MASK_SUFFIX_PREFIX_LM) && t == 0) hi = min(hi, 1);
        const uint32_t sbits = range_bits(0, hi, w0);
        return (m.flags & kFlexFlags) ? flex_word(m, t, n_prefix + w0, sbits) : sbits;
    }
    uint32_t bits = range_bits(0, prefix_valid, w0);
    if (m.flags & kMaskBits) bits &= w0 >= 0 ? mask_bits_word(m, t, w0) : 0u;
    if (m.flags & EKV_MASK_SPAN_ONLY) bits &= range_bits(span_b, span_e, w0);
    if (m.flags & EKV_MASK_SPAN_EXCLUDE) bits &= ~range_bits(span_b, span_e, w0);
    if (m.flags & EKV_MASK_BLOCK_CAUSAL) {
        const int qc = m.q_chunk0 + t / m.chunk_tokens;
        const int kc_lo = max(qc - m.window_chunks + 1, max(w0, 0) / m.chunk_stride);
        const int kc_hi = min(qc, (w0 + 31) / m.chunk_stride);
        uint32_t win = 0u;
        for (int kc = kc_lo; kc <= kc_hi; ++kc)
            win |= range_bits(kc * m.chunk_stride, kc * m.chunk_stride + m.chunk_tokens, w0);
        bits &= win;
    }
    if (m.flags & kFlexFlags) bits = flex_word(m, t, w0, bits);
    return bits;
}


// Table index of key k, and the key's row inside its block (shift/mask for power-of-two blocks).
__device__ __forceinline__ int block_index(const PoolView &p, int k, int &rib) {
    if (p.bt_shift >= 0) {
        rib = k & (p.block_tokens - 1);
        return k >> p.bt_shift;
    }
    const int idx = k / p.block_tokens;
    rib = k - idx * p.block_tokens;
    return idx;
}

__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t w) {
    const __half2 h2 = __floats2half2_rn(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
    return *(const uint32_t *)&h2;
}

// 16 Q8_0 values (int8) and their fp16 block scale -> 16 f16 values in registers
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

// Any of the eight f16 values with an all-ones exponent (a bf16 value beyond the f16 range became
// inf, or the input was inf / NaN).
__device__ __forceinline__ bool f16x8_has_inf(uint4 v) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    bool bad = false;
#pragma unroll
    for (int i = 0; i < 4; ++i) bad |= ((w[i] & 0x7C00u) == 0x7C00u) | ((w[i] & 0x7C000000u) == 0x7C000000u);
    return bad;
}

[[maybe_unused]] __device__ __forceinline__ uint4 bf16x8_to_f16x8(uint4 v) {
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2 h2 = __floats2half2_rn(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u));
        w[i] = *(const uint32_t *)&h2;
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}


using sm100::bulk_commit_group;
using sm100::bulk_wait_group_read0;
using sm100::fence_proxy_async;
using sm100::smem_addr;
using sm100::tma_store_2d;
using sm100::tma_store_5d;

// Byte offset of 16-byte unit `c` of staged Q row `r` (rows of `qstr` bytes). When a row has a
// multiple of 8 units (head_dim 64, 128, 256), the units are XOR-swizzled by r & 7, so 8
// consecutive rows of one unit land in 8 different bank groups; other widths are not swizzled.
__device__ __forceinline__ uint32_t q_stage_off(int r, int c, int qstr) {
    const int units = qstr / 16;
    const int m = (units % 8 == 0) ? 7 : 0;
    return (uint32_t)(r * qstr + ((c ^ (r & m)) << 4));
}

// ---- output epilogue through the copy engine ----
// O rows are staged as 4 KB boxes of 32 rows (one TMEM lane quarter) x 128 bytes (64 bf16 or 32
// f32 columns), 128-byte swizzled: 16-byte unit u of box row i sits at unit u ^ (i & 7), the layout
// a CU_TENSOR_MAP_SWIZZLE_128B map reads, so the 8 lanes of a store phase hit 8 distinct bank
// groups. Box (cb, quarter) is at cb * 4 + quarter, so the four quarters of column block cb form
// one 128-row box, which one lane stores with cp.async.bulk.tensor (no thread-issued global stores,
// which drain several times slower than the copy engine's from this kernel).
enum { OUT_THREADS = 0, OUT_TMA_ROWS = 1, OUT_TMA_WS = 2 };
constexpr int kOutBox = 4096;

// Stage columns [c0, c0 + EC) of this thread's row (`lane` of lane quarter `quarter`), times inv.
template <int EC>
__device__ __forceinline__ void stage_o_box(uint8_t *boxes, int quarter, int lane, int c0, const uint32_t *o, float inv,
                                            bool f32) {
    static_assert(EC == 16 || EC == 32, "column chunk");
    const int sw = lane & 7;
    if (f32) {
        uint8_t *row = boxes + ((c0 >> 5) * 4 + quarter) * kOutBox + lane * 128;
        const int u0 = (c0 & 31) >> 2;
#pragma unroll
        for (int i = 0; i < EC / 4; ++i)
            *(float4 *)(row + (((u0 + i) ^ sw) << 4)) =
                make_float4(__uint_as_float(o[4 * i]) * inv, __uint_as_float(o[4 * i + 1]) * inv,
                            __uint_as_float(o[4 * i + 2]) * inv, __uint_as_float(o[4 * i + 3]) * inv);
    } else {
        uint8_t *row = boxes + ((c0 >> 6) * 4 + quarter) * kOutBox + lane * 128;
        const int u0 = (c0 & 63) >> 3;
#pragma unroll
        for (int i = 0; i < EC / 8; ++i) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const __nv_bfloat162 b2 = __floats2bfloat162_rn(__uint_as_float(o[8 * i + 2 * e]) * inv,
                                                                __uint_as_float(o[8 * i + 2 * e + 1]) * inv);
                w[e] = *(const uint32_t *)&b2;
            }
            *(uint4 *)(row + (((u0 + i) ^ sw) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
}

// Epilogue of O columns [c_lo, c_hi) (multiples of 64) by the four warps of one column range
// (one per TMEM lane quarter), all four calling it: two 32-column TMEM loads in flight, staged as
// 32-row boxes; the four quarter boxes of a column block are contiguous, i.e. one 128-row box,
// which one lane stores as soon as the four warps have staged it (named barrier `bar_id`, 128
// threads). Box coordinates: OUT_TMA_ROWS maps the output as (head_dim, head in group, KV head,
// token, batch) with box row i = query row qrow0 + i (rows past the call's tokens fall outside the
// map); OUT_TMA_WS maps the workspace as (head_dim, unit * 128 + row). Each issuing lane waits
// once at the end until its stores have been read.
__device__ __forceinline__ void epilogue_o_tma(const AttnArgs &a, int qrow0, int rows_valid, int g, int b,
                                               const void *omap, int omode, uint8_t *boxes, int quarter, int lane,
                                               uint32_t o_taddr, int c_lo, int c_hi, bool have_o, float inv, bool f32,
                                               int64_t unit, int bar_id) {
    const int boxc = f32 ? 32 : 64;
    bool issued = false;
#pragma unroll 1
    for (int c0 = c_lo; c0 < c_hi; c0 += 64) {
        uint32_t oa[32], ob[32];
        if (have_o) {
            sm100::tmem_load32x2(o_taddr + (uint32_t)c0, o_taddr + (uint32_t)(c0 + 32), oa, ob);
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) oa[i] = ob[i] = 0u;
        }
        stage_o_box<32>(boxes, quarter, lane, c0, oa, inv, f32);
        stage_o_box<32>(boxes, quarter, lane, c0 + 32, ob, inv, f32);
        fence_proxy_async();
        asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
        // the one (bf16) or two (f32) 128-row boxes of these 64 columns, one per issuing warp
        const int cb = c0 / boxc + quarter;
        if (lane == 0 && rows_valid > 0 && cb < (c0 + 64) / boxc) {
            const uint32_t src = smem_addr(boxes + cb * 4 * kOutBox);
            if (omode == OUT_TMA_ROWS)
                tma_store_5d(omap, src, cb * boxc, qrow0 % a.group, g, qrow0 / a.group, b);
            else
                tma_store_2d(omap, src, cb * boxc, (int)(unit * kBM));
            issued = true;
        }
    }
    if (issued) {
        bulk_commit_group();
        bulk_wait_group_read0();
    }
    __syncwarp();
}

// cuTensorMapEncodeTiled from the driver the runtime loaded (no link-time libcuda dependency).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return (PFN_cuTensorMapEncodeTiled_v12000) nullptr;
        return (PFN_cuTensorMapEncodeTiled_v12000)p;
    }();
    return fn;
}

// The epilogue's store route for this call (OUT_*), and the tensor map it stores through.
// With key splits: the f32 workspace as (head_dim, unit * 128 + row), 32 x 128 boxes. Otherwise the
// output [B, Tq, Hq, D] as (head_dim, head in group, KV head, token, batch) with boxes of 128 query
// rows: min(group, 128) heads x max(1, 128 / group) tokens, which needs a group dividing 128 (then
// the map clips exactly the rows past the call's tokens). Other shapes keep the thread-store
// epilogue.
int make_out_map(const AttnArgs &a, int D, int64_t units, CUtensorMap *map) {
    std::memset(map, 0, sizeof(*map));
    const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) return OUT_THREADS;
    const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    if (a.n_splits > 1) {
        const int64_t rows = units * a.n_splits * kBM;
        if (D % 64 || rows > INT_MAX || ((uintptr_t)a.ws_o & 15)) return OUT_THREADS;
        const cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
        const cuuint64_t strides[1] = {(cuuint64_t)D * 4};
        const cuuint32_t box[2] = {32, (cuuint32_t)kBM};
        return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.ws_o, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
                   ? OUT_TMA_WS
                   : OUT_THREADS;
    }
    const bool f32 = a.out_dtype == EKV_DTYPE_F32;
    const int es = f32 ? 4 : 2, boxc = f32 ? 32 : 64;
    if (D % 64 || a.group <= 0 || kBM % a.group || ((uintptr_t)a.out & 15)) return OUT_THREADS;
    const cuuint64_t dims[5] = {(cuuint64_t)D, (cuuint64_t)a.group, (cuuint64_t)a.pool.kv_heads,
                                (cuuint64_t)a.q_tokens, (cuuint64_t)a.n_batch};
    const cuuint64_t strides[4] = {(cuuint64_t)D * es, (cuuint64_t)a.group * D * es, (cuuint64_t)a.q_heads * D * es,
                                   (cuuint64_t)a.q_tokens * a.q_heads * D * es};
    const cuuint32_t box[5] = {(cuuint32_t)boxc, (cuuint32_t)std::min(a.group, kBM), 1,
                               (cuuint32_t)std::max(1, kBM / a.group), 1};
    return enc(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, a.out, dims, strides,
               box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
               ? OUT_TMA_ROWS
               : OUT_THREADS;
}

}  // namespace
}  // namespace ekv
