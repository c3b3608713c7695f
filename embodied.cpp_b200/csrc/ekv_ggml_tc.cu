// ekv_ggml_tc.cu -- the ggml attention ops (GGML_OP_FLASH_ATTN_EXT and the pi0.5 mul_mat /
// soft_max_ext / mul_mat triple) on the tcgen05 attention kernels.
//
// A ggml backend hands over strided tensors (models/pi05.cpp:414-418, models/hy_vla.cpp:376-378 and
// :859, models/lingbot_va.cpp:1263-1266). Where the shape allows it -- head_dim 64, 128 or 256 for
// both K and V, no logit softcap, no ALiBi, a mask shared by all heads -- the call is staged into a
// workspace laid out as a one-layer bf16 pool (K/V in 64-token blocks, one sequence per K batch
// element, identity block tables), Q as bf16 rows, and the ggml mask as visibility bits, and the same
// kernels as ekv_attention run it (one CTA per 128 query rows, or CTA pairs at head_dim 256). The
// result is f32, written straight into dst when dst is laid out as flash_attn_ext's contiguous
// {Dv, Hq, Tq, B}, else scattered through dst's strides.
//
// The visibility bits keep only which entries are -inf. A mask whose visible entries are not all 0
// (an additive bias) sets a device flag while it is converted, and the CUDA-core kernel of
// ekv_ggml_fa.cu, launched behind the tensor-core call and exiting at once when the flag is clear,
// then recomputes the call with the exact additive mask.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <climits>
#include <cmath>
#include <cstdint>
#include <mutex>

#include "../../include/ekv.h"
#include "ekv_device.cuh"
#include "ekv_ggml.h"
#include "ekv_internal.h"

namespace ekv {
namespace {

constexpr int kGgBT = 64;  // tokens per staged block

struct GgTensor {
    const uint8_t *p;
    int32_t type;
    int64_t ne[4], nb[4];
};

GgTensor gg_view(const ekv_tensor *t) {
    GgTensor g;
    g.p = (const uint8_t *)t->data;
    g.type = t->type;
    for (int i = 0; i < 4; ++i) {
        g.ne[i] = t->ne[i];
        g.nb[i] = t->nb[i];
    }
    return g;
}

__device__ __forceinline__ float gg_load(int32_t type, const uint8_t *p) {
    if (type == EKV_DTYPE_F32) return *(const float *)p;
    if (type == EKV_DTYPE_F16) return f16_bits_to_f32(*(const uint16_t *)p);
    return bf16_bits_to_f32(*(const uint16_t *)p);
}

// 8 consecutive elements (stride nb0) of a row -> 8 bf16 (round to nearest even); one or two
// 16-byte loads where the elements are adjacent and aligned
__device__ __forceinline__ uint4 gg_load8_bf16(const GgTensor &t, const uint8_t *row) {
    const bool packed = ((uintptr_t)row & 15) == 0 &&
                        t.nb[0] == (t.type == EKV_DTYPE_F32 ? 4 : 2);
    if (packed && t.type == EKV_DTYPE_BF16) return *(const uint4 *)row;
    if (packed && t.type == EKV_DTYPE_F32) {
        const float4 a = *(const float4 *)row, b = *(const float4 *)(row + 16);
        const __nv_bfloat162 w0 = __floats2bfloat162_rn(a.x, a.y), w1 = __floats2bfloat162_rn(a.z, a.w);
        const __nv_bfloat162 w2 = __floats2bfloat162_rn(b.x, b.y), w3 = __floats2bfloat162_rn(b.z, b.w);
        return make_uint4(*(const uint32_t *)&w0, *(const uint32_t *)&w1, *(const uint32_t *)&w2, *(const uint32_t *)&w3);
    }
    if (packed) {  // f16
        const uint4 h = *(const uint4 *)row;
        const uint32_t hw[4] = {h.x, h.y, h.z, h.w};
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*(const __half2 *)&hw[i]);
            const __nv_bfloat162 b2 = __floats2bfloat162_rn(f.x, f.y);
            w[i] = *(const uint32_t *)&b2;
        }
        return make_uint4(w[0], w[1], w[2], w[3]);
    }
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float x0 = gg_load(t.type, row + (2 * i) * t.nb[0]);
        const float x1 = gg_load(t.type, row + (2 * i + 1) * t.nb[0]);
        const __nv_bfloat162 b2 = __floats2bfloat162_rn(x0, x1);
        w[i] = *(const uint32_t *)&b2;
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// K and V ({D, Tk, Hkv, Bk}) -> bf16 pool tiles: row j of K batch element b is row j % 64 of block
// b * nbk + j / 64. One thread per 8 consecutive d of one (kv, b, h, j) row; consecutive threads take
// consecutive d or, for a tensor whose keys are its contiguous dimension (the triple's V, {Tk, Dv}
// permuted), consecutive keys, so that a warp's loads stay coalesced. Rows j >= Tk of the last block
// are zero (their keys are masked, and a zero V row keeps P.V finite). Index arithmetic is 32-bit
// (the planner bounds the unit count).
__global__ void gg_pack_kv_kernel(const GgTensor k, const GgTensor v, const PoolView p, int nbk, bool k_keys_fastest,
                                  bool v_keys_fastest) {
    const int D = p.head_dim, W = p.swz_bytes, D8 = D / 8;
    const int rows = nbk * kGgBT, H = (int)k.ne[2];
    const int units = (int)k.ne[3] * H * rows * D8;
    for (int u2 = blockIdx.x * blockDim.x + threadIdx.x; u2 < 2 * units; u2 += gridDim.x * blockDim.x) {
        const int kv = u2 >= units;
        const int u = u2 - kv * units;
        const GgTensor &t = kv ? v : k;
        int d8, j, r;
        if (kv ? v_keys_fastest : k_keys_fastest) {
            j = u % rows;
            r = u / rows;
            d8 = r % D8;
            r /= D8;
        } else {
            d8 = u % D8;
            r = u / D8;
            j = r % rows;
            r /= rows;
        }
        const int h = r % H, b = r / H;
        uint4 w = make_uint4(0, 0, 0, 0);
        if (j < t.ne[1])
            w = gg_load8_bf16(t, t.p + (int64_t)d8 * 8 * t.nb[0] + (int64_t)j * t.nb[1] + (int64_t)h * t.nb[2] +
                                     (int64_t)b * t.nb[3]);
        const int block = b * nbk + (j >> 6), row = j & (kGgBT - 1);
        *(uint4 *)(p.prefix + prefix_tile_index(p, 0, block, kv, h) * p.tile_bytes + tile_elem_off(row, d8 * 8, D, W)) = w;
    }
}

// Q ({D, Tq, Hq, Bq}) -> bf16 [Bq][Tq][Hq][D]
__global__ void gg_pack_q_kernel(const GgTensor q, uint16_t *out) {
    const int D8 = (int)q.ne[0] / 8, H = (int)q.ne[2], T = (int)q.ne[1];
    const int units = (int)q.ne[3] * T * H * D8;
    for (int u = blockIdx.x * blockDim.x + threadIdx.x; u < units; u += gridDim.x * blockDim.x) {
        const int d8 = u % D8;
        int r = u / D8;
        const int h = r % H;
        r /= H;
        const int t = r % T, b = r / T;
        *(uint4 *)(out + (int64_t)u * 8) = gg_load8_bf16(q, q.p + (int64_t)d8 * 8 * q.nb[0] + (int64_t)t * q.nb[1] +
                                                                (int64_t)h * q.nb[2] + (int64_t)b * q.nb[3]);
    }
}

// Identity block tables, sequence lengths, the attention batch's sequence ids (query batch element
// b reads K batch element b / (Bq / Bk), ggml's broadcast) and a cleared status word and flag.
__global__ void gg_meta_kernel(int32_t *tables, int32_t *lens, int32_t *seq_ids, int32_t *status, int32_t *flag,
                               int Bk, int nbk, int Tk, int Bq) {
    const int rb = Bq / Bk;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < Bk * nbk; i += gridDim.x * blockDim.x) tables[i] = i;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < Bk; i += gridDim.x * blockDim.x) lens[i] = Tk;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < Bq; i += gridDim.x * blockDim.x) seq_ids[i] = i / rb;
    if (blockIdx.x == 0 && threadIdx.x < 4) status[threadIdx.x] = 0;
    if (blockIdx.x == 0 && threadIdx.x == 0) *flag = 0;
}

// Mask ({>= Tk, >= Tq, 1, Bm}, f16 or f32) -> visibility bits [Bm][Tq][words]: one warp per word,
// lane i reading key 32w + i. A visible entry other than 0 sets *nonbinary.
__global__ void gg_mask_bits_kernel(const GgTensor m, uint32_t *bits, int Tq, int Tk, int words, int Bm,
                                    int32_t *nonbinary) {
    const int lane = threadIdx.x & 31;
    const int64_t n_words = (int64_t)Bm * Tq * words;
    const int64_t warp0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t n_warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    bool odd = false;
    for (int64_t wi = warp0; wi < n_words; wi += n_warps) {
        const int w = (int)(wi % words);
        const int64_t r = wi / words;
        const int t = (int)(r % Tq);
        const int bm = (int)(r / Tq);
        const int key = w * 32 + lane;
        bool vis = false;
        if (key < Tk) {
            const float x = gg_load(m.type, m.p + key * m.nb[0] + t * m.nb[1] + bm * m.nb[3]);
            vis = x != -INFINITY;
            odd |= vis && x != 0.0f;
        }
        const uint32_t word = __ballot_sync(0xffffffffu, vis);
        if (lane == 0) bits[wi] = word;
    }
    if (__any_sync(0xffffffffu, odd) && lane == 0) atomicOr(nonbinary, 1);
}

// [Bq][Tq][Hq][D] f32 -> dst ({D, Hq, Tq, Bq} order of flash_attn_ext, any byte strides): one thread
// per 4 consecutive d (one 16-byte load), 32-bit index arithmetic.
__global__ void gg_scatter_out_kernel(const float *o, uint8_t *dst, int D, int Hq, int Tq, int Bq, int64_t nb0,
                                      int64_t nb1, int64_t nb2, int64_t nb3) {
    const int D4 = D / 4;
    const int n = Bq * Tq * Hq * D4;
    for (int u = blockIdx.x * blockDim.x + threadIdx.x; u < n; u += gridDim.x * blockDim.x) {
        const int d4 = u % D4;
        int r = u / D4;
        const int h = r % Hq;
        r /= Hq;
        const int t = r % Tq, b = r / Tq;
        const float4 x = *(const float4 *)(o + (int64_t)u * 4);
        uint8_t *row = dst + (int64_t)h * nb1 + (int64_t)t * nb2 + (int64_t)b * nb3 + (int64_t)d4 * 4 * nb0;
        *(float *)(row) = x.x;
        *(float *)(row + nb0) = x.y;
        *(float *)(row + 2 * nb0) = x.z;
        *(float *)(row + 3 * nb0) = x.w;
    }
}

constexpr size_t kAlign = 256;
size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

// Where a call's staged operands live in the workspace.
struct GgPlan {
    int D, Tq, Tk, Hq, Hkv, Bq, Bk, Bm, nbk, words;
    bool direct_out;
    PoolView view;
    ekv_attn_params prm;
    size_t off_kv, off_tables, off_lens, off_seq, off_status, off_q, off_out, off_bits, off_split;
    size_t split_bytes, total;
};

bool contiguous_dst(const ekv_tensor *dst) {
    const int64_t D = dst->ne[0], H = dst->ne[1], T = dst->ne[2];
    return dst->nb[0] == 4 && dst->nb[1] == 4 * D && dst->nb[2] == 4 * D * H && dst->nb[3] == 4 * D * H * T &&
           ((uintptr_t)dst->data & 15) == 0;
}

int sms_of_current_device() {
    int dev = 0, n = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

// The tensor-core staging of a call already validated against ggml's shape rules, or false where
// the call needs the CUDA-core kernel.
bool gg_plan(const ekv_tensor *q, const ekv_tensor *k, const ekv_tensor *v, const ekv_tensor *mask, float max_bias,
             float softcap, const ekv_tensor *dst, GgPlan &pl) {
    const int64_t D = q->ne[0];
    if (softcap != 0.0f || max_bias != 0.0f) return false;
    if (!(D == 64 || D == 128 || D == 256) || v->ne[0] != D) return false;
    if (mask && mask->ne[2] != 1) return false;  // a per-head mask
    if (q->ne[1] > (1 << 24) || k->ne[1] > (1 << 24) || q->ne[2] > 4096 || q->ne[3] > 65535) return false;
    pl.D = (int)D;
    pl.Tq = (int)q->ne[1];
    pl.Tk = (int)k->ne[1];
    pl.Hq = (int)q->ne[2];
    pl.Hkv = (int)k->ne[2];
    pl.Bq = (int)q->ne[3];
    pl.Bk = (int)k->ne[3];
    pl.Bm = mask ? (int)mask->ne[3] : 1;
    pl.nbk = (pl.Tk + kGgBT - 1) / kGgBT;
    pl.words = (pl.Tk + 31) / 32;
    pl.direct_out = contiguous_dst(dst);
    // 32-bit index arithmetic in the staging kernels: twice the K/V rows, and the Q / output elements
    if ((int64_t)2 * pl.Bk * pl.Hkv * pl.nbk * kGgBT * (pl.D / 8) > INT32_MAX ||
        (int64_t)pl.Bq * pl.Tq * pl.Hq * pl.D > INT32_MAX)
        return false;

    PoolView &p = pl.view;
    p = PoolView{};
    p.dtype = EKV_DTYPE_BF16;
    p.block_tokens = kGgBT;
    p.n_blocks = pl.Bk * pl.nbk;
    p.kv_heads = pl.Hkv;
    p.head_dim = pl.D;
    p.n_layers = 1;
    p.max_seqs = pl.Bk;
    p.max_blocks_per_seq = pl.nbk;
    p.suffix_rows = 0;
    p.swz_bytes = swizzle_bytes_for(pl.D);
    p.bt_shift = 6;
    p.tile_bytes = (int64_t)kGgBT * pl.D * 2;
    p.suffix_tile_bytes = 0;

    ekv_attn_params &prm = pl.prm;
    prm = ekv_attn_params{};
    prm.layer = 0;
    prm.n_batch = pl.Bq;
    prm.q_tokens = pl.Tq;
    prm.q_heads = pl.Hq;
    prm.scale = 1.0f;
    prm.out_dtype = EKV_DTYPE_F32;
    prm.use_prefix = 1;

    size_t o = 0;
    pl.off_kv = o;
    o = align_up(o + (size_t)p.n_blocks * 2 * p.kv_heads * (size_t)p.tile_bytes);
    pl.off_tables = o;
    o = align_up(o + (size_t)p.n_blocks * 4);
    pl.off_lens = o;
    o = align_up(o + (size_t)pl.Bk * 4);
    pl.off_seq = o;
    o = align_up(o + (size_t)pl.Bq * 4);
    pl.off_status = o;  // status[4], then the non-binary flag
    o = align_up(o + 8 * 4);
    pl.off_q = o;
    o = align_up(o + (size_t)pl.Bq * pl.Tq * pl.Hq * pl.D * 2);
    pl.off_out = o;
    if (!pl.direct_out) o = align_up(o + (size_t)pl.Bq * pl.Tq * pl.Hq * pl.D * 4);
    pl.off_bits = o;
    if (mask) o = align_up(o + (size_t)pl.Bm * pl.Tq * pl.words * 4);
    pl.off_split = o;
    pl.split_bytes = attention_tc_workspace(p, prm, pl.nbk * kGgBT, sms_of_current_device());
    o = align_up(o + pl.split_bytes);
    pl.total = o;
    return true;
}

int grid_for(int64_t units, int threads) {
    const int64_t g = (units + threads - 1) / threads;
    return (int)std::min<int64_t>(std::max<int64_t>(g, 1), (int64_t)sms_of_current_device() * 16);
}

std::mutex g_cache_mu;
void *g_cache_ptr[64];
size_t g_cache_bytes[64];

}  // namespace

size_t ggml_tc_workspace(const ekv_tensor *q, const ekv_tensor *k, const ekv_tensor *v, const ekv_tensor *mask,
                         float max_bias, float logit_softcap, const ekv_tensor *dst) {
    GgPlan pl;
    return gg_plan(q, k, v, mask, max_bias, logit_softcap, dst, pl) ? pl.total : 0;
}

void *ggml_tc_cached_workspace(size_t bytes) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(g_cache_mu);
    if (g_cache_bytes[dev] < bytes) {
        if (g_cache_ptr[dev]) cudaFree(g_cache_ptr[dev]);  // waits for the work that used it
        g_cache_ptr[dev] = nullptr;
        g_cache_bytes[dev] = 0;
        const size_t grow = bytes + bytes / 4;
        if (cudaMalloc(&g_cache_ptr[dev], grow) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        g_cache_bytes[dev] = grow;
    }
    return g_cache_ptr[dev];
}

int ggml_tc_run(const ekv_tensor *q, const ekv_tensor *k, const ekv_tensor *v, const ekv_tensor *mask, float scale,
                float max_bias, float logit_softcap, const ekv_tensor *dst, void *ws, size_t ws_bytes,
                cudaStream_t s, const int32_t **nonbinary) {
    GgPlan pl;
    if (!gg_plan(q, k, v, mask, max_bias, logit_softcap, dst, pl)) return EKV_ERR_UNSUPPORTED;
    if (!ws || ws_bytes < pl.total || ((uintptr_t)ws & 15)) return EKV_ERR_RANGE;
    uint8_t *w = (uint8_t *)ws;
    PoolView &p = pl.view;
    p.prefix = w + pl.off_kv;
    p.suffix = nullptr;
    p.block_tables = (int32_t *)(w + pl.off_tables);
    p.seq_lens = (int32_t *)(w + pl.off_lens);
    p.status = (int32_t *)(w + pl.off_status);
    int32_t *flag = p.status + 4;
    int32_t *seq_ids = (int32_t *)(w + pl.off_seq);
    uint16_t *qb = (uint16_t *)(w + pl.off_q);
    float *ob = pl.direct_out ? (float *)dst->data : (float *)(w + pl.off_out);
    uint32_t *bits = (uint32_t *)(w + pl.off_bits);

    constexpr int T = 256;
    gg_meta_kernel<<<grid_for(std::max<int64_t>(p.n_blocks, pl.Bq), T), T, 0, s>>>(
        p.block_tables, p.seq_lens, seq_ids, p.status, flag, pl.Bk, pl.nbk, pl.Tk, pl.Bq);
    const int64_t kv_units = (int64_t)2 * pl.Bk * pl.Hkv * pl.nbk * kGgBT * (pl.D / 8);
    gg_pack_kv_kernel<<<grid_for(kv_units, T), T, 0, s>>>(gg_view(k), gg_view(v), p, pl.nbk, k->nb[1] < k->nb[0],
                                                          v->nb[1] < v->nb[0]);
    const int64_t q_units = (int64_t)pl.Bq * pl.Tq * pl.Hq * (pl.D / 8);
    gg_pack_q_kernel<<<grid_for(q_units, T), T, 0, s>>>(gg_view(q), qb);
    int launches = 3;
    if (mask) {
        const int64_t words = (int64_t)pl.Bm * pl.Tq * pl.words;
        gg_mask_bits_kernel<<<grid_for(words * 32, T), T, 0, s>>>(gg_view(mask), bits, pl.Tq, pl.Tk, pl.words, pl.Bm,
                                                                  flag);
        ++launches;
    }
    if (cudaGetLastError() != cudaSuccess) return EKV_ERR_CUDA;
    note_launches(launches);

    AttnArgs a{};
    a.pool = p;
    a.layer = 0;
    a.n_batch = pl.Bq;
    a.q_tokens = pl.Tq;
    a.q_heads = pl.Hq;
    a.group = pl.Hq / pl.Hkv;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.mask_flags = mask ? kMaskBits : 0;
    a.suffix_len = 0;
    a.out_dtype = EKV_DTYPE_F32;
    a.use_prefix = 1;
    a.seq_ids = seq_ids;
    a.q = qb;
    a.out = ob;
    a.n_splits = 1;
    if (pl.split_bytes) {
        a.ws_o = (float *)(w + pl.off_split);
        a.n_splits = 0;  // the launcher chooses the split count for this workspace
    }
    a.wait_budget = kDefaultWaitBudget;
    a.mask_bits = mask ? bits : nullptr;
    a.mask_bits_words = pl.words;
    a.mask_bits_nb = pl.Bm;
    if (const int rc = launch_attention_tc(a, s, TcKernel::Auto)) return rc;
    if (!pl.direct_out) {
        const int64_t n = (int64_t)pl.D / 4 * pl.Hq * pl.Tq * pl.Bq;
        gg_scatter_out_kernel<<<grid_for(n, T), T, 0, s>>>(ob, (uint8_t *)dst->data, pl.D, pl.Hq, pl.Tq, pl.Bq,
                                                           dst->nb[0], dst->nb[1], dst->nb[2], dst->nb[3]);
        if (cudaGetLastError() != cudaSuccess) return EKV_ERR_CUDA;
        note_launches(1);
    }
    if (nonbinary) *nonbinary = mask ? flag : nullptr;
    return EKV_OK;
}

}  // namespace ekv
