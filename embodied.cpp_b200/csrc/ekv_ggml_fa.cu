// ekv_ggml_fa.cu -- GGML_OP_FLASH_ATTN_EXT on strided device tensors (the ggml op surface).
//
// The reference builds ggml_flash_attn_ext(Q, K, V, mask, scale, 0, 0) over permuted f32 views
// (models/hy_vla.cpp:376-378, :439-441, :492, and :859 with GQA and a mask; the causal F16 mask of
// hy_mem_causal_mask, :627 and :739; models/lingbot_va.cpp:1263-1266). A ggml backend that
// routes that op to this library passes the tensors as they are: data pointer, type, ggml ne[4]
// (ne[0] fastest) and byte strides nb[4].
// Semantics follow the op: GQA by head (h / (Hq / Hkv)) and batch broadcast, an additive mask
// broadcast over heads and batch, score = scale * q.k with the optional tanh softcap, the ALiBi
// slope when max_bias > 0, softmax in f32, and the result laid out as {Dv, Hq, Tq, B}.
//
// The pi0.5 expert layer builds the same computation as three ggml ops (models/pi05.cpp:414-418:
// mul_mat, soft_max_ext, mul_mat over permuted copies); ekv_mul_mat_soft_max_mul_mat takes that triple's
// operands and result in their own layouts.
//
// Calls whose shape the tcgen05 kernels take (head_dim 64 / 128 / 256, no softcap, no ALiBi, a mask
// shared by the heads) are staged and run there (ekv_ggml_tc.cu). The rest run here, one warp per
// query row: the row's q is staged in shared memory as f32, each lane scores one key of a 32-key
// chunk (reading its K row), the chunk's running max / sum update is a warp reduction, and each lane
// accumulates Dv/32 output columns over the chunk's V rows. The same kernel, gated by a device flag,
// redoes a tensor-core call whose mask turned out to carry additive values.
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdint>

#include "../../include/ekv.h"
#include "ekv_device.cuh"
#include "ekv_ggml.h"
#include "ekv_internal.h"

namespace ekv {
namespace {

constexpr int kFaWarps = 8;
constexpr int kFaMaxD = 512;   // q.k length
constexpr int kFaMaxDv = 256;  // output columns (8 per lane)

struct FaTensor {
    const uint8_t *p;
    int32_t type;
    int64_t ne[4], nb[4];
};

struct FaArgs {
    FaTensor q, k, v, m;
    bool has_mask, alibi;
    float scale, softcap, m0, m1;
    int n_head_log2;
    uint8_t *dst;
    int64_t dnb[4];
};

__device__ __forceinline__ float fa_load(int32_t type, const uint8_t *p) {
    if (type == EKV_DTYPE_F32) return *(const float *)p;
    if (type == EKV_DTYPE_F16) return f16_bits_to_f32(*(const uint16_t *)p);
    return bf16_bits_to_f32(*(const uint16_t *)p);
}

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
    return x;
}
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

// Grid-stride over (8-query group, head, batch) tiles; with `only_if`, nothing is done unless *only_if.
__global__ void __launch_bounds__(kFaWarps * 32) flash_attn_ext_kernel(const FaArgs a, const int32_t *only_if) {
    __shared__ float sq[kFaWarps][kFaMaxD];
    if (only_if && *(volatile const int32_t *)only_if == 0) return;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int64_t nx = (a.q.ne[1] + kFaWarps - 1) / kFaWarps, n_tiles = nx * a.q.ne[2] * a.q.ne[3];
    for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
    const int64_t iq1 = (tile % nx) * kFaWarps + warp;  // query
    const int iq2 = (int)((tile / nx) % a.q.ne[2]), iq3 = (int)(tile / (nx * a.q.ne[2]));  // head, batch
    __syncwarp();
    if (iq1 >= a.q.ne[1]) continue;
    const int D = (int)a.q.ne[0], Dv = (int)a.v.ne[0];
    const int64_t Tk = a.k.ne[1];
    const int64_t ik2 = iq2 / (a.q.ne[2] / a.k.ne[2]), ik3 = iq3 / (a.q.ne[3] / a.k.ne[3]);

    const uint8_t *qrow = a.q.p + iq1 * a.q.nb[1] + iq2 * a.q.nb[2] + iq3 * a.q.nb[3];
    for (int d = lane; d < D; d += 32) sq[warp][d] = fa_load(a.q.type, qrow + d * a.q.nb[0]);
    __syncwarp();

    const uint8_t *mrow = nullptr;
    if (a.has_mask)
        mrow = a.m.p + iq1 * a.m.nb[1] + (iq2 % a.m.ne[2]) * a.m.nb[2] + (iq3 % a.m.ne[3]) * a.m.nb[3];
    float slope = 1.0f;
    if (a.alibi)
        slope = iq2 < a.n_head_log2 ? powf(a.m0, (float)(iq2 + 1)) : powf(a.m1, (float)(2 * (iq2 - a.n_head_log2) + 1));
    const uint8_t *kbase = a.k.p + ik2 * a.k.nb[2] + ik3 * a.k.nb[3];
    const uint8_t *vbase = a.v.p + ik2 * a.v.nb[2] + ik3 * a.v.nb[3];

    float acc[kFaMaxDv / 32];
#pragma unroll
    for (int i = 0; i < kFaMaxDv / 32; ++i) acc[i] = 0.0f;
    float m_run = -INFINITY, l_run = 0.0f;
    for (int64_t k0 = 0; k0 < Tk; k0 += 32) {
        const int64_t j = k0 + lane;
        float s = -INFINITY;
        if (j < Tk) {
            const uint8_t *krow = kbase + j * a.k.nb[1];
            float dot = 0.0f;
            for (int d = 0; d < D; ++d) dot = fmaf(sq[warp][d], fa_load(a.k.type, krow + d * a.k.nb[0]), dot);
            s = dot * a.scale;
            if (a.softcap != 0.0f) s = a.softcap * tanhf(s);
            if (mrow) {
                const float mv = fa_load(a.m.type, mrow + j * a.m.nb[0]);
                s = mv == -INFINITY ? -INFINITY : s + slope * mv;
            }
        }
        const float m_new = fmaxf(m_run, warp_max(s));
        if (m_new == -INFINITY) continue;  // every key so far masked
        const float alpha = m_run == -INFINITY ? 0.0f : expf(m_run - m_new);
        const float p = s == -INFINITY ? 0.0f : expf(s - m_new);
        l_run = l_run * alpha + warp_sum(p);
        m_run = m_new;
#pragma unroll
        for (int i = 0; i < kFaMaxDv / 32; ++i) acc[i] *= alpha;
        const int nj = (int)min((int64_t)32, Tk - k0);
        for (int jj = 0; jj < nj; ++jj) {
            const float pj = __shfl_sync(0xffffffffu, p, jj);
            if (pj == 0.0f) continue;
            const uint8_t *vrow = vbase + (k0 + jj) * a.v.nb[1];
#pragma unroll
            for (int i = 0; i < kFaMaxDv / 32; ++i) {
                const int d = lane + 32 * i;
                if (d < Dv) acc[i] = fmaf(pj, fa_load(a.v.type, vrow + d * a.v.nb[0]), acc[i]);
            }
        }
    }
    const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
    uint8_t *orow = a.dst + iq2 * a.dnb[1] + iq1 * a.dnb[2] + iq3 * a.dnb[3];
#pragma unroll
    for (int i = 0; i < kFaMaxDv / 32; ++i) {
        const int d = lane + 32 * i;
        if (d < Dv) *(float *)(orow + d * a.dnb[0]) = acc[i] * inv;
    }
    }
}

int elem_size(int32_t type) {
    return type == EKV_DTYPE_F32 ? 4 : (type == EKV_DTYPE_F16 || type == EKV_DTYPE_BF16) ? 2 : 0;
}

// Shape, type and stride checks of one tensor: positive extents, strides that are multiples of the
// element size and non-negative, an element-aligned data pointer.
bool tensor_ok(const ekv_tensor *t, bool f32_only) {
    if (!t || !t->data) return false;
    const int es = elem_size(t->type);
    if (es == 0 || (f32_only && t->type != EKV_DTYPE_F32)) return false;
    if ((uintptr_t)t->data % (uintptr_t)es) return false;
    for (int i = 0; i < 4; ++i)
        if (t->ne[i] < 1 || t->nb[i] < 0 || t->nb[i] % es) return false;
    return true;
}

FaTensor fa_view(const ekv_tensor *t) {
    FaTensor f;
    f.p = (const uint8_t *)t->data;
    f.type = t->type;
    for (int i = 0; i < 4; ++i) {
        f.ne[i] = t->ne[i];
        f.nb[i] = t->nb[i];
    }
    return f;
}

}  // namespace
}  // namespace ekv

namespace ekv {
namespace {

// The op on validated-type tensors in flash_attn_ext order: v {Dv, Tk, Hkv, Bk}, dst {Dv, Hq, Tq, B}.
// Validation shared by the op's entry points (ggml's shape rules); EKV_OK for a valid call.
int check_flash_attn(const ekv_tensor *q, const ekv_tensor *k, const ekv_tensor *v, const ekv_tensor *mask, float scale,
                     float max_bias, float logit_softcap, const ekv_tensor *dst) {
    if (!tensor_ok(q, false) || !tensor_ok(k, false) || !tensor_ok(v, false) || !tensor_ok(dst, true))
        return EKV_ERR_INVALID_ARG;
    if (mask && (!tensor_ok(mask, false) || mask->type == EKV_DTYPE_BF16)) return EKV_ERR_INVALID_ARG;
    if (!std::isfinite(scale) || !std::isfinite(max_bias) || !std::isfinite(logit_softcap) || max_bias < 0.0f)
        return EKV_ERR_INVALID_ARG;
    // ggml_flash_attn_ext's shape rules
    if (k->ne[0] != q->ne[0] || v->ne[1] != k->ne[1] || v->ne[2] != k->ne[2] || v->ne[3] != k->ne[3] ||
        q->ne[2] % k->ne[2] || q->ne[3] % k->ne[3])
        return EKV_ERR_INVALID_ARG;
    if (dst->ne[0] != v->ne[0] || dst->ne[1] != q->ne[2] || dst->ne[2] != q->ne[1] || dst->ne[3] != q->ne[3])
        return EKV_ERR_INVALID_ARG;
    if (mask && (mask->ne[0] < k->ne[1] || mask->ne[1] < q->ne[1] || q->ne[2] % mask->ne[2] || q->ne[3] % mask->ne[3]))
        return EKV_ERR_INVALID_ARG;
    if (max_bias > 0.0f && !mask) return EKV_ERR_INVALID_ARG;  // ALiBi needs the mask, as in ggml
    if (q->ne[0] > kFaMaxD || v->ne[0] > kFaMaxDv) return EKV_ERR_UNSUPPORTED;
    if ((q->ne[1] + kFaWarps - 1) / kFaWarps > 0x7fffffff || q->ne[2] > 65535 || q->ne[3] > 65535)
        return EKV_ERR_UNSUPPORTED;
    return EKV_OK;
}

// The op on validated tensors in flash_attn_ext order: v {Dv, Tk, Hkv, Bk}, dst {Dv, Hq, Tq, B}.
// `ws` / `ws_bytes`: the caller's workspace for the tensor-core route, or (ws == null, use_cache)
// the library's per-device one; without either the call runs on the CUDA cores.
int run_flash_attn(const ekv_tensor *q, const ekv_tensor *k, const ekv_tensor *v, const ekv_tensor *mask, float scale,
                   float max_bias, float logit_softcap, const ekv_tensor *dst, void *ws, size_t ws_bytes,
                   bool use_cache, cudaStream_t stream) {
    if (const int rc = check_flash_attn(q, k, v, mask, scale, max_bias, logit_softcap, dst)) return rc;
    const int32_t *redo = nullptr;
    const size_t need = ggml_tc_workspace(q, k, v, mask, max_bias, logit_softcap, dst);
    if (need) {
        if (!ws && use_cache) {
            ws = ggml_tc_cached_workspace(need);
            ws_bytes = ws ? need : 0;
        }
        if (ws) {
            const int rc = ggml_tc_run(q, k, v, mask, scale, max_bias, logit_softcap, dst, ws, ws_bytes, stream, &redo);
            if (rc) return rc;
            if (!redo) return EKV_OK;
        } else if (!use_cache) {
            return EKV_ERR_RANGE;  // the tensor-core route needs the workspace the caller was told
        }
    }

    FaArgs a;
    a.q = fa_view(q);
    a.k = fa_view(k);
    a.v = fa_view(v);
    a.has_mask = mask != nullptr;
    if (mask) a.m = fa_view(mask);
    else a.m = FaTensor{};
    // as the op's compute kernel does: scale / softcap inside the tanh, softcap outside it
    a.softcap = logit_softcap;
    a.scale = logit_softcap != 0.0f ? scale / logit_softcap : scale;
    a.alibi = max_bias > 0.0f;
    const int n_head = (int)q->ne[2];
    a.n_head_log2 = 1 << (int)std::floor(std::log2((double)n_head));
    a.m0 = std::pow(2.0f, -max_bias / (float)a.n_head_log2);
    a.m1 = std::pow(2.0f, -(max_bias / 2.0f) / (float)a.n_head_log2);
    a.dst = (uint8_t *)dst->data;
    for (int i = 0; i < 4; ++i) a.dnb[i] = dst->nb[i];
    // grid-stride: the full grid, or one wave where the launch only redoes a call whose mask held
    // additive values (and exits at once when it did not)
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t n_tiles = ((q->ne[1] + kFaWarps - 1) / kFaWarps) * q->ne[2] * q->ne[3];
    const int64_t cap = redo ? (int64_t)sms : (int64_t)1 << 30;
    flash_attn_ext_kernel<<<(unsigned)std::min(n_tiles, cap), kFaWarps * 32, 0, stream>>>(a, redo);
    if (cudaGetLastError() != cudaSuccess) return EKV_ERR_CUDA;
    note_launches(1);
    return EKV_OK;
}

// `t` with dimensions i and j exchanged (a permuted view of the same bytes).
ekv_tensor swap_dims(const ekv_tensor &t, int i, int j) {
    ekv_tensor r = t;
    r.ne[i] = t.ne[j];
    r.ne[j] = t.ne[i];
    r.nb[i] = t.nb[j];
    r.nb[j] = t.nb[i];
    return r;
}

}  // namespace
}  // namespace ekv

extern "C" int ekv_flash_attn_ext(const ekv_tensor *q, const ekv_tensor *k, const ekv_tensor *v, const ekv_tensor *mask,
                                  float scale, float max_bias, float logit_softcap, const ekv_tensor *dst,
                                  ekv_stream_t stream) {
    return ekv::run_flash_attn(q, k, v, mask, scale, max_bias, logit_softcap, dst, nullptr, 0, true,
                               (cudaStream_t)stream);
}

extern "C" size_t ekv_flash_attn_ext_workspace_size(const ekv_tensor *q, const ekv_tensor *k, const ekv_tensor *v,
                                                    const ekv_tensor *mask, float max_bias, float logit_softcap,
                                                    const ekv_tensor *dst) {
    if (ekv::check_flash_attn(q, k, v, mask, 1.0f, max_bias, logit_softcap, dst)) return 0;
    return ekv::ggml_tc_workspace(q, k, v, mask, max_bias, logit_softcap, dst);
}

extern "C" int ekv_flash_attn_ext_ws(const ekv_tensor *q, const ekv_tensor *k, const ekv_tensor *v,
                                     const ekv_tensor *mask, float scale, float max_bias, float logit_softcap,
                                     const ekv_tensor *dst, void *workspace, size_t workspace_bytes,
                                     ekv_stream_t stream) {
    return ekv::run_flash_attn(q, k, v, mask, scale, max_bias, logit_softcap, dst, workspace, workspace_bytes, false,
                               (cudaStream_t)stream);
}

// mul_mat(K, Q) -> soft_max_ext(kq, mask, scale, max_bias) -> mul_mat(V, attn) of models/pi05.cpp:414-418:
// the same computation as the fused op with V given keys-fastest ({Tk, Dv, ...}, the permute(1, 2, 0, 3)
// of :412) and the result in mul_mat order {Dv, Tq, Hq, B} (before the permute of :419-420). Both are
// views of the caller's bytes with two dimensions exchanged.
namespace ekv {
namespace {
// The triple's V and result as flash_attn_ext-ordered views, or false for mismatched shapes.
bool triple_views(const ekv_tensor *k, const ekv_tensor *q, const ekv_tensor *v, const ekv_tensor *dst, ekv_tensor &vt,
                  ekv_tensor &dt) {
    if (!k || !q || !v || !dst) return false;
    // mul_mat(V, attn) contracts V's ne[0] with attn's ne[0] = keys; V's heads and batch are K's
    if (v->ne[0] != k->ne[1] || v->ne[2] != k->ne[2] || v->ne[3] != k->ne[3]) return false;
    if (dst->ne[0] != v->ne[1] || dst->ne[1] != q->ne[1] || dst->ne[2] != q->ne[2] || dst->ne[3] != q->ne[3])
        return false;
    vt = swap_dims(*v, 0, 1);
    dt = swap_dims(*dst, 1, 2);
    return true;
}
}  // namespace
}  // namespace ekv

extern "C" int ekv_mul_mat_soft_max_mul_mat(const ekv_tensor *k, const ekv_tensor *q, const ekv_tensor *v,
                                            const ekv_tensor *mask, float scale, float max_bias, const ekv_tensor *dst,
                                            ekv_stream_t stream) {
    ekv_tensor vt, dt;
    if (!ekv::triple_views(k, q, v, dst, vt, dt)) return EKV_ERR_INVALID_ARG;
    return ekv::run_flash_attn(q, k, &vt, mask, scale, max_bias, 0.0f, &dt, nullptr, 0, true, (cudaStream_t)stream);
}

extern "C" size_t ekv_mul_mat_soft_max_mul_mat_workspace_size(const ekv_tensor *k, const ekv_tensor *q,
                                                              const ekv_tensor *v, const ekv_tensor *mask,
                                                              float max_bias, const ekv_tensor *dst) {
    ekv_tensor vt, dt;
    if (!ekv::triple_views(k, q, v, dst, vt, dt)) return 0;
    return ekv_flash_attn_ext_workspace_size(q, k, &vt, mask, max_bias, 0.0f, &dt);
}

extern "C" int ekv_mul_mat_soft_max_mul_mat_ws(const ekv_tensor *k, const ekv_tensor *q, const ekv_tensor *v,
                                               const ekv_tensor *mask, float scale, float max_bias,
                                               const ekv_tensor *dst, void *workspace, size_t workspace_bytes,
                                               ekv_stream_t stream) {
    ekv_tensor vt, dt;
    if (!ekv::triple_views(k, q, v, dst, vt, dt)) return EKV_ERR_INVALID_ARG;
    return ekv::run_flash_attn(q, k, &vt, mask, scale, max_bias, 0.0f, &dt, workspace, workspace_bytes, false,
                               (cudaStream_t)stream);
}
