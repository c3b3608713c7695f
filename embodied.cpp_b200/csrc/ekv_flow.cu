// ekv_flow.cu -- the flow-matching sampler's per-step elementwise work on the device, so that a
// denoise loop needs no host round trip between steps:
//   ekv_flow_step_f32   sample += delta * velocity, the Euler step of pi0.5 (x_t + dt * v,
//                       models/pi05.cpp:856), GR00T (actions += dt * velocity,
//                       models/groot_n1.cpp:764-766) and LingBot's lingbot_scheduler_step_f32
//                       (kernels/lingbot/lingbot_flex_attn_cuda.cu:40-52, 305-319): the product and
//                       the sum each rounded (no fused multiply-add), then optionally rounded to
//                       bf16 (round to nearest even) when the sampler keeps a bf16 state
//   ekv_guidance_f32    classifier-free guidance, lingbot_model_output_guidance_f32
//                       (kernels/lingbot/lingbot_flex_attn_cuda.cu:54-73, 321-337): c = bf16(c),
//                       u = bf16(u), v = u + scale * (c - u), bf16(v), with bf16 rounding optional
// Both are HBM-bound streams: four elements per thread through 16-byte loads and stores, a grid of a
// few waves of the SMs, and a scalar tail for n not a multiple of 4 or unaligned pointers.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "ekv_device.cuh"
#include "ekv_internal.h"

namespace ekv {
namespace {

__device__ __forceinline__ float bf16_round(float x) { return bf16_bits_to_f32(f32_to_bf16_bits(x)); }

__device__ __forceinline__ float step1(float s, float v, float delta, bool round) {
    const float r = __fadd_rn(s, __fmul_rn(v, delta));
    return round ? bf16_round(r) : r;
}

__device__ __forceinline__ float guide1(float c, float u, float scale, bool use, bool round) {
    if (round) c = bf16_round(c);
    if (!use) return c;
    if (round) u = bf16_round(u);
    float v = __fadd_rn(u, __fmul_rn(scale, __fsub_rn(c, u)));
    return round ? bf16_round(v) : v;
}

__global__ void flow_step_kernel(float *__restrict__ sample, const float *__restrict__ vel, int64_t n, float delta,
                                 int round, int vec) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t n4 = vec ? n / 4 : 0;
    for (int64_t i = tid; i < n4; i += stride) {
        float4 s = ((float4 *)sample)[i];
        const float4 v = __ldg((const float4 *)vel + i);
        s.x = step1(s.x, v.x, delta, round);
        s.y = step1(s.y, v.y, delta, round);
        s.z = step1(s.z, v.z, delta, round);
        s.w = step1(s.w, v.w, delta, round);
        ((float4 *)sample)[i] = s;
    }
    for (int64_t i = 4 * n4 + tid; i < n; i += stride) sample[i] = step1(sample[i], vel[i], delta, round);
}

__global__ void guidance_kernel(float *__restrict__ cond, const float *__restrict__ uncond, int64_t n, float scale,
                                int use, int round, int vec) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t n4 = vec ? n / 4 : 0;
    for (int64_t i = tid; i < n4; i += stride) {
        float4 c = ((float4 *)cond)[i];
        const float4 u = use ? __ldg((const float4 *)uncond + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        c.x = guide1(c.x, u.x, scale, use, round);
        c.y = guide1(c.y, u.y, scale, use, round);
        c.z = guide1(c.z, u.z, scale, use, round);
        c.w = guide1(c.w, u.w, scale, use, round);
        ((float4 *)cond)[i] = c;
    }
    for (int64_t i = 4 * n4 + tid; i < n; i += stride)
        cond[i] = guide1(cond[i], use ? uncond[i] : 0.0f, scale, use, round);
}

int grid_for(int64_t work) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t blocks = (work + 255) / 256;
    return (int)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)sms * 8));
}

}  // namespace
}  // namespace ekv

extern "C" int ekv_flow_step_f32(float *sample, const float *velocity, int64_t n, float delta, int32_t bf16_round,
                                 ekv_stream_t stream) {
    if (n < 0 || (n > 0 && (!sample || !velocity))) return EKV_ERR_INVALID_ARG;
    if (n == 0) return EKV_OK;
    const int vec = !(((uintptr_t)sample | (uintptr_t)velocity) & 15);
    ekv::flow_step_kernel<<<ekv::grid_for(vec ? n / 4 + 1 : n), 256, 0, (cudaStream_t)stream>>>(
        sample, velocity, n, delta, bf16_round ? 1 : 0, vec);
    if (cudaGetLastError() != cudaSuccess) return EKV_ERR_CUDA;
    ekv::note_launches(1);
    return EKV_OK;
}

extern "C" int ekv_guidance_f32(float *cond_in_out, const float *uncond, int64_t n, float scale, int32_t use_guidance,
                                int32_t bf16_round, ekv_stream_t stream) {
    if (n < 0 || (n > 0 && (!cond_in_out || (use_guidance && !uncond)))) return EKV_ERR_INVALID_ARG;
    if (n == 0) return EKV_OK;
    const int vec = !(((uintptr_t)cond_in_out | (uintptr_t)(use_guidance ? uncond : cond_in_out)) & 15);
    ekv::guidance_kernel<<<ekv::grid_for(vec ? n / 4 + 1 : n), 256, 0, (cudaStream_t)stream>>>(
        cond_in_out, uncond, n, scale, use_guidance ? 1 : 0, bf16_round ? 1 : 0, vec);
    if (cudaGetLastError() != cudaSuccess) return EKV_ERR_CUDA;
    ekv::note_launches(1);
    return EKV_OK;
}
