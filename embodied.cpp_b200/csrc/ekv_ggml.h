// ekv_ggml.h -- the tensor-core route of the ggml attention ops (ekv_ggml_tc.cu), used by the op
// surface in ekv_ggml_fa.cu.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "../../include/ekv.h"

namespace ekv {

// Workspace bytes of the tensor-core route for a flash_attn_ext-ordered call (v {Dv, Tk, Hkv, Bk},
// dst {Dv, Hq, Tq, B}), or 0 where the call runs the CUDA-core kernel.
size_t ggml_tc_workspace(const ekv_tensor *q, const ekv_tensor *k, const ekv_tensor *v, const ekv_tensor *mask,
                         float max_bias, float logit_softcap, const ekv_tensor *dst);

// A workspace of at least `bytes` on the current device, held by the library (one per device, grown
// on demand; growing it waits for the work that used the old one).
void *ggml_tc_cached_workspace(size_t bytes);

// Enqueue the call on the tensor-core kernels. EKV_ERR_UNSUPPORTED (nothing enqueued) where the
// call needs the CUDA-core kernel, EKV_ERR_RANGE for a workspace below ggml_tc_workspace. With a
// mask, *nonbinary receives a device flag that the call sets when a visible mask entry is not 0.
int ggml_tc_run(const ekv_tensor *q, const ekv_tensor *k, const ekv_tensor *v, const ekv_tensor *mask, float scale,
                float max_bias, float logit_softcap, const ekv_tensor *dst, void *ws, size_t ws_bytes,
                cudaStream_t s, const int32_t **nonbinary);

}  // namespace ekv
