// ekv_noalloc.cu -- attention entry point that allocates no device memory.
//
// Some callers cannot call cudaMalloc at the point where attention runs: a robot controller or
// serving process that reserves its whole device-memory budget at start-up and forbids
// allocation on the control path (allocation can block, fragment, or fail mid-episode and makes
// latency non-deterministic), or a plugin host such as a ggml backend op callback, which only
// receives tensors the graph allocator has already placed and has nowhere to put a workspace.
// For them ekv_attention_noalloc runs the key-splitting attention with its scratch (the
// per-split partial outputs, running maxima and sums) in the fixed device array below instead
// of a caller-provided workspace.
#include <cuda_runtime.h>

#include <mutex>

#include "ekv_internal.h"

namespace {

// EKV_NOALLOC_SCRATCH_BYTES (16 MiB) of scratch, reserved on every GPU that loads this library
// for as long as the process lives. Every call on a device shares it and it keeps the previous
// call's contents; nothing in it has to start at zero, because each split CTA writes every
// partial row that the merge kernel reads. Calls that overlap on the GPU (different streams or
// pools on the same device without ordering between them) race on it.
static __device__ __align__(256) unsigned char g_ekv_noalloc_scratch[EKV_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
void *g_scratch_addr[kMaxDevices] = {};  // device address of the array, per device (host cache)
std::mutex g_scratch_mu;

}  // namespace

extern "C" int ekv_attention_noalloc(ekv_pool *pool, const ekv_attn_params *p, const void *q, void *out,
                                     ekv_stream_t stream) {
    if (!pool || !p || !q || !out) return EKV_ERR_INVALID_ARG;
    const int dev = pool->cfg.device;
    if (dev < 0) return EKV_ERR_UNSUPPORTED;  // host-only pool
    if (dev >= kMaxDevices) return EKV_ERR_UNSUPPORTED;
    // sized for the pool's device (its SM count sets the key splits), whatever device is current
    const size_t need = ekv_attention_workspace_size(pool, p);
    if (need > (size_t)EKV_NOALLOC_SCRATCH_BYTES) return EKV_ERR_RANGE;
    void *ws = nullptr;
    if (need) {
        std::lock_guard<std::mutex> lock(g_scratch_mu);
        if (!g_scratch_addr[dev]) {
            // Set-up, once per device, with that device current: the array's name is only a
            // host-side stand-in, the kernels need its device address. The caller's current device
            // is put back afterwards.
            int prev = 0;
            if (cudaGetDevice(&prev) != cudaSuccess) {
                cudaGetLastError();
                return EKV_ERR_CUDA;
            }
            if (prev != dev && cudaSetDevice(dev) != cudaSuccess) return EKV_ERR_CUDA;
            void *addr = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&addr, g_ekv_noalloc_scratch);
            if (prev != dev) cudaSetDevice(prev);
            if (e != cudaSuccess || !addr) {
                cudaGetLastError();
                return EKV_ERR_CUDA;
            }
            g_scratch_addr[dev] = addr;
        }
        ws = g_scratch_addr[dev];
    }
    return ekv_attention(pool, p, q, out, ws, need, stream);
}
