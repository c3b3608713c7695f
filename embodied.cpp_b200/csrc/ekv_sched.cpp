// ekv_sched.cpp -- a batching scheduler for the denoise loop over the paged pool: the reference serves
// one request at a time (serving/vla-server.cpp:240-523: receive a vla.PredictRequest, run its whole
// predict, reply); here requests queue, are admitted while sequence slots and pool blocks allow
// (first come, first served), share every layer-step call of a tick (one denoise step of every active
// request, whatever step each is at), and give their blocks back when their last step is done, so the
// next admissions reuse them. The unit of work is the request of vla.proto (serving/vla.proto:33-71,
// request_id; its prefix length stands for what images / lang_tokens / precomputed features produce).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <new>
#include <vector>

#include "ekv_internal.h"

struct ekv_sched {
    ekv_pool *pool = nullptr;
    int32_t max_batch = 0, n_steps = 0, device = 0;
    struct Req {
        uint64_t id;
        int32_t prefix_len, prefix_valid;
    };
    struct Active {
        uint64_t id;
        int32_t seq, step, prefix_len, prefix_valid;
        bool admitted;  // admitted in the current tick (its prefix K/V are due)
    };
    std::deque<Req> queue;
    std::vector<Active> active;         // in admission order
    std::vector<uint8_t> block_used;    // blocks some completed or live request has held
    int64_t reused = 0, reused_tick = 0, completed = 0;
    // host staging (pinned) and device copies of the tick's arrays, max_batch entries each: the batch's
    // seq ids and prefix_valid, then the admitted requests' seq ids, zeros, prefix lengths and first
    // rows in the packed prefix K/V
    // (a host-only pool has no device: d_arr is h_arr)
    int32_t *h_arr = nullptr, *d_arr = nullptr;
    cudaEvent_t copied = nullptr;  // the last tick's upload of h_arr has been read
    bool copy_pending = false;
    std::vector<uint64_t> ids;
    std::vector<int32_t> seqs, steps, adm_index;
};

namespace {

constexpr int kArrays = 6;  // seq ids, prefix_valid, admitted seq ids / zeros / lengths / rows

int32_t *slot(int32_t *base, int32_t max_batch, int which) { return base + (size_t)which * max_batch; }

}  // namespace

extern "C" {

int ekv_sched_create(ekv_pool *pool, int32_t max_batch, int32_t n_steps, ekv_sched **out) {
    if (!pool || !out || max_batch <= 0 || n_steps <= 0) return EKV_ERR_INVALID_ARG;
    *out = nullptr;
    if (max_batch > pool->cfg.max_seqs) return EKV_ERR_RANGE;
    ekv_sched *s = new (std::nothrow) ekv_sched();
    if (!s) return EKV_ERR_ALLOC;
    s->pool = pool;
    s->max_batch = max_batch;
    s->n_steps = n_steps;
    s->device = pool->cfg.device;
    s->block_used.assign((size_t)pool->cfg.n_blocks, 0);
    const size_t bytes = (size_t)kArrays * max_batch * sizeof(int32_t);
    if (s->device < 0) {
        s->h_arr = static_cast<int32_t *>(std::calloc(1, bytes));
        s->d_arr = s->h_arr;
        if (!s->h_arr) {
            delete s;
            return EKV_ERR_ALLOC;
        }
        *out = s;
        return EKV_OK;
    }
    int prev = 0;
    if (cudaGetDevice(&prev) != cudaSuccess || cudaSetDevice(s->device) != cudaSuccess) {
        cudaGetLastError();
        delete s;
        return EKV_ERR_CUDA;
    }
    const bool ok = cudaMallocHost((void **)&s->h_arr, bytes) == cudaSuccess &&
                    cudaMalloc((void **)&s->d_arr, bytes) == cudaSuccess &&
                    cudaMemset(s->d_arr, 0, bytes) == cudaSuccess &&
                    cudaEventCreateWithFlags(&s->copied, cudaEventDisableTiming) == cudaSuccess;
    if (ok) std::memset(s->h_arr, 0, bytes);
    if (!ok) {
        cudaGetLastError();
        if (s->h_arr) cudaFreeHost(s->h_arr);
        if (s->d_arr) cudaFree(s->d_arr);
        if (s->copied) cudaEventDestroy(s->copied);
        delete s;
    }
    cudaSetDevice(prev);
    if (!ok) return EKV_ERR_ALLOC;
    *out = s;
    return EKV_OK;
}

int ekv_sched_destroy(ekv_sched *s) {
    if (!s) return EKV_ERR_INVALID_ARG;
    for (const auto &a : s->active) ekv_seq_free(s->pool, a.seq);
    if (s->device < 0) {
        std::free(s->h_arr);
        delete s;
        return EKV_OK;
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(s->device);
    cudaDeviceSynchronize();  // kernels of the last tick may still read d_arr
    cudaFreeHost(s->h_arr);
    cudaFree(s->d_arr);
    cudaEventDestroy(s->copied);
    cudaSetDevice(prev);
    delete s;
    return EKV_OK;
}

int ekv_sched_submit(ekv_sched *s, uint64_t request_id, int32_t prefix_len, int32_t prefix_valid) {
    if (!s || prefix_len < 0 || prefix_valid < 0 || prefix_valid > prefix_len) return EKV_ERR_INVALID_ARG;
    const int64_t need = ((int64_t)prefix_len + s->pool->cfg.block_tokens - 1) / s->pool->cfg.block_tokens;
    if (need > s->pool->cfg.max_blocks_per_seq || need > s->pool->cfg.n_blocks) return EKV_ERR_RANGE;
    s->queue.push_back({request_id, prefix_len, prefix_valid});
    return EKV_OK;
}

int ekv_sched_begin_tick(ekv_sched *s, ekv_sched_batch *b, ekv_stream_t stream) {
    if (!s || !b) return EKV_ERR_INVALID_ARG;
    for (auto &a : s->active) a.admitted = false;
    s->reused_tick = 0;
    // admission, first come first served: a request that does not fit (no sequence slot, not enough
    // free blocks) waits, and so do the ones behind it
    while (!s->queue.empty() && (int32_t)s->active.size() < s->max_batch) {
        const ekv_sched::Req r = s->queue.front();
        int32_t seq = -1;
        if (ekv_seq_create(s->pool, &seq) != EKV_OK) break;
        if (ekv_seq_resize(s->pool, seq, r.prefix_len) != EKV_OK) {
            ekv_seq_free(s->pool, seq);
            break;
        }
        int32_t nt = 0, nb = 0;
        ekv_seq_get(s->pool, seq, &nt, &nb, nullptr, 0);
        std::vector<int32_t> blocks((size_t)std::max(nb, 1));
        ekv_seq_get(s->pool, seq, nullptr, nullptr, blocks.data(), nb);
        for (int32_t i = 0; i < nb; ++i) {
            uint8_t &u = s->block_used[(size_t)blocks[(size_t)i]];
            if (u) ++s->reused_tick;
            u = 1;
        }
        s->queue.pop_front();
        s->active.push_back({r.id, seq, 0, r.prefix_len, r.prefix_valid, true});
    }
    s->reused += s->reused_tick;
    // the previous tick's upload must have read the staging buffer before it is rewritten
    if (s->copy_pending) {
        if (cudaEventSynchronize(s->copied) != cudaSuccess) return EKV_ERR_CUDA;
        s->copy_pending = false;
    }
    const int32_t n = (int32_t)s->active.size(), M = s->max_batch;
    s->ids.resize((size_t)n);
    s->seqs.resize((size_t)n);
    s->steps.resize((size_t)n);
    s->adm_index.clear();
    int32_t n_adm = 0, max_adm = 0, packed_rows = 0;
    for (int32_t i = 0; i < n; ++i) {
        const auto &a = s->active[(size_t)i];
        s->ids[(size_t)i] = a.id;
        s->seqs[(size_t)i] = a.seq;
        s->steps[(size_t)i] = a.step;
        slot(s->h_arr, M, 0)[i] = a.seq;
        slot(s->h_arr, M, 1)[i] = a.prefix_valid;
        if (a.admitted) {
            slot(s->h_arr, M, 2)[n_adm] = a.seq;
            slot(s->h_arr, M, 3)[n_adm] = 0;
            slot(s->h_arr, M, 4)[n_adm] = a.prefix_len;
            slot(s->h_arr, M, 5)[n_adm] = packed_rows;
            packed_rows += a.prefix_len;
            s->adm_index.push_back(i);
            max_adm = std::max(max_adm, a.prefix_len);
            ++n_adm;
        }
    }
    int rc = ekv_pool_sync(s->pool, stream);  // block tables of the admitted (and freed) sequences
    if (!rc && s->device >= 0 && n > 0) {
        int prev = 0;
        cudaGetDevice(&prev);
        if (prev != s->device) cudaSetDevice(s->device);
        if (cudaMemcpyAsync(s->d_arr, s->h_arr, (size_t)kArrays * M * sizeof(int32_t), cudaMemcpyHostToDevice,
                            (cudaStream_t)stream) != cudaSuccess ||
            cudaEventRecord(s->copied, (cudaStream_t)stream) != cudaSuccess)
            rc = EKV_ERR_CUDA;
        else
            s->copy_pending = true;
        if (prev != s->device) cudaSetDevice(prev);
    }
    if (rc) return rc;
    b->n_batch = n;
    b->request_ids = s->ids.data();
    b->seq_ids_host = s->seqs.data();
    b->steps = s->steps.data();
    b->seq_ids = slot(s->d_arr, M, 0);
    b->prefix_valid = slot(s->d_arr, M, 1);
    b->n_admitted = n_adm;
    b->max_admitted_prefix = max_adm;
    b->admitted_index = s->adm_index.data();
    b->admitted_seq_ids = slot(s->d_arr, M, 2);
    b->admitted_zeros = slot(s->d_arr, M, 3);
    b->admitted_prefix_len = slot(s->d_arr, M, 4);
    b->admitted_src_row = slot(s->d_arr, M, 5);
    b->admitted_rows = packed_rows;
    b->blocks_reused = s->reused_tick;
    b->queued = (int32_t)s->queue.size();
    return EKV_OK;
}

int ekv_sched_end_tick(ekv_sched *s, uint64_t *finished, int32_t cap, int32_t *n_finished) {
    if (!s || (cap > 0 && !finished)) return EKV_ERR_INVALID_ARG;
    int32_t nf = 0;
    std::vector<ekv_sched::Active> keep;
    keep.reserve(s->active.size());
    for (auto &a : s->active) {
        if (++a.step < s->n_steps) {
            keep.push_back(a);
            continue;
        }
        ekv_seq_free(s->pool, a.seq);  // its blocks go back to the free list for the next admissions
        if (nf < cap) finished[nf] = a.id;
        ++nf;
        ++s->completed;
    }
    s->active.swap(keep);
    if (n_finished) *n_finished = nf;
    return EKV_OK;
}

int ekv_sched_stats(const ekv_sched *s, int64_t *completed, int64_t *blocks_reused, int32_t *active, int32_t *queued) {
    if (!s) return EKV_ERR_INVALID_ARG;
    if (completed) *completed = s->completed;
    if (blocks_reused) *blocks_reused = s->reused;
    if (active) *active = (int32_t)s->active.size();
    if (queued) *queued = (int32_t)s->queue.size();
    return EKV_OK;
}

}  // extern "C"
