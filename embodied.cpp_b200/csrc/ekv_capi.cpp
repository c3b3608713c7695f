// ekv_capi.cpp -- C-ABI entry points and the host-side pool manager (block allocator, block
// tables, sequence slots). Every entry point validates its arguments before enqueuing work.
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <new>

#include "ekv_internal.h"

using ekv::PoolView;

namespace {

constexpr size_t kAlign = 1024;

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

bool valid_seq(const ekv_pool *p, int32_t id) {
    return p && id >= 0 && id < p->cfg.max_seqs && p->seqs[(size_t)id].live;
}

int32_t blocks_for(const ekv_pool *p, int32_t n_tokens) {
    return (n_tokens + p->cfg.block_tokens - 1) / p->cfg.block_tokens;
}

// The predicted range within the sequence's length (empty ranges normalised to [0, 0)).
void clamp_pred(ekv_pool::Seq &q) {
    q.pred_hi = std::min(q.pred_hi, q.n_tokens);
    q.pred_lo = std::min(q.pred_lo, q.pred_hi);
    if (q.pred_hi <= q.pred_lo) q.pred_lo = q.pred_hi = 0;
}

void mark_dirty(ekv_pool *p, int32_t id) {
    p->dirty[(size_t)id] = 1;
    p->any_dirty = true;
}

// Makes the pool's device current for one entry point and restores the caller's current device when
// the entry point returns (a library inside a host such as a ggml backend must not move its device).
class DeviceScope {
  public:
    explicit DeviceScope(const ekv_pool *p) {
        if (p->cfg.device < 0) {
            rc_ = EKV_ERR_UNSUPPORTED;  // host-only pool
            return;
        }
        if (cudaGetDevice(&prev_) != cudaSuccess) {
            cudaGetLastError();
            rc_ = EKV_ERR_CUDA;
            return;
        }
        if (prev_ != p->cfg.device && cudaSetDevice(p->cfg.device) != cudaSuccess) {
            rc_ = EKV_ERR_CUDA;
            return;
        }
        switched_ = prev_ != p->cfg.device;
    }
    ~DeviceScope() {
        if (switched_) cudaSetDevice(prev_);
    }
    DeviceScope(const DeviceScope &) = delete;
    DeviceScope &operator=(const DeviceScope &) = delete;
    int rc() const { return rc_; }

  private:
    int prev_ = 0;
    int rc_ = EKV_OK;
    bool switched_ = false;
};

}  // namespace

namespace ekv {
static std::atomic<unsigned long long> g_launches{0};
void note_launches(int n) { g_launches.fetch_add((unsigned long long)n, std::memory_order_relaxed); }
static std::atomic<int> g_debug_stall{0};
bool take_debug_stall() { return g_debug_stall.exchange(0, std::memory_order_relaxed) != 0; }
}  // namespace ekv

extern "C" {

const char *ekv_version(void) { return "ekv 0.1 (sm_100a)"; }

uint64_t ekv_launch_count(void) { return ekv::g_launches.load(std::memory_order_relaxed); }

int ekv_debug_expire_wait(int32_t enable) {
    ekv::g_debug_stall.store(enable ? 1 : 0, std::memory_order_relaxed);
    return EKV_OK;
}

const char *ekv_strerror(int code) {
    switch (code) {
        case EKV_OK: return "ok";
        case EKV_ERR_INVALID_ARG: return "invalid argument";
        case EKV_ERR_CUDA: return "CUDA runtime error";
        case EKV_ERR_POOL_EXHAUSTED: return "pool exhausted";
        case EKV_ERR_NO_SEQ: return "unknown sequence";
        case EKV_ERR_RANGE: return "position or length out of range";
        case EKV_ERR_UNSUPPORTED: return "unsupported shape or dtype";
        case EKV_ERR_DEVICE: return "kernel reported a bad index";
        case EKV_ERR_TIMEOUT: return "kernel wait budget ran out";
        case EKV_ERR_ALLOC: return "allocation failed";
        default: return "unknown error";
    }
}

int ekv_pool_create(const ekv_pool_config *cfg, ekv_pool **out) {
    if (!cfg || !out) return EKV_ERR_INVALID_ARG;
    *out = nullptr;
    const ekv_pool_config c = *cfg;
    if (c.dtype != EKV_DTYPE_BF16 && c.dtype != EKV_DTYPE_Q8_0) return EKV_ERR_UNSUPPORTED;
    if (c.block_tokens <= 0 || c.block_tokens % 8 || c.block_tokens > 256) return EKV_ERR_INVALID_ARG;
    if (c.head_dim <= 0 || c.head_dim > 256 || c.head_dim % 16) return EKV_ERR_UNSUPPORTED;
    if (c.dtype == EKV_DTYPE_Q8_0 && c.head_dim % 32) return EKV_ERR_UNSUPPORTED;
    if (c.n_blocks <= 0 || c.kv_heads <= 0 || c.n_layers <= 0 || c.max_seqs <= 0 ||
        c.max_blocks_per_seq <= 0 || c.suffix_tokens < 0 || c.suffix_tokens > 4096)
        return EKV_ERR_INVALID_ARG;

    ekv_pool *p = new (std::nothrow) ekv_pool();
    if (!p) return EKV_ERR_ALLOC;
    p->cfg = c;
    const DeviceScope dev_scope(p);
    if (c.device >= 0 && dev_scope.rc()) {
        delete p;
        return dev_scope.rc();
    }
    p->sms = 148;
    if (c.device >= 0 && cudaDeviceGetAttribute(&p->sms, cudaDevAttrMultiProcessorCount, c.device) != cudaSuccess) {
        delete p;
        return EKV_ERR_CUDA;
    }
    PoolView &v = p->view;
    v.dtype = c.dtype;
    v.block_tokens = c.block_tokens;
    v.n_blocks = c.n_blocks;
    v.kv_heads = c.kv_heads;
    v.head_dim = c.head_dim;
    v.n_layers = c.n_layers;
    v.max_seqs = c.max_seqs;
    v.max_blocks_per_seq = c.max_blocks_per_seq;
    v.suffix_rows = (c.suffix_tokens + 15) / 16 * 16;
    v.swz_bytes = ekv::swizzle_bytes_for(c.head_dim);
    v.bt_shift = -1;
    for (int sh = 0; sh < 16; ++sh)
        if ((1 << sh) == c.block_tokens) v.bt_shift = sh;
    v.tile_bytes = c.dtype == EKV_DTYPE_BF16
                       ? (int64_t)c.block_tokens * c.head_dim * 2
                       : (int64_t)c.block_tokens * c.head_dim + (int64_t)c.block_tokens * (c.head_dim / 32) * 2;
    v.suffix_tile_bytes = (int64_t)v.suffix_rows * c.head_dim * 2;

    p->bytes_prefix = align_up((size_t)c.n_layers * c.n_blocks * 2 * c.kv_heads * (size_t)v.tile_bytes, kAlign);
    p->bytes_suffix = align_up((size_t)c.n_layers * c.max_seqs * 2 * c.kv_heads * (size_t)v.suffix_tile_bytes, kAlign);
    const size_t bytes_tables = align_up((size_t)c.max_seqs * c.max_blocks_per_seq * 4, kAlign);
    const size_t bytes_lens = align_up((size_t)c.max_seqs * 4, kAlign);
    const size_t bytes_status = kAlign;
    p->bytes_total = p->bytes_prefix + p->bytes_suffix + bytes_tables + bytes_lens + bytes_status;

    if (c.device < 0) {
        // Host-only pool: block tables and sequences without device memory (for testing the
        // allocator where no GPU is present). Data operations on it fail with EKV_ERR_UNSUPPORTED.
        for (int32_t b = 0; b < c.n_blocks; ++b) p->free_blocks.insert(p->free_blocks.end(), b);
        p->seqs.resize((size_t)c.max_seqs);
        p->dirty.assign((size_t)c.max_seqs, 0);
        for (int32_t s = 0; s < c.max_seqs; ++s) p->free_seq_ids.insert(p->free_seq_ids.end(), s);
        *out = p;
        return EKV_OK;
    }
    if (cudaMalloc(&p->dev_base, p->bytes_total) != cudaSuccess) {
        cudaGetLastError();
        delete p;
        return EKV_ERR_ALLOC;
    }
    if (cudaMallocHost((void **)&p->h_status, 4 * sizeof(int32_t)) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(p->dev_base);
        delete p;
        return EKV_ERR_ALLOC;
    }
    if (cudaMemset(p->dev_base, 0, p->bytes_total) != cudaSuccess) {
        cudaFreeHost(p->h_status);
        cudaFree(p->dev_base);
        delete p;
        return EKV_ERR_CUDA;
    }
    uint8_t *base = (uint8_t *)p->dev_base;
    v.prefix = base;
    v.suffix = base + p->bytes_prefix;
    v.block_tables = (int32_t *)(base + p->bytes_prefix + p->bytes_suffix);
    v.seq_lens = (int32_t *)(base + p->bytes_prefix + p->bytes_suffix + bytes_tables);
    v.status = (int32_t *)(base + p->bytes_prefix + p->bytes_suffix + bytes_tables + bytes_lens);

    for (int32_t b = 0; b < c.n_blocks; ++b) p->free_blocks.insert(p->free_blocks.end(), b);
    p->seqs.resize((size_t)c.max_seqs);
    p->dirty.assign((size_t)c.max_seqs, 0);
    for (int32_t s = 0; s < c.max_seqs; ++s) p->free_seq_ids.insert(p->free_seq_ids.end(), s);
    if (cudaDeviceSynchronize() != cudaSuccess) {
        cudaFreeHost(p->h_status);
        cudaFree(p->dev_base);
        delete p;
        return EKV_ERR_CUDA;
    }
    *out = p;
    return EKV_OK;
}

int ekv_pool_destroy(ekv_pool *p) {
    if (!p) return EKV_ERR_INVALID_ARG;
    if (p->cfg.device < 0) {
        delete p;
        return EKV_OK;
    }
    const DeviceScope dev_scope(p);
    cudaDeviceSynchronize();
    if (p->h_status) cudaFreeHost(p->h_status);
    if (p->dev_base) cudaFree(p->dev_base);
    delete p;
    return EKV_OK;
}

int ekv_pool_get_info(const ekv_pool *p, ekv_pool_info *info) {
    if (!p || !info) return EKV_ERR_INVALID_ARG;
    info->bytes_total = p->bytes_total;
    info->bytes_prefix = p->bytes_prefix;
    info->bytes_suffix = p->bytes_suffix;
    info->block_bytes = (size_t)p->view.tile_bytes * 2 * p->cfg.kv_heads;
    info->free_blocks = (int32_t)p->free_blocks.size();
    info->live_seqs = p->cfg.max_seqs - (int32_t)p->free_seq_ids.size();
    info->prefix_base = p->view.prefix;
    info->suffix_base = p->view.suffix;
    info->block_tables = p->view.block_tables;
    info->seq_lens = p->view.seq_lens;
    return EKV_OK;
}

int ekv_pool_status(ekv_pool *p, int32_t *code, ekv_stream_t stream) {
    if (!p || !code) return EKV_ERR_INVALID_ARG;
    if (p->cfg.device < 0) {
        *code = EKV_OK;
        return EKV_OK;
    }
    const DeviceScope dev_scope(p);
    if (const int e = dev_scope.rc()) return e;
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemcpyAsync(p->h_status, p->view.status, 4 * sizeof(int32_t), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemsetAsync(p->view.status, 0, 4 * sizeof(int32_t), s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return EKV_ERR_CUDA;
    *code = p->h_status[0];
    return EKV_OK;
}

int ekv_pool_sync(ekv_pool *p, ekv_stream_t stream) {
    if (!p) return EKV_ERR_INVALID_ARG;
    if (!p->any_dirty || p->cfg.device < 0) return EKV_OK;
    const DeviceScope dev_scope(p);
    if (const int e = dev_scope.rc()) return e;
    cudaStream_t s = (cudaStream_t)stream;
    const int32_t W = p->cfg.max_blocks_per_seq;
    // Pageable sources: cudaMemcpyAsync stages them before returning, so the host vectors may
    // change right after this call.
    std::vector<int32_t> row((size_t)W);
    for (int32_t id = 0; id < p->cfg.max_seqs; ++id) {
        if (!p->dirty[(size_t)id]) continue;
        const ekv_pool::Seq &q = p->seqs[(size_t)id];
        std::fill(row.begin(), row.end(), -1);
        std::copy(q.blocks.begin(), q.blocks.end(), row.begin());
        const int32_t len = q.live ? q.n_tokens : 0;
        if (cudaMemcpyAsync(p->view.block_tables + (size_t)id * W, row.data(), (size_t)W * 4,
                            cudaMemcpyHostToDevice, s) != cudaSuccess ||
            cudaMemcpyAsync(p->view.seq_lens + id, &len, 4, cudaMemcpyHostToDevice, s) != cudaSuccess)
            return EKV_ERR_CUDA;
        p->dirty[(size_t)id] = 0;
    }
    p->any_dirty = false;
    return EKV_OK;
}

int ekv_seq_create(ekv_pool *p, int32_t *seq_id) {
    if (!p || !seq_id) return EKV_ERR_INVALID_ARG;
    if (p->free_seq_ids.empty()) return EKV_ERR_POOL_EXHAUSTED;
    const int32_t id = *p->free_seq_ids.begin();
    p->free_seq_ids.erase(p->free_seq_ids.begin());
    ekv_pool::Seq &q = p->seqs[(size_t)id];
    q.live = true;
    q.n_tokens = 0;
    q.blocks.clear();
    q.pred_lo = q.pred_hi = 0;
    mark_dirty(p, id);
    *seq_id = id;
    return EKV_OK;
}

int ekv_seq_free(ekv_pool *p, int32_t id) {
    if (!valid_seq(p, id)) return EKV_ERR_NO_SEQ;
    ekv_pool::Seq &q = p->seqs[(size_t)id];
    for (int32_t b : q.blocks) p->free_blocks.insert(b);
    q.blocks.clear();
    q.n_tokens = 0;
    q.pred_lo = q.pred_hi = 0;
    q.live = false;
    p->free_seq_ids.insert(id);
    mark_dirty(p, id);
    return EKV_OK;
}

int ekv_seq_resize(ekv_pool *p, int32_t id, int32_t n_tokens) {
    if (!valid_seq(p, id)) return EKV_ERR_NO_SEQ;
    if (n_tokens < 0) return EKV_ERR_INVALID_ARG;
    ekv_pool::Seq &q = p->seqs[(size_t)id];
    const int32_t need = blocks_for(p, n_tokens);
    if (need > p->cfg.max_blocks_per_seq) return EKV_ERR_RANGE;
    const int32_t have = (int32_t)q.blocks.size();
    if (need > have) {
        if ((int32_t)p->free_blocks.size() < need - have) return EKV_ERR_POOL_EXHAUSTED;
        for (int32_t i = have; i < need; ++i) {
            q.blocks.push_back(*p->free_blocks.begin());
            p->free_blocks.erase(p->free_blocks.begin());
        }
    } else {
        for (int32_t i = need; i < have; ++i) p->free_blocks.insert(q.blocks[(size_t)i]);
        q.blocks.resize((size_t)need);
    }
    q.n_tokens = n_tokens;
    clamp_pred(q);
    mark_dirty(p, id);
    return EKV_OK;
}

int ekv_seq_set_blocks(ekv_pool *p, int32_t id, const int32_t *blocks, int32_t n_blocks,
                       int32_t n_tokens) {
    if (!valid_seq(p, id)) return EKV_ERR_NO_SEQ;
    if ((!blocks && n_blocks) || n_blocks < 0 || n_tokens < 0) return EKV_ERR_INVALID_ARG;
    if (n_blocks > p->cfg.max_blocks_per_seq || blocks_for(p, n_tokens) > n_blocks) return EKV_ERR_RANGE;
    ekv_pool::Seq &q = p->seqs[(size_t)id];
    // Every requested block must be free or already owned by this sequence, and distinct.
    std::set<int32_t> own(q.blocks.begin(), q.blocks.end()), seen;
    for (int32_t i = 0; i < n_blocks; ++i) {
        const int32_t b = blocks[i];
        if (b < 0 || b >= p->cfg.n_blocks) return EKV_ERR_INVALID_ARG;
        if (!seen.insert(b).second) return EKV_ERR_INVALID_ARG;
        if (!own.count(b) && !p->free_blocks.count(b)) return EKV_ERR_POOL_EXHAUSTED;
    }
    for (int32_t b : q.blocks) p->free_blocks.insert(b);
    q.blocks.assign(blocks, blocks + n_blocks);
    for (int32_t b : q.blocks) p->free_blocks.erase(b);
    q.n_tokens = n_tokens;
    q.pred_lo = q.pred_hi = 0;
    mark_dirty(p, id);
    return EKV_OK;
}

int ekv_seq_evict_front(ekv_pool *p, int32_t id, int32_t n_blocks) {
    if (!valid_seq(p, id)) return EKV_ERR_NO_SEQ;
    ekv_pool::Seq &q = p->seqs[(size_t)id];
    if (n_blocks < 0 || n_blocks > (int32_t)q.blocks.size()) return EKV_ERR_RANGE;
    for (int32_t i = 0; i < n_blocks; ++i) p->free_blocks.insert(q.blocks[(size_t)i]);
    q.blocks.erase(q.blocks.begin(), q.blocks.begin() + n_blocks);
    const int32_t shift = n_blocks * p->cfg.block_tokens;
    q.n_tokens = std::max(0, q.n_tokens - shift);
    q.pred_lo = std::max(0, q.pred_lo - shift);
    q.pred_hi = std::max(0, q.pred_hi - shift);
    clamp_pred(q);
    mark_dirty(p, id);
    return EKV_OK;
}

int ekv_seq_append_tokens(ekv_pool *p, int32_t id, int32_t n_tokens, int32_t pred) {
    if (!valid_seq(p, id)) return EKV_ERR_NO_SEQ;
    if (n_tokens < 0) return EKV_ERR_INVALID_ARG;
    ekv_pool::Seq &q = p->seqs[(size_t)id];
    const int32_t old = q.n_tokens;
    const bool has_pred = q.pred_hi > q.pred_lo;
    if (pred && has_pred && q.pred_hi != old) return EKV_ERR_UNSUPPORTED;  // a second predicted range
    if ((int64_t)old + n_tokens > INT32_MAX) return EKV_ERR_RANGE;
    if (const int rc = ekv_seq_resize(p, id, old + n_tokens)) return rc;
    if (pred && n_tokens > 0) {
        if (!has_pred) q.pred_lo = old;
        q.pred_hi = old + n_tokens;
    }
    return EKV_OK;
}

int ekv_seq_clear_pred(ekv_pool *p, int32_t id) {
    if (!valid_seq(p, id)) return EKV_ERR_NO_SEQ;
    ekv_pool::Seq &q = p->seqs[(size_t)id];
    if (q.pred_hi <= q.pred_lo) return EKV_OK;
    const int32_t bt = p->cfg.block_tokens, lo = q.pred_lo, hi = q.pred_hi;
    if (hi == q.n_tokens) {
        q.pred_lo = q.pred_hi = 0;
        return ekv_seq_resize(p, id, lo);  // truncation cannot fail
    }
    if (lo % bt || hi % bt) return EKV_ERR_UNSUPPORTED;
    for (int32_t i = lo / bt; i < hi / bt; ++i) p->free_blocks.insert(q.blocks[(size_t)i]);
    q.blocks.erase(q.blocks.begin() + lo / bt, q.blocks.begin() + hi / bt);
    q.n_tokens -= hi - lo;
    q.pred_lo = q.pred_hi = 0;
    mark_dirty(p, id);
    return EKV_OK;
}

int ekv_seq_restore(ekv_pool *p, int32_t id, int32_t n_tokens) {
    if (!valid_seq(p, id)) return EKV_ERR_NO_SEQ;
    ekv_pool::Seq &q = p->seqs[(size_t)id];
    if (n_tokens < 0 || n_tokens > q.n_tokens) return EKV_ERR_RANGE;
    return ekv_seq_resize(p, id, q.n_tokens - n_tokens);
}

int ekv_seq_get_pred(const ekv_pool *p, int32_t id, int32_t *lo, int32_t *hi) {
    if (!valid_seq(p, id)) return EKV_ERR_NO_SEQ;
    const ekv_pool::Seq &q = p->seqs[(size_t)id];
    if (lo) *lo = q.pred_lo;
    if (hi) *hi = q.pred_hi;
    return EKV_OK;
}

int ekv_seq_get(const ekv_pool *p, int32_t id, int32_t *n_tokens, int32_t *n_blocks,
                int32_t *blocks, int32_t cap) {
    if (!valid_seq(p, id)) return EKV_ERR_NO_SEQ;
    const ekv_pool::Seq &q = p->seqs[(size_t)id];
    if (n_tokens) *n_tokens = q.n_tokens;
    if (n_blocks) *n_blocks = (int32_t)q.blocks.size();
    if (blocks) {
        const int32_t n = std::min(cap, (int32_t)q.blocks.size());
        for (int32_t i = 0; i < n; ++i) blocks[i] = q.blocks[(size_t)i];
    }
    return EKV_OK;
}

int ekv_append(ekv_pool *p, int32_t layer, int32_t n_batch, const int32_t *seq_ids,
               const int32_t *dst_pos, const int32_t *n_rows, const int32_t *src_row,
               int32_t max_rows, const void *k, const void *v, ekv_stream_t stream) {
    if (!p || !seq_ids || !dst_pos || !n_rows || !src_row || !k || !v) return EKV_ERR_INVALID_ARG;
    if (layer < 0 || layer >= p->cfg.n_layers || n_batch < 0 || max_rows < 0) return EKV_ERR_INVALID_ARG;
    if (n_batch == 0 || max_rows == 0) return EKV_OK;
    const DeviceScope dev_scope(p);
    if (const int e = dev_scope.rc()) return e;
    return ekv::launch_append(p->view, layer, n_batch, seq_ids, dst_pos, n_rows, src_row, max_rows,
                              k, v, (cudaStream_t)stream);
}

int ekv_append_suffix(ekv_pool *p, int32_t layer, int32_t n_batch, const int32_t *seq_ids,
                      int32_t n_rows, const void *k, const void *v, ekv_stream_t stream) {
    if (!p || !seq_ids || !k || !v) return EKV_ERR_INVALID_ARG;
    if (layer < 0 || layer >= p->cfg.n_layers || n_batch < 0 || n_rows < 0) return EKV_ERR_INVALID_ARG;
    if (n_rows > p->cfg.suffix_tokens) return EKV_ERR_RANGE;
    if (n_batch == 0 || n_rows == 0) return EKV_OK;
    const DeviceScope dev_scope(p);
    if (const int e = dev_scope.rc()) return e;
    return ekv::launch_append_suffix(p->view, layer, n_batch, seq_ids, n_rows, k, v, (cudaStream_t)stream);
}

int ekv_gather(ekv_pool *p, int32_t layer, int32_t id, int32_t pos0, int32_t n_rows, int32_t format,
               void *k_out, void *v_out, ekv_stream_t stream) {
    if (!p || !k_out || !v_out) return EKV_ERR_INVALID_ARG;
    if (format != EKV_GATHER_NATIVE && format != EKV_GATHER_F32) return EKV_ERR_INVALID_ARG;
    if (layer < 0 || layer >= p->cfg.n_layers) return EKV_ERR_INVALID_ARG;
    if (!valid_seq(p, id)) return EKV_ERR_NO_SEQ;
    if (pos0 < 0 || n_rows < 0 || pos0 + n_rows > p->seqs[(size_t)id].n_tokens) return EKV_ERR_RANGE;
    if (n_rows == 0) return EKV_OK;
    const DeviceScope dev_scope(p);
    if (const int e = dev_scope.rc()) return e;
    return ekv::launch_gather(p->view, layer, id, pos0, n_rows, format, k_out, v_out, (cudaStream_t)stream);
}

int ekv_gather_suffix(ekv_pool *p, int32_t layer, int32_t id, int32_t n_rows, int32_t format,
                      void *k_out, void *v_out, ekv_stream_t stream) {
    if (!p || !k_out || !v_out) return EKV_ERR_INVALID_ARG;
    if (format != EKV_GATHER_NATIVE && format != EKV_GATHER_F32) return EKV_ERR_INVALID_ARG;
    if (layer < 0 || layer >= p->cfg.n_layers) return EKV_ERR_INVALID_ARG;
    if (!valid_seq(p, id)) return EKV_ERR_NO_SEQ;
    if (n_rows < 0 || n_rows > p->cfg.suffix_tokens) return EKV_ERR_RANGE;
    if (n_rows == 0) return EKV_OK;
    const DeviceScope dev_scope(p);
    if (const int e = dev_scope.rc()) return e;
    return ekv::launch_gather_suffix(p->view, layer, id, n_rows, format, k_out, v_out, (cudaStream_t)stream);
}

static int fill_attn_args(ekv_pool *p, const ekv_attn_params *prm, const void *q, void *out,
                          ekv::AttnArgs &a) {
    if (!p || !prm || !q || !out || !prm->seq_ids) return EKV_ERR_INVALID_ARG;
    if (((uintptr_t)q | (uintptr_t)out) & 15) return EKV_ERR_INVALID_ARG;  // 16-byte vector loads/stores
    const ekv_pool_config &c = p->cfg;
    if (prm->layer < 0 || prm->layer >= c.n_layers) return EKV_ERR_INVALID_ARG;
    if (prm->n_batch <= 0 || prm->q_tokens <= 0 || prm->q_heads <= 0) return EKV_ERR_INVALID_ARG;
    if (prm->q_heads % c.kv_heads) return EKV_ERR_INVALID_ARG;
    if (prm->suffix_len < 0 || prm->suffix_len > c.suffix_tokens) return EKV_ERR_RANGE;
    if (prm->out_dtype != EKV_DTYPE_BF16 && prm->out_dtype != EKV_DTYPE_F32) return EKV_ERR_UNSUPPORTED;
    if (!(prm->scale > 0.0f) || !std::isfinite(prm->scale)) return EKV_ERR_INVALID_ARG;
    if ((prm->mask_flags & EKV_MASK_BLOCK_CAUSAL) &&
        (prm->chunk_tokens <= 0 || prm->chunk_stride < prm->chunk_tokens || prm->window_chunks <= 0))
        return EKV_ERR_INVALID_ARG;
    if ((prm->mask_flags & (EKV_MASK_SPAN_ONLY | EKV_MASK_SPAN_EXCLUDE)) && (!prm->span_begin || !prm->span_end))
        return EKV_ERR_INVALID_ARG;
    if ((prm->mask_flags & (EKV_MASK_FLEX_SELF | EKV_MASK_FLEX_CROSS)) &&
        (!prm->flex_meta || prm->flex_stride < 0 || (prm->n_batch > 1 && prm->flex_stride == 0) || prm->flex_q0 < 0 ||
         prm->flex_k0 < 0 || prm->flex_window < 0))
        return EKV_ERR_INVALID_ARG;
    if (prm->mask_flags & ~(EKV_MASK_SUFFIX_CAUSAL | EKV_MASK_SUFFIX_PREFIX_LM | EKV_MASK_SPAN_ONLY | EKV_MASK_SPAN_EXCLUDE |
                            EKV_MASK_BLOCK_CAUSAL | EKV_MASK_FLEX_SELF | EKV_MASK_FLEX_CROSS))
        return EKV_ERR_INVALID_ARG;
    a = ekv::AttnArgs{};
    a.pool = p->view;
    a.layer = prm->layer;
    a.n_batch = prm->n_batch;
    a.q_tokens = prm->q_tokens;
    a.q_heads = prm->q_heads;
    a.group = prm->q_heads / c.kv_heads;
    a.scale_log2 = prm->scale * 1.4426950408889634f;
    a.mask_flags = prm->mask_flags;
    a.chunk_tokens = prm->chunk_tokens;
    a.chunk_stride = prm->chunk_stride;
    a.window_chunks = prm->window_chunks;
    a.q_chunk0 = prm->q_chunk0;
    a.suffix_len = prm->suffix_len;
    a.out_dtype = prm->out_dtype;
    a.use_prefix = prm->use_prefix;
    a.seq_ids = prm->seq_ids;
    a.prefix_len = prm->prefix_len;
    a.prefix_valid = prm->prefix_valid;
    a.span_begin = prm->span_begin;
    a.span_end = prm->span_end;
    a.flex_meta = prm->flex_meta;
    a.flex_stride = prm->flex_stride;
    a.flex_q0 = prm->flex_q0;
    a.flex_k0 = prm->flex_k0;
    a.flex_window = prm->flex_window;
    a.q = (const uint16_t *)q;
    a.out = out;
    a.n_splits = 1;
    a.wait_budget = ekv::kDefaultWaitBudget;
    a.debug_stall = 0;
    return EKV_OK;
}

size_t ekv_attention_workspace_size(const ekv_pool *p, const ekv_attn_params *prm) {
    if (!p || !prm) return 0;
    return ekv::attention_tc_workspace(p->view, *prm, p->cfg.max_blocks_per_seq * p->cfg.block_tokens, p->sms);
}

int ekv_attention_algo(ekv_pool *p, const ekv_attn_params *prm, const void *q, void *out,
                       void *workspace, size_t workspace_bytes, int32_t algo, ekv_stream_t stream) {
    ekv::AttnArgs a;
    const int rc = fill_attn_args(p, prm, q, out, a);
    if (rc) return rc;
    const DeviceScope dev_scope(p);
    if (const int e = dev_scope.rc()) return e;
    if (algo == EKV_ALGO_SIMT) return ekv::launch_attention_simt(a, (cudaStream_t)stream);
    if (algo != EKV_ALGO_TC && algo != EKV_ALGO_TC_PAIR && algo != EKV_ALGO_TC_CTA && algo != EKV_ALGO_TC_PAIR64 &&
        algo != EKV_ALGO_TC_HEADS)
        return EKV_ERR_INVALID_ARG;
    const size_t need = ekv::attention_tc_workspace(p->view, *prm, p->cfg.max_blocks_per_seq * p->cfg.block_tokens, p->sms);
    if (workspace && ((uintptr_t)workspace & 15)) return EKV_ERR_INVALID_ARG;
    if (workspace && need && workspace_bytes >= need) {
        // The split count and the workspace carve-up are recomputed by the launcher.
        a.ws_o = (float *)workspace;
        a.n_splits = 0;  // 0 = let the launcher choose from the workspace it was given
    }
    const ekv::TcKernel k = algo == EKV_ALGO_TC_PAIR     ? ekv::TcKernel::Pair
                            : algo == EKV_ALGO_TC_CTA    ? ekv::TcKernel::OneCta
                            : algo == EKV_ALGO_TC_PAIR64 ? ekv::TcKernel::Pair64
                            : algo == EKV_ALGO_TC_HEADS  ? ekv::TcKernel::Heads
                                                         : ekv::TcKernel::Auto;
    return ekv::launch_attention_tc(a, (cudaStream_t)stream, k);
}

int ekv_attention(ekv_pool *p, const ekv_attn_params *prm, const void *q, void *out, void *workspace,
                  size_t workspace_bytes, ekv_stream_t stream) {
    return ekv_attention_algo(p, prm, q, out, workspace, workspace_bytes, EKV_ALGO_TC, stream);
}

int ekv_project_qkv_rope(ekv_pool *p, int32_t layer, int32_t n_batch, const int32_t *seq_ids, int32_t tokens,
                         int32_t q_heads, int32_t hidden, const void *x, const void *wq, const void *wk, const void *wv,
                         const int32_t *positions, float rope_base, void *q_out, void *k_out, void *v_out,
                         ekv_stream_t stream) {
    if (!p || !x || !wq || !wk || !wv || !positions || !q_out) return EKV_ERR_INVALID_ARG;
    if ((k_out == nullptr) != (v_out == nullptr)) return EKV_ERR_INVALID_ARG;
    const ekv_pool_config &c = p->cfg;
    if (layer < 0 || layer >= c.n_layers || n_batch <= 0 || tokens <= 0 || q_heads <= 0 || q_heads % c.kv_heads)
        return EKV_ERR_INVALID_ARG;
    if (hidden <= 0 || hidden % 64 || !(rope_base > 0.0f) || !std::isfinite(rope_base)) return EKV_ERR_INVALID_ARG;
    if ((int64_t)n_batch * tokens > INT_MAX / 2) return EKV_ERR_INVALID_ARG;
    if (((uintptr_t)x | (uintptr_t)wq | (uintptr_t)wk | (uintptr_t)wv | (uintptr_t)q_out | (uintptr_t)k_out |
         (uintptr_t)v_out) & 15)
        return EKV_ERR_INVALID_ARG;
    if (c.head_dim != 64 && c.head_dim != 128 && c.head_dim != 256) return EKV_ERR_UNSUPPORTED;
    if (!k_out) {  // into the suffix slots
        if (!seq_ids || c.suffix_tokens == 0) return EKV_ERR_INVALID_ARG;
        if (tokens > c.suffix_tokens) return EKV_ERR_RANGE;
    }
    const DeviceScope dev_scope(p);
    if (const int e = dev_scope.rc()) return e;
    return ekv::launch_project_qkv(p->view, layer, n_batch, seq_ids, tokens, q_heads, hidden, x, wq, wk, wv, positions,
                                   rope_base, q_out, k_out, v_out, (cudaStream_t)stream);
}

int ekv_append_suffix_attention(ekv_pool *p, const ekv_attn_params *prm, const void *k_suffix,
                                const void *v_suffix, const void *q, void *out, void *workspace,
                                size_t workspace_bytes, ekv_stream_t stream) {
    if (!p || !prm || !k_suffix || !v_suffix) return EKV_ERR_INVALID_ARG;
    if (prm->layer < 0 || prm->layer >= p->cfg.n_layers || prm->n_batch < 0 || prm->suffix_len < 0)
        return EKV_ERR_INVALID_ARG;
    if (prm->suffix_len > p->cfg.suffix_tokens) return EKV_ERR_RANGE;
    if (((uintptr_t)k_suffix | (uintptr_t)v_suffix) & 15) return EKV_ERR_INVALID_ARG;
    if (p->cfg.suffix_tokens == 0) return EKV_ERR_INVALID_ARG;
    ekv::AttnArgs a;
    if (const int rc = fill_attn_args(p, prm, q, out, a)) return rc;
    if (workspace && ((uintptr_t)workspace & 15)) return EKV_ERR_INVALID_ARG;
    const DeviceScope dev_scope(p);
    if (const int e = dev_scope.rc()) return e;
    const cudaStream_t s = (cudaStream_t)stream;
    if (p->cfg.head_dim == 256) {
        // the CTA-pair kernel reads the suffix from the caller's buffers; the slot is not written
        a.k_sfx = (const uint16_t *)k_suffix;
        a.v_sfx = (const uint16_t *)v_suffix;
    } else if (prm->suffix_len > 0) {
        const int rc = ekv::launch_append_suffix(p->view, prm->layer, prm->n_batch, prm->seq_ids, prm->suffix_len,
                                                 k_suffix, v_suffix, s);
        if (rc) return rc;
    }
    const size_t need = ekv::attention_tc_workspace(p->view, *prm, p->cfg.max_blocks_per_seq * p->cfg.block_tokens, p->sms);
    if (workspace && need && workspace_bytes >= need) {
        a.ws_o = (float *)workspace;
        a.n_splits = 0;
    }
    return ekv::launch_attention_tc(a, s, ekv::TcKernel::Auto);
}

}  // extern "C"
