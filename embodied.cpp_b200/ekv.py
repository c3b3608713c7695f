"""Python binding of libekv.so, the B200 paged KV-cache + masked-attention library.

A thin ctypes mirror of include/ekv.h for tests, the benchmark and Python callers: the pool
(`Pool`), sequence/block-table management, append / gather, and attention. Device buffers are
torch CUDA tensors (passed by data pointer); every call is asynchronous on the given (or
current) torch stream, like the C-ABI.

There is no fallback: if libekv.so is missing or fails to load, importing this module raises.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

HERE = os.path.dirname(os.path.abspath(__file__))
# EKV_LIB_PATH selects another build of the same library (e.g. a tracing build).
LIB_PATH = os.environ.get("EKV_LIB_PATH") or os.path.join(HERE, "libekv.so")

OK = 0
ERR_INVALID_ARG, ERR_CUDA, ERR_POOL_EXHAUSTED, ERR_NO_SEQ = -1, -2, -3, -4
ERR_RANGE, ERR_UNSUPPORTED, ERR_DEVICE, ERR_TIMEOUT, ERR_ALLOC = -5, -6, -7, -8, -9

DTYPE_F32, DTYPE_F16, DTYPE_Q8_0, DTYPE_BF16 = 0, 1, 8, 30
GATHER_NATIVE, GATHER_F32 = 0, 1
MASK_SUFFIX_CAUSAL = 1 << 0
MASK_SUFFIX_PREFIX_LM = 1 << 1
MASK_SPAN_ONLY = 1 << 2
MASK_SPAN_EXCLUDE = 1 << 3
MASK_BLOCK_CAUSAL = 1 << 4
MASK_FLEX_SELF = 1 << 5
MASK_FLEX_CROSS = 1 << 6


def flex_meta_word(seq: int, frame: int, clean: bool) -> int:
    """EKV_FLEX_META: the metadata word of a token for the FLEX masks (negative seq = padding)."""
    if seq < 0:
        return 0
    w = ((seq + 1) << 24) | ((1 if clean else 0) << 23) | (frame & 0x7FFFFF)
    return w - (1 << 32) if w >= (1 << 31) else w
ALGO_TC, ALGO_SIMT, ALGO_TC_PAIR, ALGO_TC_CTA, ALGO_TC_PAIR64, ALGO_TC_HEADS = 0, 1, 2, 3, 4, 5

# Device-side error codes written into the pool status word by kernels.
DEV_ERR_BAD_BLOCK, DEV_ERR_BAD_SEQ, DEV_ERR_BAD_POS, DEV_ERR_TIMEOUT, DEV_ERR_F16_RANGE = 1, 2, 3, 4, 5


class PoolConfig(C.Structure):
    _fields_ = [("device", C.c_int32), ("dtype", C.c_int32), ("block_tokens", C.c_int32),
                ("n_blocks", C.c_int32), ("kv_heads", C.c_int32), ("head_dim", C.c_int32),
                ("n_layers", C.c_int32), ("max_seqs", C.c_int32), ("max_blocks_per_seq", C.c_int32),
                ("suffix_tokens", C.c_int32)]


class PoolInfo(C.Structure):
    _fields_ = [("bytes_total", C.c_size_t), ("bytes_prefix", C.c_size_t),
                ("bytes_suffix", C.c_size_t), ("block_bytes", C.c_size_t),
                ("free_blocks", C.c_int32), ("live_seqs", C.c_int32),
                ("prefix_base", C.c_void_p), ("suffix_base", C.c_void_p),
                ("block_tables", C.c_void_p), ("seq_lens", C.c_void_p)]


class AttnParams(C.Structure):
    _fields_ = [("layer", C.c_int32), ("n_batch", C.c_int32), ("q_tokens", C.c_int32),
                ("q_heads", C.c_int32), ("scale", C.c_float), ("mask_flags", C.c_int32),
                ("chunk_tokens", C.c_int32), ("chunk_stride", C.c_int32),
                ("window_chunks", C.c_int32), ("q_chunk0", C.c_int32), ("suffix_len", C.c_int32),
                ("out_dtype", C.c_int32), ("use_prefix", C.c_int32), ("reserved", C.c_int32),
                ("seq_ids", C.c_void_p), ("prefix_len", C.c_void_p), ("prefix_valid", C.c_void_p),
                ("span_begin", C.c_void_p), ("span_end", C.c_void_p), ("flex_meta", C.c_void_p),
                ("flex_stride", C.c_int32), ("flex_q0", C.c_int32), ("flex_k0", C.c_int32),
                ("flex_window", C.c_int32)]


class SchedBatch(C.Structure):
    _fields_ = [("n_batch", C.c_int32), ("request_ids", C.POINTER(C.c_uint64)),
                ("seq_ids_host", C.POINTER(C.c_int32)), ("steps", C.POINTER(C.c_int32)),
                ("seq_ids", C.c_void_p), ("prefix_valid", C.c_void_p), ("n_admitted", C.c_int32),
                ("max_admitted_prefix", C.c_int32), ("admitted_index", C.POINTER(C.c_int32)),
                ("admitted_seq_ids", C.c_void_p), ("admitted_zeros", C.c_void_p),
                ("admitted_prefix_len", C.c_void_p), ("admitted_src_row", C.c_void_p), ("admitted_rows", C.c_int32),
                ("blocks_reused", C.c_int64), ("queued", C.c_int32)]


class Tensor(C.Structure):
    """ekv_tensor: a ggml-ordered strided device tensor (ne[0] fastest, nb in bytes)."""
    _fields_ = [("data", C.c_void_p), ("type", C.c_int32), ("ne", C.c_int64 * 4), ("nb", C.c_int64 * 4)]


# Every symbol include/ekv.h declares; tests check that the library exports all of them.
EXPORTED = [
    "ekv_pool_create", "ekv_pool_destroy", "ekv_pool_get_info", "ekv_pool_status", "ekv_pool_sync",
    "ekv_seq_create", "ekv_seq_free", "ekv_seq_resize", "ekv_seq_set_blocks", "ekv_seq_evict_front",
    "ekv_seq_append_tokens", "ekv_seq_clear_pred", "ekv_seq_restore", "ekv_seq_get_pred",
    "ekv_seq_get", "ekv_append", "ekv_append_suffix", "ekv_gather", "ekv_gather_suffix",
    "ekv_attention_workspace_size", "ekv_attention", "ekv_attention_algo", "ekv_version",
    "ekv_strerror", "ekv_attention_noalloc", "ekv_flash_attn_ext",
    "ekv_mul_mat_soft_max_mul_mat", "ekv_flash_attn_ext_workspace_size", "ekv_flash_attn_ext_ws",
    "ekv_mul_mat_soft_max_mul_mat_workspace_size", "ekv_mul_mat_soft_max_mul_mat_ws", "ekv_append_suffix_attention", "ekv_launch_count", "ekv_debug_expire_wait",
    "ekv_flow_step_f32", "ekv_guidance_f32", "ekv_sched_create", "ekv_sched_destroy", "ekv_sched_submit",
    "ekv_sched_begin_tick", "ekv_sched_end_tick", "ekv_sched_stats", "ekv_project_qkv_rope",
]
NOALLOC_SCRATCH_BYTES = 16 << 20  # EKV_NOALLOC_SCRATCH_BYTES


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python embodied.cpp_b200/build.py`"
                          " (there is no CPU fallback)")
    L = C.CDLL(LIB_PATH)
    vp, i32, pi32 = C.c_void_p, C.c_int32, C.POINTER(C.c_int32)
    sig = {
        "ekv_pool_create": ([C.POINTER(PoolConfig), C.POINTER(vp)], C.c_int),
        "ekv_pool_destroy": ([vp], C.c_int),
        "ekv_pool_get_info": ([vp, C.POINTER(PoolInfo)], C.c_int),
        "ekv_pool_status": ([vp, pi32, vp], C.c_int),
        "ekv_pool_sync": ([vp, vp], C.c_int),
        "ekv_seq_create": ([vp, pi32], C.c_int),
        "ekv_seq_free": ([vp, i32], C.c_int),
        "ekv_seq_resize": ([vp, i32, i32], C.c_int),
        "ekv_seq_set_blocks": ([vp, i32, pi32, i32, i32], C.c_int),
        "ekv_seq_evict_front": ([vp, i32, i32], C.c_int),
        "ekv_seq_append_tokens": ([vp, i32, i32, i32], C.c_int),
        "ekv_seq_clear_pred": ([vp, i32], C.c_int),
        "ekv_debug_expire_wait": ([i32], C.c_int),
        "ekv_flow_step_f32": ([vp, vp, C.c_int64, C.c_float, i32, vp], C.c_int),
        "ekv_guidance_f32": ([vp, vp, C.c_int64, C.c_float, i32, i32, vp], C.c_int),
        "ekv_seq_restore": ([vp, i32, i32], C.c_int),
        "ekv_sched_create": ([vp, i32, i32, C.POINTER(vp)], C.c_int),
        "ekv_sched_destroy": ([vp], C.c_int),
        "ekv_sched_submit": ([vp, C.c_uint64, i32, i32], C.c_int),
        "ekv_sched_begin_tick": ([vp, C.POINTER(SchedBatch), vp], C.c_int),
        "ekv_sched_end_tick": ([vp, C.POINTER(C.c_uint64), i32, pi32], C.c_int),
        "ekv_sched_stats": ([vp, C.POINTER(C.c_int64), C.POINTER(C.c_int64), pi32, pi32], C.c_int),
        "ekv_seq_get_pred": ([vp, i32, pi32, pi32], C.c_int),
        "ekv_seq_get": ([vp, i32, pi32, pi32, pi32, i32], C.c_int),
        "ekv_append": ([vp, i32, i32, vp, vp, vp, vp, i32, vp, vp, vp], C.c_int),
        "ekv_append_suffix": ([vp, i32, i32, vp, i32, vp, vp, vp], C.c_int),
        "ekv_gather": ([vp, i32, i32, i32, i32, i32, vp, vp, vp], C.c_int),
        "ekv_gather_suffix": ([vp, i32, i32, i32, i32, vp, vp, vp], C.c_int),
        "ekv_attention_workspace_size": ([vp, C.POINTER(AttnParams)], C.c_size_t),
        "ekv_attention": ([vp, C.POINTER(AttnParams), vp, vp, vp, C.c_size_t, vp], C.c_int),
        "ekv_attention_algo": ([vp, C.POINTER(AttnParams), vp, vp, vp, C.c_size_t, i32, vp], C.c_int),
        "ekv_attention_noalloc": ([vp, C.POINTER(AttnParams), vp, vp, vp], C.c_int),
        "ekv_append_suffix_attention": ([vp, C.POINTER(AttnParams), vp, vp, vp, vp, vp, C.c_size_t, vp], C.c_int),
        "ekv_flash_attn_ext": ([C.POINTER(Tensor)] * 4 + [C.c_float] * 3 + [C.POINTER(Tensor), vp], C.c_int),
        "ekv_mul_mat_soft_max_mul_mat": ([C.POINTER(Tensor)] * 4 + [C.c_float] * 2 + [C.POINTER(Tensor), vp],
                                         C.c_int),
        "ekv_flash_attn_ext_workspace_size": ([C.POINTER(Tensor)] * 4 + [C.c_float] * 2 + [C.POINTER(Tensor)],
                                              C.c_size_t),
        "ekv_flash_attn_ext_ws": ([C.POINTER(Tensor)] * 4 + [C.c_float] * 3 + [C.POINTER(Tensor), vp, C.c_size_t, vp],
                                  C.c_int),
        "ekv_mul_mat_soft_max_mul_mat_workspace_size": ([C.POINTER(Tensor)] * 4 + [C.c_float, C.POINTER(Tensor)],
                                                        C.c_size_t),
        "ekv_mul_mat_soft_max_mul_mat_ws": ([C.POINTER(Tensor)] * 4 + [C.c_float] * 2 + [C.POINTER(Tensor), vp,
                                                                                         C.c_size_t, vp], C.c_int),
        "ekv_project_qkv_rope": ([vp, i32, i32, vp, i32, i32, i32, vp, vp, vp, vp, vp, C.c_float, vp, vp, vp, vp],
                                 C.c_int),
        "ekv_version": ([], C.c_char_p),
        "ekv_launch_count": ([], C.c_uint64),
        "ekv_strerror": ([C.c_int], C.c_char_p),
    }
    for name, (args, res) in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = res
    return L


lib = _load()


class EkvError(RuntimeError):
    def __init__(self, code, what):
        super().__init__(f"{what}: {lib.ekv_strerror(code).decode()} ({code})")
        self.code = code


def check(code, what="ekv"):
    if code != OK:
        raise EkvError(code, what)
    return code


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream(stream):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


@dataclass
class SeqView:
    n_tokens: int
    blocks: list


class Pool:
    """A paged KV pool on one device (ekv_pool_create / ekv_pool_destroy)."""

    def __init__(self, *, device=0, dtype=DTYPE_BF16, block_tokens=16, n_blocks=1024, kv_heads=1,
                 head_dim=256, n_layers=1, max_seqs=64, max_blocks_per_seq=64, suffix_tokens=0):
        self.cfg = PoolConfig(device, dtype, block_tokens, n_blocks, kv_heads, head_dim, n_layers,
                              max_seqs, max_blocks_per_seq, suffix_tokens)
        h = C.c_void_p()
        check(lib.ekv_pool_create(C.byref(self.cfg), C.byref(h)), "ekv_pool_create")
        self.h = h

    def close(self):
        if self.h:
            check(lib.ekv_pool_destroy(self.h), "ekv_pool_destroy")
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def info(self) -> PoolInfo:
        i = PoolInfo()
        check(lib.ekv_pool_get_info(self.h, C.byref(i)), "ekv_pool_get_info")
        return i

    def status(self, stream=None) -> int:
        code = C.c_int32()
        check(lib.ekv_pool_status(self.h, C.byref(code), _stream(stream)), "ekv_pool_status")
        return code.value

    def sync(self, stream=None):
        check(lib.ekv_pool_sync(self.h, _stream(stream)), "ekv_pool_sync")

    # ---- sequences ----
    def seq_create(self) -> int:
        s = C.c_int32()
        check(lib.ekv_seq_create(self.h, C.byref(s)), "ekv_seq_create")
        return s.value

    def seq_free(self, seq):
        check(lib.ekv_seq_free(self.h, seq), "ekv_seq_free")

    def seq_resize(self, seq, n_tokens):
        check(lib.ekv_seq_resize(self.h, seq, n_tokens), "ekv_seq_resize")

    def seq_set_blocks(self, seq, blocks, n_tokens):
        arr = (C.c_int32 * len(blocks))(*blocks)
        check(lib.ekv_seq_set_blocks(self.h, seq, arr, len(blocks), n_tokens), "ekv_seq_set_blocks")

    def seq_evict_front(self, seq, n_blocks):
        check(lib.ekv_seq_evict_front(self.h, seq, n_blocks), "ekv_seq_evict_front")

    def seq_append_tokens(self, seq, n_tokens, pred=False):
        check(lib.ekv_seq_append_tokens(self.h, seq, n_tokens, 1 if pred else 0), "ekv_seq_append_tokens")

    def seq_clear_pred(self, seq):
        check(lib.ekv_seq_clear_pred(self.h, seq), "ekv_seq_clear_pred")

    def seq_restore(self, seq, n_tokens):
        check(lib.ekv_seq_restore(self.h, seq, n_tokens), "ekv_seq_restore")

    def seq_get_pred(self, seq):
        lo, hi = C.c_int32(), C.c_int32()
        check(lib.ekv_seq_get_pred(self.h, seq, C.byref(lo), C.byref(hi)), "ekv_seq_get_pred")
        return lo.value, hi.value

    def seq_get(self, seq) -> SeqView:
        nt, nb = C.c_int32(), C.c_int32()
        check(lib.ekv_seq_get(self.h, seq, C.byref(nt), C.byref(nb), None, 0), "ekv_seq_get")
        arr = (C.c_int32 * max(1, nb.value))()
        check(lib.ekv_seq_get(self.h, seq, None, None, arr, nb.value), "ekv_seq_get")
        return SeqView(nt.value, list(arr)[: nb.value])

    # ---- data ----
    def append(self, layer, seq_ids, dst_pos, n_rows, src_row, max_rows, k, v, stream=None):
        check(lib.ekv_append(self.h, layer, seq_ids.numel(), _ptr(seq_ids), _ptr(dst_pos),
                             _ptr(n_rows), _ptr(src_row), max_rows, _ptr(k), _ptr(v),
                             _stream(stream)), "ekv_append")

    def append_suffix(self, layer, seq_ids, k, v, stream=None):
        n_rows = k.shape[1]
        check(lib.ekv_append_suffix(self.h, layer, seq_ids.numel(), _ptr(seq_ids), n_rows, _ptr(k),
                                    _ptr(v), _stream(stream)), "ekv_append_suffix")

    def gather(self, layer, seq, pos0, n_rows, fmt, k_out, v_out, stream=None):
        check(lib.ekv_gather(self.h, layer, seq, pos0, n_rows, fmt, _ptr(k_out), _ptr(v_out),
                             _stream(stream)), "ekv_gather")

    def gather_suffix(self, layer, seq, n_rows, fmt, k_out, v_out, stream=None):
        check(lib.ekv_gather_suffix(self.h, layer, seq, n_rows, fmt, _ptr(k_out), _ptr(v_out),
                                    _stream(stream)), "ekv_gather_suffix")

    def attention_params(self, *, layer, seq_ids, q_tokens, q_heads, scale, mask_flags=0,
                         chunk_tokens=0, chunk_stride=0, window_chunks=0, q_chunk0=0,
                         suffix_len=0, out_dtype=DTYPE_BF16, use_prefix=True, prefix_len=None,
                         prefix_valid=None, span_begin=None, span_end=None, flex_meta=None, flex_stride=0,
                         flex_q0=0, flex_k0=0, flex_window=0) -> AttnParams:
        p = AttnParams(layer, seq_ids.numel(), q_tokens, q_heads, scale, mask_flags, chunk_tokens,
                       chunk_stride, window_chunks, q_chunk0, suffix_len, out_dtype,
                       1 if use_prefix else 0, 0, seq_ids.data_ptr(),
                       None if prefix_len is None else prefix_len.data_ptr(),
                       None if prefix_valid is None else prefix_valid.data_ptr(),
                       None if span_begin is None else span_begin.data_ptr(),
                       None if span_end is None else span_end.data_ptr(),
                       None if flex_meta is None else flex_meta.data_ptr(), flex_stride, flex_q0, flex_k0,
                       flex_window)
        p._keep = (seq_ids, prefix_len, prefix_valid, span_begin, span_end, flex_meta)
        return p

    def workspace_size(self, params: AttnParams) -> int:
        return lib.ekv_attention_workspace_size(self.h, C.byref(params))

    def attention(self, params: AttnParams, q, out, workspace=None, algo=ALGO_TC, stream=None):
        ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
        check(lib.ekv_attention_algo(self.h, C.byref(params), _ptr(q), _ptr(out), _ptr(workspace),
                                     ws_bytes, algo, _stream(stream)), "ekv_attention")

    def append_suffix_attention(self, params: AttnParams, k_suffix, v_suffix, q, out, workspace=None, stream=None):
        """ekv_append_suffix_attention: this layer-step's suffix K/V ([n_batch][suffix_len][kv_heads]
        [head_dim] bf16) into the slots, then attention, in one call."""
        ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
        check(lib.ekv_append_suffix_attention(self.h, C.byref(params), _ptr(k_suffix), _ptr(v_suffix), _ptr(q),
                                              _ptr(out), _ptr(workspace), ws_bytes, _stream(stream)),
              "ekv_append_suffix_attention")


def project_qkv_rope(pool: "Pool", layer, seq_ids, x, wq, wk, wv, positions, rope_base, q_out, k_out=None, v_out=None,
                     *, tokens, q_heads, stream=None):
    """ekv_project_qkv_rope: x [n_batch * tokens, hidden] bf16, weights [out, hidden] bf16, positions int32
    [n_batch * tokens]; q_out [n_batch, tokens, q_heads, head_dim] bf16; K/V into the pool's suffix slots
    (k_out / v_out None) or into k_out / v_out [n_batch, tokens, kv_heads, head_dim] bf16."""
    rows, hidden = x.shape
    n_batch = rows // tokens
    check(lib.ekv_project_qkv_rope(pool.h, layer, n_batch, _ptr(seq_ids), tokens, q_heads, hidden, _ptr(x), _ptr(wq),
                                   _ptr(wk), _ptr(wv), _ptr(positions), rope_base, _ptr(q_out), _ptr(k_out),
                                   _ptr(v_out), _stream(stream)), "ekv_project_qkv_rope")


class DevArray:
    """A device (or, for a host-only pool, host) int32 array owned by the library: what
    Pool.attention_params and Pool.append read from a tensor (numel, data_ptr)."""

    def __init__(self, ptr, n):
        self.ptr, self.n = ptr or 0, n

    def numel(self):
        return self.n

    def data_ptr(self):
        return self.ptr


@dataclass
class Tick:
    """One tick of the scheduler (ekv_sched_batch): every active request runs its next denoise step."""
    n_batch: int
    request_ids: list
    seq_ids_host: list
    steps: list
    seq_ids: DevArray
    prefix_valid: DevArray
    admitted_index: list
    admitted_seq_ids: DevArray
    admitted_zeros: DevArray
    admitted_prefix_len: DevArray
    admitted_src_row: DevArray
    admitted_rows: int
    max_admitted_prefix: int
    blocks_reused: int
    queued: int


class Scheduler:
    """Batching scheduler over a pool (ekv_sched_*): first come first served admission, one denoise
    step of every active request per tick, blocks freed (and reused) on completion."""

    def __init__(self, pool: Pool, max_batch: int, n_steps: int):
        self.pool = pool
        self.h = C.c_void_p()
        check(lib.ekv_sched_create(pool.h, max_batch, n_steps, C.byref(self.h)), "ekv_sched_create")

    def close(self):
        if self.h:
            lib.ekv_sched_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def submit(self, request_id, prefix_len, prefix_valid=None):
        pv = prefix_len if prefix_valid is None else prefix_valid
        check(lib.ekv_sched_submit(self.h, request_id, prefix_len, pv), "ekv_sched_submit")

    def begin_tick(self, stream=None) -> Tick:
        b = SchedBatch()
        s = None if self.pool.cfg.device < 0 else _stream(stream)
        check(lib.ekv_sched_begin_tick(self.h, C.byref(b), s), "ekv_sched_begin_tick")
        n, na = b.n_batch, b.n_admitted
        return Tick(n, list(b.request_ids[:n]) if n else [], list(b.seq_ids_host[:n]) if n else [],
                    list(b.steps[:n]) if n else [], DevArray(b.seq_ids, n), DevArray(b.prefix_valid, n),
                    list(b.admitted_index[:na]) if na else [], DevArray(b.admitted_seq_ids, na),
                    DevArray(b.admitted_zeros, na), DevArray(b.admitted_prefix_len, na),
                    DevArray(b.admitted_src_row, na), b.admitted_rows, b.max_admitted_prefix,
                    b.blocks_reused, b.queued)

    def end_tick(self, cap=4096) -> list:
        arr = (C.c_uint64 * cap)()
        nf = C.c_int32()
        check(lib.ekv_sched_end_tick(self.h, arr, cap, C.byref(nf)), "ekv_sched_end_tick")
        return list(arr[: min(nf.value, cap)])

    def stats(self) -> dict:
        c, r, a, q = C.c_int64(), C.c_int64(), C.c_int32(), C.c_int32()
        check(lib.ekv_sched_stats(self.h, C.byref(c), C.byref(r), C.byref(a), C.byref(q)), "ekv_sched_stats")
        return dict(completed=c.value, blocks_reused=r.value, active=a.value, queued=q.value)


def flow_step(sample, velocity, delta, bf16_round=False, stream=None):
    """ekv_flow_step_f32 on contiguous f32 torch tensors of equal size (sample updated in place)."""
    check(lib.ekv_flow_step_f32(_ptr(sample), _ptr(velocity), sample.numel(), float(delta), 1 if bf16_round else 0,
                                _stream(stream)), "ekv_flow_step_f32")


def guidance(cond, uncond, scale, use_guidance=True, bf16_round=False, stream=None):
    """ekv_guidance_f32 on contiguous f32 torch tensors (cond updated in place)."""
    check(lib.ekv_guidance_f32(_ptr(cond), _ptr(uncond), cond.numel(), float(scale), 1 if use_guidance else 0,
                               1 if bf16_round else 0, _stream(stream)), "ekv_guidance_f32")


_TORCH_DTYPES = {"torch.float32": DTYPE_F32, "torch.float16": DTYPE_F16, "torch.bfloat16": DTYPE_BF16}


def ggml_view(t) -> Tensor:
    """Describe a torch tensor (up to 4-D, any strides) as ekv_tensor in ggml order: the torch shape
    reversed, so a [B, H, T, D] tensor is ne = {D, T, H, B} and nb = its strides in bytes."""
    if t.dim() > 4:
        raise ValueError("at most 4 dimensions")
    dt = _TORCH_DTYPES.get(str(t.dtype))
    if dt is None:
        raise ValueError(f"unsupported dtype {t.dtype}")
    shape = [1] * (4 - t.dim()) + list(t.shape)
    strides = [0] * (4 - t.dim()) + list(t.stride())
    es = t.element_size()
    g = Tensor()
    g.data = t.data_ptr()
    g.type = dt
    for i in range(4):
        g.ne[i] = shape[3 - i]
        g.nb[i] = strides[3 - i] * es
    return g


def flash_attn_ext(q, k, v, mask, dst, *, scale, max_bias=0.0, logit_softcap=0.0, workspace=None, stream=None):
    """ggml_flash_attn_ext on torch tensors given in reversed ggml order: q [B, Hq, Tq, D],
    k [Bk, Hkv, Tk, D], v [Bk, Hkv, Tk, Dv], mask [Mb, Mh, >=Tq, >=Tk] (or None) and the f32
    result dst [B, Tq, Hq, Dv]; any of them may be a permuted or sliced view. With `workspace` (a
    uint8 device tensor of flash_attn_ext_workspace_size bytes) the call stages into it
    (ekv_flash_attn_ext_ws), else into the library's per-device workspace."""
    gm = None if mask is None else C.byref(ggml_view(mask))
    args = (C.byref(ggml_view(q)), C.byref(ggml_view(k)), C.byref(ggml_view(v)), gm, scale, max_bias, logit_softcap,
            C.byref(ggml_view(dst)))
    if workspace is None:
        check(lib.ekv_flash_attn_ext(*args, _stream(stream)), "ekv_flash_attn_ext")
    else:
        check(lib.ekv_flash_attn_ext_ws(*args, _ptr(workspace), workspace.numel() * workspace.element_size(),
                                        _stream(stream)), "ekv_flash_attn_ext_ws")


def flash_attn_ext_workspace_size(q, k, v, mask, dst, *, max_bias=0.0, logit_softcap=0.0) -> int:
    """Bytes of the tensor-core staging of this flash_attn_ext call (0: it runs on the CUDA cores)."""
    gm = None if mask is None else C.byref(ggml_view(mask))
    return lib.ekv_flash_attn_ext_workspace_size(C.byref(ggml_view(q)), C.byref(ggml_view(k)), C.byref(ggml_view(v)),
                                                 gm, max_bias, logit_softcap, C.byref(ggml_view(dst)))


def mul_mat_soft_max_mul_mat(k, q, v, mask, dst, *, scale, max_bias=0.0, workspace=None, stream=None):
    """The ggml triple mul_mat(K, Q) -> soft_max_ext -> mul_mat(V, .) on torch tensors in reversed ggml
    order: k [Bk, Hkv, Tk, D], q [B, Hq, Tq, D], v [Bk, Hkv, Dv, Tk] (keys fastest), mask
    [Mb, Mh, >=Tq, >=Tk] or None, f32 dst [B, Hq, Tq, Dv]. `workspace` as for flash_attn_ext."""
    gm = None if mask is None else C.byref(ggml_view(mask))
    args = (C.byref(ggml_view(k)), C.byref(ggml_view(q)), C.byref(ggml_view(v)), gm, scale, max_bias,
            C.byref(ggml_view(dst)))
    if workspace is None:
        check(lib.ekv_mul_mat_soft_max_mul_mat(*args, _stream(stream)), "ekv_mul_mat_soft_max_mul_mat")
    else:
        check(lib.ekv_mul_mat_soft_max_mul_mat_ws(*args, _ptr(workspace), workspace.numel() * workspace.element_size(),
                                                  _stream(stream)), "ekv_mul_mat_soft_max_mul_mat_ws")


def mul_mat_soft_max_mul_mat_workspace_size(k, q, v, mask, dst, *, max_bias=0.0) -> int:
    gm = None if mask is None else C.byref(ggml_view(mask))
    return lib.ekv_mul_mat_soft_max_mul_mat_workspace_size(C.byref(ggml_view(k)), C.byref(ggml_view(q)),
                                                           C.byref(ggml_view(v)), gm, max_bias,
                                                           C.byref(ggml_view(dst)))


def version() -> str:
    return lib.ekv_version().decode()
