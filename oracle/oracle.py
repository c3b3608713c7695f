"""ctypes binding of the CPU oracle (libekv_oracle.so). TEST INFRASTRUCTURE ONLY.

The oracle restates the reference's arithmetic for the denoise-loop attention path on the CPU
(see ekv_oracle.h for the reference lines). It is the parity checker for tests/, for
__graft_entry__.smoke(), and the CPU baseline timed by bench.py. The product library
(embodied.cpp_b200/ekv.py over libekv.so) never imports this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libekv_oracle.so")

MASK_SUFFIX_CAUSAL = 1 << 0
MASK_SUFFIX_PREFIX_LM = 1 << 1
MASK_SPAN_ONLY = 1 << 2
MASK_SPAN_EXCLUDE = 1 << 3
MASK_BLOCK_CAUSAL = 1 << 4
MASK_FLEX_SELF = 1 << 5
MASK_FLEX_CROSS = 1 << 6


class Seq(C.Structure):
    _fields_ = [("n_prefix", C.c_int32), ("prefix_valid", C.c_int32),
                ("span_begin", C.c_int32), ("span_end", C.c_int32), ("n_suffix", C.c_int32),
                ("flex_meta", C.c_void_p)]


class Mask(C.Structure):
    _fields_ = [("flags", C.c_int32), ("chunk_tokens", C.c_int32), ("chunk_stride", C.c_int32),
                ("window_chunks", C.c_int32), ("q_chunk0", C.c_int32), ("flex_q0", C.c_int32),
                ("flex_k0", C.c_int32), ("flex_window", C.c_int32)]


class AttnArgs(C.Structure):
    _fields_ = [("B", C.c_int32), ("Tq", C.c_int32), ("Hq", C.c_int32), ("Hkv", C.c_int32),
                ("D", C.c_int32), ("Lk_max", C.c_int32), ("scale", C.c_float),
                ("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p),
                ("dense_mask", C.c_void_p), ("seqs", C.c_void_p), ("mask", Mask),
                ("out", C.c_void_p)]


class CacheArgs(C.Structure):
    _fields_ = [("B", C.c_int32), ("Tq", C.c_int32), ("Hq", C.c_int32), ("Hkv", C.c_int32),
                ("D", C.c_int32), ("n_layers", C.c_int32), ("kv_is_q8", C.c_int32),
                ("max_prefix", C.c_int32), ("n_suffix", C.c_int32), ("scale", C.c_float),
                ("n_prefix", C.c_void_p), ("prefix_valid", C.c_void_p),
                ("prefix_k", C.c_void_p), ("prefix_v", C.c_void_p),
                ("suffix_k", C.c_void_p), ("suffix_v", C.c_void_p),
                ("q", C.c_void_p), ("n_calls", C.c_int32), ("out", C.c_void_p)]


_lib = None


def build():
    """Compile libekv_oracle.so with the committed Makefile (gcc, no fast-math)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH) or (
                os.path.getmtime(LIB_PATH) < os.path.getmtime(os.path.join(HERE, "ekv_oracle.c"))):
            build()
        L = C.CDLL(LIB_PATH)
        L.ekvo_f32_to_bf16.restype = C.c_uint16
        L.ekvo_f32_to_bf16.argtypes = [C.c_float]
        L.ekvo_f32_to_f16.restype = C.c_uint16
        L.ekvo_f32_to_f16.argtypes = [C.c_float]
        L.ekvo_f16_to_f32.restype = C.c_float
        L.ekvo_f16_to_f32.argtypes = [C.c_uint16]
        L.ekvo_f32_to_bf16_n.argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
        L.ekvo_bf16_to_f32_n.argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
        L.ekvo_quantize_q8_0.argtypes = [C.c_void_p, C.c_int64, C.c_void_p]
        L.ekvo_dequantize_q8_0.argtypes = [C.c_void_p, C.c_int64, C.c_void_p]
        L.ekvo_attention_rows.argtypes = [C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_int]
        L.ekvo_allowed.restype = C.c_int
        L.ekvo_allowed.argtypes = [C.POINTER(Mask), C.POINTER(Seq), C.c_int32, C.c_int32]
        L.ekvo_attention_f32.restype = C.c_int
        L.ekvo_attention_f32.argtypes = [C.POINTER(AttnArgs), C.c_int]
        L.ekvo_attention_f64.restype = C.c_int
        L.ekvo_attention_f64.argtypes = [C.POINTER(AttnArgs), C.c_void_p]
        L.ekvo_cache_attention_run.restype = C.c_int
        L.ekvo_cache_attention_run.argtypes = [C.POINTER(CacheArgs), C.c_int]
        _lib = L
    return _lib


def _ptr(a):
    return a.ctypes.data_as(C.c_void_p)


# ---- number formats -------------------------------------------------------------------------

def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().ekvo_f32_to_bf16_n(_ptr(x), _ptr(out), x.size)
    return out


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, dtype=np.float32)
    lib().ekvo_bf16_to_f32_n(_ptr(h), _ptr(out), h.size)
    return out


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    L = lib()
    return np.array([L.ekvo_f32_to_f16(float(v)) for v in x], dtype=np.uint16)


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """x: f32 with last dim a multiple of 32 -> uint8 [..., last/32*34] ggml block_q8_0 bytes."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    assert x.shape[-1] % 32 == 0
    out = np.empty(x.shape[:-1] + (x.shape[-1] // 32 * 34,), dtype=np.uint8)
    lib().ekvo_quantize_q8_0(_ptr(x), x.size, _ptr(out))
    return out


def dequantize_q8_0(blocks: np.ndarray) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    assert blocks.shape[-1] % 34 == 0
    n = blocks.shape[-1] // 34 * 32
    out = np.empty(blocks.shape[:-1] + (n,), dtype=np.float32)
    lib().ekvo_dequantize_q8_0(_ptr(blocks), out.size, _ptr(out))
    return out


# ---- masks and attention --------------------------------------------------------------------

def make_mask(flags=0, chunk_tokens=0, chunk_stride=0, window_chunks=0, q_chunk0=0, flex_q0=0, flex_k0=0,
              flex_window=0) -> Mask:
    return Mask(flags, chunk_tokens, chunk_stride, window_chunks, q_chunk0, flex_q0, flex_k0, flex_window)


def flex_meta_word(seq: int, frame: int, noise: int) -> int:
    """Pack a token's (seq_id, frame_id, noise_id) of the reference's LingBotFlexMaskMeta
    (models/lingbot_va.cpp:9273-9280; seq -1 = padding, noise 1 = clean) as an int32 metadata word."""
    if seq < 0:
        return 0
    w = ((seq + 1) << 24) | ((noise & 1) << 23) | (frame & 0x7FFFFF)
    return w - (1 << 32) if w >= (1 << 31) else w


def make_seqs(n_prefix, prefix_valid=None, span=None, n_suffix=0, flex_meta=None):
    """n_prefix etc. are per-request sequences (or scalars broadcast over B); flex_meta is a list of
    per-request int32 metadata arrays (kept alive by the returned array)."""
    n_prefix = np.atleast_1d(np.asarray(n_prefix, dtype=np.int32))
    B = n_prefix.size
    pv = n_prefix if prefix_valid is None else np.broadcast_to(np.asarray(prefix_valid, np.int32), (B,))
    if span is None:
        sb = np.zeros(B, np.int32)
        se = np.zeros(B, np.int32)
    else:
        sb = np.broadcast_to(np.asarray(span[0], np.int32), (B,))
        se = np.broadcast_to(np.asarray(span[1], np.int32), (B,))
    ns = np.broadcast_to(np.asarray(n_suffix, np.int32), (B,))
    arr = (Seq * B)()
    keep = []
    for i in range(B):
        fm = None
        if flex_meta is not None:
            m = np.ascontiguousarray(flex_meta[i], np.int32)
            keep.append(m)
            fm = m.ctypes.data
        arr[i] = Seq(int(n_prefix[i]), int(pv[i]), int(sb[i]), int(se[i]), int(ns[i]), fm)
    arr._keep = keep
    return arr


def allowed_matrix(mask: Mask, seq: Seq, Tq: int, Lk: int) -> np.ndarray:
    L = lib()
    out = np.zeros((Tq, Lk), dtype=bool)
    for q in range(Tq):
        for k in range(Lk):
            out[q, k] = bool(L.ekvo_allowed(C.byref(mask), C.byref(seq), q, k))
    return out


def attention(q, k, v, seqs, mask: Mask, scale: float, dense_mask=None, precision="f32",
              n_threads=0):
    """q [B,Tq,Hq,D], k/v [B,Lk,Hkv,D] as f32 (prefix keys then suffix keys)."""
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    B, Tq, Hq, D = q.shape
    Lk, Hkv = k.shape[1], k.shape[2]
    dm = None if dense_mask is None else np.ascontiguousarray(dense_mask, np.float32)
    out = np.zeros(q.shape, np.float32)
    args = AttnArgs(B, Tq, Hq, Hkv, D, Lk, scale, _ptr(q).value, _ptr(k).value, _ptr(v).value,
                    None if dm is None else _ptr(dm).value, C.addressof(seqs), mask,
                    _ptr(out).value)
    if precision == "f64":
        out64 = np.zeros(q.shape, np.float64)
        rc = lib().ekvo_attention_f64(C.byref(args), _ptr(out64))
        assert rc == 0
        return out64
    rc = lib().ekvo_attention_f32(C.byref(args), n_threads or os.cpu_count() or 1)
    assert rc == 0
    return out


def attention_rows(q, k, v, seqs, mask: Mask, scale: float, rows, n_threads=0):
    """The f32 oracle for a sample of query rows: rows is an int array [n][3] of (b, t, h); returns
    [n][D]. q [B,Tq,Hq,D], k/v [B,Lk,Hkv,D] f32 (prefix keys then suffix keys)."""
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    rows = np.ascontiguousarray(rows, np.int32)
    B, Tq, Hq, D = q.shape
    Lk, Hkv = k.shape[1], k.shape[2]
    out = np.zeros((rows.shape[0], D), np.float32)
    args = AttnArgs(B, Tq, Hq, Hkv, D, Lk, scale, _ptr(q).value, _ptr(k).value, _ptr(v).value, None,
                    C.addressof(seqs), mask, _ptr(out).value)
    rc = lib().ekvo_attention_rows(C.byref(args), rows.shape[0], _ptr(rows), _ptr(out), n_threads or os.cpu_count() or 1)
    assert rc == 0
    return out


def cache_attention_run(args: CacheArgs, n_threads: int) -> int:
    return lib().ekvo_cache_attention_run(C.byref(args), n_threads)


def alibi_slopes(n_head: int, max_bias: float) -> np.ndarray:
    """ALiBi slope of each head as ggml computes it for soft_max_ext / flash_attn_ext (llama.cpp
    b9016, ggml-cpu ops.cpp): n_head_log2 = 2^floor(log2(n_head)), m0 = 2^(-max_bias/n_head_log2),
    m1 = 2^(-max_bias/2/n_head_log2); head h < n_head_log2 gets m0^(h+1), the rest
    m1^(2(h-n_head_log2)+1); every slope is 1 when max_bias == 0."""
    if max_bias <= 0.0:
        return np.ones(n_head, np.float64)
    n_log2 = 1 << int(np.floor(np.log2(n_head)))
    m0 = 2.0 ** (-max_bias / n_log2)
    m1 = 2.0 ** (-(max_bias / 2.0) / n_log2)
    h = np.arange(n_head)
    return np.where(h < n_log2, m0 ** (h + 1), m1 ** (2 * (h - n_log2) + 1))


def flash_attn_ext(q, k, v, mask=None, *, scale, max_bias=0.0, logit_softcap=0.0):
    """GGML_OP_FLASH_ATTN_EXT restated in float64 (ggml_flash_attn_ext and its CPU kernel,
    llama.cpp b9016 `ggml/src/ggml.c` and `ggml-cpu/ops.cpp`, an absent dependency pinned by the
    reference's patches/init_third_party.sh:21-22; call sites models/hy_vla.cpp:376-378, :439-441,
    :492, :859 and models/lingbot_va.cpp:1263-1266).

    Arrays are in reversed ggml order: q [B, Hq, Tq, D], k [Bk, Hkv, Tk, D], v [Bk, Hkv, Tk, Dv],
    mask [Mb, Mh, >=Tq, >=Tk] or None. Head h reads KV head h // (Hq // Hkv), batch b reads
    b // (B // Bk); the mask broadcasts as mask[b % Mb, h % Mh]. Each score is
    scale * q.k (with softcap: softcap * tanh(scale / softcap * q.k)) plus slope(h) * mask; keys whose
    mask is -inf are skipped; a row with no key left gives 0. Returns dst [B, Tq, Hq, Dv]."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    B, Hq, Tq, _ = q.shape
    Bk, Hkv, Tk, _ = k.shape
    Dv = v.shape[3]
    slopes = alibi_slopes(Hq, max_bias)
    sc = scale / logit_softcap if logit_softcap != 0.0 else scale
    out = np.zeros((B, Tq, Hq, Dv), np.float64)
    for b in range(B):
        kb = b // (B // Bk)
        for h in range(Hq):
            kh = h // (Hq // Hkv)
            s = (q[b, h] @ k[kb, kh].T) * sc
            if logit_softcap != 0.0:
                s = logit_softcap * np.tanh(s)
            if mask is not None:
                mv = np.asarray(mask[b % mask.shape[0], h % mask.shape[1], :Tq, :Tk], np.float64)
                s = np.where(np.isneginf(mv), -np.inf, s + slopes[h] * mv)
            m = s.max(axis=1, keepdims=True)
            live = np.isfinite(m)
            p = np.where(live, np.exp(s - np.where(live, m, 0.0)), 0.0)
            den = p.sum(axis=1, keepdims=True)
            o = p @ v[kb, kh]
            out[b, :, h] = np.where(den > 0, o / np.where(den > 0, den, 1.0), 0.0)
    return out


def attention_ggml_q8_0(q, k, v, n_prefix, scale):
    """The pi0.5 attention as ggml's CPU backend would compute it over a Q8_0 key/value cache
    (models/pi05.cpp:406-418 with the cached tensors stored as GGML_TYPE_Q8_0), float64.

    ggml's Q8_0 mul_mat converts src1 to the type's dot-product partner, Q8_0 itself (llama.cpp
    b9016, ggml-cpu: the vec_dot_type of Q8_0), so S = dot(q8(Q), q8(K)): every 32-value block of each
    query row is quantised with the same gguf rule as the keys. The 50 suffix keys joined by the
    concat of :406 are quantised with the prefix (the concat writes into the Q8_0 tensor). V is read
    dequantised (a permuted Q8_0 tensor is made contiguous as float). Softmax in float.
    q [B, Tq, Hq, D], k/v [B, Lk, Hkv, D] f32 (pre-quantisation values: prefix, then suffix);
    n_prefix is unused by the arithmetic (all keys are cached the same way) and kept for symmetry
    with `attention`. Returns [B, Tq, Hq, D]. Used to bound the difference between a Q8_0 ggml path
    and this library's f16 MMAs over exactly dequantised keys (both within the 5e-2 tolerance)."""
    q = np.asarray(q, np.float32)
    B, Tq, Hq, D = q.shape
    Lk, Hkv = k.shape[1], k.shape[2]
    rt = lambda x: dequantize_q8_0(quantize_q8_0(np.ascontiguousarray(x, np.float32).reshape(-1, D))).reshape(x.shape)
    qh, kh, vh = rt(q).astype(np.float64), rt(k).astype(np.float64), rt(v).astype(np.float64)
    g = Hq // Hkv
    out = np.zeros((B, Tq, Hq, D), np.float64)
    for b in range(B):
        for h in range(Hq):
            s = (qh[b, :, h] @ kh[b, :, h // g].T) * scale
            p = np.exp(s - s.max(axis=1, keepdims=True))
            out[b, :, h] = (p / p.sum(axis=1, keepdims=True)) @ vh[b, :, h // g]
    del n_prefix
    return out


def flow_step(sample, velocity, delta, bf16_round=False):
    """The sampler's Euler step as the reference computes it in f32: sample + (velocity * delta),
    the product and the sum each rounded to f32 (lingbot_scheduler_step_f32's __fmul_rn / __fadd_rn,
    kernels/lingbot/lingbot_flex_attn_cuda.cu:40-52; x_t + scale(velocity, dt), models/pi05.cpp:856),
    then bf16 round-to-nearest-even when bf16_round (lingbot_bf16_round_device, :36-38)."""
    s = np.asarray(sample, np.float32)
    r = (s + (np.asarray(velocity, np.float32) * np.float32(delta)).astype(np.float32)).astype(np.float32)
    return bf16_to_f32(f32_to_bf16(r)) if bf16_round else r


def guidance(cond, uncond, scale, use_guidance=True, bf16_round=False):
    """Classifier-free guidance of lingbot_model_output_guidance_f32 (kernels/lingbot/
    lingbot_flex_attn_cuda.cu:54-73): c (bf16-rounded when asked), then u + scale * (c - u) with each
    operation rounded to f32 and the result bf16-rounded when asked."""
    rnd = (lambda x: bf16_to_f32(f32_to_bf16(np.asarray(x, np.float32)))) if bf16_round else (lambda x: x)
    c = rnd(np.asarray(cond, np.float32))
    if not use_guidance:
        return c
    u = rnd(np.asarray(uncond, np.float32))
    d = (c - u).astype(np.float32)
    v = (u + (np.float32(scale) * d).astype(np.float32)).astype(np.float32)
    return rnd(v)


def rope_neox(x: np.ndarray, pos: np.ndarray, base: float) -> np.ndarray:
    """RoPE in ggml's NEOX mode as models/pi05.cpp:391-401 applies it (ggml_rope_ext(t, positions, n_dims =
    head_dim, GGML_ROPE_TYPE_NEOX, n_ctx_orig 0, freq_base rope_base, freq_scale 1, ext_factor 0,
    attn_factor 1)): ggml (llama.cpp b9016, an absent dependency) keeps theta in float32, starting at the
    token's position and multiplied by theta_scale = base^(-2/n_dims) after every dimension pair; pair i
    rotates dims i and i + n_dims/2 by theta: (x0 cos - x1 sin, x0 sin + x1 cos). x: [rows, ..., D] float32,
    pos: [rows] int. Returns float32."""
    x = np.asarray(x, np.float32)
    d = x.shape[-1]
    h = d // 2
    theta_scale = np.float32(np.power(np.float32(base), np.float32(-2.0 / d), dtype=np.float32))
    theta = np.asarray(pos, np.float32).reshape((-1,) + (1,) * (x.ndim - 2))
    out = np.empty_like(x)
    for i in range(h):
        c = np.cos(theta).astype(np.float32)
        s = np.sin(theta).astype(np.float32)
        x0, x1 = x[..., i], x[..., i + h]
        out[..., i] = x0 * c - x1 * s
        out[..., i + h] = x0 * s + x1 * c
        theta = (theta * theta_scale).astype(np.float32)
    return out


def project_qkv_rope(x, wq, wk, wv, pos, base, q_heads, kv_heads):
    """The action expert's q/k/v projection of one layer-step with RoPE (models/pi05.cpp:391-401):
    q = mul_mat(Wq, x), k = mul_mat(Wk, x), v = mul_mat(Wv, x) over bf16 weights [out][hidden] and bf16
    activations (ggml's bf16 mul_mat rounds the f32 activations to bf16), f32 dot products; RoPE NEOX on q
    and k at the tokens' positions; returned as float32 values of the bf16 results (q [rows, Hq, D],
    k and v [rows, Hkv, D])."""
    xf = np.asarray(x, np.float32)
    d = np.asarray(wq).shape[0] // q_heads
    rows = xf.shape[0]
    q = (xf @ np.asarray(wq, np.float32).T).reshape(rows, q_heads, d)
    k = (xf @ np.asarray(wk, np.float32).T).reshape(rows, kv_heads, d)
    v = (xf @ np.asarray(wv, np.float32).T).reshape(rows, kv_heads, d)
    q = rope_neox(q, pos, base)
    k = rope_neox(k, pos, base)
    r = lambda a: bf16_to_f32(f32_to_bf16(np.ascontiguousarray(a, np.float32)))
    return r(q), r(k), r(v)
