"""The multi-head small-query kernel (EKV_ALGO_TC_HEADS, ekv_attn_heads.cu) against the CPU oracle,
through the C-ABI: GR00T's DiT action-head attention (models/groot_n1.cpp:328-364) -- 17 queries per
head, one KV head per query head, head_dim 48 -- over a cached backbone with the image / text span
masks (:708-718), padding, the suffix-only self layer, a prefix followed by suffix keys, head_dim 64,
16-, 32- and 64-token blocks, more units than SMs (persistent CTAs walking several units), units
with nothing visible, tables longer than the kernel's per-unit block cache, and the shapes it must
refuse. The default algorithm picks this kernel for such calls (checked bit for bit).
"""
import numpy as np
import pytest
import torch

import ekv
from cases import Filled, bf16_randn
from test_gpu_parity import check, oracle_attention, run_attention

pytestmark = pytest.mark.gpu
TOL = 2e-2


@pytest.mark.parametrize("bt", [16, 64])
@pytest.mark.parametrize("flag", [0, ekv.MASK_SPAN_ONLY, ekv.MASK_SPAN_EXCLUDE])
def test_groot_cross_layer(bt, flag):
    """Cross-attention of 17 queries x 32 heads x 48 over a 300-token backbone: the image span [0, 256)
    (SPAN_ONLY), the text keys after it (SPAN_EXCLUDE), or every key, with padding on some requests."""
    B, T, H, D, P = 10, 17, 32, 48, 300
    gen = torch.Generator().manual_seed(bt + flag)
    f = Filled(dtype=ekv.DTYPE_BF16, B=B, prefix_lens=[P] * B, Hkv=H, D=D, block_tokens=bt, seed=bt + flag)
    q = bf16_randn(gen, (B, T, H, D))
    valid = [P - 7 * (b % 3) for b in range(B)]
    span = ([0] * B, [256] * B)
    kw = dict(mask_flags=flag, prefix_valid=valid)
    if flag:
        kw["span"] = span
    got = run_attention(f, 0, q, Hq=H, scale=D ** -0.5, algo=ekv.ALGO_TC_HEADS, **kw)
    want = oracle_attention(f, 0, q, scale=D ** -0.5, **kw)
    check(got, want, TOL)


@pytest.mark.parametrize("out_dtype", [ekv.DTYPE_F32, ekv.DTYPE_BF16])
def test_groot_self_layer(out_dtype):
    """The self layer: the 17 tokens attend only each other (use_prefix = 0), keys from the suffix slot
    (24 rows per head, so the MMAs read 8 zero rows past the last head of a unit)."""
    B, T, H, D = 12, 17, 32, 48
    gen = torch.Generator().manual_seed(31)
    f = Filled(dtype=ekv.DTYPE_BF16, B=B, prefix_lens=[20] * B, Hkv=H, D=D, suffix_len=T, seed=31)
    q = bf16_randn(gen, (B, T, H, D))
    got = run_attention(f, 0, q, Hq=H, scale=D ** -0.5, algo=ekv.ALGO_TC_HEADS, use_prefix=False,
                        out_dtype=out_dtype)
    want = oracle_attention(f, 0, q, scale=D ** -0.5, use_prefix=False)
    check(got, want, TOL)


@pytest.mark.parametrize("D,bt,T", [(64, 32, 32), (64, 16, 1), (48, 32, 9)])
@pytest.mark.parametrize("flag", [0, ekv.MASK_SUFFIX_CAUSAL, ekv.MASK_SUFFIX_PREFIX_LM])
def test_prefix_then_suffix(D, bt, T, flag):
    """Ragged prefixes followed by suffix keys, the suffix masks, 8 KV heads (two units per request),
    1 to 32 query tokens, head_dim 48 and 64."""
    B, H = 5, 8
    rng = np.random.default_rng(D + bt + T)
    gen = torch.Generator().manual_seed(D + bt + T)
    plens = [int(x) for x in rng.integers(1, 260, size=B)]
    f = Filled(dtype=ekv.DTYPE_BF16, B=B, prefix_lens=plens, Hkv=H, D=D, block_tokens=bt, suffix_len=T,
               seed=D + bt)
    q = bf16_randn(gen, (B, T, H, D))
    valid = [max(0, p - int(rng.integers(0, 30))) for p in plens]
    got = run_attention(f, 0, q, Hq=H, scale=D ** -0.5, algo=ekv.ALGO_TC_HEADS, mask_flags=flag, prefix_valid=valid)
    want = oracle_attention(f, 0, q, scale=D ** -0.5, mask_flags=flag, prefix_valid=valid)
    check(got, want, TOL)


def test_many_units_ragged_and_empty():
    """More units than SMs (each persistent CTA walks several units), ragged prefixes up to 1,100 keys
    (more blocks than a unit plan caches, so later blocks are looked up directly), requests with
    nothing visible (zero rows), and the default algorithm choosing this kernel (bit for bit)."""
    B, T, H, D = 60, 17, 16, 48
    rng = np.random.default_rng(7)
    gen = torch.Generator().manual_seed(7)
    plens = [int(x) for x in rng.integers(1, 1100, size=B)]
    plens[3] = 1100
    f = Filled(dtype=ekv.DTYPE_BF16, B=B, prefix_lens=plens, Hkv=H, D=D, block_tokens=16, seed=7)
    q = bf16_randn(gen, (B, T, H, D))
    valid = list(plens)
    valid[5] = 0
    valid[11] = 0
    got = run_attention(f, 0, q, Hq=H, scale=D ** -0.5, algo=ekv.ALGO_TC_HEADS, prefix_valid=valid)
    want = oracle_attention(f, 0, q, scale=D ** -0.5, prefix_valid=valid)
    check(got, want, TOL)
    assert np.all(got[5] == 0) and np.all(got[11] == 0)
    auto = run_attention(f, 0, q, Hq=H, scale=D ** -0.5, algo=ekv.ALGO_TC, prefix_valid=valid)
    assert np.array_equal(auto, got)


def test_block_causal_and_packed_path_agree():
    """A chunked block-causal prefix (LingBot's window form) under the heads kernel, and the one-CTA
    packed-unit kernel (EKV_ALGO_TC_CTA) on the same GR00T-shaped call."""
    B, T, H, D = 6, 17, 32, 48
    gen = torch.Generator().manual_seed(9)
    f = Filled(dtype=ekv.DTYPE_BF16, B=B, prefix_lens=[400] * B, Hkv=H, D=D, block_tokens=64, seed=9)
    q = bf16_randn(gen, (B, T, H, D))
    block = (100, 128, 2, 3)  # chunk tokens, stride, window chunks, query chunk
    got = run_attention(f, 0, q, Hq=H, scale=D ** -0.5, algo=ekv.ALGO_TC_HEADS, mask_flags=ekv.MASK_BLOCK_CAUSAL,
                        block=block)
    want = oracle_attention(f, 0, q, scale=D ** -0.5, mask_flags=ekv.MASK_BLOCK_CAUSAL, block=block)
    check(got, want, TOL)
    cta = run_attention(f, 0, q, Hq=H, scale=D ** -0.5, algo=ekv.ALGO_TC_CTA, mask_flags=ekv.MASK_BLOCK_CAUSAL,
                        block=block)
    check(cta, want, TOL)


def test_bad_sequence_gives_zeros_and_status():
    B, T, H, D = 4, 17, 8, 48
    gen = torch.Generator().manual_seed(13)
    f = Filled(dtype=ekv.DTYPE_BF16, B=B, prefix_lens=[100] * B, Hkv=H, D=D, seed=13)
    q = bf16_randn(gen, (B, T, H, D)).cuda()
    ids = f.seq_ids.clone()
    ids[2] = 10_000
    prm = f.pool.attention_params(layer=0, seq_ids=ids, q_tokens=T, q_heads=H, scale=D ** -0.5,
                                  out_dtype=ekv.DTYPE_F32)
    out = torch.full((B, T, H, D), float("nan"), dtype=torch.float32, device="cuda")
    f.pool.attention(prm, q, out, algo=ekv.ALGO_TC_HEADS)
    torch.cuda.synchronize()
    assert f.pool.status() == ekv.DEV_ERR_BAD_SEQ
    o = out.cpu().numpy()
    assert np.all(o[2] == 0) and np.isfinite(o).all()


@pytest.mark.parametrize("case", ["gqa", "d128", "tokens33", "q8"])
def test_refuses_other_shapes(case):
    """Shapes outside the kernel: nothing is enqueued and EKV_ERR_UNSUPPORTED is returned."""
    D = {"d128": 128}.get(case, 48)
    dtype = ekv.DTYPE_Q8_0 if case == "q8" else ekv.DTYPE_BF16
    if case == "q8":
        D = 64
    Hkv, Hq = (4, 8) if case == "gqa" else (4, 4)
    T = 33 if case == "tokens33" else 17
    f = Filled(dtype=dtype, B=2, prefix_lens=[40, 50], Hkv=Hkv, D=D, seed=17)
    q = torch.zeros((2, T, Hq, D), dtype=torch.bfloat16, device="cuda")
    out = torch.zeros((2, T, Hq, D), dtype=torch.float32, device="cuda")
    prm = f.pool.attention_params(layer=0, seq_ids=f.seq_ids, q_tokens=T, q_heads=Hq, scale=0.1,
                                  out_dtype=ekv.DTYPE_F32)
    rc = ekv.lib.ekv_attention_algo(f.pool.h, ekv.C.byref(prm), q.data_ptr(), out.data_ptr(), None, 0,
                                    ekv.ALGO_TC_HEADS, None)
    assert rc == ekv.ERR_UNSUPPORTED
