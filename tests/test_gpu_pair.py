"""head_dim 256 on CTA pairs (tcgen05 cta_group::2, EKV_ALGO_TC_PAIR) against the CPU oracle and
against the default one-CTA tensor-core kernel, through the C-ABI.

The pair kernel splits every K/V tile between the two CTAs of a cluster (K rows by key, V columns by
head_dim) and runs 256 query rows per pair, so the cases cover: query-row counts that leave the
second CTA of the last pair partly or entirely empty; one and two KV heads; 16- and 64-token blocks;
bf16 and Q8_0 pools; every mask family; key splits through a workspace; prefixes that end inside a
tile and inside a block."""
import numpy as np
import pytest
import torch

import ekv
from cases import Filled, bf16_randn
from test_gpu_parity import TOL, check, oracle_attention, run_attention

pytestmark = pytest.mark.gpu

D = 256


def both(f, q, *, Hq, scale, **kw):
    """The CTA-pair kernel (128-key tiles where the shape allows, as the default runs it) and the
    one-CTA kernel; the 64-key pair kernel is checked against the one-CTA kernel on the way."""
    got = run_attention(f, 0, q, Hq=Hq, scale=scale, algo=ekv.ALGO_TC_PAIR, **kw)
    single = run_attention(f, 0, q, Hq=Hq, scale=scale, algo=ekv.ALGO_TC_CTA, **kw)
    pair64 = run_attention(f, 0, q, Hq=Hq, scale=scale, algo=ekv.ALGO_TC_PAIR64, **kw)
    tol = TOL[f.dtype]
    assert np.abs(pair64 - single).max() <= tol
    return got, single


@pytest.mark.parametrize("dtype", [ekv.DTYPE_BF16, ekv.DTYPE_Q8_0])
@pytest.mark.parametrize("tokens,heads,hkv", [(50, 8, 1), (37, 8, 1), (16, 8, 1), (3, 8, 1), (20, 8, 2)])
def test_pair_row_counts(dtype, tokens, heads, hkv):
    """400, 296, 128, 24 and 80 query rows per KV head: a full pair plus a part-empty one, a pair
    whose second CTA is empty, and GQA with two KV heads."""
    gen = torch.Generator().manual_seed(21)
    plens = [758, 301, 64, 33]
    f = Filled(dtype=dtype, B=4, prefix_lens=plens, Hkv=hkv, D=D, suffix_len=tokens, seed=21)
    q = bf16_randn(gen, (4, tokens, heads, D))
    got, single = both(f, q, Hq=heads, scale=1 / 16)
    want = oracle_attention(f, 0, q, scale=1 / 16)
    check(got, want, TOL[dtype])
    check(single, want, TOL[dtype])
    assert np.abs(got - single).max() <= TOL[dtype]


@pytest.mark.parametrize("dtype", [ekv.DTYPE_BF16, ekv.DTYPE_Q8_0])
@pytest.mark.parametrize("flag", [ekv.MASK_SUFFIX_CAUSAL, ekv.MASK_SUFFIX_PREFIX_LM, ekv.MASK_SPAN_EXCLUDE,
                                  ekv.MASK_SPAN_ONLY])
def test_pair_masks(dtype, flag):
    gen = torch.Generator().manual_seed(22)
    f = Filled(dtype=dtype, B=3, prefix_lens=[300, 517, 96], Hkv=1, D=D, suffix_len=50, seed=22)
    q = bf16_randn(gen, (3, 50, 8, D))
    span = ([20, 100, 0], [276, 400, 64])
    valid = [300, 500, 90]
    kw = dict(mask_flags=flag, prefix_valid=valid)
    if flag in (ekv.MASK_SPAN_EXCLUDE, ekv.MASK_SPAN_ONLY):
        kw["span"] = span
    got, single = both(f, q, Hq=8, scale=1 / 16, **kw)
    want = oracle_attention(f, 0, q, scale=1 / 16, **kw)
    check(got, want, TOL[dtype])
    check(single, want, TOL[dtype])


@pytest.mark.parametrize("dtype", [ekv.DTYPE_BF16, ekv.DTYPE_Q8_0])
def test_pair_block_causal_64_token_blocks(dtype):
    """Block-causal window over 64-token blocks (a block is larger than a CTA's 32-key K half)."""
    gen = torch.Generator().manual_seed(23)
    n_chunks, ct, stride = 3, 40, 64
    f = Filled(dtype=dtype, B=2, prefix_lens=[n_chunks * stride] * 2, Hkv=1, D=D, block_tokens=64, seed=23)
    q = bf16_randn(gen, (2, ct, 8, D))
    block = (ct, stride, 2, n_chunks - 1)
    got, single = both(f, q, Hq=8, scale=1 / 16, mask_flags=ekv.MASK_BLOCK_CAUSAL, block=block)
    want = oracle_attention(f, 0, q, scale=1 / 16, mask_flags=ekv.MASK_BLOCK_CAUSAL, block=block)
    check(got, want, TOL[dtype])
    check(single, want, TOL[dtype])


@pytest.mark.parametrize("dtype", [ekv.DTYPE_BF16, ekv.DTYPE_Q8_0])
def test_pair_split_keys(dtype):
    """Few pairs and long prefixes: the launcher splits keys across pairs through the workspace and
    merges the partial outputs."""
    gen = torch.Generator().manual_seed(24)
    f = Filled(dtype=dtype, B=2, prefix_lens=[2000, 1459], Hkv=1, D=D, suffix_len=10, seed=24)
    q = bf16_randn(gen, (2, 10, 8, D))
    prm = f.pool.attention_params(layer=0, seq_ids=f.seq_ids, q_tokens=10, q_heads=8, scale=1 / 16,
                                  suffix_len=f.suffix_len, out_dtype=ekv.DTYPE_F32)
    assert f.pool.workspace_size(prm) > 0  # the splitter engages for this shape
    want = oracle_attention(f, 0, q, scale=1 / 16)
    for algo in (ekv.ALGO_TC_PAIR, ekv.ALGO_TC_PAIR64):
        a = run_attention(f, 0, q, Hq=8, scale=1 / 16, algo=algo)
        b = run_attention(f, 0, q, Hq=8, scale=1 / 16, algo=algo, workspace=True)
        check(a, want, TOL[dtype])
        check(b, want, TOL[dtype])


def test_pair_bf16_output_pi05_batch():
    """The bench shape at a small batch, bf16 output: pair and single-CTA kernels agree to bf16
    rounding of the same f32 results."""
    gen = torch.Generator().manual_seed(25)
    plens = [700, 816, 759, 701, 788, 730, 777, 812]
    f = Filled(dtype=ekv.DTYPE_Q8_0, B=8, prefix_lens=plens, Hkv=1, D=D, suffix_len=50, seed=25)
    q = bf16_randn(gen, (8, 50, 8, D))
    got, single = both(f, q, Hq=8, scale=1 / 16, out_dtype=ekv.DTYPE_BF16)
    want = oracle_attention(f, 0, q, scale=1 / 16)
    check(got, want, TOL[ekv.DTYPE_Q8_0])
    assert np.abs(got - single).max() <= 2e-2


@pytest.mark.parametrize("dtype", [ekv.DTYPE_BF16, ekv.DTYPE_Q8_0])
@pytest.mark.parametrize("B,ws,d", [(6, False, 256), (2, True, 256), (3, False, 128)])
def test_append_suffix_attention_matches_two_calls(dtype, B, ws, d):
    """ekv_append_suffix_attention gives the same output, bit for bit, as ekv_append_suffix followed
    by ekv_attention, over several layer-steps with a fresh suffix each time, with and without key
    splits. At head_dim 256 the pair kernel reads the suffix from the caller's buffers (the slot,
    clobbered beforehand, stays as it was); at head_dim 128 the call appends into the slot first."""
    gen = torch.Generator().manual_seed(40 + B)
    plens = [int(x) for x in np.random.default_rng(B).integers(200, 820, size=B)]
    T, Hq = 50, 8
    f = Filled(dtype=dtype, B=B, prefix_lens=plens, Hkv=1, D=d, suffix_len=T, n_layers=2, seed=40 + B)
    prm = [f.pool.attention_params(layer=l, seq_ids=f.seq_ids, q_tokens=T, q_heads=Hq, scale=d ** -0.5,
                                   suffix_len=T, out_dtype=ekv.DTYPE_F32) for l in range(2)]
    wsb = None
    if ws:
        n = f.pool.workspace_size(prm[0])
        wsb = torch.empty(max(n, 16), dtype=torch.uint8, device="cuda")
    for step in range(3):
        for l in range(2):
            sk = bf16_randn(gen, (B, T, 1, d)).cuda()
            sv = bf16_randn(gen, (B, T, 1, d)).cuda()
            q = bf16_randn(gen, (B, T, Hq, d)).cuda()
            two = torch.empty((B, T, Hq, d), dtype=torch.float32, device="cuda")
            one = torch.empty_like(two)
            f.pool.append_suffix(l, f.seq_ids, sk, sv)
            f.pool.attention(prm[l], q, two, workspace=wsb)
            ks_two = torch.empty((T, 1, d), dtype=torch.bfloat16, device="cuda")
            vs_two = torch.empty_like(ks_two)
            f.pool.gather_suffix(l, f.seqs[0], T, ekv.GATHER_NATIVE, ks_two, vs_two)
            # clobber the slot so that the fused call must write it again
            f.pool.append_suffix(l, f.seq_ids, torch.zeros_like(sk), torch.zeros_like(sv))
            f.pool.append_suffix_attention(prm[l], sk, sv, q, one, workspace=wsb)
            ks_one = torch.empty_like(ks_two)
            vs_one = torch.empty_like(ks_two)
            f.pool.gather_suffix(l, f.seqs[0], T, ekv.GATHER_NATIVE, ks_one, vs_one)
            torch.cuda.synchronize()
            assert f.pool.status() == 0
            assert torch.equal(one, two), (step, l)
            if d == 256:
                assert not torch.any(ks_one.view(torch.int16)) and not torch.any(vs_one.view(torch.int16))
            else:
                assert torch.equal(ks_one.view(torch.int16), ks_two.view(torch.int16))
                assert torch.equal(vs_one.view(torch.int16), vs_two.view(torch.int16))


@pytest.mark.parametrize("dtype", [ekv.DTYPE_BF16, ekv.DTYPE_Q8_0])
@pytest.mark.parametrize("flag,T,hkv", [(ekv.MASK_SUFFIX_CAUSAL, 50, 1), (ekv.MASK_SUFFIX_PREFIX_LM, 51, 1),
                                        (ekv.MASK_SPAN_EXCLUDE, 100, 2), (0, 1, 1), (0, 64, 2), (0, 128, 1)])
def test_direct_suffix_masks_and_lengths(dtype, flag, T, hkv):
    """The pair kernel's direct suffix read against the oracle and against append + attention,
    bit for bit: causal and prefix-LM suffix masks, spans, GQA, suffix lengths of 1, 51, 64, 100 and
    128 rows (one, two and exactly two full suffix tiles), ragged prefixes with padding."""
    gen = torch.Generator().manual_seed(60 + T)
    B, Hq = 3, 4 * hkv
    plens = [517, 64, 300]
    f = Filled(dtype=dtype, B=B, prefix_lens=plens, Hkv=hkv, D=D, suffix_len=T, seed=60 + T)
    valid = [500, 60, 290]
    span = ([20, 0, 10], [400, 64, 200])
    dev = lambda v: torch.tensor(v, dtype=torch.int32, device="cuda")
    kw = dict(mask_flags=flag, suffix_len=T, out_dtype=ekv.DTYPE_F32, prefix_valid=dev(valid))
    if flag == ekv.MASK_SPAN_EXCLUDE:
        kw.update(span_begin=dev(span[0]), span_end=dev(span[1]))
    prm = f.pool.attention_params(layer=0, seq_ids=f.seq_ids, q_tokens=T, q_heads=Hq, scale=1 / 16, **kw)
    sk = bf16_randn(gen, (B, T, hkv, D))
    sv = bf16_randn(gen, (B, T, hkv, D))
    q = bf16_randn(gen, (B, T, Hq, D)).cuda()
    fused = torch.empty((B, T, Hq, D), dtype=torch.float32, device="cuda")
    f.pool.append_suffix(0, f.seq_ids, torch.zeros_like(sk).cuda(), torch.zeros_like(sv).cuda())
    f.pool.append_suffix_attention(prm, sk.cuda(), sv.cuda(), q, fused)
    two = torch.empty_like(fused)
    f.pool.append_suffix(0, f.seq_ids, sk.cuda(), sv.cuda())
    f.pool.attention(prm, q, two)
    torch.cuda.synchronize()
    assert f.pool.status() == 0
    assert torch.equal(fused, two)
    f.sk[0], f.sv[0] = sk, sv  # the oracle reads this layer's suffix from the builder
    okw = dict(mask_flags=flag, prefix_valid=valid)
    if flag == ekv.MASK_SPAN_EXCLUDE:
        okw["span"] = span
    want = oracle_attention(f, 0, q.cpu(), scale=1 / 16, **okw)
    check(fused.cpu().numpy(), want, TOL[dtype])
