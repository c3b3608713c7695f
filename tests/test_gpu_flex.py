"""LingBot-VA flex masks (EKV_MASK_FLEX_SELF / EKV_MASK_FLEX_CROSS) on the GPU against the CPU oracle,
through the C-ABI: the reference's token metadata layouts (build_flex_mask_meta, flex_self_allowed,
flex_cross_allowed, models/lingbot_va.cpp:9283-9348) from the golden fixture, with the keys split
between the paged prefix and the suffix slot, two batch elements with different metadata rows, GQA,
head dims 64 / 128 / 256 (one-CTA kernel, both CTA-pair kernels, the CUDA-core kernel), bf16 and
Q8_0 caches."""
import os

import numpy as np
import pytest
import torch

import ekv
import oracle
from cases import Filled, bf16_randn, to_f32_np
from test_gpu_parity import TOL, check

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "lingbot_flex.npz")


def layout_words(layout):
    g = np.load(GOLDEN)
    seq, frame, noise = g[f"{layout}_seq"], g[f"{layout}_frame"], g[f"{layout}_noise"]
    words = np.array([oracle.flex_meta_word(int(s), int(f), int(z)) if s >= 0 else 0
                      for s, f, z in zip(seq, frame, noise)], np.int32)
    text = np.array([oracle.flex_meta_word(int(t), 0, 0) for t in g[f"{layout}_text"]], np.int32)
    return words, text, int(g[f"{layout}_window"])


def run(f, q, Hq, D, flags, meta, stride, q0, k0, window, algo, ws=False):
    dev = lambda a: torch.tensor(np.asarray(a, np.int32), device="cuda")
    m = dev(meta)
    prm = f.pool.attention_params(layer=0, seq_ids=f.seq_ids, q_tokens=q.shape[1], q_heads=Hq, scale=D ** -0.5,
                                  mask_flags=flags, suffix_len=f.suffix_len, out_dtype=ekv.DTYPE_F32,
                                  flex_meta=m, flex_stride=stride, flex_q0=q0, flex_k0=k0, flex_window=window)
    out = torch.full(q.shape, float("nan"), dtype=torch.float32, device="cuda")
    wsb = None
    if ws:
        n = f.pool.workspace_size(prm)
        wsb = torch.empty(max(n, 16), dtype=torch.uint8, device="cuda")
    f.pool.attention(prm, q.cuda().contiguous(), out, workspace=wsb, algo=algo)
    torch.cuda.synchronize()
    assert f.pool.status() == 0
    return out.cpu().numpy()


CASES = [("chunks", 128, 4, 2, ekv.DTYPE_BF16), ("chunks", 128, 4, 2, ekv.DTYPE_Q8_0),
         ("batch2", 256, 2, 1, ekv.DTYPE_BF16), ("batch2", 256, 2, 1, ekv.DTYPE_Q8_0),
         ("runtime", 64, 4, 4, ekv.DTYPE_BF16)]


@pytest.mark.parametrize("algo", [ekv.ALGO_TC, ekv.ALGO_TC_CTA, ekv.ALGO_SIMT, ekv.ALGO_TC_PAIR64])
@pytest.mark.parametrize("layout,D,Hq,Hkv,dtype", CASES)
def test_flex_self(algo, layout, D, Hq, Hkv, dtype):
    """Self-attention of every token of the layout over itself: the first n - 9 tokens' K/V in the
    paged prefix, the last 9 in the suffix slot; batch element 1 carries the metadata rolled by 7."""
    words, _, window = layout_words(layout)
    n, ns = len(words), 9
    meta = np.stack([words, np.roll(words, 7)])
    gen = torch.Generator().manual_seed(70 + n)
    f = Filled(dtype=dtype, B=2, prefix_lens=[n - ns, n - ns], Hkv=Hkv, D=D, suffix_len=ns, block_tokens=16,
               seed=70 + n)
    q = bf16_randn(gen, (2, n, Hq, D))
    got = run(f, q, Hq, D, ekv.MASK_FLEX_SELF, meta.ravel(), n, 0, 0, window, algo)
    k, v = f.oracle_kv(0)
    seqs = oracle.make_seqs([n - ns] * 2, n_suffix=ns, flex_meta=[meta[0], meta[1]])
    want = oracle.attention(to_f32_np(q), k, v, seqs, oracle.make_mask(oracle.MASK_FLEX_SELF, flex_window=window),
                            D ** -0.5)
    check(got, want, TOL[dtype])


@pytest.mark.parametrize("algo", [ekv.ALGO_TC, ekv.ALGO_SIMT])
@pytest.mark.parametrize("layout,D,Hq,Hkv,dtype", CASES)
def test_flex_cross(algo, layout, D, Hq, Hkv, dtype):
    """Cross-attention of the layout's tokens to its text tokens (the keys, in the paged prefix):
    metadata rows hold the query words, then the text words (flex_k0 = tokens)."""
    words, text, _ = layout_words(layout)
    n, T = len(words), len(text)
    meta = np.concatenate([words, text])
    gen = torch.Generator().manual_seed(80 + n)
    f = Filled(dtype=dtype, B=2, prefix_lens=[T, T], Hkv=Hkv, D=D, suffix_len=0, seed=80 + n)
    q = bf16_randn(gen, (2, n, Hq, D))
    got = run(f, q, Hq, D, ekv.MASK_FLEX_CROSS, np.concatenate([meta, meta]), n + T, 0, n, 0, algo)
    k, v = f.oracle_kv(0)
    seqs = oracle.make_seqs([T] * 2, n_suffix=0, flex_meta=[meta, meta])
    want = oracle.attention(to_f32_np(q), k, v, seqs, oracle.make_mask(oracle.MASK_FLEX_CROSS, flex_k0=n),
                            D ** -0.5)
    check(got, want, TOL[dtype])


def test_flex_self_with_key_splits():
    """A long flex-masked prefix on few CTAs: the launcher splits its keys (workspace) and merges."""
    words, _, window = layout_words("chunks")
    reps = 12  # the layout repeated: frame ids shifted by 40 per repeat, one sequence
    rows = []
    for r in range(reps):
        for w in words:
            u = int(w) & 0xFFFFFFFF
            rows.append(0 if u == 0 else ((u & ~0x7FFFFF) | ((u & 0x7FFFFF) + 40 * r)))
    meta = np.array([x - (1 << 32) if x >= (1 << 31) else x for x in rows], np.int64).astype(np.int32)
    n = len(meta)
    gen = torch.Generator().manual_seed(90)
    f = Filled(dtype=ekv.DTYPE_BF16, B=1, prefix_lens=[n], Hkv=1, D=128, suffix_len=0, seed=90)
    q = bf16_randn(gen, (1, 40, 2, 128))
    got = run(f, q, 2, 128, ekv.MASK_FLEX_SELF, meta, n, n - 40, 0, window, ekv.ALGO_TC, ws=True)
    k, v = f.oracle_kv(0)
    seqs = oracle.make_seqs([n], n_suffix=0, flex_meta=[meta])
    want = oracle.attention(to_f32_np(q), k, v, seqs,
                            oracle.make_mask(oracle.MASK_FLEX_SELF, flex_q0=n - 40, flex_window=window), 128 ** -0.5)
    check(got, want, 2e-2)
