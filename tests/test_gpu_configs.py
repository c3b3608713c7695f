"""GPU parity at the BASELINE configs' own shapes, through the C-ABI, against the CPU oracle.

The calls run at full size; the oracle checks a seeded sample of query rows (every row where that is
cheap) with the same f32 arithmetic as the full oracle (ekvo_attention_rows):
  config 1  pi0.5 bf16, batch 1: prefix 816 = 768 image + 48 text slots, valid text U[20, 48] (the
            rest padding), 8 query heads over 1 KV head, head_dim 256, 50 suffix tokens; with the
            key-split workspace (the launcher splits a batch-1 call) and without
  config 2  pi0.5 Q8_0, batch 64, prefixes U[700, 816] in 16-token blocks with shuffled tables, the
            bench's one-call layer-step (ekv_append_suffix_attention), bf16 output
  config 3  GR00T, batch 128: 17 queries x 32 heads x 48 over a 300-token backbone with the image
            span [0, 256) (SPAN_ONLY) and text (SPAN_EXCLUDE) masks, and the self layer over the 17
  config 4  LingBot, one episode: chunks of 1560 tokens at stride 1600 in 64-token blocks, 24 heads x
            128, block-causal window of 8 chunks; 10 chunks, so that the oldest chunk is evicted twice
  config 5  serving, Q8_0, batch 256, prefixes U[600, 1000]
"""
import numpy as np
import pytest
import torch

import ekv
import oracle
from cases import Filled, bf16_randn, to_f32_np
from test_gpu_parity import TOL

pytestmark = pytest.mark.gpu


def sample_rows(rng, B, Tq, Hq, per_b):
    rows = []
    for b in range(B):
        for i in rng.choice(Tq * Hq, size=min(per_b, Tq * Hq), replace=False):
            rows.append((b, int(i) // Hq, int(i) % Hq))
    return np.array(rows, np.int32)


def check_rows(got, want_rows, rows, tol):
    g = got[rows[:, 0], rows[:, 1], rows[:, 2]]
    assert np.isfinite(got).all()
    err = float(np.abs(g - want_rows).max())
    assert err <= tol, f"max-abs {err} > {tol}"
    return err


def dev(a):
    return torch.tensor(np.asarray(a, np.int32), device="cuda")


@pytest.mark.parametrize("workspace", [True, False])
def test_config1_pi05_bf16_batch1(workspace):
    rng = np.random.default_rng(101)
    gen = torch.Generator().manual_seed(101)
    valid = [768 + int(rng.integers(20, 49))]
    f = Filled(dtype=ekv.DTYPE_BF16, B=1, prefix_lens=[816], Hkv=1, D=256, suffix_len=50, seed=101)
    q = bf16_randn(gen, (1, 50, 8, 256))
    prm = f.pool.attention_params(layer=0, seq_ids=f.seq_ids, q_tokens=50, q_heads=8, scale=1 / 16, suffix_len=50,
                                  out_dtype=ekv.DTYPE_F32, prefix_valid=dev(valid))
    ws = None
    if workspace:
        n = f.pool.workspace_size(prm)
        assert n > 0  # batch 1 splits its keys across CTA pairs
        ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    out = torch.empty((1, 50, 8, 256), dtype=torch.float32, device="cuda")
    f.pool.attention(prm, q.cuda(), out, workspace=ws)
    torch.cuda.synchronize()
    assert f.pool.status() == 0
    k, v = f.oracle_kv(0)
    want = oracle.attention(to_f32_np(q), k, v, oracle.make_seqs([816], prefix_valid=valid, n_suffix=50),
                            oracle.make_mask(), 1 / 16)
    err = np.abs(out.cpu().numpy() - want).max()
    assert err <= TOL[ekv.DTYPE_BF16], err


def test_config2_pi05_q8_batch64_layer_step():
    rng = np.random.default_rng(102)
    gen = torch.Generator().manual_seed(102)
    B = 64
    plens = [int(x) for x in rng.integers(700, 817, size=B)]
    f = Filled(dtype=ekv.DTYPE_Q8_0, B=B, prefix_lens=plens, Hkv=1, D=256, suffix_len=50, seed=102)
    sk, sv = bf16_randn(gen, (B, 50, 1, 256)), bf16_randn(gen, (B, 50, 1, 256))
    q = bf16_randn(gen, (B, 50, 8, 256))
    prm = f.pool.attention_params(layer=0, seq_ids=f.seq_ids, q_tokens=50, q_heads=8, scale=1 / 16, suffix_len=50,
                                  out_dtype=ekv.DTYPE_BF16)
    out = torch.empty((B, 50, 8, 256), dtype=torch.bfloat16, device="cuda")
    f.pool.append_suffix_attention(prm, sk.cuda(), sv.cuda(), q.cuda(), out)
    torch.cuda.synchronize()
    assert f.pool.status() == 0
    f.sk[0], f.sv[0] = sk, sv
    k, v = f.oracle_kv(0)
    rows = sample_rows(rng, B, 50, 8, 8)
    want = oracle.attention_rows(to_f32_np(q), k, v, oracle.make_seqs(plens, n_suffix=50), oracle.make_mask(),
                                 1 / 16, rows)
    check_rows(out.float().cpu().numpy(), want, rows, TOL[ekv.DTYPE_Q8_0])


def test_config3_groot_batch128():
    rng = np.random.default_rng(103)
    gen = torch.Generator().manual_seed(103)
    B, T, H, DH, P, IMG = 128, 17, 32, 48, 300, 256
    f = Filled(dtype=ekv.DTYPE_BF16, B=B, prefix_lens=[P] * B, Hkv=H, D=DH, suffix_len=T, seed=103)
    q = bf16_randn(gen, (B, T, H, DH))
    span_b, span_e = dev(np.zeros(B)), dev(np.full(B, IMG))
    k, v = f.oracle_kv(0)
    for flag in (ekv.MASK_SPAN_ONLY, ekv.MASK_SPAN_EXCLUDE):
        prm = f.pool.attention_params(layer=0, seq_ids=f.seq_ids, q_tokens=T, q_heads=H, scale=DH ** -0.5,
                                      mask_flags=flag, span_begin=span_b, span_end=span_e, out_dtype=ekv.DTYPE_F32)
        out = torch.empty((B, T, H, DH), dtype=torch.float32, device="cuda")
        f.pool.attention(prm, q.cuda(), out)
        torch.cuda.synchronize()
        assert f.pool.status() == 0
        rows = sample_rows(rng, B, T, H, 6)
        want = oracle.attention_rows(to_f32_np(q), k, v, oracle.make_seqs([P] * B, span=(0, IMG), n_suffix=0),
                                     oracle.make_mask(flag), DH ** -0.5, rows)
        check_rows(out.cpu().numpy(), want, rows, TOL[ekv.DTYPE_BF16])
    # the self layer: suffix only (the 17 tokens' own K/V passed with the call)
    sk, sv = bf16_randn(gen, (B, T, H, DH)), bf16_randn(gen, (B, T, H, DH))
    prm = f.pool.attention_params(layer=0, seq_ids=f.seq_ids, q_tokens=T, q_heads=H, scale=DH ** -0.5, suffix_len=T,
                                  use_prefix=False, out_dtype=ekv.DTYPE_F32)
    out = torch.empty((B, T, H, DH), dtype=torch.float32, device="cuda")
    f.pool.append_suffix_attention(prm, sk.cuda(), sv.cuda(), q.cuda(), out)
    torch.cuda.synchronize()
    assert f.pool.status() == 0
    rows = sample_rows(rng, B, T, H, 6)
    want = oracle.attention_rows(to_f32_np(q), to_f32_np(sk), to_f32_np(sv), oracle.make_seqs([0] * B, n_suffix=T),
                                 oracle.make_mask(), DH ** -0.5, rows)
    check_rows(out.cpu().numpy(), want, rows, TOL[ekv.DTYPE_BF16])


def test_config4_lingbot_window_with_eviction():
    rng = np.random.default_rng(104)
    gen = torch.Generator().manual_seed(104)
    CT, STRIDE, WIN, H, DH, BT = 1560, 1600, 8, 24, 128, 64
    bpc = STRIDE // BT
    pool = ekv.Pool(device=0, dtype=ekv.DTYPE_BF16, block_tokens=BT, n_blocks=(WIN + 1) * bpc, kv_heads=H,
                    head_dim=DH, n_layers=1, max_seqs=1, max_blocks_per_seq=(WIN + 1) * bpc)
    seq = pool.seq_create()
    seq_ids = dev([seq])
    held_k, held_v = [], []  # the window's chunks, oldest first
    for c in range(10):
        held = min(c, WIN - 1) + 1
        if c >= WIN:
            pool.seq_evict_front(seq, bpc)
            held_k.pop(0)
            held_v.pop(0)
        pool.seq_resize(seq, held * STRIDE)
        pool.sync()
        kc, vc, qc = (bf16_randn(gen, (CT, H, DH)) for _ in range(3))
        pool.append(0, seq_ids, dev([(held - 1) * STRIDE]), dev([CT]), dev([0]), CT, kc.cuda(), vc.cuda())
        held_k.append(kc)
        held_v.append(vc)
        prm = pool.attention_params(layer=0, seq_ids=seq_ids, q_tokens=CT, q_heads=H, scale=DH ** -0.5,
                                    mask_flags=ekv.MASK_BLOCK_CAUSAL, chunk_tokens=CT, chunk_stride=STRIDE,
                                    window_chunks=WIN, q_chunk0=held - 1, out_dtype=ekv.DTYPE_F32)
        n = pool.workspace_size(prm)
        ws = torch.empty(max(n, 16), dtype=torch.uint8, device="cuda")
        out = torch.empty((1, CT, H, DH), dtype=torch.float32, device="cuda")
        pool.attention(prm, qc[None].cuda(), out, workspace=ws)
        torch.cuda.synchronize()
        assert pool.status() == 0
        if c in (0, 3, 7, 8, 9):
            L = held * STRIDE
            k = np.zeros((1, L, H, DH), np.float32)
            v = np.zeros_like(k)
            for i in range(held):
                k[0, i * STRIDE:i * STRIDE + CT] = to_f32_np(held_k[i])
                v[0, i * STRIDE:i * STRIDE + CT] = to_f32_np(held_v[i])
            rows = sample_rows(rng, 1, CT, H, 48)
            want = oracle.attention_rows(to_f32_np(qc)[None], k, v, oracle.make_seqs([L], n_suffix=0),
                                         oracle.make_mask(oracle.MASK_BLOCK_CAUSAL, CT, STRIDE, WIN, held - 1),
                                         DH ** -0.5, rows)
            check_rows(out.cpu().numpy(), want, rows, TOL[ekv.DTYPE_BF16])
    pool.close()


def test_config5_serving_q8_batch256():
    rng = np.random.default_rng(105)
    gen = torch.Generator().manual_seed(105)
    B = 256
    plens = [int(x) for x in rng.integers(600, 1001, size=B)]
    f = Filled(dtype=ekv.DTYPE_Q8_0, B=B, prefix_lens=plens, Hkv=1, D=256, suffix_len=50, seed=105)
    q = bf16_randn(gen, (B, 50, 8, 256))
    prm = f.pool.attention_params(layer=0, seq_ids=f.seq_ids, q_tokens=50, q_heads=8, scale=1 / 16, suffix_len=50,
                                  out_dtype=ekv.DTYPE_BF16)
    out = torch.empty((B, 50, 8, 256), dtype=torch.bfloat16, device="cuda")
    f.pool.attention(prm, q.cuda(), out)
    torch.cuda.synchronize()
    assert f.pool.status() == 0
    k, v = f.oracle_kv(0)
    rows = sample_rows(rng, B, 50, 8, 3)
    want = oracle.attention_rows(to_f32_np(q), k, v, oracle.make_seqs(plens, n_suffix=50), oracle.make_mask(),
                                 1 / 16, rows)
    check_rows(out.float().cpu().numpy(), want, rows, TOL[ekv.DTYPE_Q8_0])
