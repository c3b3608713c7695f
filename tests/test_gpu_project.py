"""The layer-step's Q/K/V projection with RoPE (ekv_project_qkv_rope, tcgen05) against the CPU oracle,
through the C-ABI: q = Wq x, k = Wk x, v = Wv x over bf16 weights and activations with f32 accumulation,
RoPE in ggml's NEOX mode on q and k at the suffix positions (models/pi05.cpp:391-402, positions
n_prefix + i, :876-879), results rounded to bf16. K and V land in the pool's suffix slots (checked by
gathering them back, and by attention over the pool) or in the caller's row-major buffers.
"""
import numpy as np
import pytest
import torch

import ekv
import oracle
from cases import Filled, bf16_randn, to_f32_np
from test_gpu_parity import check

pytestmark = pytest.mark.gpu


def setup(B, T, hidden, Hq, Hkv, D, plens, seed, suffix_cap=None):
    gen = torch.Generator().manual_seed(seed)
    f = Filled(dtype=ekv.DTYPE_BF16, B=B, prefix_lens=plens, Hkv=Hkv, D=D, suffix_len=0,
               suffix_cap=suffix_cap if suffix_cap is not None else T, seed=seed)
    x = bf16_randn(gen, (B * T, hidden), 0.5)
    ws = hidden ** -0.5
    wq, wk, wv = (bf16_randn(gen, (h * D, hidden), ws) for h in (Hq, Hkv, Hkv))
    pos = np.concatenate([np.arange(T) + p for p in plens]).astype(np.int32)
    return f, x, wq, wk, wv, pos


def run(f, x, wq, wk, wv, pos, *, T, Hq, base=10000.0, row_major=False):
    B = f.B
    D, Hkv = f.D, f.Hkv
    q = torch.full((B, T, Hq, D), float("nan"), dtype=torch.bfloat16, device="cuda")
    k = v = None
    if row_major:
        k = torch.full((B, T, Hkv, D), float("nan"), dtype=torch.bfloat16, device="cuda")
        v = torch.full_like(k, float("nan"))
    ekv.project_qkv_rope(f.pool, 0, f.seq_ids, x.cuda(), wq.cuda(), wk.cuda(), wv.cuda(),
                         torch.tensor(pos, device="cuda"), base, q, k, v, tokens=T, q_heads=Hq)
    torch.cuda.synchronize()
    assert f.pool.status() == 0
    return q, k, v


def expect(x, wq, wk, wv, pos, Hq, Hkv, base=10000.0):
    return oracle.project_qkv_rope(to_f32_np(x), to_f32_np(wq), to_f32_np(wk), to_f32_np(wv), pos, base, Hq, Hkv)


def agree(got, want):
    """bf16 results: within the bf16 tolerance everywhere and bit-identical almost everywhere (f32 sums in a
    different order can move a value across a bf16 rounding boundary)."""
    g = got.float().cpu().numpy().reshape(want.shape)
    check(g, want, 2e-2)
    assert np.mean(g == want) > 0.99


def test_pi05_shape_into_slots_and_attention():
    """pi0.5 expert layer-step (hidden 1024, 8 query heads over 1 KV head of 256, 50 action tokens) for 3
    requests: q, the slot K/V gathered back, and attention over prefix + projected suffix."""
    B, T, hidden, Hq, Hkv, D = 3, 50, 1024, 8, 1, 256
    plens = [816, 700, 777]
    f, x, wq, wk, wv, pos = setup(B, T, hidden, Hq, Hkv, D, plens, 51)
    q, _, _ = run(f, x, wq, wk, wv, pos, T=T, Hq=Hq)
    eq, ek, ev = expect(x, wq, wk, wv, pos, Hq, Hkv)
    agree(q, eq.reshape(B, T, Hq, D))
    for b in range(B):
        ks = torch.empty((T, Hkv, D), dtype=torch.bfloat16, device="cuda")
        vs = torch.empty_like(ks)
        f.pool.gather_suffix(0, f.seqs[b], T, ekv.GATHER_NATIVE, ks, vs)
        torch.cuda.synchronize()
        agree(ks, ek[b * T:(b + 1) * T])
        agree(vs, ev[b * T:(b + 1) * T])
    # attention over the cached prefix and the projected suffix, as the denoise loop runs it next
    f.suffix_len = T
    f.sk = [torch.tensor(oracle.f32_to_bf16(ek.reshape(B, T, Hkv, D))).view(torch.bfloat16)]
    f.sv = [torch.tensor(oracle.f32_to_bf16(ev.reshape(B, T, Hkv, D))).view(torch.bfloat16)]
    prm = f.pool.attention_params(layer=0, seq_ids=f.seq_ids, q_tokens=T, q_heads=Hq, scale=1 / 16, suffix_len=T,
                                  out_dtype=ekv.DTYPE_F32)
    out = torch.empty((B, T, Hq, D), dtype=torch.float32, device="cuda")
    f.pool.attention(prm, q, out)
    torch.cuda.synchronize()
    assert f.pool.status() == 0
    k_all, v_all = f.oracle_kv(0)
    want = oracle.attention(to_f32_np(q), k_all, v_all, oracle.make_seqs(plens, n_suffix=T), oracle.make_mask(), 1 / 16)
    check(out.cpu().numpy(), want, 2e-2)


@pytest.mark.parametrize("D,Hq,Hkv,B,T,p0", [(128, 4, 2, 3, 17, 37), (64, 6, 3, 2, 70, 37), (256, 8, 1, 1, 50, 37),
                                             (128, 2, 2, 2, 40, 60000)])
def test_row_major_outputs_and_ragged_rows(D, Hq, Hkv, B, T, p0):
    """Row-major K/V outputs (the buffers of ekv_append_suffix_attention), GQA, head dims 64 / 128 / 256,
    row counts that leave the last 128-row tile partly empty, hidden 512, and positions near 60,000 (angles
    of thousands of turns)."""
    hidden = 512
    f, x, wq, wk, wv, pos = setup(B, T, hidden, Hq, Hkv, D, [37 * (b + 1) for b in range(B)], D + T,
                                  suffix_cap=max(T, 8))
    pos = pos - 37 + p0
    q, k, v = run(f, x, wq, wk, wv, pos, T=T, Hq=Hq, base=500.0, row_major=True)
    eq, ek, ev = expect(x, wq, wk, wv, pos, Hq, Hkv, base=500.0)
    agree(q, eq.reshape(B, T, Hq, D))
    agree(k, ek.reshape(B, T, Hkv, D))
    agree(v, ev.reshape(B, T, Hkv, D))


def test_outputs_16_byte_aligned_only():
    """q_out / k_out / v_out that are 16-byte but not 32-byte aligned (views 8 elements into larger buffers)
    take the 16-byte store path and give the same bits as 32-byte aligned outputs."""
    B, T, hidden, Hq, Hkv, D = 2, 40, 256, 4, 2, 128
    f, x, wq, wk, wv, pos = setup(B, T, hidden, Hq, Hkv, D, [20, 30], 77)
    q_a, k_a, v_a = run(f, x, wq, wk, wv, pos, T=T, Hq=Hq, row_major=True)
    bufs = [torch.full((B * T * h * D + 8,), float("nan"), dtype=torch.bfloat16, device="cuda") for h in (Hq, Hkv, Hkv)]
    q_u, k_u, v_u = (b_[8:].view(B, T, h, D) for b_, h in zip(bufs, (Hq, Hkv, Hkv)))
    assert q_u.data_ptr() % 32 == 16
    ekv.project_qkv_rope(f.pool, 0, f.seq_ids, x.cuda(), wq.cuda(), wk.cuda(), wv.cuda(), torch.tensor(pos, device="cuda"),
                         10000.0, q_u, k_u, v_u, tokens=T, q_heads=Hq)
    torch.cuda.synchronize()
    assert f.pool.status() == 0
    for got, want in ((q_u, q_a), (k_u, k_a), (v_u, v_a)):
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("case", ["hidden", "tokens", "align", "one_of_kv"])
def test_rejects_bad_arguments(case):
    B, T, hidden, Hq, Hkv, D = 2, 8, 128, 2, 1, 64
    f, x, wq, wk, wv, pos = setup(B, T, hidden, Hq, Hkv, D, [10, 20], 3)
    dev = lambda t: t.cuda()
    xq, pq = dev(x), torch.tensor(pos, device="cuda")
    q = torch.empty((B, T, Hq, D), dtype=torch.bfloat16, device="cuda")
    k = torch.empty((B, T, Hkv, D), dtype=torch.bfloat16, device="cuda")
    args = dict(hidden=hidden, tokens=T, xp=xq.data_ptr(), kp=None, vp=None)
    want = ekv.ERR_INVALID_ARG
    if case == "hidden":
        args["hidden"] = 100
    elif case == "tokens":
        args["tokens"] = 9  # more than the pool's suffix slot
        want = ekv.ERR_RANGE
    elif case == "align":
        args["xp"] = xq.data_ptr() + 2
    else:
        args["kp"] = k.data_ptr()
    rc = ekv.lib.ekv_project_qkv_rope(f.pool.h, 0, B, f.seq_ids.data_ptr(), args["tokens"], Hq, args["hidden"],
                                      args["xp"], dev(wq).data_ptr(), dev(wk).data_ptr(), dev(wv).data_ptr(),
                                      pq.data_ptr(), 10000.0, q.data_ptr(), args["kp"], args["vp"], None)
    assert rc == want
