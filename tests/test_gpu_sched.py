"""The batching scheduler on the GPU: requests stream through a small Q8_0 (and bf16) pool, are
admitted as blocks come free, run their denoise steps batched with whatever else is active, and give
their blocks back. Every layer-step output of every request is checked against the oracle run on that
request alone, so a request served from reused blocks (or next to different neighbours) must give the
same result as one served alone."""
import numpy as np
import pytest
import torch

import ekv
import oracle
from cases import bf16_randn, to_f32_np
from test_gpu_parity import TOL

pytestmark = pytest.mark.gpu

D, HQ, TQ, BT, L = 256, 8, 16, 16, 2


def _inputs(rid, plen, n_steps):
    gen = torch.Generator().manual_seed(7000 + rid)
    pk = [bf16_randn(gen, (plen, 1, D)) for _ in range(L)]
    pv = [bf16_randn(gen, (plen, 1, D)) for _ in range(L)]
    sk = [[bf16_randn(gen, (TQ, 1, D)) for _ in range(L)] for _ in range(n_steps)]
    sv = [[bf16_randn(gen, (TQ, 1, D)) for _ in range(L)] for _ in range(n_steps)]
    q = [[bf16_randn(gen, (TQ, HQ, D)) for _ in range(L)] for _ in range(n_steps)]
    return pk, pv, sk, sv, q


@pytest.mark.parametrize("dtype", [ekv.DTYPE_Q8_0, ekv.DTYPE_BF16])
def test_served_requests_match_the_oracle(dtype):
    rng = np.random.default_rng(55)
    n_req, max_batch, n_steps = 10, 4, 3
    plens = [int(x) for x in rng.integers(100, 301, size=n_req)]
    pvalid = [int(rng.integers(p - 40, p + 1)) for p in plens]
    # room for about three requests at a time: admissions wait for blocks and then reuse them
    n_blocks = 3 * ((300 + BT - 1) // BT)
    pool = ekv.Pool(device=0, dtype=dtype, block_tokens=BT, n_blocks=n_blocks, kv_heads=1, head_dim=D, n_layers=L,
                    max_seqs=max_batch, max_blocks_per_seq=(300 + BT - 1) // BT, suffix_tokens=TQ)
    sched = ekv.Scheduler(pool, max_batch, n_steps)
    inp = {r: _inputs(r, plens[r], n_steps) for r in range(n_req)}
    for r in range(n_req):
        sched.submit(r, plens[r], pvalid[r])
    outs, reused, max_active = {}, 0, 0
    for _ in range(200):
        t = sched.begin_tick()
        if t.n_batch == 0 and t.queued == 0:
            break
        reused += t.blocks_reused
        max_active = max(max_active, t.n_batch)
        if t.admitted_index:
            adm = [t.request_ids[i] for i in t.admitted_index]
            for l in range(L):
                kp = torch.cat([inp[r][0][l] for r in adm]).cuda()
                vp = torch.cat([inp[r][1][l] for r in adm]).cuda()
                assert kp.shape[0] == t.admitted_rows
                pool.append(l, t.admitted_seq_ids, t.admitted_zeros, t.admitted_prefix_len, t.admitted_src_row,
                            t.max_admitted_prefix, kp, vp)
        for l in range(L):
            prm = pool.attention_params(layer=l, seq_ids=t.seq_ids, q_tokens=TQ, q_heads=HQ, scale=1 / 16,
                                        suffix_len=TQ, out_dtype=ekv.DTYPE_F32, prefix_valid=t.prefix_valid)
            sel = list(zip(t.request_ids, t.steps))
            sk = torch.stack([inp[r][2][s][l] for r, s in sel]).cuda()
            sv = torch.stack([inp[r][3][s][l] for r, s in sel]).cuda()
            q = torch.stack([inp[r][4][s][l] for r, s in sel]).cuda()
            out = torch.empty((t.n_batch, TQ, HQ, D), dtype=torch.float32, device="cuda")
            ws_n = pool.workspace_size(prm)
            ws = torch.empty(ws_n, dtype=torch.uint8, device="cuda") if ws_n else None
            pool.append_suffix_attention(prm, sk, sv, q, out, workspace=ws)
            o = out.cpu()
            for i, (r, s) in enumerate(sel):
                outs[(r, s, l)] = o[i].numpy()
        sched.end_tick()
    torch.cuda.synchronize()
    assert pool.status() == 0
    st = sched.stats()
    assert st["completed"] == n_req and st["active"] == 0 and st["queued"] == 0
    assert reused > 0 and st["blocks_reused"] == reused
    assert 2 <= max_active <= max_batch
    assert len(outs) == n_req * n_steps * L
    for r in range(n_req):
        n = plens[r]
        pk, pv, sk, sv, q = inp[r]
        for l in range(L):
            kpre, vpre = to_f32_np(pk[l]), to_f32_np(pv[l])
            if dtype == ekv.DTYPE_Q8_0:
                kpre = oracle.dequantize_q8_0(oracle.quantize_q8_0(kpre.reshape(n, -1))).reshape(kpre.shape)
                vpre = oracle.dequantize_q8_0(oracle.quantize_q8_0(vpre.reshape(n, -1))).reshape(vpre.shape)
            for s in range(n_steps):
                k = np.concatenate([kpre, to_f32_np(sk[s][l])])[None]
                v = np.concatenate([vpre, to_f32_np(sv[s][l])])[None]
                want = oracle.attention(to_f32_np(q[s][l])[None], k, v,
                                        oracle.make_seqs([n], prefix_valid=[pvalid[r]], n_suffix=TQ),
                                        oracle.make_mask(), 1 / 16)[0]
                err = float(np.abs(outs[(r, s, l)] - want).max())
                assert err <= TOL[dtype], (r, s, l, err)
    sched.close()
