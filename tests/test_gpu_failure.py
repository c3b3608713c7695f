"""Failure handling on the GPU without a fault: a bounded wait inside the 64-key CTA-pair kernel is
made to run out (ekv_debug_expire_wait: the MMA-issuing thread waits on a barrier nothing arrives on,
every wait of the launch limited to about 10 ms). The launch must end by itself, report the timeout
through the pool's status word, and leave the context usable: the next call is correct."""
import time

import numpy as np
import pytest
import torch

import ekv
import oracle
from cases import Filled, bf16_randn, to_f32_np

pytestmark = pytest.mark.gpu

DEV_ERR_TIMEOUT = 4  # the kernels' status code for an expired wait (ekv_pool_status)


@pytest.mark.parametrize("dtype", [ekv.DTYPE_Q8_0, ekv.DTYPE_BF16])
def test_expired_wait_reports_timeout_and_context_stays_usable(dtype):
    gen = torch.Generator().manual_seed(300)
    f = Filled(dtype=dtype, B=2, prefix_lens=[300, 517], Hkv=1, D=256, suffix_len=50, seed=300)
    q = bf16_randn(gen, (2, 50, 8, 256)).cuda()
    prm = f.pool.attention_params(layer=0, seq_ids=f.seq_ids, q_tokens=50, q_heads=8, scale=1 / 16, suffix_len=50,
                                  out_dtype=ekv.DTYPE_F32)
    out = torch.full((2, 50, 8, 256), float("nan"), dtype=torch.float32, device="cuda")
    assert f.pool.status() == 0
    ekv.lib.ekv_debug_expire_wait(1)
    try:
        t0 = time.perf_counter()
        f.pool.attention(prm, q, out, algo=ekv.ALGO_TC_PAIR64)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    finally:
        ekv.lib.ekv_debug_expire_wait(0)
    assert f.pool.status() == DEV_ERR_TIMEOUT
    assert elapsed < 5.0
    assert torch.isfinite(out).all()  # the launch that gave up wrote zeros, not garbage
    # the context is usable and the hook was consumed by that one launch
    out.fill_(float("nan"))
    f.pool.attention(prm, q, out, algo=ekv.ALGO_TC_PAIR64)
    torch.cuda.synchronize()
    assert f.pool.status() == 0
    k, v = f.oracle_kv(0)
    want = oracle.attention(to_f32_np(q), k, v, oracle.make_seqs([300, 517], n_suffix=50), oracle.make_mask(), 1 / 16)
    tol = 5e-2 if dtype == ekv.DTYPE_Q8_0 else 2e-2
    assert np.abs(out.cpu().numpy() - want).max() <= tol
    f.pool.close()
