"""ekv_attention_noalloc: attention whose key-split scratch is a fixed device array, for callers
that cannot allocate device memory where attention runs (a controller or server with a device
budget fixed at start-up, or a plugin host with nowhere to put a workspace). Checked through
the C-ABI against ekv_attention with a caller-provided workspace and against the CPU oracle, on two
calls in a row (the second reuses the scratch the first left behind), for the one-CTA kernel
(head_dim 128) and both CTA-pair kernels (head_dim 256, bf16 and Q8_0 pools), whose key splits
run through the array. This file is collected last on purpose."""
import ctypes as C

import numpy as np
import pytest
import torch

import ekv
import oracle
from cases import Filled, bf16_randn, to_f32_np

pytestmark = pytest.mark.gpu

TOL = {ekv.DTYPE_BF16: 2e-2, ekv.DTYPE_Q8_0: 5e-2}


def noalloc(pool, prm, q, out):
    return ekv.lib.ekv_attention_noalloc(pool.h, C.byref(prm), C.c_void_p(q.data_ptr()),
                                         C.c_void_p(out.data_ptr()),
                                         C.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("dtype,D", [(ekv.DTYPE_BF16, 128), (ekv.DTYPE_Q8_0, 128), (ekv.DTYPE_BF16, 256),
                                     (ekv.DTYPE_Q8_0, 256)])
def test_noalloc_matches_workspace_entry_point(dtype, D):
    f = Filled(dtype=dtype, B=2, prefix_lens=[2000, 1500], Hkv=1, D=D, suffix_len=10, seed=21)
    q = bf16_randn(torch.Generator().manual_seed(21), (2, 10, 8, D)).cuda()
    prm = f.pool.attention_params(layer=0, seq_ids=f.seq_ids, q_tokens=10, q_heads=8, scale=1 / np.sqrt(D),
                                  suffix_len=10, out_dtype=ekv.DTYPE_F32)
    k, v = f.oracle_kv(0)
    want = oracle.attention(to_f32_np(q), k, v, oracle.make_seqs([2000, 1500], n_suffix=10), oracle.make_mask(),
                            1 / np.sqrt(D))
    need = f.pool.workspace_size(prm)
    assert 0 < need <= ekv.NOALLOC_SCRATCH_BYTES  # the key-splitting path is the one exercised
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    ref = torch.empty((2, 10, 8, D), dtype=torch.float32, device="cuda")
    f.pool.attention(prm, q, ref, workspace=ws)
    torch.cuda.synchronize()
    assert f.pool.status() == 0
    assert np.abs(ref.cpu().numpy() - want).max() <= TOL[dtype]
    for _ in range(2):
        out = torch.full((2, 10, 8, D), float("nan"), dtype=torch.float32, device="cuda")
        assert noalloc(f.pool, prm, q, out) == ekv.OK
        torch.cuda.synchronize()
        assert f.pool.status() == 0
        got = out.cpu().numpy()
        assert np.isfinite(got).all()
        assert np.abs(got - ref.cpu().numpy()).max() <= TOL[dtype]
        assert np.abs(got - want).max() <= TOL[dtype]
    f.pool.close()


def test_noalloc_rejects_calls_beyond_the_scratch():
    # 24 KV heads x 13 query tiles with up to 12,800 keys wants far more split scratch than the
    # fixed array holds: the call is refused before anything is launched.
    pool = ekv.Pool(device=0, dtype=ekv.DTYPE_BF16, block_tokens=64, n_blocks=4, kv_heads=24, head_dim=128,
                    n_layers=1, max_seqs=1, max_blocks_per_seq=200, suffix_tokens=0)
    seq_ids = torch.zeros(1, dtype=torch.int32, device="cuda")
    prm = pool.attention_params(layer=0, seq_ids=seq_ids, q_tokens=1560, q_heads=24, scale=0.088,
                                out_dtype=ekv.DTYPE_BF16)
    assert pool.workspace_size(prm) > ekv.NOALLOC_SCRATCH_BYTES
    q = torch.zeros(8, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(8, dtype=torch.bfloat16, device="cuda")
    assert noalloc(pool, prm, q, out) == ekv.ERR_RANGE
    pool.close()
