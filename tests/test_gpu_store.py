"""GPU checks of the pool's predicted-token roll-back through the C-ABI: LingBot-VA's rollout appends
a chunk's predicted K/V, attends, clears them (LingBotKVCache::clear_pred, models/lingbot_va.cpp:
8954-8966) and appends the chunk's clean K/V, which take the predicted rows' positions. The gathered
cache must equal, bit for bit, the cache the clean tokens alone would give (bf16 values, or ggml
block_q8_0 bytes from the gguf rule), and attention must see only the clean tokens."""
import numpy as np
import pytest
import torch

import ekv
import oracle
from cases import bf16_randn, to_f32_np

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.tensor(np.asarray(a, np.int32), device="cuda")


@pytest.mark.parametrize("dtype,bt", [(ekv.DTYPE_BF16, 16), (ekv.DTYPE_Q8_0, 16), (ekv.DTYPE_BF16, 64)])
def test_predict_clear_append_clean(dtype, bt):
    gen = torch.Generator().manual_seed(200 + bt)
    H, D = 2, 128
    pool = ekv.Pool(device=0, dtype=dtype, block_tokens=bt, n_blocks=32, kv_heads=H, head_dim=D, n_layers=1,
                    max_seqs=2, max_blocks_per_seq=16)
    s = pool.seq_create()
    ids = dev([s])
    base_k, base_v = bf16_randn(gen, (70, H, D)), bf16_randn(gen, (70, H, D))
    pred_k, pred_v = bf16_randn(gen, (45, H, D)) * 9, bf16_randn(gen, (45, H, D)) * 9
    clean_k, clean_v = bf16_randn(gen, (45, H, D)), bf16_randn(gen, (45, H, D))
    pool.seq_append_tokens(s, 70)
    pool.sync()
    pool.append(0, ids, dev([0]), dev([70]), dev([0]), 70, base_k.cuda(), base_v.cuda())
    # the predicted chunk, attended over, then rolled back
    pool.seq_append_tokens(s, 45, pred=True)
    pool.sync()
    pool.append(0, ids, dev([70]), dev([45]), dev([0]), 45, pred_k.cuda(), pred_v.cuda())
    q = bf16_randn(gen, (1, 5, 4, D))
    prm = pool.attention_params(layer=0, seq_ids=ids, q_tokens=5, q_heads=4, scale=D ** -0.5, out_dtype=ekv.DTYPE_F32)
    out = torch.empty((1, 5, 4, D), dtype=torch.float32, device="cuda")
    pool.attention(prm, q.cuda(), out)
    assert pool.seq_get_pred(s) == (70, 115)
    pool.seq_clear_pred(s)
    pool.seq_append_tokens(s, 45)
    pool.sync()
    pool.append(0, ids, dev([70]), dev([45]), dev([0]), 45, clean_k.cuda(), clean_v.cuda())
    torch.cuda.synchronize()
    assert pool.seq_get(s).n_tokens == 115 and pool.status() == 0
    want_k = torch.cat([base_k, clean_k])
    want_v = torch.cat([base_v, clean_v])
    if dtype == ekv.DTYPE_BF16:
        k = torch.empty((115, H, D), dtype=torch.bfloat16, device="cuda")
    else:
        k = torch.empty((115, H, D // 32 * 34), dtype=torch.uint8, device="cuda")
    v = torch.empty_like(k)
    pool.gather(0, s, 0, 115, ekv.GATHER_NATIVE, k, v)
    torch.cuda.synchronize()
    if dtype == ekv.DTYPE_BF16:
        assert torch.equal(k.cpu().view(torch.int16), want_k.view(torch.int16))
        assert torch.equal(v.cpu().view(torch.int16), want_v.view(torch.int16))
    else:
        np.testing.assert_array_equal(k.cpu().numpy(), oracle.quantize_q8_0(to_f32_np(want_k).reshape(115, H, D)))
        np.testing.assert_array_equal(v.cpu().numpy(), oracle.quantize_q8_0(to_f32_np(want_v).reshape(115, H, D)))
    # attention after the roll-back sees the clean tokens only
    pool.attention(prm, q.cuda(), out)
    torch.cuda.synchronize()
    kf, vf = to_f32_np(want_k)[None], to_f32_np(want_v)[None]
    if dtype == ekv.DTYPE_Q8_0:
        kf = oracle.dequantize_q8_0(oracle.quantize_q8_0(kf.reshape(115, -1))).reshape(kf.shape)
        vf = oracle.dequantize_q8_0(oracle.quantize_q8_0(vf.reshape(115, -1))).reshape(vf.shape)
    want = oracle.attention(to_f32_np(q), kf, vf, oracle.make_seqs([115]), oracle.make_mask(), D ** -0.5)
    assert np.abs(out.cpu().numpy() - want).max() <= (5e-2 if dtype == ekv.DTYPE_Q8_0 else 2e-2)
    pool.close()
