"""GPU parity of libekv.so against the CPU oracle, through the C-ABI.

Bit-exact: append / gather / evict contents (bf16 and ggml Q8_0 bytes) and block tables.
Attention: max-abs error within the BASELINE tolerances, 2e-2 for bf16 caches and 5e-2 for Q8_0
caches (fp32 accumulation), for both the tcgen05 kernel and the CUDA-core cross-check kernel,
over every mask family of the reference (pi0.5 bidirectional + padding, SmolVLA causal suffix,
HY-VLA prefix-LM, GR00T text/image spans, LingBot block-causal window).
"""
import numpy as np
import pytest
import torch

import ekv
import oracle
from cases import Filled, bf16_randn, to_f32_np

pytestmark = pytest.mark.gpu

TOL = {ekv.DTYPE_BF16: 2e-2, ekv.DTYPE_Q8_0: 5e-2}
ALGOS = [ekv.ALGO_TC, ekv.ALGO_TC_CTA, ekv.ALGO_SIMT]


def gather_prefix(f, layer, b, fmt):
    n = f.prefix_lens[b]
    D, Hkv = f.D, f.Hkv
    if fmt == ekv.GATHER_F32:
        k = torch.empty((n, Hkv, D), dtype=torch.float32, device="cuda")
    elif f.dtype == ekv.DTYPE_BF16:
        k = torch.empty((n, Hkv, D), dtype=torch.bfloat16, device="cuda")
    else:
        k = torch.empty((n, Hkv, D // 32 * 34), dtype=torch.uint8, device="cuda")
    v = torch.empty_like(k)
    f.pool.gather(layer, f.seqs[b], 0, n, fmt, k, v)
    torch.cuda.synchronize()
    return k.cpu(), v.cpu()


@pytest.mark.parametrize("bt", [16, 64])
def test_append_gather_bf16_bit_exact(bt):
    f = Filled(dtype=ekv.DTYPE_BF16, B=3, prefix_lens=[37, 130, 64], Hkv=2, D=128, n_layers=2,
               block_tokens=bt, suffix_len=50, seed=1)
    for layer in range(2):
        for b in range(3):
            n = f.prefix_lens[b]
            k, v = gather_prefix(f, layer, b, ekv.GATHER_NATIVE)
            assert torch.equal(k.view(torch.int16), f.pk[layer][b, :n].view(torch.int16))
            assert torch.equal(v.view(torch.int16), f.pv[layer][b, :n].view(torch.int16))
            kf, vf = gather_prefix(f, layer, b, ekv.GATHER_F32)
            assert torch.equal(kf, f.pk[layer][b, :n].float())
            ks = torch.empty((50, 2, 128), dtype=torch.bfloat16, device="cuda")
            vs = torch.empty_like(ks)
            f.pool.gather_suffix(layer, f.seqs[b], 50, ekv.GATHER_NATIVE, ks, vs)
            torch.cuda.synchronize()
            assert torch.equal(ks.cpu().view(torch.int16), f.sk[layer][b, :50].view(torch.int16))
            assert torch.equal(vs.cpu().view(torch.int16), f.sv[layer][b, :50].view(torch.int16))
    assert f.pool.status() == 0


@pytest.mark.parametrize("D", [64, 256])
def test_append_gather_q8_0_bit_exact(D):
    f = Filled(dtype=ekv.DTYPE_Q8_0, B=3, prefix_lens=[16, 45, 101], Hkv=1, D=D, block_tokens=16, seed=2)
    for b in range(3):
        n = f.prefix_lens[b]
        k, v = gather_prefix(f, 0, b, ekv.GATHER_NATIVE)
        want_k = oracle.quantize_q8_0(to_f32_np(f.pk[0][b, :n]).reshape(n, 1, D))
        want_v = oracle.quantize_q8_0(to_f32_np(f.pv[0][b, :n]).reshape(n, 1, D))
        np.testing.assert_array_equal(k.numpy(), want_k)
        np.testing.assert_array_equal(v.numpy(), want_v)
        kf, _ = gather_prefix(f, 0, b, ekv.GATHER_F32)
        np.testing.assert_array_equal(kf.numpy().view(np.uint32),
                                      oracle.dequantize_q8_0(want_k).view(np.uint32))
    assert f.pool.status() == 0


def test_q8_0_append_edge_values():
    """Zero groups, exact .5 ties after scaling, tiny (fp16-subnormal) scales, large values."""
    g = np.load(__file__.replace("test_gpu_parity.py", "golden/q8_0_gguf.npz"))
    x = g["x"]  # [n_groups][32] f32, bf16-representable or not: round to bf16 first
    xb = torch.from_numpy(x).to(torch.bfloat16)
    n_rows = xb.shape[0] // 8
    D = 256
    rows = xb[: n_rows * 8].reshape(n_rows, 1, D)
    pool = ekv.Pool(device=0, dtype=ekv.DTYPE_Q8_0, block_tokens=16, n_blocks=8, kv_heads=1, head_dim=D,
                    n_layers=1, max_seqs=1, max_blocks_per_seq=8)
    s = pool.seq_create()
    pool.seq_resize(s, n_rows)
    pool.sync()
    dev = lambda a: torch.tensor(a, dtype=torch.int32, device="cuda")
    kd = rows.contiguous().cuda()
    pool.append(0, dev([s]), dev([0]), dev([n_rows]), dev([0]), n_rows, kd, kd)
    k = torch.empty((n_rows, 1, D // 32 * 34), dtype=torch.uint8, device="cuda")
    v = torch.empty_like(k)
    pool.gather(0, s, 0, n_rows, ekv.GATHER_NATIVE, k, v)
    torch.cuda.synchronize()
    want = oracle.quantize_q8_0(rows.float().numpy())
    np.testing.assert_array_equal(k.cpu().numpy(), want)


def test_evict_front_and_block_reuse():
    f = Filled(dtype=ekv.DTYPE_BF16, B=1, prefix_lens=[64 * 5], Hkv=1, D=128, block_tokens=64, seed=3,
               shuffle=False)
    before = f.pool.seq_get(f.seqs[0]).blocks
    f.pool.seq_evict_front(f.seqs[0], 2)
    after = f.pool.seq_get(f.seqs[0])
    assert after.blocks == before[2:] and after.n_tokens == 64 * 3
    f.pool.sync()
    k = torch.empty((64 * 3, 1, 128), dtype=torch.bfloat16, device="cuda")
    v = torch.empty_like(k)
    f.pool.gather(0, f.seqs[0], 0, 64 * 3, ekv.GATHER_NATIVE, k, v)
    torch.cuda.synchronize()
    assert torch.equal(k.cpu().view(torch.int16), f.pk[0][0, 128:].view(torch.int16))
    # the evicted blocks are handed out first to the next growth (lowest index first)
    f.pool.seq_resize(f.seqs[0], 64 * 4)
    assert f.pool.seq_get(f.seqs[0]).blocks[-1] == min(before[:2])
    assert f.pool.status() == 0


def run_attention(f, layer, q, *, Hq, scale, algo, out_dtype=ekv.DTYPE_F32, mask_flags=0, use_prefix=True,
                  prefix_valid=None, span=None, block=None, workspace=False):
    B, Tq = q.shape[0], q.shape[1]
    dev = lambda a: None if a is None else torch.tensor(a, dtype=torch.int32, device="cuda")
    kw = {}
    if block:
        kw = dict(chunk_tokens=block[0], chunk_stride=block[1], window_chunks=block[2], q_chunk0=block[3])
    prm = f.pool.attention_params(layer=layer, seq_ids=f.seq_ids, q_tokens=Tq, q_heads=Hq, scale=scale,
                                  mask_flags=mask_flags, suffix_len=f.suffix_len, out_dtype=out_dtype,
                                  use_prefix=use_prefix, prefix_valid=dev(prefix_valid),
                                  span_begin=dev(None if span is None else span[0]),
                                  span_end=dev(None if span is None else span[1]), **kw)
    out = torch.full(q.shape, float("nan"), dtype=torch.float32 if out_dtype == ekv.DTYPE_F32 else torch.bfloat16,
                     device="cuda")
    ws = None
    if workspace:
        n = f.pool.workspace_size(prm)
        ws = torch.empty(max(n, 4), dtype=torch.uint8, device="cuda") if n else None
    f.pool.attention(prm, q.cuda().contiguous(), out, workspace=ws, algo=algo)
    torch.cuda.synchronize()
    assert f.pool.status() == 0
    return out.float().cpu().numpy()


def oracle_attention(f, layer, q, *, scale, mask_flags=0, use_prefix=True, prefix_valid=None, span=None,
                     block=None):
    k, v = f.oracle_kv(layer)
    B = f.B
    n_prefix = f.prefix_lens if use_prefix else [0] * B
    if not use_prefix:
        Ls = f.suffix_len
        k2 = np.zeros((B, Ls, f.Hkv, f.D), np.float32)
        v2 = np.zeros_like(k2)
        for b in range(B):
            k2[b] = k[b, f.prefix_lens[b]:f.prefix_lens[b] + Ls]
            v2[b] = v[b, f.prefix_lens[b]:f.prefix_lens[b] + Ls]
        k, v = k2, v2
    seqs = oracle.make_seqs(n_prefix, prefix_valid=prefix_valid if prefix_valid is not None else n_prefix,
                            span=span, n_suffix=f.suffix_len)
    m = oracle.make_mask(mask_flags, *(block or (0, 0, 0, 0)))
    return oracle.attention(to_f32_np(q), k, v, seqs, m, scale)


def check(got, want, tol):
    assert np.isfinite(got).all()
    err = np.abs(got - want).max()
    assert err <= tol, f"max-abs {err} > {tol}"
    return err


@pytest.mark.parametrize("algo", ALGOS)
@pytest.mark.parametrize("dtype", [ekv.DTYPE_BF16, ekv.DTYPE_Q8_0])
def test_attention_pi05_shape(algo, dtype):
    """pi0.5: 8 query heads, 1 KV head, D=256, prefix with padded text tail, 50 suffix tokens
    attending bidirectionally (models/pi05.cpp:406-421, mask all zero :880-882; padding as
    models/smolvla.cpp:707-716)."""
    gen = torch.Generator().manual_seed(5)
    plens = [816, 700, 777]
    valid = [768 + 20, 700, 768 - 5]
    f = Filled(dtype=dtype, B=3, prefix_lens=plens, Hkv=1, D=256, suffix_len=50, seed=5)
    q = bf16_randn(gen, (3, 50, 8, 256))
    got = run_attention(f, 0, q, Hq=8, scale=1 / 16, algo=algo, prefix_valid=valid)
    want = oracle_attention(f, 0, q, scale=1 / 16, prefix_valid=valid)
    check(got, want, TOL[dtype])


@pytest.mark.parametrize("algo", ALGOS)
@pytest.mark.parametrize("flag", [ekv.MASK_SUFFIX_CAUSAL, ekv.MASK_SUFFIX_PREFIX_LM])
def test_attention_suffix_masks(algo, flag):
    """SmolVLA causal suffix (models/smolvla.cpp:718-720), HY-VLA prefix-LM row 0
    (models/hy_vla.cpp:2355-2367); GQA with 2 KV heads."""
    gen = torch.Generator().manual_seed(6)
    f = Filled(dtype=ekv.DTYPE_BF16, B=2, prefix_lens=[90, 141], Hkv=2, D=64, suffix_len=37, seed=6)
    q = bf16_randn(gen, (2, 37, 6, 64))
    got = run_attention(f, 0, q, Hq=6, scale=0.125, algo=algo, mask_flags=flag, prefix_valid=[80, 141])
    want = oracle_attention(f, 0, q, scale=0.125, mask_flags=flag, prefix_valid=[80, 141])
    check(got, want, 2e-2)


@pytest.mark.parametrize("algo", ALGOS)
@pytest.mark.parametrize("flag", [ekv.MASK_SPAN_EXCLUDE, ekv.MASK_SPAN_ONLY])
def test_attention_groot_cross_and_self(algo, flag):
    """GR00T DiT: 32 heads x 48 (MHA), 17 queries over a cached 300-token backbone with text
    (outside the image span) / image (inside) masks (models/groot_n1.cpp:708-718); then the
    self-attention layer over the 17 suffix tokens only."""
    gen = torch.Generator().manual_seed(7)
    f = Filled(dtype=ekv.DTYPE_BF16, B=3, prefix_lens=[300, 300, 300], Hkv=32, D=48, suffix_len=17, seed=7,
               block_tokens=16)
    q = bf16_randn(gen, (3, 17, 32, 48))
    span = ([20, 30, 0], [276, 286, 256])
    valid = [300, 290, 280]
    scale = 1 / np.sqrt(48)
    f.suffix_len_saved = f.suffix_len
    # cross layer: prefix only
    f.suffix_len = 0
    got = run_attention(f, 0, q, Hq=32, scale=scale, algo=algo, mask_flags=flag, prefix_valid=valid, span=span)
    want = oracle_attention(f, 0, q, scale=scale, mask_flags=flag, prefix_valid=valid, span=span)
    check(got, want, 2e-2)
    # self layer: suffix only
    f.suffix_len = 17
    got = run_attention(f, 0, q, Hq=32, scale=scale, algo=algo, use_prefix=False)
    want = oracle_attention(f, 0, q, scale=scale, use_prefix=False)
    check(got, want, 2e-2)


@pytest.mark.parametrize("algo", ALGOS)
def test_attention_lingbot_block_causal(algo):
    """LingBot-shaped block-causal window over a paged bf16 cache with 64-token blocks: chunks of
    100 valid tokens padded to 128 key slots, window of 2 chunks, queries = the newest chunk;
    12 heads x 128 (MHA)."""
    gen = torch.Generator().manual_seed(8)
    n_chunks, ct, stride = 3, 100, 128
    f = Filled(dtype=ekv.DTYPE_BF16, B=2, prefix_lens=[n_chunks * stride] * 2, Hkv=4, D=128, block_tokens=64,
               seed=8)
    q = bf16_randn(gen, (2, ct, 4, 128))
    block = (ct, stride, 2, n_chunks - 1)
    got = run_attention(f, 0, q, Hq=4, scale=1 / np.sqrt(128), algo=algo, mask_flags=ekv.MASK_BLOCK_CAUSAL,
                        block=block)
    want = oracle_attention(f, 0, q, scale=1 / np.sqrt(128), mask_flags=ekv.MASK_BLOCK_CAUSAL, block=block)
    check(got, want, 2e-2)


@pytest.mark.parametrize("dtype", [ekv.DTYPE_BF16, ekv.DTYPE_Q8_0])
def test_attention_split_keys_matches_unsplit(dtype):
    """Key splitting across CTAs (workspace given) agrees with the single-pass kernel and the
    oracle; long prefixes, few query tiles so the splitter engages."""
    gen = torch.Generator().manual_seed(9)
    f = Filled(dtype=dtype, B=2, prefix_lens=[2000, 1500], Hkv=1, D=128, suffix_len=10, seed=9)
    q = bf16_randn(gen, (2, 10, 8, 128))
    a = run_attention(f, 0, q, Hq=8, scale=1 / np.sqrt(128), algo=ekv.ALGO_TC)
    b = run_attention(f, 0, q, Hq=8, scale=1 / np.sqrt(128), algo=ekv.ALGO_TC, workspace=True)
    want = oracle_attention(f, 0, q, scale=1 / np.sqrt(128))
    check(a, want, TOL[dtype])
    check(b, want, TOL[dtype])


@pytest.mark.parametrize("out_dtype", [ekv.DTYPE_F32, ekv.DTYPE_BF16])
@pytest.mark.parametrize("Hq,Hkv,Tq", [(16, 1, 9), (32, 2, 5), (64, 1, 3), (128, 1, 3), (2, 1, 70), (12, 4, 11)])
def test_attention_output_row_boxes(out_dtype, Hq, Hkv, Tq):
    """The tensor-core epilogue stores 32 query rows at a time: min(group, 32) heads x
    max(1, 32 / group) tokens. Groups from 2 to 128 (both box shapes), row counts that end inside a
    32-row quarter and inside a 128-row tile, and a group of 3 that keeps the thread-store epilogue.
    The output starts as NaN, so an unwritten row fails the finiteness check."""
    gen = torch.Generator().manual_seed(12)
    f = Filled(dtype=ekv.DTYPE_BF16, B=2, prefix_lens=[150, 77], Hkv=Hkv, D=64, suffix_len=Tq, seed=12)
    q = bf16_randn(gen, (2, Tq, Hq, 64))
    want = oracle_attention(f, 0, q, scale=0.125)
    got = run_attention(f, 0, q, Hq=Hq, scale=0.125, algo=ekv.ALGO_TC, out_dtype=out_dtype)
    check(got, want, 2e-2)
    got = run_attention(f, 0, q, Hq=Hq, scale=0.125, algo=ekv.ALGO_TC, out_dtype=out_dtype, workspace=True)
    check(got, want, 2e-2)


def test_attention_bf16_output_and_fully_masked_rows():
    """bf16 output; a request whose every key is masked returns zeros
    (models/lingbot_va.cpp:9503-9506)."""
    gen = torch.Generator().manual_seed(10)
    f = Filled(dtype=ekv.DTYPE_BF16, B=2, prefix_lens=[64, 64], Hkv=1, D=256, seed=10)
    q = bf16_randn(gen, (2, 4, 8, 256))
    for algo in ALGOS:
        got = run_attention(f, 0, q, Hq=8, scale=1 / 16, algo=algo, out_dtype=ekv.DTYPE_BF16, prefix_valid=[64, 0])
        want = oracle_attention(f, 0, q, scale=1 / 16, prefix_valid=[64, 0])
        check(got, want, 2e-2)
        assert (got[1] == 0).all()


def _cudart():
    import ctypes as C
    import glob
    import os
    import nvidia.cuda_runtime
    lib = glob.glob(os.path.join(os.path.dirname(nvidia.cuda_runtime.__file__), "lib", "libcudart.so*"))[0]
    rt = C.CDLL(lib)
    rt.cudaMemcpy.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
    return rt


def test_kernel_reports_bad_block_table():
    """A corrupted device block table is caught by the kernels' bounds checks and reported in the
    status word instead of being dereferenced."""
    import ctypes as C
    f = Filled(dtype=ekv.DTYPE_BF16, B=1, prefix_lens=[128], Hkv=1, D=128, seed=11)
    info = f.pool.info()
    bad = C.c_int32(10 ** 6)
    entry = info.block_tables + 4 * (f.seqs[0] * f.pool.cfg.max_blocks_per_seq + 1)
    torch.cuda.synchronize()
    assert _cudart().cudaMemcpy(entry, C.addressof(bad), 4, 1) == 0  # host -> device
    k = torch.empty((128, 1, 128), dtype=torch.bfloat16, device="cuda")
    v = torch.empty_like(k)
    f.pool.gather(0, f.seqs[0], 0, 128, ekv.GATHER_NATIVE, k, v)
    torch.cuda.synchronize()
    assert f.pool.status() == ekv.DEV_ERR_BAD_BLOCK
    assert f.pool.status() == 0  # reading clears it
    q = bf16_randn(torch.Generator().manual_seed(1), (1, 4, 8, 128))
    for algo in ALGOS:
        prm = f.pool.attention_params(layer=0, seq_ids=f.seq_ids, q_tokens=4, q_heads=8, scale=0.1,
                                      out_dtype=ekv.DTYPE_F32)
        out = torch.empty((1, 4, 8, 128), dtype=torch.float32, device="cuda")
        f.pool.attention(prm, q.cuda(), out, algo=algo)
        torch.cuda.synchronize()
        assert f.pool.status() == ekv.DEV_ERR_BAD_BLOCK


@pytest.mark.parametrize("D,Hq,Hkv,T,B", [(48, 32, 32, 17, 6), (64, 16, 8, 17, 24), (128, 8, 8, 9, 30)])
@pytest.mark.parametrize("flag", [0, ekv.MASK_SPAN_EXCLUDE, ekv.MASK_SPAN_ONLY])
def test_attention_packed_units(D, Hq, Hkv, T, B, flag):
    """More (request, KV head) units of at most 64 query rows than SMs (GR00T's 17 queries x 32
    heads at batch 6 and up): the one-CTA kernel packs several units into one CTA's 128 rows, each
    row seeing only its unit's keys. Ragged prefixes, padding, spans, GQA, bf16 and f32 output, and
    the suffix-only self layer."""
    gen = torch.Generator().manual_seed(D + B)
    rng = np.random.default_rng(D + B)
    plens = [int(x) for x in rng.integers(1, 400, size=B)]
    f = Filled(dtype=ekv.DTYPE_BF16, B=B, prefix_lens=plens, Hkv=Hkv, D=D, suffix_len=T, seed=D + B,
               block_tokens=16)
    q = bf16_randn(gen, (B, T, Hq, D))
    valid = [max(1, p - int(rng.integers(0, 20))) for p in plens]
    span = ([int(rng.integers(0, v)) for v in valid], [v for v in valid])
    scale = 1 / np.sqrt(D)
    f.suffix_len = 0
    kw = dict(mask_flags=flag, prefix_valid=valid)
    if flag:
        kw["span"] = span
    got = run_attention(f, 0, q, Hq=Hq, scale=scale, algo=ekv.ALGO_TC, **kw)
    want = oracle_attention(f, 0, q, scale=scale, **kw)
    check(got, want, 2e-2)
    f.suffix_len = T
    got = run_attention(f, 0, q, Hq=Hq, scale=scale, algo=ekv.ALGO_TC, use_prefix=False)
    want = oracle_attention(f, 0, q, scale=scale, use_prefix=False)
    check(got, want, 2e-2)
    got = run_attention(f, 0, q, Hq=Hq, scale=scale, algo=ekv.ALGO_TC, out_dtype=ekv.DTYPE_BF16)
    want = oracle_attention(f, 0, q, scale=scale)
    check(got, want, 2e-2)


def test_q8_0_attention_against_ggml_q8_0_path():
    """The tcgen05 Q8_0 path against the emulated ggml CPU Q8_0 path (queries and suffix keys
    quantised for the dot products as ggml's Q8_0 mul_mat does) within the Q8_0 tolerance."""
    gen = torch.Generator().manual_seed(12)
    plens = [300, 517]
    f = Filled(dtype=ekv.DTYPE_Q8_0, B=2, prefix_lens=plens, Hkv=1, D=256, suffix_len=50, seed=12)
    q = bf16_randn(gen, (2, 50, 8, 256))
    got = run_attention(f, 0, q, Hq=8, scale=1 / 16, algo=ekv.ALGO_TC)
    for b, n in enumerate(plens):
        k = np.concatenate([to_f32_np(f.pk[0][b, :n]), to_f32_np(f.sk[0][b, :50])])[None]
        v = np.concatenate([to_f32_np(f.pv[0][b, :n]), to_f32_np(f.sv[0][b, :50])])[None]
        want = oracle.attention_ggml_q8_0(to_f32_np(q[b:b + 1]), k, v, n, 1 / 16)
        check(got[b:b + 1], want, TOL[ekv.DTYPE_Q8_0])


@pytest.mark.parametrize("algo,D", [(ekv.ALGO_TC, 256), (ekv.ALGO_TC_PAIR, 256), (ekv.ALGO_TC_CTA, 256),
                                    (ekv.ALGO_TC, 128)])
@pytest.mark.parametrize("where", ["q", "suffix"])
def test_q8_0_f16_range_is_reported(algo, D, where):
    """Q8_0 pools multiply in f16: a bf16 query or suffix value beyond the f16 range (65504) would become
    inf there. Every tcgen05 kernel records DEV_ERR_F16_RANGE in the status word instead of returning
    silently wrong rows; values inside the range leave the status clear."""
    gen = torch.Generator().manual_seed(31)
    f = Filled(dtype=ekv.DTYPE_Q8_0, B=2, prefix_lens=[90, 130], Hkv=1, D=D, suffix_len=20, seed=31)
    q = bf16_randn(gen, (2, 20, 8, D))
    run_attention(f, 0, q, Hq=8, scale=D ** -0.5, algo=algo)  # in range: status clear (checked inside)
    if where == "q":
        q[1, 3, 2, 7] = 1.0e5
    else:
        big = f.sk[0].clone()
        big[0, 5, 0, 11] = -2.0e5
        f.pool.append_suffix(0, f.seq_ids, big[:, :20].contiguous().cuda(), f.sv[0][:, :20].contiguous().cuda())
    prm = f.pool.attention_params(layer=0, seq_ids=f.seq_ids, q_tokens=20, q_heads=8, scale=D ** -0.5,
                                  suffix_len=20, out_dtype=ekv.DTYPE_F32)
    out = torch.empty((2, 20, 8, D), dtype=torch.float32, device="cuda")
    f.pool.attention(prm, q.cuda().contiguous(), out, algo=algo)
    torch.cuda.synchronize()
    assert f.pool.status() == ekv.DEV_ERR_F16_RANGE
