"""ekv_flash_attn_ext: GGML_OP_FLASH_ATTN_EXT on ggml-strided device tensors.

CPU: the float64 oracle is pinned to the LingBot known-answer vectors and to the pinned
attention oracle; the C-ABI rejects malformed tensors before any CUDA call (no kernel runs).
GPU: parity with the oracle on the reference's call shapes (models/hy_vla.cpp:376-378 permuted
self-attention, :439-441 time attention under hy_mem_causal_mask, :859 GQA with a mask;
models/lingbot_va.cpp:1263-1266), plus softcap, ALiBi, f16/bf16 inputs, batch broadcast, the
largest head dims, fully masked rows and strided outputs. Calls the tcgen05 kernels take (head_dim
64/128/256, no softcap or ALiBi, a head-shared mask) run there on bf16 operands: max-abs 2e-2, the
bf16 tolerance of the attention path; the rest run on the CUDA cores in f32: max-abs 2e-4 against
float64 (inputs are rounded to their storage type before the oracle sees them).
"""
import ctypes as C
import os

import numpy as np
import pytest

import ekv
import oracle

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TOL = 2e-4     # CUDA-core route, f32
TOL_TC = 2e-2  # tensor-core route, bf16 operands, f32 accumulation


# ---------------------------------------------------------------- oracle pins (CPU)

def test_oracle_matches_lingbot_known_answer():
    g = np.load(os.path.join(GOLD, "lingbot_smoke.npz"))
    S, H, D = g["q"].shape
    dense = np.where(g["mask"].astype(bool), 0.0, -np.inf)[None, None]
    t = lambda a: np.transpose(a, (1, 0, 2))[None]  # [S, H, D] -> [1, H, S, D]
    out = oracle.flash_attn_ext(t(g["q"]), t(g["k"]), t(g["v"]), dense, scale=float(g["scale"]))
    assert np.abs(out[0] - g["ref"]).max() < 1e-12


def test_oracle_matches_attention_oracle_gqa_mask():
    rng = np.random.default_rng(3)
    B, Tq, Hq, Hkv, D, Lk = 2, 6, 4, 2, 32, 23
    q, k, v = (rng.standard_normal(sh).astype(np.float32) for sh in
               ((B, Tq, Hq, D), (B, Lk, Hkv, D), (B, Lk, Hkv, D)))
    dense = np.where(rng.random((B, Tq, Lk)) < 0.3, -np.inf, 0.0)
    dense[:, :, 0] = 0.0
    seqs = oracle.make_seqs([Lk] * B, n_suffix=0)
    want = oracle.attention(q, k, v, seqs, oracle.make_mask(), 0.25, dense_mask=dense, precision="f64")
    got = oracle.flash_attn_ext(q.transpose(0, 2, 1, 3), k.transpose(0, 2, 1, 3), v.transpose(0, 2, 1, 3),
                                dense[:, None], scale=0.25)
    assert np.abs(got - want).max() < 1e-12


def test_oracle_alibi_and_softcap_rules():
    s = oracle.alibi_slopes(12, 8.0)
    np.testing.assert_allclose(s[[0, 7, 8, 11]], [0.5, 2.0 ** -8, 2.0 ** -0.5, 2.0 ** -3.5], rtol=1e-14)
    assert np.all(oracle.alibi_slopes(5, 0.0) == 1.0)
    rng = np.random.default_rng(4)
    q, k, v = (rng.standard_normal((1, 1, 3, 8)) for _ in range(3))
    got = oracle.flash_attn_ext(q, k, v, scale=0.7, logit_softcap=2.0)
    s = 2.0 * np.tanh(0.7 / 2.0 * (q[0, 0] @ k[0, 0].T))
    p = np.exp(s - s.max(1, keepdims=True))
    assert np.abs(got[0, :, 0] - (p / p.sum(1, keepdims=True)) @ v[0, 0]).max() < 1e-12


# ---------------------------------------------------------------- C-ABI validation (CPU)

def fake(ne, type=ekv.DTYPE_F32, nb=None, data=1 << 20):
    es = 4 if type == ekv.DTYPE_F32 else 2
    if nb is None:
        nb = [es]
        for i in range(3):
            nb.append(nb[-1] * ne[i])
    t = ekv.Tensor()
    t.data, t.type = data, type
    for i in range(4):
        t.ne[i], t.nb[i] = ne[i], nb[i]
    return t


def call(q, k, v, m, dst, scale=0.125, max_bias=0.0, softcap=0.0):
    r = lambda t: None if t is None else C.byref(t)
    return ekv.lib.ekv_flash_attn_ext(r(q), r(k), r(v), r(m), scale, max_bias, softcap, r(dst), None)


def good():
    return dict(q=fake([64, 5, 8, 2]), k=fake([64, 9, 2, 1]), v=fake([32, 9, 2, 1]),
                m=fake([16, 8, 1, 1], ekv.DTYPE_F16), dst=fake([32, 8, 5, 2]))


@pytest.mark.parametrize("name,patch,code", [
    ("k head dim", dict(k=fake([48, 9, 2, 1])), ekv.ERR_INVALID_ARG),
    ("v length", dict(v=fake([32, 8, 2, 1])), ekv.ERR_INVALID_ARG),
    ("gqa ratio", dict(k=fake([64, 9, 3, 1]), v=fake([32, 9, 3, 1])), ekv.ERR_INVALID_ARG),
    ("batch ratio", dict(q=fake([64, 5, 8, 3]), dst=fake([32, 8, 5, 3]), k=fake([64, 9, 2, 2]),
                         v=fake([32, 9, 2, 2])), ekv.ERR_INVALID_ARG),
    ("dst shape", dict(dst=fake([32, 5, 8, 2])), ekv.ERR_INVALID_ARG),
    ("dst type", dict(dst=fake([32, 8, 5, 2], ekv.DTYPE_F16)), ekv.ERR_INVALID_ARG),
    ("mask short", dict(m=fake([8, 8, 1, 1], ekv.DTYPE_F16)), ekv.ERR_INVALID_ARG),
    ("mask rows", dict(m=fake([16, 4, 1, 1], ekv.DTYPE_F16)), ekv.ERR_INVALID_ARG),
    ("mask heads", dict(m=fake([16, 8, 3, 1], ekv.DTYPE_F16)), ekv.ERR_INVALID_ARG),
    ("mask bf16", dict(m=fake([16, 8, 1, 1], ekv.DTYPE_BF16)), ekv.ERR_INVALID_ARG),
    ("q type", dict(q=fake([64, 5, 8, 2], ekv.DTYPE_Q8_0)), ekv.ERR_INVALID_ARG),
    ("odd stride", dict(q=fake([64, 5, 8, 2], nb=[4, 258, 1290, 10320])), ekv.ERR_INVALID_ARG),
    ("misaligned", dict(q=fake([64, 5, 8, 2], data=(1 << 20) + 2)), ekv.ERR_INVALID_ARG),
    ("null data", dict(k=fake([64, 9, 2, 1], data=0)), ekv.ERR_INVALID_ARG),
    ("null dst", dict(dst=None), ekv.ERR_INVALID_ARG),
    ("empty", dict(q=fake([64, 0, 8, 2])), ekv.ERR_INVALID_ARG),
    ("D too large", dict(q=fake([640, 5, 8, 2]), k=fake([640, 9, 2, 1])), ekv.ERR_UNSUPPORTED),
    ("Dv too large", dict(v=fake([320, 9, 2, 1]), dst=fake([320, 8, 5, 2])), ekv.ERR_UNSUPPORTED),
])
def test_capi_rejects(name, patch, code):
    a = good()
    a.update(patch)
    assert call(a["q"], a["k"], a["v"], a["m"], a["dst"]) == code, name


def test_capi_rejects_scalars():
    a = good()
    args = (a["q"], a["k"], a["v"], a["m"], a["dst"])
    assert call(*args, scale=float("nan")) == ekv.ERR_INVALID_ARG
    assert call(*args, max_bias=-1.0) == ekv.ERR_INVALID_ARG
    assert call(*args, softcap=float("inf")) == ekv.ERR_INVALID_ARG
    assert call(a["q"], a["k"], a["v"], None, a["dst"], max_bias=8.0) == ekv.ERR_INVALID_ARG


# ---------------------------------------------------------------- GPU parity

def _np(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


TOL_OF = {}


def run(q, k, v, mask, *, scale, max_bias=0.0, softcap=0.0, dst=None):
    """One call; also records in TOL_OF[id(dst)] the tolerance of the route it took (the tensor-core
    route launches the staging kernels and the attention, the CUDA-core route one kernel)."""
    import torch
    B, Hq, Tq, _ = q.shape
    Dv = v.shape[3]
    if dst is None:
        dst = torch.full((B, Tq, Hq, Dv), float("nan"), dtype=torch.float32, device="cuda")
    tc = ekv.flash_attn_ext_workspace_size(q, k, v, mask, dst, max_bias=max_bias, logit_softcap=softcap) > 0
    n0 = ekv.lib.ekv_launch_count()
    ekv.flash_attn_ext(q, k, v, mask, dst, scale=scale, max_bias=max_bias, logit_softcap=softcap)
    torch.cuda.synchronize()
    launched = ekv.lib.ekv_launch_count() - n0
    assert (launched >= 4) == tc, (launched, tc)
    want = oracle.flash_attn_ext(_np(q), _np(k), _np(v), None if mask is None else _np(mask),
                                 scale=scale, max_bias=max_bias, logit_softcap=softcap)
    TOL_OF[id(dst)] = TOL_TC if tc else TOL
    return dst, want


def tol(dst):
    return TOL_OF[id(dst)]


def causal_f16(n, device):
    import torch
    r = torch.arange(n, device=device)
    return torch.where(r[None, :] <= r[:, None], 0.0, float("-inf")).to(torch.float16)


@pytest.mark.gpu
def test_hy_self_attention_permuted_views():
    """models/hy_vla.cpp:365-378: q/k/v are column slices of one fused qkv row-major buffer,
    reshaped to heads and permuted, so every operand is non-contiguous."""
    import torch
    torch.manual_seed(0)
    seq, H, D = 77, 6, 64
    qkv = torch.randn(seq, 3 * H * D, device="cuda")
    views = [qkv[:, i * H * D:(i + 1) * H * D].view(seq, H, D).permute(1, 0, 2)[None] for i in range(3)]
    dst, want = run(*views, None, scale=D ** -0.5)
    assert np.abs(_np(dst) - want).max() < tol(dst)


@pytest.mark.gpu
@pytest.mark.parametrize("frames", [1, 3, 9])
def test_hy_time_attention_causal_mask(frames):
    """models/hy_vla.cpp:430-441: patches batched in ne[3], a [T, T] F16 causal mask
    (hy_mem_causal_mask) broadcast over heads and patches."""
    import torch
    torch.manual_seed(frames)
    P, H, D = 20, 4, 64
    q4, k4, v4 = (torch.randn(frames, P, H, D, device="cuda") for _ in range(3))
    Q, K, V = (t.permute(1, 2, 0, 3) for t in (q4, k4, v4))  # [P, H, T, D] views
    mask = causal_f16(frames, "cuda")[None, None]
    dst, want = run(Q, K, V, mask, scale=D ** -0.5)
    assert np.abs(_np(dst) - want).max() < tol(dst)


@pytest.mark.gpu
@pytest.mark.parametrize("hq,hkv", [(8, 1), (8, 2), (16, 16)])
def test_hy_expert_gqa_mask(hq, hkv):
    """models/hy_vla.cpp:845-859: GQA heads with an additive F16 mask over the suffix."""
    import torch
    torch.manual_seed(hq + hkv)
    seq, D = 51, 128
    q = torch.randn(seq, hq, D, device="cuda").permute(1, 0, 2)[None]
    k = torch.randn(seq, hkv, D, device="cuda").permute(1, 0, 2)[None]
    v = torch.randn(seq, hkv, D, device="cuda").permute(1, 0, 2)[None]
    pad = 64  # ggml pads the mask's rows and columns; extra entries are ignored
    m = torch.zeros(pad, pad, device="cuda")
    m[:seq, :seq] = torch.where(torch.rand(seq, seq, device="cuda") < 0.25, float("-inf"), 0.0)
    m[:, 0] = 0.0
    mask = m.to(torch.float16)[None, None]
    dst, want = run(q, k, v, mask, scale=D ** -0.5)
    assert np.abs(_np(dst) - want).max() < tol(dst)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_half_inputs_and_f32_mask_per_head(dtype):
    import torch
    torch.manual_seed(7)
    dt = torch.float16 if dtype == "f16" else torch.bfloat16
    B, Hq, Hkv, Tq, Tk, D = 2, 4, 2, 33, 70, 96
    q = torch.randn(B, Hq, Tq, D, device="cuda").to(dt)
    k = torch.randn(B, Hkv, Tk, D, device="cuda").to(dt)
    v = torch.randn(B, Hkv, Tk, D, device="cuda").to(dt)
    mask = torch.randn(B, Hq, Tq, Tk, device="cuda")
    mask[..., 5:9] = float("-inf")
    dst, want = run(q, k, v, mask, scale=0.1)
    assert np.abs(_np(dst) - want).max() < tol(dst)


@pytest.mark.gpu
def test_softcap_alibi_and_batch_broadcast():
    import torch
    torch.manual_seed(11)
    B, Bk, Hq, Hkv, Tq, Tk, D = 4, 2, 12, 3, 17, 45, 64
    q = torch.randn(B, Hq, Tq, D, device="cuda")
    k = torch.randn(Bk, Hkv, Tk, D, device="cuda")
    v = torch.randn(Bk, Hkv, Tk, D, device="cuda")
    mask = (-torch.arange(Tk, device="cuda").float().abs()).expand(1, 1, Tq, Tk).contiguous()
    dst, want = run(q, k, v, mask, scale=0.125, max_bias=8.0, softcap=20.0)
    assert np.abs(_np(dst) - want).max() < tol(dst)
    dst, want = run(q, k, v, None, scale=0.125, softcap=5.0)
    assert np.abs(_np(dst) - want).max() < tol(dst)


@pytest.mark.gpu
@pytest.mark.parametrize("d,dv,tk", [(512, 256, 33), (256, 256, 1), (40, 24, 31), (64, 128, 300)])
def test_head_dims_and_key_counts(d, dv, tk):
    import torch
    torch.manual_seed(d + dv + tk)
    q = torch.randn(1, 2, 9, d, device="cuda") * 0.2
    k = torch.randn(1, 2, tk, d, device="cuda") * 0.2
    v = torch.randn(1, 2, tk, dv, device="cuda")
    dst, want = run(q, k, v, None, scale=1.0)
    assert np.abs(_np(dst) - want).max() < tol(dst)


@pytest.mark.gpu
def test_fully_masked_rows_and_strided_dst():
    """Rows whose every key is -inf give 0 (the op's S == 0 rule); dst may be a strided view
    inside a larger buffer, and nothing outside it is written."""
    import torch
    torch.manual_seed(5)
    B, H, Tq, Tk, D = 1, 2, 8, 40, 64
    q, k, v = (torch.randn(B, H, n, D, device="cuda") for n in (Tq, Tk, Tk))
    mask = torch.zeros(1, 1, Tq, Tk, device="cuda", dtype=torch.float16)
    mask[0, 0, 3] = float("-inf")
    mask[0, 0, 6, :35] = float("-inf")
    big = torch.full((B, Tq, H + 1, D + 16), 7.0, device="cuda")
    dst = big[:, :, 1:, 8:8 + D]
    dst, want = run(q, k, v, mask, scale=0.125, dst=dst)
    got = _np(dst)
    assert np.all(got[:, 3] == 0.0)
    assert np.abs(got - want).max() < tol(dst)
    rest = big.clone()
    rest[:, :, 1:, 8:8 + D] = 7.0
    assert torch.all(rest == 7.0)


@pytest.mark.gpu
def test_lingbot_known_answer_on_gpu():
    """models/lingbot_va.cpp:1263-1266 shapes from the LingBot smoke vectors, through the op."""
    import torch
    g = np.load(os.path.join(GOLD, "lingbot_smoke.npz"))
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda().permute(1, 0, 2)[None]
    mask = torch.from_numpy(np.where(g["mask"].astype(bool), 0.0, -np.inf).astype(np.float16)).cuda()[None, None]
    S, H, D = g["q"].shape
    dst = torch.empty(1, S, H, D, device="cuda")
    ekv.flash_attn_ext(t(g["q"]), t(g["k"]), t(g["v"]), mask, dst, scale=float(g["scale"]))
    torch.cuda.synchronize()
    assert np.abs(dst[0].cpu().numpy() - g["ref"]).max() < float(g["tol"])


# ---------------------------------------------------------------- the mul_mat / soft_max_ext / mul_mat triple

def call_triple(k, q, v, m, dst, scale=0.0625, max_bias=0.0):
    r = lambda t: None if t is None else C.byref(t)
    return ekv.lib.ekv_mul_mat_soft_max_mul_mat(r(k), r(q), r(v), r(m), scale, max_bias, r(dst), None)


def good_triple():
    # pi0.5 shapes (models/pi05.cpp:410-418): K {256, 866, 1}, Q {256, 50, 8}, V {866, 256, 1}
    return dict(k=fake([256, 866, 1, 1]), q=fake([256, 50, 8, 1]), v=fake([866, 256, 1, 1]),
                m=fake([866, 50, 1, 1]), dst=fake([256, 50, 8, 1]))


@pytest.mark.parametrize("name,patch", [
    ("v keys", dict(v=fake([865, 256, 1, 1]))),
    ("v heads", dict(v=fake([866, 256, 2, 1]))),
    ("dst order", dict(dst=fake([256, 8, 50, 1]))),
    ("dst dv", dict(dst=fake([128, 50, 8, 1]))),
    ("k dim", dict(k=fake([128, 866, 1, 1]))),
    ("mask short", dict(m=fake([800, 50, 1, 1]))),
    ("null v", dict(v=None)),
])
def test_triple_capi_rejects(name, patch):
    a = good_triple()
    a.update(patch)
    assert call_triple(a["k"], a["q"], a["v"], a["m"], a["dst"]) == ekv.ERR_INVALID_ARG, name


@pytest.mark.gpu
@pytest.mark.parametrize("contig_v", [True, False])
@pytest.mark.parametrize("masked", [False, True])
def test_triple_pi05_layer(contig_v, masked):
    """models/pi05.cpp:404-418 on one layer-step: K/V = concat(cached prefix, 50 new rows), Q 50 x 8
    heads over 1 KV head, D = 256, scale 1/16; V keys-fastest as the permute of :412 makes it (a
    contiguous copy) or as a strided view; the f32 mask of :815 (zeros) or SmolVLA-style padding."""
    import torch
    torch.manual_seed(21 + contig_v + 2 * masked)
    Tq, Hq, D, Lp = 50, 8, 256, 816
    Tk = Lp + Tq
    kf = (torch.randn(Tk, D, device="cuda") * 0.5).to(torch.bfloat16).float()
    vf = (torch.randn(Tk, D, device="cuda") * 0.5).to(torch.bfloat16).float()
    q = (torch.randn(1, Hq, Tq, D, device="cuda") * 0.5).to(torch.bfloat16).float()
    k = kf[None, None]                                         # ggml {D, Tk, 1, 1}
    v = vf.t().contiguous()[None, None] if contig_v else vf.t()[None, None]  # ggml {Tk, D, 1, 1}
    mask = torch.zeros(1, 1, Tq, Tk, device="cuda")
    if masked:
        mask[..., 790:Lp] = float("-inf")                      # padded text positions
    dst = torch.full((1, Hq, Tq, D), float("nan"), device="cuda")
    ekv.mul_mat_soft_max_mul_mat(k, q, v, mask, dst, scale=1.0 / 16)
    torch.cuda.synchronize()
    want = oracle.flash_attn_ext(_np(q), _np(k), _np(vf)[None, None], _np(mask), scale=1.0 / 16)
    assert np.abs(_np(dst) - want.transpose(0, 2, 1, 3)).max() < TOL_TC


@pytest.mark.gpu
def test_triple_fully_masked_row_gives_zero():
    """A query row whose every key is masked: ggml's soft_max_ext would give NaN there (max -inf,
    exp(-inf - -inf)); the fused triple gives 0, as the fused flash_attn_ext op and
    dense_masked_attention_ref (models/lingbot_va.cpp:9503-9506) do. The other rows are unchanged."""
    import torch
    torch.manual_seed(33)
    Tq, Hq, D, Tk = 6, 2, 64, 40
    k = (torch.randn(1, 1, Tk, D, device="cuda") * 0.5)
    vf = (torch.randn(Tk, D, device="cuda") * 0.5)
    q = (torch.randn(1, Hq, Tq, D, device="cuda") * 0.5)
    mask = torch.zeros(1, 1, Tq, Tk, device="cuda")
    mask[..., 2, :] = float("-inf")                            # row 2 sees no key
    mask[..., 4, 10:] = float("-inf")
    dst = torch.full((1, Hq, Tq, D), float("nan"), device="cuda")
    ekv.mul_mat_soft_max_mul_mat(k, q, vf.t()[None, None], mask, dst, scale=0.125)
    torch.cuda.synchronize()
    got = _np(dst)
    assert np.all(got[:, :, 2] == 0.0)
    want = oracle.flash_attn_ext(_np(q), _np(k), _np(vf)[None, None], _np(mask), scale=0.125)
    assert np.abs(got - want.transpose(0, 2, 1, 3)).max() < TOL_TC


# ---------------------------------------------------------------- the tensor-core route

def test_workspace_size_picks_the_route():
    """Host logic only: which calls the tensor-core route takes, and that its workspace covers the
    staged K/V (two bf16 copies in 64-token blocks), Q and the mask bits."""
    def ws(q, k, v, m, dst, max_bias=0.0, softcap=0.0):
        r = lambda t: None if t is None else C.byref(t)
        return ekv.lib.ekv_flash_attn_ext_workspace_size(r(q), r(k), r(v), r(m), max_bias, softcap, r(dst))
    q, k, v = fake([128, 50, 8, 4]), fake([128, 300, 2, 4]), fake([128, 300, 2, 4])
    m, dst = fake([300, 50, 1, 1], ekv.DTYPE_F16), fake([128, 8, 50, 4])
    n = ws(q, k, v, m, dst)
    assert n >= 4 * 2 * 2 * 320 * 128 * 2 + 4 * 50 * 8 * 128 * 2
    assert ws(q, k, v, None, dst) > 0
    assert ws(q, k, v, m, dst, softcap=10.0) == 0                        # softcap: CUDA cores
    assert ws(q, k, v, m, dst, max_bias=8.0) == 0                        # ALiBi: CUDA cores
    assert ws(q, k, v, fake([300, 50, 8, 1], ekv.DTYPE_F16), dst) == 0   # per-head mask
    assert ws(fake([96, 50, 8, 4]), fake([96, 300, 2, 4]), fake([96, 300, 2, 4]), m, fake([96, 8, 50, 4])) == 0
    assert ws(q, k, fake([64, 300, 2, 4]), m, fake([64, 8, 50, 4])) == 0  # Dv != D
    assert ws(q, fake([64, 300, 2, 4]), v, m, dst) == 0                  # invalid call


@pytest.mark.gpu
@pytest.mark.parametrize("d", [64, 128, 256])
def test_tensor_core_route_gqa_batch_broadcast_and_mask(d):
    """GQA, K/V batch broadcast (B = 2 Bk), a binary F16 mask per batch element with padding and a
    causal block, f16 K/V: the staged call on the tcgen05 kernels against the oracle."""
    import torch
    torch.manual_seed(d)
    B, Bk, Hq, Hkv, Tq, Tk = 4, 2, 8, 2, 37, 203
    q = torch.randn(B, Hq, Tq, d, device="cuda") * 0.5
    k = (torch.randn(Bk, Hkv, Tk, d, device="cuda") * 0.5).to(torch.float16)
    v = (torch.randn(Bk, Hkv, Tk, d, device="cuda") * 0.5).to(torch.float16)
    m = torch.zeros(B, 1, Tq + 3, Tk + 13, device="cuda")
    m[:, :, :, 150:180] = float("-inf")
    m[1, :, :, :40] = float("-inf")
    m[2, :, 5:9, 100:] = float("-inf")
    dst, want = run(q, k, v, m.to(torch.float16), scale=d ** -0.5)
    assert tol(dst) == TOL_TC
    assert np.abs(_np(dst) - want).max() < TOL_TC


@pytest.mark.gpu
def test_additive_mask_is_redone_exactly():
    """A head-shared mask with additive (finite, non-zero) entries on a tensor-core shape: the
    conversion flags it and the CUDA-core kernel redoes the call, so the result is f32-exact."""
    import torch
    torch.manual_seed(77)
    B, Hq, Hkv, Tq, Tk, D = 2, 4, 4, 21, 90, 64
    q, k, v = (torch.randn(B, h, n, D, device="cuda") for h, n in ((Hq, Tq), (Hkv, Tk), (Hkv, Tk)))
    mask = torch.randn(B, 1, Tq, Tk, device="cuda")
    mask[..., 7:11] = float("-inf")
    dst, want = run(q, k, v, mask, scale=0.125)
    assert np.abs(_np(dst) - want).max() < TOL


@pytest.mark.gpu
def test_explicit_workspace_and_too_small():
    import torch
    torch.manual_seed(3)
    B, H, Tq, Tk, D = 2, 8, 50, 866, 256
    q = torch.randn(B, H, Tq, D, device="cuda") * 0.5
    k = torch.randn(B, 1, Tk, D, device="cuda") * 0.5
    v = torch.randn(B, 1, Tk, D, device="cuda") * 0.5
    dst = torch.empty(B, Tq, H, D, device="cuda")
    n = ekv.flash_attn_ext_workspace_size(q, k, v, None, dst)
    assert n > 0
    small = torch.empty(n - 256, dtype=torch.uint8, device="cuda")
    with pytest.raises(ekv.EkvError) as e:
        ekv.flash_attn_ext(q, k, v, None, dst, scale=1 / 16, workspace=small)
    assert e.value.code == ekv.ERR_RANGE
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    ekv.flash_attn_ext(q, k, v, None, dst, scale=1 / 16, workspace=ws)
    torch.cuda.synchronize()
    want = oracle.flash_attn_ext(_np(q), _np(k), _np(v), None, scale=1 / 16)
    assert np.abs(_np(dst) - want).max() < TOL_TC
    # the triple with its own workspace
    vt = v.transpose(2, 3)
    dt = torch.empty(B, H, Tq, D, device="cuda")
    nt = ekv.mul_mat_soft_max_mul_mat_workspace_size(k, q, vt, None, dt)
    assert nt > 0
    ekv.mul_mat_soft_max_mul_mat(k, q, vt, None, dt, scale=1 / 16, workspace=torch.empty(nt, dtype=torch.uint8,
                                                                                          device="cuda"))
    torch.cuda.synchronize()
    assert np.abs(_np(dt) - want.transpose(0, 2, 1, 3)).max() < TOL_TC
