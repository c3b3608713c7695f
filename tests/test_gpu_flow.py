"""The sampler's per-step kernels (ekv_flow_step_f32, ekv_guidance_f32) against the oracle, bit for bit:
f32 products and sums each rounded, optional bf16 rounding; sizes that are and are not multiples of four,
16-byte aligned and unaligned pointers, and the pi0.5 / GR00T / LingBot state shapes."""
import numpy as np
import pytest
import torch

import ekv
import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,offset", [(64 * 50 * 32, 0), (128 * 16 * 32, 0), (1001, 0), (1001, 1), (3, 0), (0, 0)])
@pytest.mark.parametrize("bf16_round", [False, True])
def test_flow_step_bit_exact(n, offset, bf16_round):
    rng = np.random.default_rng(n + offset)
    s = rng.standard_normal(n + offset).astype(np.float32) * 3
    v = rng.standard_normal(n + offset).astype(np.float32)
    if n > 4:
        s[1], v[2] = np.float32(1e30), np.float32(-2e-38)  # large and subnormal operands
    ds, dv = torch.from_numpy(s).cuda(), torch.from_numpy(v).cuda()
    ekv.flow_step(ds[offset:], dv[offset:], -0.1, bf16_round)
    torch.cuda.synchronize()
    want = oracle.flow_step(s[offset:], v[offset:], -0.1, bf16_round)
    np.testing.assert_array_equal(ds[offset:].cpu().numpy().view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("use,bf16_round", [(True, False), (True, True), (False, True), (False, False)])
def test_guidance_bit_exact(use, bf16_round):
    rng = np.random.default_rng(7)
    n = 24 * 30 * 17 + 3
    c = rng.standard_normal(n).astype(np.float32)
    u = rng.standard_normal(n).astype(np.float32)
    dc, du = torch.from_numpy(c).cuda(), torch.from_numpy(u).cuda()
    ekv.guidance(dc, du, 5.0, use, bf16_round)
    torch.cuda.synchronize()
    want = oracle.guidance(c, u, 5.0, use, bf16_round)
    np.testing.assert_array_equal(dc.cpu().numpy().view(np.uint32), np.asarray(want, np.float32).view(np.uint32))


def test_flow_loop_on_device_matches_host_loop():
    """GR00T's 4-step loop (models/groot_n1.cpp:721-768) with the action update on the device: the
    same actions as the host loop's float updates, with no copy between steps."""
    rng = np.random.default_rng(11)
    steps, B, H, A = 4, 128, 16, 32
    x = rng.standard_normal((B, H, A)).astype(np.float32)
    vel = rng.standard_normal((steps, B, H, A)).astype(np.float32)
    dx, dvel = torch.from_numpy(x.copy()).cuda(), torch.from_numpy(vel).cuda()
    dt = 1.0 / steps
    for k in range(steps):
        ekv.flow_step(dx, dvel[k], dt)
        x = oracle.flow_step(x, vel[k], dt)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(dx.cpu().numpy().view(np.uint32), x.view(np.uint32))
