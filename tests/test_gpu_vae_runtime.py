"""VAE runtime device steps against the reference's own moments_to_latent
(seedvr2_vae.cpp:454-478, built from its source by oracle/Makefile) and
decode's unscaling (:583-587).  Without a posterior sample the latent is
mean * 0.9152 and must match bit for bit; with one, the only difference is
the device's expf against the host's (at most 2 ulp of the factor), so the
gate is max|gpu - ref| <= 4e-7 * max|ref| per element scale.  The unscaling
is a correctly rounded division on both sides: bit for bit."""
import numpy as np
import pytest

from seedvr2_ncnn_b200 import abi

pytestmark = pytest.mark.gpu


def _moments(d, h, w, seed):
    rng = np.random.default_rng(seed)
    m = np.empty((32, d, h, w), np.float32)
    m[:16] = rng.standard_normal((16, d, h, w)).astype(np.float32)
    # log-variances across both clamps (-30, 20)
    m[16:] = rng.uniform(-40.0, 30.0, (16, d, h, w)).astype(np.float32)
    return m


@pytest.mark.parametrize("shape", [(3, 16, 24), (1, 8, 8), (5, 12, 20)])
def test_moments_to_latent_vs_reference(gpu_ctx, s2lib, shape):
    import torch

    from oracle import oracle

    d, h, w = shape
    m = _moments(d, h, w, sum(shape))
    try:
        ref_mean = oracle.ref_moments_to_latent(m, False)
    except FileNotFoundError:
        pytest.skip("reference VAE runtime checker not built (oracle/_ref)")
    got = s2lib.vae_moments_to_latent(gpu_ctx, torch.from_numpy(m).cuda())
    np.testing.assert_array_equal(got.cpu().numpy(), ref_mean)

    ref = oracle.ref_moments_to_latent(m, True, 666)
    noise = torch.from_numpy(s2lib.vae_posterior_noise(666, 16 * d * h * w).reshape(16, d, h, w)).cuda()
    got = s2lib.vae_moments_to_latent(gpu_ctx, torch.from_numpy(m).cuda(), noise).cpu().numpy()
    torch.cuda.synchronize()
    assert gpu_ctx.status() == 0
    # per element: |mean| + exp(0.5 lv) |noise| bounds the terms whose rounding differs
    scale = (np.abs(m[:16]) + np.exp(0.5 * np.clip(m[16:], -30, 20)) * np.abs(noise.cpu().numpy())) * 0.9152
    assert np.all(np.abs(got - ref) <= 4e-7 * scale + 1e-30)


def test_unscale_latent(gpu_ctx, s2lib):
    import torch

    x = np.random.default_rng(4).standard_normal(16 * 3 * 40 * 56).astype(np.float32) * 7
    t = torch.from_numpy(x.copy()).cuda()
    s2lib.vae_unscale_latent(gpu_ctx, t)
    np.testing.assert_array_equal(t.cpu().numpy(), x / np.float32(s2lib.VAE_SCALING_FACTOR))
