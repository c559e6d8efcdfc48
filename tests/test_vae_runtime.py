"""VAE runtime host steps (no GPU): the temporal segment plan of
extract_temporal_slices (seedvr2_vae.cpp:408-451), the frame-count rules of
encode_moments / decode (:551-565, :578-599), and the posterior noise, pinned
bit for bit against the reference's own moments_to_latent (:454-478, built
from its source by oracle/Makefile): with zero means and zero log-variances
it returns noise * 0.9152."""
import numpy as np
import pytest

from seedvr2_ncnn_b200 import abi

DISABLED, INITIALIZING, ACTIVE = 0, 1, 2


def _segments(frames, first, active):
    """extract_temporal_slices' loop, restated."""
    if frames <= first:
        return [(0, frames, DISABLED)]
    out, start = [], 0
    while start < frames:
        count = min(first if start == 0 else active, frames - start)
        out.append((start, count, INITIALIZING if start == 0 else ACTIVE))
        start += count
    return out


@pytest.mark.parametrize("first,active", [(5, 4), (2, 1), (1, 1), (3, 7)])
def test_temporal_segments(first, active):
    for frames in range(1, 50):
        assert abs_list(abi.vae_temporal_segments(frames, first, active)) == _segments(frames, first, active)


def abs_list(v):
    return [tuple(int(x) for x in s) for s in v]


def test_temporal_segments_invalid():
    lib = abi.lib()
    for args in ((0, 5, 4), (9, 0, 4), (9, 5, 0), (-3, 5, 4)):
        assert lib.s2_vae_temporal_segments(*args, 0, None) == -1


def test_frame_counts():
    for f in range(1, 42):
        want = (f - 1) // 4 + 1 if (f <= 5 or (f - 1) % 4 == 0) else -1
        assert abi.vae_encode_frames(f) == want
    assert abi.vae_encode_frames(0) == -1
    for n in range(1, 12):
        assert abi.vae_decode_frames(n) == (n - 1) * 4 + 1
    assert abi.vae_decode_frames(0) == -1


def test_posterior_noise_matches_reference():
    from oracle import oracle

    d, h, w = 2, 8, 12
    plane = d * h * w
    moments = np.zeros((32, d, h, w), np.float32)
    for seed in (666, 1, 2**63 + 5):
        try:
            ref = oracle.ref_moments_to_latent(moments, True, seed)
        except FileNotFoundError:
            pytest.skip("reference VAE runtime checker not built (oracle/_ref)")
        noise = abi.vae_posterior_noise(seed, 16 * plane)
        np.testing.assert_array_equal(noise.reshape(16, d, h, w) * np.float32(abi.VAE_SCALING_FACTOR), ref)
    a, b = abi.vae_posterior_noise(7, 4096), abi.vae_posterior_noise(8, 4096)
    assert not np.array_equal(a, b)
    assert abs(float(a.mean())) < 0.1 and abs(float(a.std()) - 1.0) < 0.1
