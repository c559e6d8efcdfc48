"""GPU parity of the VAE DecomposedConv3D implicit GEMM (s2_conv3d_*, through
the C ABI) against the reference's own layer (golden fixture) and the CPU
oracle.

Gates: against the fp32 reference, cosine >= 0.9995 and
max|gpu - ref| / max|ref| <= 2e-2 (the GPU computes with bf16 operands);
against the oracle fed the same bf16-rounded inputs and weights,
max|gpu - ref| / max|ref| <= 1e-3 (fp32 accumulation order only).  The
temporal memory is carried across chunks exactly as the reference's.
"""
import numpy as np
import pytest

from tests.conftest import cosine, rel_maxabs
from tests.golden.gen_golden import CONV_CASES, conv_weights

pytestmark = pytest.mark.gpu


def _run_gpu(gpu_ctx, s2lib, cfg, b, w, xs, states):
    import torch

    layer = s2lib.Conv3d(gpu_ctx, cfg, b, w)
    outs = []
    for x, st in zip(xs, states):
        outs.append(layer.forward(torch.from_numpy(np.ascontiguousarray(x)).cuda(), st).cpu().numpy())
    torch.cuda.synchronize()
    assert gpu_ctx.status() == 0
    layer.close()
    return outs


def _run_port(port, cfg, b, w, xs, states, bf16):
    rnd = port.round_bf16 if bf16 else (lambda a: np.asarray(a, np.float32))
    mem, outs = None, []
    for x, st in zip(xs, states):
        y, nm = port.conv3d_forward(cfg, b, rnd(w), rnd(x), mem if st == 2 else None)
        outs.append(y)
        mem = nm if st != 0 else None
    return outs


@pytest.mark.parametrize("name", [c[0] for c in CONV_CASES])
def test_conv3d_golden(gpu_ctx, s2lib, port, golden, name):
    g = golden["vae_conv"]
    chunks = [c[3] for c in CONV_CASES if c[0] == name][0]
    cfg = g[f"{name}__cfg"].tolist()
    b = g[f"{name}__b"] if f"{name}__b" in g else None
    w = g[f"{name}__w"]
    xs = [g[f"{name}__x{i}"] for i in range(chunks)]
    states = [int(g[f"{name}__state{i}"]) for i in range(chunks)]
    got = _run_gpu(gpu_ctx, s2lib, cfg, b, w, xs, states)
    emu = _run_port(port, cfg, b, w, xs, states, True)
    for i in range(chunks):
        ref = g[f"{name}__y{i}"]
        assert got[i].shape == ref.shape
        assert cosine(got[i], ref) >= 0.9995 and rel_maxabs(got[i], ref) <= 2e-2, (name, i)
        assert rel_maxabs(got[i], emu[i]) <= 1e-3, (name, i)


@pytest.mark.parametrize("cfg,shape,chunks", [
    # wide rows (two 128-pixel segments), channel counts off the 64 / 128 tiles
    ([200, 136, 3, 3, 3, 1, 1, 2, 1, 1, 1, 1, 1, 1, 1, 1], (136, 3, 6, 160), 1),
    # pointwise, 128 -> 128
    ([128, 128, 1, 1, 1, 1, 1, 0, 1, 1, 1, 1, 0, 0, 1, 1], (128, 2, 9, 40), 1),
    # VAE-like 3x3x3 with the temporal memory over three chunks
    ([64, 64, 3, 3, 3, 1, 1, 2, 1, 1, 1, 1, 1, 1, 1, 1], (64, 2, 12, 20), 3),
    # three RGB channels in (padded to one 8-channel row), temporal stride 2, no bias
    ([32, 3, 3, 3, 3, 2, 1, 2, 1, 1, 1, 1, 1, 1, 1, 0], (3, 5, 16, 16), 2),
])
def test_conv3d_vs_oracle(gpu_ctx, s2lib, port, cfg, shape, chunks):
    rng = np.random.default_rng(sum(cfg) + chunks)
    b, w = conv_weights(rng, cfg)
    xs = [rng.standard_normal(shape).astype(np.float32) for _ in range(chunks)]
    states = [0] if chunks == 1 else [1] + [2] * (chunks - 1)
    got = _run_gpu(gpu_ctx, s2lib, cfg, b, w, xs, states)
    ref = _run_port(port, cfg, b, w, xs, states, False)
    emu = _run_port(port, cfg, b, w, xs, states, True)
    for i in range(chunks):
        assert got[i].shape == ref[i].shape
        assert cosine(got[i], ref[i]) >= 0.9995 and rel_maxabs(got[i], ref[i]) <= 2e-2, i
        assert rel_maxabs(got[i], emu[i]) <= 1e-3, i


def test_conv3d_rejects_like_the_reference(gpu_ctx, s2lib):
    import torch

    rng = np.random.default_rng(4)
    cfg = [16, 8, 3, 3, 3, 1, 1, 0, 1, 1, 1, 1, 1, 1, 1, 1]
    b, w = conv_weights(rng, cfg)
    layer = s2lib.Conv3d(gpu_ctx, cfg, b, w)
    L = s2lib.lib()
    x = torch.zeros((8, 4, 6, 6), device="cuda")
    out = torch.zeros((16, 4 * 6 * 6), device="cuda")  # up to 4 output frames of 6 x 6 per channel

    def fwd(c, d, state, hw=6):
        return L.s2_conv3d_forward(layer.handle, x.data_ptr(), d * hw * hw, hw, hw, d, c, state, out.data_ptr(),
                                   4 * 6 * 6)

    assert fwd(7, 4, 0) == -1          # channel count other than num_input
    assert fwd(8, 2, 0) == -1          # head_frames 0: two frames are fewer than the kernel's three
    assert fwd(8, 4, 1) == 0           # initializing: caches the last two frames
    assert fwd(8, 1, 2) == 0           # active: two cached frames + one new frame -> one output frame
    assert fwd(8, 1, 2, hw=5) == -1    # cached frames of another size
    # grouped convolutions and spatial strides above 2, which this build does not implement, are refused
    for i, v in ((14, 2), (8, 3)):
        bad = list(cfg)
        bad[i] = v
        with pytest.raises(s2lib.S2Error):
            s2lib.Conv3d(gpu_ctx, bad, b, w)
    torch.cuda.synchronize()
    layer.close()


# ---- VAE resampling layers (VAEDownsample3D / VAEUpsample3D) ----
def _resample_cases():
    from tests.golden.gen_golden import RESAMPLE_CASES

    return [c[0] for c in RESAMPLE_CASES]


@pytest.mark.parametrize("name", _resample_cases())
def test_resample_golden(gpu_ctx, s2lib, port, golden, name):
    """Against the reference's own layers (golden, fp32): the DiT gate.  The downsample (one conv, spatial
    stride 2 through the tensor map's traversal stride) also against the oracle fed bf16-rounded inputs and
    weights: rel <= 1e-3; the upsample chains two convs around a shuffle, so its bf16-emulated comparison
    allows 5e-3 (a bf16 rounding of the intermediate can flip)."""
    import torch

    from oracle import oracle

    g = golden["vae_conv"]
    kind = int(g[f"{name}__kind"])
    blob = g[f"{name}__blob"]
    layer = s2lib.VaeResample(gpu_ctx, kind, blob)
    emu = (oracle.PortDownsample if kind == 0 else oracle.PortUpsample)(port, blob, emulate_bf16=True)
    i = 0
    while f"{name}__x{i}" in g:
        x, st = g[f"{name}__x{i}"], int(g[f"{name}__state{i}"])
        got = layer.forward(torch.from_numpy(x).cuda(), st).cpu().numpy()
        ref = g[f"{name}__y{i}"]
        assert got.shape == ref.shape, (name, i)
        assert cosine(got, ref) >= 0.9995 and rel_maxabs(got, ref) <= 2e-2, (name, i)
        assert rel_maxabs(got, emu.forward(x, st)) <= (1e-3 if kind == 0 else 5e-3), (name, i)
        i += 1
    torch.cuda.synchronize()
    assert gpu_ctx.status() == 0
    layer.close()


def test_resample_decoder_shapes(gpu_ctx, s2lib, port):
    """A 2x spatial downsample of 128 channels on 3 frames of 64 x 96 and a 2x / 2x upsample of 64 channels
    on 2 frames of 24 x 40, against the oracle in fp32 (the DiT gate)."""
    import torch

    from oracle import oracle
    from tests.golden.gen_golden import conv_blob

    rng = np.random.default_rng(99)
    down = np.concatenate([np.asarray([128, 1, 1], np.float32), conv_blob(rng, 128, 128, 3, 3, 1, 2, 2, 0, True)])
    up = np.concatenate([np.asarray([64, 2, 2, 1], np.float32), conv_blob(rng, 64, 64, 3, 3, 1, 2, 1, 1, True),
                         conv_blob(rng, 512, 64, 3, 3, 1, 2, 1, 1, True)])
    for kind, blob, shape in ((0, down, (128, 3, 64, 96)), (1, up, (64, 2, 24, 40))):
        x = rng.standard_normal(shape).astype(np.float32)
        layer = s2lib.VaeResample(gpu_ctx, kind, blob)
        got = layer.forward(torch.from_numpy(x).cuda(), s2lib.S2_VAE_MEMORY_DISABLED).cpu().numpy()
        ref = (oracle.PortDownsample if kind == 0 else oracle.PortUpsample)(port, blob).forward(x, 0)
        assert got.shape == ref.shape
        assert cosine(got, ref) >= 0.9995 and rel_maxabs(got, ref) <= 2e-2, kind
        layer.close()


# ---- VAEChunkedMHA ----
@pytest.mark.parametrize("E,T", [(16, 20), (64, 100), (512, 1440), (64, 9000)])
def test_vae_mha_vs_oracle(gpu_ctx, s2lib, port, golden, E, T):
    """Against the oracle's restatement of the reference's CPU path (fp32): the DiT gate.  (16, 20) and
    (64, 100) are the golden cases; 512 x 1440 is a VAE mid-block width; 9000 tokens run in two query
    chunks."""
    import torch

    from tests.golden.gen_golden import mha_weights

    g = golden["vae_conv"]
    name = f"mha{E}"
    if (E, T) in ((16, 20), (64, 100)):
        w, x = g[f"{name}__w"], g[f"{name}__x"]
        ref = g[f"{name}__y"]
    else:
        rng = np.random.default_rng(E + T)
        w = mha_weights(rng, E) * (0.5 if E == 512 else 1.0)
        x = rng.standard_normal((T, E)).astype(np.float32)
        ref = port.mha_forward(E, 1, float(1.0 / np.sqrt(E)), w, x)
    layer = s2lib.VaeMha(gpu_ctx, E, 1, float(1.0 / np.sqrt(E)), w)
    got = layer.forward(torch.from_numpy(np.ascontiguousarray(x)).cuda()).cpu().numpy()
    torch.cuda.synchronize()
    assert gpu_ctx.status() == 0
    assert cosine(got, ref) >= 0.9995 and rel_maxabs(got, ref) <= 2e-2, (E, T)
    layer.close()
