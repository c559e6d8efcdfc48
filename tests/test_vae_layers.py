"""The VAE's ncnn-surface layer classes (DecomposedConv3D, VAEDownsample3D,
VAEUpsample3D, VAEChunkedMHA in libseedvr2_ncnn.so) driven the way ncnn's Net
drives the reference's: creator -> load_param -> load_model (one flat .bin
sequence) -> create_pipeline -> forward under the thread's VAE memory state.

CPU tests: the load-time codes equal the reference's own layers' on the same
blobs, this build's documented limits, and a clean error without a GPU.
GPU tests: forward against the golden outputs of the reference's layers,
chunk by chunk with the temporal memory carried in the layer (cosine >=
0.9995, max|a-b|/max|b| <= 2e-2: bf16 operands, fp32 accumulation), and
reset_temporal_memory.
"""
import os

import numpy as np
import pytest

from tests.conftest import cosine, rel_maxabs
from tests.golden.gen_golden import CONV_CASES, MHA_CASES, RESAMPLE_CASES, conv_blob, mha_weights


@pytest.fixture(scope="module")
def layers(s2lib):
    from seedvr2_ncnn_b200 import layers as L

    L.lib()
    return L


@pytest.fixture(scope="module")
def refvae():
    from oracle import oracle

    if not os.path.exists(oracle.REF_VAE_SO):
        pytest.skip("oracle/_ref/libs2_ref_vae.so not built (reference tree absent)")
    return oracle


def _conv(co=6, ci=4, k=3, kt=3, st=1, head=2, sw=1, pad=1, bias=True, seed=0):
    return conv_blob(np.random.default_rng(seed), co, ci, k, kt, st, head, sw, pad, bias)


def _with(blob, i, v):
    b = np.array(blob, np.float32)
    b[i] = v
    return b


def _load_cases():
    """(name, kind, blob): valid blobs and every load-time rejection the reference has."""
    good = _conv()
    yield "conv", 0, good
    yield "conv_nobias", 0, _conv(bias=False)
    yield "conv_cfg_short", 0, good[:10]
    yield "conv_empty", 0, good[:0]
    yield "conv_bias_short", 0, good[:16 + 3]
    yield "conv_weights_short", 0, good[:-1]
    for i, v in ((0, 0), (1, 0), (2, 0), (3, -1), (4, 0), (5, 0), (6, 0), (8, 0), (9, 0), (10, 0), (11, 0), (14, 0),
                 (7, -1)):
        yield f"conv_cfg{i}={v}", 0, _with(good, i, v)
    yield "conv_groups_indivisible", 0, _with(good, 14, 3)  # 4 inputs % 3
    yield "conv_pad_negative", 0, _with(good, 12, -1)
    down = np.concatenate([np.asarray([6, 1, 1], np.float32), _conv(co=6, ci=6, sw=2, pad=0)])
    yield "down", 1, down
    yield "down_pad_right_only", 1, _with(down, 2, 0)
    yield "down_no_pad", 1, _with(_with(down, 1, 0), 2, 0)
    yield "down_channels0", 1, _with(down, 0, 0)
    yield "down_pad_negative", 1, _with(down, 1, -1)
    yield "down_short", 1, down[:2]
    yield "down_conv_short", 1, down[:-5]
    up = np.concatenate([np.asarray([4, 2, 2, 1], np.float32), _conv(co=4, ci=4), _conv(co=32, ci=4, seed=1)])
    yield "up", 2, up
    yield "up_ratio3", 2, _with(up, 1, 3)
    yield "up_spatial3", 2, _with(up, 2, 3)
    yield "up_head_mismatch", 2, _with(up, 3, 0)
    yield "up_channels0", 2, _with(up, 0, 0)
    yield "up_short", 2, up[:3]
    yield "up_upscale_short", 2, up[:-7]
    yield "up_t1", 2, np.concatenate([np.asarray([4, 1, 2, 0], np.float32), _conv(co=4, ci=4),
                                      _conv(co=16, ci=4, seed=2)])


@pytest.mark.parametrize("name,kind,blob", list(_load_cases()), ids=[c[0] for c in _load_cases()])
def test_vae_load_codes_match_reference(layers, refvae, name, kind, blob):
    assert layers.vae_load_code(kind, blob) == refvae.ref_vae_load(kind, blob), name


def test_vae_load_codes_cover_every_outcome(layers):
    codes = {layers.vae_load_code(k, b) for _, k, b in _load_cases()}
    assert codes == {0, -1, -100}


def test_vae_build_limits(layers, refvae):
    """Grouped convolutions and spatial strides above 2 load in the reference; this build's implicit GEMM
    rejects them at create_pipeline with -1."""
    for blob in (_with(_with(_conv(co=6, ci=4), 14, 2), 1, 4), _with(_conv(), 8, 3)):
        assert refvae.ref_vae_load(0, blob) == 0
        assert layers.vae_load_code(0, blob) == -1


def _mha_cases():
    E = 16
    w = mha_weights(np.random.default_rng(3), E)
    sc = float(1.0 / np.sqrt(E))
    yield "ok", dict(E=E, heads=1, scale=sc, weights=w)
    yield "embed0", dict(E=0, heads=1, scale=sc, weights=w, wds=E * E)
    yield "heads_indivisible", dict(E=E, heads=3, scale=sc, weights=w)
    yield "wds_indivisible", dict(E=E, heads=1, scale=sc, weights=w, wds=E * E + 1)
    yield "wds0", dict(E=E, heads=1, scale=sc, weights=w, wds=0)
    yield "kdim0", dict(E=E, heads=1, scale=sc, weights=w, kdim=0)
    yield "vdim0", dict(E=E, heads=1, scale=sc, weights=w, vdim=0)
    yield "chunk0", dict(E=E, heads=1, scale=sc, weights=w, chunk=0)
    yield "weights_short", dict(E=E, heads=1, scale=sc, weights=w[:-1])
    yield "weights_empty", dict(E=E, heads=1, scale=sc, weights=w[:0])


@pytest.mark.parametrize("name,kw", list(_mha_cases()), ids=[c[0] for c in _mha_cases()])
def test_mha_load_codes_match_reference(layers, refvae, name, kw):
    E = kw["E"]
    ip = [E, kw["heads"], kw.get("wds") or E * E, kw.get("kdim", E), kw.get("vdim", E), kw.get("chunk", 128)]
    if kw.get("wds") == 0:
        ip[2] = 0
    qdim = ip[2] // E if E and ip[2] > 0 else 1
    x = np.random.default_rng(4).standard_normal((5, max(qdim, 1))).astype(np.float32)
    want = refvae.ref_mha_code(ip, kw["scale"], kw["weights"], x)
    got = layers.mha_load_code(E, kw["heads"], kw["scale"], kw["weights"], wds=ip[2], kdim=ip[3], vdim=ip[4],
                               chunk=ip[5])
    assert got == want, (name, got, want)


def test_mha_build_limits(layers, refvae):
    """Two heads or a k / v width other than embed_dim load in the reference; this build (the VAE's one
    512-wide head as GEMMs) rejects them at create_pipeline with -1."""
    E = 16
    w = mha_weights(np.random.default_rng(5), E)
    x = np.zeros((3, E), np.float32)
    assert refvae.ref_mha_code([E, 2, E * E, E, E, 128], 0.25, w, x) == 0
    assert layers.mha_load_code(E, 2, 0.25, w) == -1


def test_vae_layers_without_gpu_are_a_clean_error(layers):
    import torch

    if torch.cuda.is_available():
        pytest.skip("GPU present")
    layer = layers.VaeLayer(0, _conv())
    with pytest.raises(layers.LayerError) as e:
        layer.forward(np.zeros((4, 3, 5, 5), np.float32), 0)
    assert e.value.code == -5
    layer.close()
    mha = layers.VaeMhaLayer(16, 1, 0.25, mha_weights(np.random.default_rng(6), 16))
    with pytest.raises(layers.LayerError) as e:
        mha.forward(np.zeros((3, 16), np.float32))
    assert e.value.code == -5
    mha.close()


def test_forward_rejects_blobs_like_the_reference(layers, refvae):
    """Blob checks that run before any device work (wrong channel count) return -1 on both sides."""
    blob = _conv()
    ref = refvae.RefConv3d(blob[:16].astype(np.int32), blob[16:22], blob[22:].reshape(3, 6, 4, 3, 3))
    with pytest.raises(ValueError, match="-1"):
        ref.forward(np.zeros((5, 3, 5, 5), np.float32), 0)
    layer = layers.VaeLayer(0, blob)
    with pytest.raises(layers.LayerError) as e:
        layer.forward(np.zeros((5, 3, 5, 5), np.float32), 0)
    assert e.value.code == -1
    layer.close()


# ---------------------------------------------------------------- GPU
def _conv_blob_from_golden(g, name):
    cfg = g[f"{name}__cfg"].astype(np.float32)
    parts = [cfg] + ([g[f"{name}__b"]] if f"{name}__b" in g else []) + [g[f"{name}__w"].ravel()]
    return np.concatenate(parts).astype(np.float32)


@pytest.mark.gpu
@pytest.mark.parametrize("name", [c[0] for c in CONV_CASES])
def test_conv3d_layer_vs_golden(layers, golden, name):
    g = golden["vae_conv"]
    chunks = [c[3] for c in CONV_CASES if c[0] == name][0]
    layer = layers.VaeLayer(layers.DECOMPOSED_CONV3D, _conv_blob_from_golden(g, name))
    for i in range(chunks):
        got = layer.forward(g[f"{name}__x{i}"], int(g[f"{name}__state{i}"]))
        ref = g[f"{name}__y{i}"]
        assert got.shape == ref.shape, (name, i)
        assert cosine(got, ref) >= 0.9995 and rel_maxabs(got, ref) <= 2e-2, (name, i)
    layer.close()


@pytest.mark.gpu
@pytest.mark.parametrize("name", [c[0] for c in RESAMPLE_CASES])
def test_resample_layer_vs_golden(layers, golden, name):
    g = golden["vae_conv"]
    kind = int(g[f"{name}__kind"])
    layer = layers.VaeLayer(layers.VAE_DOWNSAMPLE3D if kind == 0 else layers.VAE_UPSAMPLE3D, g[f"{name}__blob"])
    i = 0
    while f"{name}__x{i}" in g:
        got = layer.forward(g[f"{name}__x{i}"], int(g[f"{name}__state{i}"]))
        ref = g[f"{name}__y{i}"]
        assert got.shape == ref.shape, (name, i)
        assert cosine(got, ref) >= 0.9995 and rel_maxabs(got, ref) <= 2e-2, (name, i)
        i += 1
    layer.close()


@pytest.mark.gpu
def test_reset_temporal_memory_matches_reference(layers, refvae):
    """INITIALIZING caches frames, reset_temporal_memory drops them: an ACTIVE chunk after the reset uses
    the head frames again, on both sides."""
    rng = np.random.default_rng(12)
    blob = _conv(co=8, ci=8, seed=7)
    cfg, b, w = blob[:16].astype(np.int32), blob[16:24], blob[24:].reshape(3, 8, 8, 3, 3)
    xs = [rng.standard_normal((8, 3, 6, 7)).astype(np.float32) for _ in range(2)]
    ref = refvae.RefConv3d(cfg, b, w)
    ref.forward(xs[0], 1)
    ref_reset = refvae.RefConv3d(cfg, b, w)  # a fresh layer = one whose memory was reset
    want = ref_reset.forward(xs[1], 2)
    layer = layers.VaeLayer(0, blob)
    layer.forward(xs[0], 1)
    layer.reset_temporal_memory()
    got = layer.forward(xs[1], 2)
    assert got.shape == want.shape
    assert cosine(got, want) >= 0.9995 and rel_maxabs(got, want) <= 2e-2
    layer.close()


@pytest.mark.gpu
@pytest.mark.parametrize("name,E,T", MHA_CASES)
def test_mha_layer_vs_golden(layers, golden, name, E, T):
    g = golden["vae_conv"]
    layer = layers.VaeMhaLayer(E, 1, float(1.0 / np.sqrt(E)), g[f"{name}__w"])
    got = layer.forward(g[f"{name}__x"])
    ref = g[f"{name}__y"]
    assert cosine(got, ref) >= 0.9995 and rel_maxabs(got, ref) <= 2e-2, name
    layer.close()
