"""The ncnn-surface layer classes (libseedvr2_ncnn.so) driven exactly like the
reference's own layers: same creator / ParamDict / ModelBin / blob calls.

CPU tests check the surface (library loads, validation error codes equal the
reference's on the same bad inputs, no GPU -> a clean error).  GPU tests check
forward() against the golden outputs of the reference's layer code and
against that code itself on identical inputs (cosine >= 0.9995,
max|a-b|/max|b| <= 2e-2).
"""
import numpy as np
import pytest

from tests.conftest import cosine, rel_maxabs


@pytest.fixture(scope="module")
def layers(s2lib):
    from seedvr2_ncnn_b200 import layers as L

    L.lib()
    return L


def _bad_cases(g):
    base = dict(heads=int(g["heads"]), head_dim=int(g["head_dim"]), target=g["target"], shifted=0,
                eps=float(g["eps"]), rope_pairs=int(g["rope_pairs"]), norms=g["norms"], freqs=g["freqs"],
                shapes=g["shapes"], text_lengths=g["text_lengths"], video_qkv=g["video_qkv"],
                text_qkv=g["text_qkv"])
    yield dict(base, rope_pairs=22, freqs=np.ones(22, np.float32))                 # 6*22 > head_dim
    yield dict(base, text_lengths=np.asarray([5, 2], np.int32))                     # token count mismatch
    yield dict(base, text_lengths=np.asarray([5, 0], np.int32))                     # empty text


def test_validation_codes_match_reference(layers, ref, golden):
    g = golden["awa"]
    for case in _bad_cases(g):
        code, _, _ = layers.awa_forward(**case)
        with pytest.raises(ValueError) as e:
            ref.awa_forward(**case)
        assert f"returned {code}" in str(e.value), (code, str(e.value))


def test_shared_linear_validation(layers, ref):
    x = np.zeros((3, 16), np.float32)
    code, _, _ = layers.shared_linear(x, x, np.zeros((0, 16), np.float32))  # num_output 0 -> load_param -1
    assert code == -1
    with pytest.raises(ValueError, match="returned -1"):
        ref.shared_linear(x, x, np.zeros((0, 16), np.float32))


def test_no_gpu_is_a_clean_error(layers, golden):
    import torch

    if torch.cuda.is_available():
        pytest.skip("GPU present")
    g = golden["awa"]
    code, _, _ = layers.awa_forward(heads=int(g["heads"]), head_dim=int(g["head_dim"]), target=g["target"],
                                    shifted=0, eps=float(g["eps"]), rope_pairs=int(g["rope_pairs"]), norms=g["norms"],
                                    freqs=g["freqs"], shapes=g["shapes"], text_lengths=g["text_lengths"],
                                    video_qkv=g["video_qkv"], text_qkv=g["text_qkv"])
    assert code == -5


@pytest.mark.gpu
@pytest.mark.parametrize("shifted", [0, 1])
@pytest.mark.parametrize("bf16", [0, 1])
def test_awa_layer_vs_golden(layers, golden, shifted, bf16):
    g = golden["awa"]
    code, vo, to = layers.awa_forward(heads=int(g["heads"]), head_dim=int(g["head_dim"]), target=g["target"],
                                      shifted=shifted, eps=float(g["eps"]), rope_pairs=int(g["rope_pairs"]),
                                      norms=g["norms"], freqs=g["freqs"], shapes=g["shapes"],
                                      text_lengths=g["text_lengths"], video_qkv=g["video_qkv"],
                                      text_qkv=g["text_qkv"], bf16=bool(bf16))
    assert code == 0
    for got, key in ((vo, f"video_out_s{shifted}_b{bf16}"), (to, f"text_out_s{shifted}_b{bf16}")):
        assert cosine(got, g[key]) >= 0.9995 and rel_maxabs(got, g[key]) <= 2e-2


@pytest.mark.gpu
def test_awa_layer_vs_reference_split_int32_shared_norm(layers, ref):
    """8-blob form, int32 shape blobs, shared norms: both layer implementations, same calls."""
    rng = np.random.default_rng(8)
    heads, hd = 3, 128
    shapes = np.array([[2, 5, 7], [1, 3, 9]], np.int32)
    tl = np.array([4, 7], np.int32)
    nv, nt = int(np.prod(shapes, axis=1).sum()), int(tl.sum())
    inner = heads * hd
    split = [rng.standard_normal((nv if i < 3 else nt, inner)).astype(np.float32) for i in range(6)]
    norms = (1 + 0.02 * rng.standard_normal((4, hd))).astype(np.float32)
    norms[2:] = norms[:2]
    freqs = (1.0 / 10000 ** (np.arange(21) * 2 / 42)).astype(np.float32)
    kw = dict(heads=heads, head_dim=hd, target=[2, 1, 3], shifted=1, eps=1e-5, rope_pairs=21, norms=norms,
              freqs=freqs, shapes=shapes, text_lengths=tl, split=split, shared_norm=True, shape_int32=True)
    code, vo, to = layers.awa_forward(**kw)
    assert code == 0
    rv, rt = ref.awa_forward(**kw)
    for a, b in ((vo, rv), (to, rt)):
        assert cosine(a, b) >= 0.9995 and rel_maxabs(a, b) <= 2e-2


@pytest.mark.gpu
def test_shared_linear_layer_vs_golden(layers, golden):
    g = golden["linear"]
    for bias, vk, tk in ((g["bias"], "video_out_bias", "text_out_bias"), (None, "video_out_nobias",
                                                                          "text_out_nobias")):
        code, vo, to = layers.shared_linear(g["video"], g["text"], g["weight"], bias)
        assert code == 0
        for a, key in ((vo, vk), (to, tk)):
            assert cosine(a, g[key]) >= 0.9995 and rel_maxabs(a, g[key]) <= 2e-2


@pytest.mark.parametrize("src", ["adaptive_window_attention.cpp", "shared_linear.cpp", "vae_layers.cpp"])
def test_layer_sources_compile_against_ncnn_headers(src):
    """With -DS2_WITH_NCNN the layer sources include ncnn's own layer.h / modelbin.h / paramdict.h; checked
    here against the oracle shim's copies of that API (the subset the reference's layers use)."""
    import os
    import subprocess

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    r = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-DS2_WITH_NCNN",
                        "-I" + os.path.join(root, "oracle", "ncnn_shim"), "-I" + os.path.join(cuda, "include"),
                        os.path.join(root, "seedvr2_ncnn_b200", "csrc", "layers", src)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
