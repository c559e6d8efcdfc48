"""CPU: the VAE's DecomposedConv3D (src/seedvr2/decomposed_conv3d.cpp) -- our C
restatement (oracle/s2_oracle.c: s2o_conv3d_forward) against the golden fixture
made by the reference's own layer built here (tests/golden/vae_conv.npz), and
against that build directly on random configurations, including the temporal
memory carried across chunks.  Bit-exact (same fp32 operation order)."""
import numpy as np
import pytest

from tests.golden.gen_golden import CONV_CASES, conv_weights


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _run_port(port, cfg, b, w, xs, states):
    mem, outs = None, []
    for x, st in zip(xs, states):
        y, nm = port.conv3d_forward(cfg, b, w, x, mem if st == 2 else None)
        outs.append(y)
        mem = nm if st != 0 else None
    return outs


@pytest.mark.parametrize("name", [c[0] for c in CONV_CASES])
def test_port_conv3d_matches_golden(port, golden, name):
    g = golden["vae_conv"]
    chunks = [c[3] for c in CONV_CASES if c[0] == name][0]
    cfg = g[f"{name}__cfg"]
    b = g[f"{name}__b"] if f"{name}__b" in g else None
    xs = [g[f"{name}__x{i}"] for i in range(chunks)]
    states = [int(g[f"{name}__state{i}"]) for i in range(chunks)]
    for i, y in enumerate(_run_port(port, cfg, b, g[f"{name}__w"], xs, states)):
        assert np.array_equal(_bits(y), _bits(g[f"{name}__y{i}"])), (name, i)


def test_port_conv3d_vs_reference_random(port):
    from oracle import oracle

    if not __import__("os").path.exists(oracle.REF_VAE_SO):
        pytest.skip("oracle/_ref/libs2_ref_vae.so not built (reference tree absent)")
    rng = np.random.default_rng(21)
    for _ in range(12):
        kt = int(rng.integers(1, 4))
        st = int(rng.integers(1, kt + 1))
        k = int(rng.choice([1, 3]))
        pad = int(rng.integers(0, 2)) if k == 3 else 0
        cfg = [int(rng.integers(1, 9)), int(rng.integers(1, 7)), k, k, kt, st, int(rng.integers(1, 3)),
               int(rng.integers(0, 3)), 1, 1, 1, 1, pad, pad, 1, int(rng.integers(0, 2))]
        extent = cfg[6] * (kt - 1) + 1
        d = max(1, extent - cfg[7]) + int(rng.integers(0, 3))
        c, h, w = cfg[1], int(rng.integers(3, 9)), int(rng.integers(3, 9))
        b, wt = conv_weights(rng, cfg)
        ref = oracle.RefConv3d(cfg, b, wt)
        chunks = int(rng.integers(1, 4))
        xs = [rng.standard_normal((c, d, h, w)).astype(np.float32) for _ in range(chunks)]
        states = [0] if chunks == 1 else [1] + [2] * (chunks - 1)
        got = _run_port(port, cfg, b, wt, xs, states)
        for i, (x, s) in enumerate(zip(xs, states)):
            try:
                want = ref.forward(x, s)
            except ValueError:
                break  # too few padded frames for this chunk: both sides reject it
            assert np.array_equal(_bits(got[i]), _bits(want)), (cfg, i)


@pytest.mark.parametrize("name", [c[0] for c in __import__("tests.golden.gen_golden", fromlist=["x"]).RESAMPLE_CASES])
def test_port_resample_matches_golden(port, golden, name):
    """VAEDownsample3D / VAEUpsample3D restated (pad / shuffle in numpy around the C conv) against the
    reference's own layers (golden)."""
    from oracle import oracle

    g = golden["vae_conv"]
    kind = int(g[f"{name}__kind"])
    layer = (oracle.PortDownsample if kind == 0 else oracle.PortUpsample)(port, g[f"{name}__blob"])
    i = 0
    while f"{name}__x{i}" in g:
        y = layer.forward(g[f"{name}__x{i}"], int(g[f"{name}__state{i}"]))
        assert np.array_equal(_bits(y), _bits(g[f"{name}__y{i}"])), (name, i)
        i += 1


def test_port_mha_matches_golden_and_reference(port, golden):
    """VAEChunkedMHA's CPU path (ncnn MultiHeadAttention, restated) -- port vs the reference's layer."""
    from oracle import oracle
    from tests.golden.gen_golden import MHA_CASES

    g = golden["vae_conv"]
    for name, E, T in MHA_CASES:
        y = port.mha_forward(E, 1, float(1.0 / np.sqrt(E)), g[f"{name}__w"], g[f"{name}__x"])
        assert np.array_equal(_bits(y), _bits(g[f"{name}__y"])), name
    if __import__("os").path.exists(oracle.REF_VAE_SO):
        rng = np.random.default_rng(8)
        for E, H, T in ((32, 2, 41), (24, 1, 9)):
            w = np.concatenate([(0.1 * rng.standard_normal(n)).astype(np.float32) for n in [E * E, E] * 4])
            x = rng.standard_normal((T, E)).astype(np.float32)
            sc = float(1.0 / np.sqrt(E // H))
            assert np.array_equal(_bits(port.mha_forward(E, H, sc, w, x)),
                                  _bits(oracle.ref_mha_forward(E, H, sc, w, x)))
