"""CPU: the DiT input/output formats around the block stack -- patchify_video,
unpatchify_prediction and make_timestep_embedding (src/seedvr2/seedvr2_dit.cpp:167-326)
-- pinned three ways: our C restatement (oracle/s2_oracle.c) against the golden
fixture made from the reference's own code (tests/golden/dit_io.npz), against
that code built here (oracle/_ref/libs2_ref_dit_io.so) on random shapes, and
the error codes of invalid / empty calls.  Plus the frontend / tail
restatement's own invariants.  Bit-exact throughout (these are copies and the
reference's fp32 expression order)."""
import numpy as np
import pytest

from tests.golden.gen_golden import DIT_IO_CASES, DIT_IO_ERRORS


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _code(fn):
    try:
        fn()
        return 0
    except ValueError as e:
        return int(e.args[0])


@pytest.mark.parametrize("name", [c[0] for c in DIT_IO_CASES])
def test_port_patchify_matches_golden(port, golden, name):
    g = golden["dit_io"]
    shapes = g[f"{name}__shapes"].tolist()
    got = port.patchify_video(g[f"{name}__video"], shapes)
    assert np.array_equal(_bits(got), _bits(g[f"{name}__patches"]))
    got = port.unpatchify_prediction(g[f"{name}__pred"], shapes)
    assert np.array_equal(_bits(got), _bits(g[f"{name}__unpatched"]))


def test_port_timestep_embedding_matches_golden(port, golden):
    g = golden["dit_io"]
    assert np.array_equal(_bits(port.timestep_embedding(g["timesteps"])), _bits(g["timestep_embedding"]))


def test_port_error_codes_match_golden(port, golden):
    codes = []
    for fn, shapes, rows in DIT_IO_ERRORS:
        if fn == "patchify":
            codes.append(_code(lambda: port.patchify_video(np.zeros((max(rows, 1), 33), np.float32), shapes, rows)))
        else:
            codes.append(_code(lambda: port.unpatchify_prediction(np.zeros((max(rows, 1), 64), np.float32), shapes,
                                                                   rows)))
    assert codes == golden["dit_io"]["error_codes"].tolist()


def test_patchify_roundtrip_identity(port):
    """unpatchify(patchify(x)) restores the tokens when the 16 prediction channels are the first
    16 latent channels of each 33-channel group (a size-independent property)."""
    rng = np.random.default_rng(5)
    shapes = [[3, 10, 14], [1, 2, 2]]
    n = sum(t * h * w for t, h, w in shapes)
    x = rng.standard_normal((n, 33)).astype(np.float32)
    p = port.patchify_video(x, shapes)
    pred = np.concatenate([p[:, q * 33:q * 33 + 16] for q in range(4)], axis=1)
    back = port.unpatchify_prediction(pred, shapes)
    assert np.array_equal(_bits(back), _bits(x[:, :16]))


def test_port_vs_reference_random(port, refio):
    rng = np.random.default_rng(11)
    for _ in range(40):
        batch = int(rng.integers(1, 4))
        shapes = [[int(rng.integers(1, 5)), 2 * int(rng.integers(1, 9)), 2 * int(rng.integers(1, 9))]
                  for _ in range(batch)]
        n = sum(t * h * w for t, h, w in shapes)
        x = rng.standard_normal((n, 33)).astype(np.float32)
        a, b = port.patchify_video(x, shapes), refio.patchify_video(x, shapes)
        assert np.array_equal(_bits(a), _bits(b))
        pr = rng.standard_normal((a.shape[0], 64)).astype(np.float32)
        assert np.array_equal(_bits(port.unpatchify_prediction(pr, shapes)), _bits(refio.unpatchify_prediction(pr,
                                                                                                               shapes)))
    t = np.concatenate([rng.uniform(0, 1000, 200), rng.uniform(-50, 50, 50), [0.0, 1e-7, 1e6]]).astype(np.float32)
    assert np.array_equal(_bits(port.timestep_embedding(t)), _bits(refio.timestep_embedding(t)))


def test_frontend_tail_restatement_shapes(port):
    """The frontend / tail restatement's I/O contract: modulation [6][batch][D], per-sample rows,
    prediction [tokens][16]; a zero tail weight leaves exactly the bias."""
    rng = np.random.default_rng(2)
    D = 64
    n = lambda *s: (0.02 * rng.standard_normal(s)).astype(np.float32)  # noqa: E731
    io = dict(w_vid_in=n(D, 132), b_vid_in=n(D), w_txt_in=n(D, 5120), b_txt_in=n(D), w_emb0=n(D, 256),
              b_emb0=n(D), w_emb1=n(D, D), b_emb1=n(D), w_emb2=n(6 * D, D), b_emb2=n(6 * D),
              tail_ada=np.stack([n(D), 1 + n(D)]), w_out=np.zeros((64, D), np.float32), b_out=n(64))
    shapes = [[1, 4, 6], [2, 2, 2]]
    tokens = sum(t * h * w for t, h, w in shapes)
    v, t, mod = port.frontend_forward(io, shapes, [10.0, 500.0], rng.standard_normal((tokens, 33)),
                                      rng.standard_normal((7, 5120)))
    assert v.shape == (tokens // 4, D) and t.shape == (7, D) and mod.shape == (6, 2, D)
    pred = port.tail_forward(io, shapes, v, mod)
    assert pred.shape == (tokens, 16)
    # patch (0, 0, 0) of the first sample (w = 6) covers tokens 0, 1, 6, 7 in (y, x) order
    bias = io["b_out"].reshape(4, 16)
    for q, tok in enumerate([0, 1, 6, 7]):
        assert np.allclose(pred[tok], bias[q])


# ---- denoise loop pieces (src/seedvr2/seedvr2_pipeline.cpp) ----
def test_port_apply_cfg_matches_golden(port, golden):
    from tests.golden.gen_golden import CFG_CASES

    g = golden["dit_io"]
    for i, (_, scale, rescale) in enumerate(CFG_CASES):
        got = port.apply_cfg(g[f"cfg{i}__pos"], g[f"cfg{i}__neg"], scale, rescale)
        assert np.array_equal(_bits(got), _bits(g[f"cfg{i}__out"])), i


def test_port_apply_cfg_vs_reference_random(port, refio):
    rng = np.random.default_rng(12)
    for _ in range(20):
        rows = int(rng.integers(1, 300))
        pos = rng.standard_normal((rows, 16)).astype(np.float32)
        neg = rng.standard_normal((rows, 16)).astype(np.float32)
        scale, rescale = float(rng.uniform(1, 8)), float(rng.choice([0.0, rng.uniform(0, 1)]))
        assert np.array_equal(_bits(port.apply_cfg(pos, neg, scale, rescale)),
                              _bits(refio.apply_cfg(pos, neg, scale, rescale)))
    # a constant guided prediction (std 0) is left as is
    one = np.ones((4, 16), np.float32)
    assert np.array_equal(port.apply_cfg(one, one, 2.0, 0.5), one)


def test_denoise_schedule_and_assembly(port):
    """Timesteps 1000 * (n - s) / n in fp32 and deltas to the next one; the DiT input row is
    [latent 16 | condition 16 | 1]."""
    for n in (1, 3, 7, 50):
        ts = [port.denoise_schedule(n, s) for s in range(n)]
        assert ts[0][0] == 1000.0
        assert all(np.float32(t) == np.float32(np.float32(1000.0) * np.float32(n - s) / np.float32(n))
                   for s, (t, _) in enumerate(ts))
        assert abs(sum(d for _, d in ts) + 1.0) < 1e-5
    rng = np.random.default_rng(3)
    lat = rng.standard_normal((16, 40)).astype(np.float32)
    cond = rng.standard_normal((16, 40)).astype(np.float32)
    rows = port.assemble_dit_input(lat, cond)
    assert np.array_equal(rows[:, :16], lat.T) and np.array_equal(rows[:, 16:32], cond.T)
    assert (rows[:, 32] == 1).all()
    pred = rng.standard_normal((40, 16)).astype(np.float32)
    upd = port.euler_update(lat, pred, np.float32(-0.25))
    assert np.array_equal(upd, lat + np.float32(-0.25) * pred.T)
