"""CPU: pins the oracle (our C restatement) against the golden fixtures made
by the reference's own layer code, and against that code directly where it
is built."""
import numpy as np
import pytest

from oracle import oracle

PLAN_KEYS = ("windows", "sample_window_count", "video_indices", "inverse_video_indices", "local_positions")


def _plan_cases(golden):
    g = golden["plans"]
    return sorted({k.split("__")[0] for k in g.files})


def test_port_plans_match_golden(port, golden):
    import hashlib

    g = golden["plans"]
    cases = _plan_cases(golden)
    assert len(cases) >= 20
    for case in cases:
        shapes = g[f"{case}__shapes"]
        target = g[f"{case}__target"]
        shifted = int(case.endswith("_s1"))
        p = port.plan(shapes, target, shifted, mode=oracle.WINDOW_TARGET)
        np.testing.assert_array_equal(p.windows, g[f"{case}__windows"], err_msg=case)
        np.testing.assert_array_equal(p.sample_window_count, g[f"{case}__sample_window_count"], err_msg=case)
        for name in ("video_indices", "inverse_video_indices", "local_positions"):
            arr = getattr(p, name)
            digest = hashlib.sha256(np.ascontiguousarray(arr, np.int32).tobytes()).hexdigest()
            assert digest == bytes(g[f"{case}__sha_{name}"]).decode(), (case, name)
            if f"{case}__{name}" in g.files:
                np.testing.assert_array_equal(arr, g[f"{case}__{name}"], err_msg=case)


def test_port_awa_matches_golden(port, golden):
    g = golden["awa"]
    for shifted in (0, 1):
        for bf16 in (0, 1):
            vo, to = port.awa_forward(heads=int(g["heads"]), head_dim=int(g["head_dim"]), window=g["target"],
                                      shifted=shifted, eps=float(g["eps"]), rope_pairs=int(g["rope_pairs"]),
                                      norms=g["norms"], freqs=g["freqs"], shapes=g["shapes"],
                                      text_lengths=g["text_lengths"], video_qkv=g["video_qkv"],
                                      text_qkv=g["text_qkv"], bf16=bool(bf16))
            np.testing.assert_allclose(vo, g[f"video_out_s{shifted}_b{bf16}"], rtol=0, atol=2e-6)
            np.testing.assert_allclose(to, g[f"text_out_s{shifted}_b{bf16}"], rtol=0, atol=2e-6)


def test_port_awa_split_equals_fused(port, golden):
    g = golden["awa"]
    inner = int(g["heads"]) * int(g["head_dim"])
    v, t = g["video_qkv"], g["text_qkv"]
    split = [v[:, :inner], v[:, inner:2 * inner], v[:, 2 * inner:], t[:, :inner], t[:, inner:2 * inner],
             t[:, 2 * inner:]]
    kw = dict(heads=int(g["heads"]), head_dim=int(g["head_dim"]), window=g["target"], shifted=1,
              eps=float(g["eps"]), rope_pairs=int(g["rope_pairs"]), norms=g["norms"], freqs=g["freqs"],
              shapes=g["shapes"], text_lengths=g["text_lengths"])
    a = port.awa_forward(video_qkv=v, text_qkv=t, **kw)
    b = port.awa_forward(split=split, **kw)
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[1], b[1])


def test_port_linear_matches_golden(port, golden):
    g = golden["linear"]
    np.testing.assert_allclose(port.linear(g["video"], g["weight"], g["bias"]), g["video_out_bias"], atol=1e-5)
    np.testing.assert_allclose(port.linear(g["text"], g["weight"], g["bias"]), g["text_out_bias"], atol=1e-5)
    np.testing.assert_allclose(port.linear(g["video"], g["weight"]), g["video_out_nobias"], atol=1e-5)


def test_round_bf16_c_vs_numpy(port):
    rng = np.random.default_rng(5)
    x = np.concatenate([rng.standard_normal(2000).astype(np.float32) * 10.0 ** rng.integers(-30, 30, 2000),
                        np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 3.3895314e38, 1e-45], np.float32)])
    x = x.astype(np.float32)
    c = np.array([port.lib.s2o_round_bf16(float(v)) for v in x], np.float32)
    n = port.round_bf16(x)
    np.testing.assert_array_equal(c.view(np.uint32), n.view(np.uint32))


def test_plan_invariants_random(port):
    """Coverage / inverse permutation (adaptive_window_attention.cpp:642-653) on ragged shapes, both modes."""
    rng = np.random.default_rng(11)
    for _ in range(300):
        shapes = rng.integers(1, 40, size=(int(rng.integers(1, 4)), 3))
        win = rng.integers(1, 9, size=3)
        mode = int(rng.integers(0, 2))
        shifted = int(rng.integers(0, 2))
        p = port.plan(shapes, win, shifted, mode=mode)
        n = int(np.prod(shapes, axis=1).sum())
        assert sorted(p.video_indices.tolist()) == list(range(n))
        np.testing.assert_array_equal(p.video_indices[p.inverse_video_indices], np.arange(n))
        assert p.windows[:, 8].sum() == n
        assert (p.windows[:, 8] > 0).all()


def test_plan_rejects_bad_shapes(port):
    for shapes, win in (([[0, 4, 4]], [1, 1, 1]), ([[1, 4, 4]], [0, 1, 1]), ([[1, -3, 4]], [1, 1, 1])):
        with pytest.raises(ValueError):
            port.plan(shapes, win, 0)


def test_port_vs_reference_random(port, ref):
    """Our restatement is bit-identical with the reference's own code (plan and AWA)."""
    rng = np.random.default_rng(3)
    for _ in range(400):
        shape = [int(rng.integers(1, 30)), int(rng.integers(1, 120)), int(rng.integers(1, 200))]
        tgt = [int(v) for v in rng.integers(1, 8, 3)]
        sh = int(rng.integers(0, 2))
        a = ref.plan([shape], tgt, sh)
        b = port.plan([shape], tgt, sh)
        for k in PLAN_KEYS:
            np.testing.assert_array_equal(a.as_dict()[k], b.as_dict()[k])
    heads, hd = 3, 128
    shapes = np.array([[2, 5, 7], [1, 3, 9]], np.int32)
    tl = np.array([4, 7], np.int32)
    nv, nt = int(np.prod(shapes, axis=1).sum()), int(tl.sum())
    vq = rng.standard_normal((nv, 3 * heads * hd)).astype(np.float32)
    tq = rng.standard_normal((nt, 3 * heads * hd)).astype(np.float32)
    norms = (1 + 0.02 * rng.standard_normal((4, hd))).astype(np.float32)
    fr = (1.0 / 10000 ** (np.arange(20) * 2 / 40)).astype(np.float32)
    for sh in (0, 1):
        for bf in (0, 1):
            kw = dict(heads=heads, head_dim=hd, shifted=sh, eps=1e-5, rope_pairs=20, norms=norms, freqs=fr,
                      shapes=shapes, text_lengths=tl, video_qkv=vq, text_qkv=tq, bf16=bool(bf))
            a = ref.awa_forward(target=[2, 1, 3], **kw)
            b = port.awa_forward(window=[2, 1, 3], **kw)
            np.testing.assert_array_equal(a[0], b[0])
            np.testing.assert_array_equal(a[1], b[1])


def test_reference_error_codes(ref):
    """forward() validation codes (adaptive_window_attention.cpp:766-831) seen through the ncnn surface."""
    heads, hd = 1, 128
    norms = np.ones((4, hd), np.float32)
    fr = np.ones(21, np.float32)
    vq = np.zeros((4, 3 * hd), np.float32)
    tq = np.zeros((2, 3 * hd), np.float32)
    with pytest.raises(ValueError, match="-1"):
        ref.awa_forward(heads=heads, head_dim=hd, target=[1, 1, 1], shifted=0, eps=1e-5, rope_pairs=22, norms=norms,
                        freqs=np.ones(22, np.float32), shapes=[[1, 2, 2]], text_lengths=[2], video_qkv=vq,
                        text_qkv=tq)
    with pytest.raises(ValueError, match="-1"):
        ref.awa_forward(heads=heads, head_dim=hd, target=[1, 1, 1], shifted=0, eps=1e-5, rope_pairs=21, norms=norms,
                        freqs=fr, shapes=[[1, 2, 3]], text_lengths=[2], video_qkv=vq, text_qkv=tq)


def test_block_oracle_bf16_emulation_close(port):
    """The block restatement with bf16 activation rounding stays within the
    per-block tolerance of the fp32 one (sanity of the tolerance itself)."""
    from tests.conftest import cosine, rel_maxabs

    rng = np.random.default_rng(7)
    D, heads, hd, F, pairs = 256, 2, 128, 512, 21
    shapes, tl = [[1, 6, 8]], [5]
    w = dict(ada=(rng.standard_normal((6, D)) / np.sqrt(D) + np.array([0, 1, 0, 0, 1, 0])[:, None]),
             w_qkv=0.02 * rng.standard_normal((3 * D, D)), b_qkv=0.02 * rng.standard_normal(3 * D),
             w_out=0.02 * rng.standard_normal((D, D)), b_out=0.02 * rng.standard_normal(D),
             w_up=0.02 * rng.standard_normal((F, D)), b_up=0.02 * rng.standard_normal(F),
             w_down=0.02 * rng.standard_normal((D, F)), b_down=0.02 * rng.standard_normal(D),
             qk_norm=1 + 0.02 * rng.standard_normal((4, hd)),
             freqs=1.0 / 10000 ** (np.arange(pairs) * 2 / (2 * pairs)))
    mod = rng.standard_normal((1, 6, D))
    xv = rng.standard_normal((48, D))
    xt = rng.standard_normal((5, D))
    dims = [D, heads, hd, F, pairs, oracle.WINDOW_EXTENT, 1, 3, 4, 1]
    a = port.block_forward(dims=dims, eps_norm=1e-5, eps_qk=1e-5, weights=w, modulation=mod, shapes=shapes,
                           text_lengths=tl, x_video=xv, x_text=xt)
    b = port.block_forward(dims=dims, eps_norm=1e-5, eps_qk=1e-5, weights=w, modulation=mod, shapes=shapes,
                           text_lengths=tl, x_video=xv, x_text=xt, emulate_bf16=True)
    for x, y in zip(b, a):
        assert cosine(x, y) >= 0.9995
        assert rel_maxabs(x, y) <= 2e-2


@pytest.mark.parametrize("layer", [0, 1])
def test_block_oracle_norm_forms_vs_numpy(port, layer):
    """The block restatement's two AdaLN forms (RMSNorm, LayerNorm; no affine) against numpy glue in float64
    around the restatement's own attention: h = norm(x) * scale + shift, QKV, AWA, out + gate residual,
    norm, up, GELU-tanh, down + gate residual."""
    rng = np.random.default_rng(11 + layer)
    D, heads, hd, F, pairs = 256, 2, 128, 512, 21
    shapes, tl = [[1, 6, 8]], [5]
    w = dict(ada=(rng.standard_normal((6, D)) / np.sqrt(D) + np.array([0, 1, 0, 0, 1, 0])[:, None]),
             w_qkv=0.02 * rng.standard_normal((3 * D, D)), b_qkv=0.02 * rng.standard_normal(3 * D),
             w_out=0.02 * rng.standard_normal((D, D)), b_out=0.02 * rng.standard_normal(D),
             w_up=0.02 * rng.standard_normal((F, D)), b_up=0.02 * rng.standard_normal(F),
             w_down=0.02 * rng.standard_normal((D, F)), b_down=0.02 * rng.standard_normal(D),
             qk_norm=1 + 0.02 * rng.standard_normal((4, hd)),
             freqs=1.0 / 10000 ** (np.arange(pairs) * 2 / (2 * pairs)))
    mod = rng.standard_normal((1, 6, D))
    xv = rng.standard_normal((48, D)) + 3.0 * rng.standard_normal((48, 1))  # row offsets: mean matters
    xt = rng.standard_normal((5, D))
    dims = [D, heads, hd, F, pairs, oracle.WINDOW_EXTENT, 1, 3, 4, 1, layer]
    gv, gt = port.block_forward(dims=dims, eps_norm=1e-5, eps_qk=1e-5, weights=w, modulation=mod, shapes=shapes,
                                text_lengths=tl, x_video=xv, x_text=xt)

    m = mod[0] + w["ada"]
    x = np.concatenate([xv, xt]).astype(np.float64)

    def norm(x, k):
        c = x - x.mean(1, keepdims=True) if layer else x
        return c / np.sqrt((c * c).mean(1, keepdims=True) + 1e-5) * m[k + 1] + m[k]

    h = norm(x, 0)
    qkv = h @ w["w_qkv"].T + w["b_qkv"]
    cv, ct = port.awa_forward(heads=heads, head_dim=hd, window=[1, 3, 4], shifted=1, eps=1e-5, rope_pairs=pairs,
                              norms=w["qk_norm"], freqs=w["freqs"], shapes=shapes, text_lengths=tl,
                              video_qkv=qkv[:48], text_qkv=qkv[48:], mode=oracle.WINDOW_EXTENT)
    x = x + (np.concatenate([cv, ct]) @ w["w_out"].T + w["b_out"]) * m[2]
    u = norm(x, 3) @ w["w_up"].T + w["b_up"]
    u = 0.5 * u * (1 + np.tanh(0.7978845608028654 * (u + 0.044715 * u ** 3)))
    x = x + (u @ w["w_down"].T + w["b_down"]) * m[5]
    np.testing.assert_allclose(np.concatenate([gv, gt]), x, rtol=2e-4, atol=2e-4)
