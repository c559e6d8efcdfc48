"""GPU parity of the individual kernels, called through the C ABI.

SharedLinear and the norm pass are floating-point kernels and are checked
against a plain torch fp32 computation on the same bf16 inputs.  The window
attention is checked against the golden fixtures written by the reference's
own layer code and against the CPU oracle.  Gates (north star): cosine
>= 0.9995 and max|gpu - ref| / max|ref| <= 2e-2.
"""
import numpy as np
import pytest

from tests.conftest import cosine, rel_maxabs

pytestmark = pytest.mark.gpu

COS_MIN = 0.9995
REL_MAX = 2e-2


def _t(a, dtype=None):
    import torch

    t = torch.as_tensor(np.ascontiguousarray(a)).cuda()
    return t.to(dtype) if dtype is not None else t


def _ref_linear(a, w, bias):
    out = a.float() @ w.float().T
    return out + bias if bias is not None else out


@pytest.mark.parametrize("M0,M1,N,K", [(300, 0, 512, 256), (1, 0, 256, 64), (257, 58, 520, 136), (129, 3, 8, 72),
                                       (1000, 0, 2560, 2560), (5000, 333, 2600, 192),
                                       # one GPU's rows of an 8-GPU 720p step; the long-K gate-residual case
                                       # runs as split-K CTA pairs (two half-K units reduce-added into the output)
                                       (2758, 0, 2560, 2560), (2500, 58, 2560, 10240),
                                       # 79 pair tiles for 74 pairs: a narrow tail of 256 x 128 units whose
                                       # second halves lie wholly past N
                                       (20000, 0, 8, 64)])
@pytest.mark.parametrize("epi", ["store_bf16", "store_f32", "gelu", "gate_residual"])
def test_shared_linear_vs_torch(gpu_ctx, s2lib, M0, M1, N, K, epi):
    import torch

    g = torch.Generator(device="cuda").manual_seed(M0 * 7 + N + K)
    a0 = torch.randn(M0, K, device="cuda", generator=g).bfloat16()
    a1 = torch.randn(M1, K, device="cuda", generator=g).bfloat16() if M1 else None
    w = (0.05 * torch.randn(N, K, device="cuda", generator=g)).bfloat16()
    bias = 0.1 * torch.randn(N, device="cuda", generator=g)
    gate = torch.randn(N, device="cuda", generator=g)
    outs = []
    for a in ([a0] + ([a1] if a1 is not None else [])):
        outs.append(_ref_linear(a, w, bias))
    if epi == "store_bf16":
        o0, o1 = s2lib.shared_linear(gpu_ctx, a0, w, bias, a1=a1, out_dtype=s2lib.S2_DTYPE_BF16)
        refs = outs
    elif epi == "store_f32":
        o0, o1 = s2lib.shared_linear(gpu_ctx, a0, w, bias, a1=a1, out_dtype=s2lib.S2_DTYPE_F32)
        refs = outs
    elif epi == "gelu":
        o0, o1 = s2lib.shared_linear(gpu_ctx, a0, w, bias, a1=a1, epilogue=s2lib.S2_EPI_GELU_TANH)
        refs = [torch.nn.functional.gelu(o, approximate="tanh") for o in outs]
    else:
        r0 = torch.randn(M0, N, device="cuda", generator=g)
        r1 = torch.randn(M1, N, device="cuda", generator=g) if M1 else None
        refs = [r0 + outs[0] * gate] + ([r1 + outs[1] * gate] if M1 else [])
        o0, o1 = s2lib.shared_linear(gpu_ctx, a0, w, bias, a1=a1, epilogue=s2lib.S2_EPI_GATE_RESIDUAL, gate=gate,
                                     out_dtype=s2lib.S2_DTYPE_F32, out0=r0, out1=r1)
    torch.cuda.synchronize()
    assert gpu_ctx.status() == 0
    got = [o0] + ([o1] if M1 else [])
    for x, y in zip(got, refs):
        x = x.float().cpu().numpy()
        y = y.float().cpu().numpy()
        assert cosine(x, y) >= 0.9999
        assert rel_maxabs(x, y) <= 1e-2


@pytest.mark.parametrize("M0,M1", [(2758, 0), (2500, 58)])
def test_split_k_gate_residual_reproducible(gpu_ctx, s2lib, M0, M1):
    """Split-K units (K = 10240 at these M: 110 CTA-pair tiles for 74 pairs,
    run as 220 half-K units) reduce-add both halves into the fp32 residual;
    the second half waits for the first, so repeated runs agree bit for bit
    (the 8-GPU step relies on it for the text rows every rank computes)."""
    import torch

    g = torch.Generator(device="cuda").manual_seed(5)
    N, K = 2560, 10240
    a0 = torch.randn(M0, K, device="cuda", generator=g).bfloat16()
    a1 = torch.randn(M1, K, device="cuda", generator=g).bfloat16() if M1 else None
    w = (0.05 * torch.randn(N, K, device="cuda", generator=g)).bfloat16()
    bias = 0.1 * torch.randn(N, device="cuda", generator=g)
    gate = torch.randn(N, device="cuda", generator=g)
    r0 = torch.randn(M0, N, device="cuda", generator=g)
    r1 = torch.randn(M1, N, device="cuda", generator=g) if M1 else None
    runs = []
    for _ in range(6):
        o0, o1 = r0.clone(), (r1.clone() if M1 else None)
        s2lib.shared_linear(gpu_ctx, a0, w, bias, a1=a1, epilogue=s2lib.S2_EPI_GATE_RESIDUAL, gate=gate,
                            out_dtype=s2lib.S2_DTYPE_F32, out0=o0, out1=o1)
        runs.append(torch.cat([o0] + ([o1] if M1 else [])))
    torch.cuda.synchronize()
    assert gpu_ctx.status() == 0
    for x in runs[1:]:
        assert torch.equal(x, runs[0])


def test_shared_linear_full_width_qkv(gpu_ctx, s2lib):
    """720p QKV projection shape (M = 21600 + 58, N = 7680, K = 2560), rows sampled."""
    import torch

    g = torch.Generator(device="cuda").manual_seed(1)
    M, N, K = 21658, 7680, 2560
    a = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = (0.02 * torch.randn(N, K, device="cuda", generator=g)).bfloat16()
    bias = 0.02 * torch.randn(N, device="cuda", generator=g)
    out, _ = s2lib.shared_linear(gpu_ctx, a, w, bias)
    rows = torch.cat([torch.arange(0, 256), torch.arange(M - 300, M), torch.randint(0, M, (512,), generator=None)])
    rows = rows.cuda()
    ref = _ref_linear(a[rows], w, bias)
    x, y = out[rows].float().cpu().numpy(), ref.cpu().numpy()
    assert cosine(x, y) >= 0.9999 and rel_maxabs(x, y) <= 1e-2


def test_ada_rmsnorm_vs_torch(gpu_ctx, s2lib):
    import torch

    g = torch.Generator(device="cuda").manual_seed(2)
    for rows, D in ((1, 8), (333, 2560), (58, 512)):
        x = 3 * torch.randn(rows, D, device="cuda", generator=g)
        shift = torch.randn(D, device="cuda", generator=g)
        scale = torch.randn(D, device="cuda", generator=g)
        y = s2lib.ada_rmsnorm(gpu_ctx, x, 1e-5, shift, scale)
        ref = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-5) * scale + shift
        np.testing.assert_allclose(y.float().cpu().numpy(), ref.cpu().numpy(), rtol=1e-2, atol=2e-2)


def test_ada_layernorm_vs_torch(gpu_ctx, s2lib):
    """The LayerNorm form of the AdaLN pass against torch's fp32 layer_norm (no affine), then scale + shift;
    rows with a large common offset check that the variance is taken about the mean."""
    import torch

    g = torch.Generator(device="cuda").manual_seed(3)
    for rows, D in ((1, 8), (333, 2560), (58, 512), (17, 2000)):
        x = 3 * torch.randn(rows, D, device="cuda", generator=g) + 20 * torch.randn(rows, 1, device="cuda",
                                                                                 generator=g)
        shift = torch.randn(D, device="cuda", generator=g)
        scale = torch.randn(D, device="cuda", generator=g)
        y = s2lib.ada_layernorm(gpu_ctx, x, 1e-5, shift, scale)
        ref = torch.nn.functional.layer_norm(x, (D,), eps=1e-5) * scale + shift
        np.testing.assert_allclose(y.float().cpu().numpy(), ref.cpu().numpy(), rtol=1e-2, atol=2e-2)


def _awa_kwargs(g):
    return dict(heads=int(g["heads"]), head_dim=int(g["head_dim"]), window=[int(v) for v in g["target"]],
                window_mode=0, eps=float(g["eps"]), rope_pairs=int(g["rope_pairs"]),
                shapes=g["shapes"].tolist(), text_lengths=g["text_lengths"].tolist())


@pytest.mark.parametrize("shifted", [0, 1])
@pytest.mark.parametrize("bf16", [0, 1])
def test_awa_vs_golden(gpu_ctx, s2lib, golden, shifted, bf16):
    """2-sample batch, text lengths 5/3, ragged windows: GPU vs the reference's own CPU forward."""
    g = golden["awa"]
    kw = _awa_kwargs(g)
    vo, to = s2lib.awa_forward(gpu_ctx, shifted=shifted, norms=_t(g["norms"]), freqs=_t(g["freqs"]),
                               video_qkv=_t(g["video_qkv"]), text_qkv=_t(g["text_qkv"]), official_bf16=bool(bf16),
                               **kw)
    assert gpu_ctx.status() == 0
    for got, key in ((vo, f"video_out_s{shifted}_b{bf16}"), (to, f"text_out_s{shifted}_b{bf16}")):
        got = got.cpu().numpy()
        ref = g[key]
        assert cosine(got, ref) >= COS_MIN, key
        assert rel_maxabs(got, ref) <= REL_MAX, key


def test_awa_split_bf16_inputs(gpu_ctx, s2lib, golden):
    """8-blob (split) form with bf16 inputs and bf16 outputs equals the fused fp32 form within bf16."""
    import torch

    g = golden["awa"]
    kw = _awa_kwargs(g)
    inner = kw["heads"] * kw["head_dim"]
    v = _t(g["video_qkv"])
    t = _t(g["text_qkv"])
    split = [x.bfloat16().contiguous() for x in (v[:, :inner], v[:, inner:2 * inner], v[:, 2 * inner:],
                                                   t[:, :inner], t[:, inner:2 * inner], t[:, 2 * inner:])]
    a = s2lib.awa_forward(gpu_ctx, shifted=1, norms=_t(g["norms"]), freqs=_t(g["freqs"]), split=split,
                          out_dtype=s2lib.S2_DTYPE_BF16, **kw)
    b = s2lib.awa_forward(gpu_ctx, shifted=1, norms=_t(g["norms"]), freqs=_t(g["freqs"]),
                          video_qkv=v.bfloat16(), text_qkv=t.bfloat16(), **kw)
    for x, y in zip(a, b):
        assert cosine(x.float().cpu().numpy(), y.cpu().numpy()) >= 0.9999
    torch.cuda.synchronize()


@pytest.mark.parametrize("shape,window,shifted,heads", [
    ([1, 32, 32], [1, 16, 16], 0, 20),    # BASELINE config 1 geometry, full width
    ([1, 64, 64], [1, 16, 16], 1, 2),     # config 2 shifted: 25 windows of 64..256 tokens
    ([2, 15, 20], [2, 15, 20], 0, 2),     # one 600-token window (720p window, 5 kv tiles + text)
    ([3, 7, 11], [2, 3, 4], 1, 3),        # odd extents, tiny shifted boundary windows
    # BASELINE config 4 sweep of window lengths L (video tokens per window; + 58 text rows)
    ([2, 16, 16], [1, 8, 8], 0, 2),       # L = 64: 8 windows of one query tile each
    ([1, 32, 32], [1, 16, 16], 1, 2),     # L = 256 shifted: 9 windows of 64..256 tokens
    ([1, 32, 64], [1, 32, 64], 0, 2),     # L = 2048: 17 key tiles, 9 query-tile pairs
])
def test_awa_vs_oracle_explicit_windows(gpu_ctx, s2lib, port, shape, window, shifted, heads):
    from oracle import oracle

    rng = np.random.default_rng(sum(shape) + heads)
    hd, T, pairs = 128, 58, 21
    inner = heads * hd
    nv = int(np.prod(shape))
    vq = rng.standard_normal((nv, 3 * inner)).astype(np.float32)
    tq = rng.standard_normal((T, 3 * inner)).astype(np.float32)
    norms = (1 + 0.02 * rng.standard_normal((4, hd))).astype(np.float32)
    freqs = (1.0 / 10000 ** (np.arange(pairs) * 2 / 42)).astype(np.float32)
    ref_v, ref_t = port.awa_forward(heads=heads, head_dim=hd, window=window, shifted=shifted, eps=1e-5,
                                    rope_pairs=pairs, norms=norms, freqs=freqs, shapes=[shape], text_lengths=[T],
                                    video_qkv=vq, text_qkv=tq, mode=oracle.WINDOW_EXTENT)
    vo, to = s2lib.awa_forward(gpu_ctx, heads=heads, head_dim=hd, window=window,
                               window_mode=s2lib.S2_WINDOW_EXTENT, shifted=shifted, eps=1e-5, rope_pairs=pairs,
                               norms=_t(norms), freqs=_t(freqs), shapes=[shape], text_lengths=[T],
                               video_qkv=_t(vq), text_qkv=_t(tq))
    assert gpu_ctx.status() == 0
    for got, ref in ((vo.cpu().numpy(), ref_v), (to.cpu().numpy(), ref_t)):
        assert cosine(got, ref) >= COS_MIN
        assert rel_maxabs(got, ref) <= REL_MAX


def test_awa_rejects_bad_args(gpu_ctx, s2lib, golden):
    g = golden["awa"]
    kw = _awa_kwargs(g)
    kw["rope_pairs"] = 22  # 6 * 22 > 128 (adaptive_window_attention.cpp:769)
    with pytest.raises(s2lib.S2Error) as e:
        s2lib.awa_forward(gpu_ctx, shifted=0, norms=_t(g["norms"]), freqs=_t(np.ones(22, np.float32)),
                          video_qkv=_t(g["video_qkv"]), text_qkv=_t(g["text_qkv"]), **kw)
    assert e.value.code == s2lib.S2_ERR_INVALID
    kw = _awa_kwargs(g)
    kw["text_lengths"] = [5, 0]
    with pytest.raises(s2lib.S2Error):
        s2lib.awa_forward(gpu_ctx, shifted=0, norms=_t(g["norms"]), freqs=_t(g["freqs"]),
                          video_qkv=_t(g["video_qkv"]), text_qkv=_t(g["text_qkv"]), **kw)


def test_counters(gpu_ctx, s2lib, golden):
    g = golden["awa"]
    gpu_ctx.profile(True)
    s2lib.awa_forward(gpu_ctx, shifted=0, norms=_t(g["norms"]), freqs=_t(g["freqs"]), video_qkv=_t(g["video_qkv"]),
                      text_qkv=_t(g["text_qkv"]), **_awa_kwargs(g))
    c = gpu_ctx.counters()
    gpu_ctx.profile(False)
    assert c["window_attention"]["launches"] == 1 and c["window_attention"]["ms"] > 0
    assert c["window_attention"]["flops"] > 0
    assert c["prepare_qkv"]["launches"] == 1 and c["text_pool"]["launches"] == 1
