"""s2_awa_forward_static -- the AdaptiveWindowAttention forward for callers
that cannot allocate device memory (plugins whose host owns all device
memory, processes under a hard memory cap, loops that must not risk the
device-wide synchronisation of cudaMalloc/cudaFree).  Its scratch is one
static device array inside the library.

This file is collected last on purpose: it runs after every other test (and
also passes alone in a fresh process).  It calls the entry point through the
C ABI twice in a row with different inputs -- so the second call sees the
first call's leftovers in the shared scratch -- and checks each result
against the allocating s2_awa_forward within the tolerance the other
attention tests use (cosine >= 0.9995, max|a-b|/max|b| <= 2e-2; the two
paths run the same kernels, so they should in fact agree exactly).
"""
import ctypes as C

import numpy as np
import pytest

from tests.conftest import cosine, rel_maxabs

pytestmark = pytest.mark.gpu

S2_STATIC_BYTES = 64 << 20  # S2_AWA_STATIC_SCRATCH_BYTES


def _case(rng, heads, shape, T):
    inner = heads * 128
    nv = int(np.prod(shape))
    return (rng.standard_normal((nv, 3 * inner)).astype(np.float32),
            rng.standard_normal((T, 3 * inner)).astype(np.float32),
            (1 + 0.02 * rng.standard_normal((4, 128))).astype(np.float32))


def _static_call(abi, prm, shapes, tls, vq, tq, inner, out_dtype, vo, to, stream):
    flat = [int(v) for s in shapes for v in s]
    esz = vq.element_size()
    in_dtype = abi.S2_DTYPE_BF16 if esz == 2 else abi.S2_DTYPE_F32
    v0, t0 = vq.data_ptr(), tq.data_ptr()
    return abi.lib().s2_awa_forward_static(
        C.byref(prm), (C.c_int * len(flat))(*flat), (C.c_int * len(tls))(*tls), len(shapes), in_dtype,
        v0, v0 + inner * esz, v0 + 2 * inner * esz, vq.stride(0), t0, t0 + inner * esz, t0 + 2 * inner * esz,
        tq.stride(0), out_dtype, vo.data_ptr(), to.data_ptr(), stream)


def test_static_scratch_entry_matches_allocating_entry():
    import torch

    from seedvr2_ncnn_b200 import abi

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    ctx = abi.Context(0)
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(77)
    freqs = torch.from_numpy((1.0 / 10000 ** (np.arange(21) * 2 / 42)).astype(np.float32)).cuda()
    # two different calls: 2-sample shifted batch (fp32 in/out), then a 20-head
    # 1x32x32 video with 58 text tokens (bf16 in/out)
    cases = [
        dict(heads=3, shapes=[[2, 9, 14], [1, 5, 7]], tls=[6, 11], window=[2, 4, 5], mode=abi.S2_WINDOW_EXTENT,
             shifted=1, dtype=torch.float32, out=abi.S2_DTYPE_F32),
        dict(heads=20, shapes=[[1, 32, 32]], tls=[58], window=[4, 3, 3], mode=abi.S2_WINDOW_TARGET, shifted=0,
             dtype=torch.bfloat16, out=abi.S2_DTYPE_BF16),
    ]
    for call, cs in enumerate(cases):
        heads, inner = cs["heads"], cs["heads"] * 128
        vq_np, tq_np, norms_np = _case(rng, heads, [sum(int(np.prod(s)) for s in cs["shapes"])], sum(cs["tls"]))
        vq = torch.from_numpy(vq_np).cuda().to(cs["dtype"])
        tq = torch.from_numpy(tq_np).cuda().to(cs["dtype"])
        norms = torch.from_numpy(norms_np).cuda()
        ref_v, ref_t = abi.awa_forward(ctx, heads=heads, head_dim=128, window=cs["window"], window_mode=cs["mode"],
                                       shifted=cs["shifted"], eps=1e-5, rope_pairs=21, norms=norms, freqs=freqs,
                                       shapes=cs["shapes"], text_lengths=cs["tls"], video_qkv=vq, text_qkv=tq,
                                       out_dtype=cs["out"])
        prm = abi.AwaParams()
        prm.heads, prm.head_dim = heads, 128
        prm.window[:] = cs["window"]
        prm.window_mode, prm.shifted, prm.epsilon, prm.rope_pairs = cs["mode"], cs["shifted"], 1e-5, 21
        prm.official_bf16_attention = 0
        prm.norm_weights, prm.rope_freqs = norms.data_ptr(), freqs.data_ptr()
        odt = torch.float32 if cs["out"] == abi.S2_DTYPE_F32 else torch.bfloat16
        vo = torch.full_like(ref_v, float("nan"), dtype=odt)
        to = torch.full_like(ref_t, float("nan"), dtype=odt)
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        r = _static_call(abi, prm, cs["shapes"], cs["tls"], vq, tq, inner, cs["out"], vo, to, stream)
        assert r == abi.S2_OK, abi.error_string(r)
        # the call only enqueues: device-side failures are read back here
        assert abi.lib().s2_awa_static_status(stream) == abi.S2_OK
        torch.cuda.synchronize()
        if call > 0:
            # the first call may load the library's module (and with it the
            # static array); later calls take no device memory at all
            assert torch.cuda.mem_get_info()[0] == free_before
        for got, ref in ((vo, ref_v), (to, ref_t)):
            g, f = got.float().cpu().numpy(), ref.float().cpu().numpy()
            assert np.isfinite(g).all()
            assert cosine(g, f) >= 0.9995
            assert rel_maxabs(g, f) <= 2e-2
    assert ctx.status() == 0

    # a call past the fixed scratch is rejected without touching the GPU
    big = torch.zeros((1, 3 * 20 * 128), device="cuda")
    prm.heads = 20
    r = abi.lib().s2_awa_forward_static(
        C.byref(prm), (C.c_int * 3)(8, 64, 64), (C.c_int * 1)(58), 1, abi.S2_DTYPE_F32, big.data_ptr(),
        big.data_ptr(), big.data_ptr(), 3 * 2560, big.data_ptr(), big.data_ptr(), big.data_ptr(), 3 * 2560,
        abi.S2_DTYPE_F32, big.data_ptr(), big.data_ptr(), stream)
    assert r == abi.S2_ERR_TOO_LARGE
    ctx.close()


def test_static_planner_matches_allocating_planner(golden):
    """The static entry point builds its window plan with its own heap-free walk.  On every golden plan
    shape that fits the fixed scratch (the reference's target-count windows, shifted and unshifted, ragged
    and 2-sample cases), its outputs must equal the allocating entry point's bit for bit: both run the
    same kernels, so any difference in a window, a token's position or its RoPE coordinates would show."""
    import torch

    from seedvr2_ncnn_b200 import abi

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    ctx = abi.Context(0)
    stream = torch.cuda.current_stream().cuda_stream
    g = golden["plans"]
    rng = np.random.default_rng(5)
    heads, inner, T = 1, 128, 7
    freqs = torch.from_numpy((1.0 / 10000 ** (np.arange(21) * 2 / 42)).astype(np.float32)).cuda()
    norms = torch.from_numpy((1 + 0.02 * rng.standard_normal((4, 128))).astype(np.float32)).cuda()
    checked = 0
    for case in sorted({k.split("__")[0] for k in g.files}):
        shapes = g[f"{case}__shapes"].tolist()
        target = g[f"{case}__target"].tolist()
        shifted = int(case.endswith("_s1"))
        nv = sum(int(np.prod(s)) for s in shapes)
        nw = int(g[f"{case}__windows"].shape[0])
        if (nv + nw * T) * inner * 2 * 3 + nw * T * inner * 4 > (S2_STATIC_BYTES * 3) // 4:
            continue
        tls = [T] * len(shapes)
        vq = torch.from_numpy(rng.standard_normal((nv, 3 * inner)).astype(np.float32)).cuda().to(torch.bfloat16)
        tq = torch.from_numpy(rng.standard_normal((T * len(shapes), 3 * inner)).astype(np.float32)).cuda().to(
            torch.bfloat16)
        ref_v, ref_t = abi.awa_forward(ctx, heads=heads, head_dim=128, window=target,
                                       window_mode=abi.S2_WINDOW_TARGET, shifted=shifted, eps=1e-5, rope_pairs=21,
                                       norms=norms, freqs=freqs, shapes=shapes, text_lengths=tls, video_qkv=vq,
                                       text_qkv=tq, out_dtype=abi.S2_DTYPE_F32)
        prm = abi.AwaParams()
        prm.heads, prm.head_dim = heads, 128
        prm.window[:] = target
        prm.window_mode, prm.shifted, prm.epsilon, prm.rope_pairs = abi.S2_WINDOW_TARGET, shifted, 1e-5, 21
        prm.official_bf16_attention = 0
        prm.norm_weights, prm.rope_freqs = norms.data_ptr(), freqs.data_ptr()
        vo = torch.full_like(ref_v, float("nan"))
        to = torch.full_like(ref_t, float("nan"))
        torch.cuda.synchronize()
        r = _static_call(abi, prm, shapes, tls, vq, tq, inner, abi.S2_DTYPE_F32, vo, to, stream)
        assert r == abi.S2_OK, (case, abi.error_string(r))
        assert abi.lib().s2_awa_static_status(stream) == abi.S2_OK, case
        assert torch.equal(vo, ref_v), case
        assert torch.equal(to, ref_t), case
        checked += 1
    assert checked >= 8
    assert ctx.status() == 0
    ctx.close()
