"""GPU parity of the DiT input/output formats and the frontend / tail nets
(through the C ABI) against the reference's own code (golden fixture) and the
CPU oracle.

Gates:
* patchify / unpatchify: bit-exact (pure copies); error codes identical.
* timestep embedding: the phase is the reference's fp32 product (host-made
  frequencies), so only sinf/cosf rounding differs: |gpu - ref| <= 5e-7.
* frontend / tail with the oracle emulating the device's bf16 activations and
  bf16-valued weights: rel max-abs <= 1e-3 (video, text, prediction),
  <= 1e-4 (modulation, an fp32 matrix-vector chain); at 720p also against the
  plain fp32 oracle (fp32 activations): the block gate below.
* whole DiT step (frontend, blocks, tail) vs the oracle chain in fp32: the
  block gate, cosine >= 0.9995 and rel max-abs <= 2e-2.
"""
import numpy as np
import pytest

from tests.conftest import cosine, rel_maxabs
from tests.golden.gen_golden import DIT_IO_CASES, DIT_IO_ERRORS

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _bf16(port, a):
    return port.round_bf16(np.asarray(a, np.float32))


def make_io_weights(rng, port, D, bias=True):
    n = lambda *s: _bf16(port, 0.02 * rng.standard_normal(s))  # noqa: E731
    b = lambda *s: (0.02 * rng.standard_normal(s)).astype(np.float32) if bias else None  # noqa: E731
    ada = (rng.standard_normal((2, D)) / np.sqrt(D)).astype(np.float32)
    ada[1] += 1.0
    return dict(w_vid_in=n(D, 132), b_vid_in=b(D), w_txt_in=n(D, 5120), b_txt_in=b(D), w_emb0=n(D, 256),
                b_emb0=b(D), w_emb1=n(D, D), b_emb1=b(D), w_emb2=n(6 * D, D), b_emb2=b(6 * D), tail_ada=ada,
                w_out=n(64, D), b_out=b(64))


@pytest.mark.parametrize("name", [c[0] for c in DIT_IO_CASES])
def test_patchify_unpatchify_bit_exact_golden(gpu_ctx, s2lib, golden, name):
    import torch

    g = golden["dit_io"]
    shapes = g[f"{name}__shapes"].tolist()
    p = s2lib.patchify_video(gpu_ctx, torch.from_numpy(g[f"{name}__video"]).cuda(), shapes)
    u = s2lib.unpatchify_prediction(gpu_ctx, torch.from_numpy(g[f"{name}__pred"]).cuda(), shapes)
    torch.cuda.synchronize()
    assert np.array_equal(_bits(p.cpu().numpy()), _bits(g[f"{name}__patches"]))
    assert np.array_equal(_bits(u.cpu().numpy()), _bits(g[f"{name}__unpatched"]))


def test_patchify_unpatchify_random_vs_port(gpu_ctx, s2lib, port):
    import torch

    rng = np.random.default_rng(8)
    for shapes in ([[6, 90, 160]], [[5, 2, 30], [1, 64, 2], [3, 10, 10]], [[21, 34, 60]]):
        n = sum(t * h * w for t, h, w in shapes)
        x = rng.standard_normal((n, 33)).astype(np.float32)
        p = s2lib.patchify_video(gpu_ctx, torch.from_numpy(x).cuda(), shapes)
        ref_p = port.patchify_video(x, shapes)
        pr = rng.standard_normal((ref_p.shape[0], 64)).astype(np.float32)
        u = s2lib.unpatchify_prediction(gpu_ctx, torch.from_numpy(pr).cuda(), shapes)
        torch.cuda.synchronize()
        assert np.array_equal(_bits(p.cpu().numpy()), _bits(ref_p))
        assert np.array_equal(_bits(u.cpu().numpy()), _bits(port.unpatchify_prediction(pr, shapes)))


def test_token_format_error_codes(gpu_ctx, s2lib, golden):
    import torch

    codes = []
    buf = torch.zeros((64, 64), dtype=torch.float32, device="cuda")
    out = torch.zeros((256, 132), dtype=torch.float32, device="cuda")
    L = s2lib.lib()
    for fn, shapes, rows in DIT_IO_ERRORS:
        flat = s2lib._ints([v for s in shapes for v in s] or [0])
        if fn == "patchify":
            codes.append(L.s2_patchify_video(gpu_ctx.handle, buf.data_ptr(), rows, flat, len(shapes), out.data_ptr()))
        else:
            codes.append(L.s2_unpatchify_prediction(gpu_ctx.handle, buf.data_ptr(), rows, flat, len(shapes),
                                                    out.data_ptr()))
    torch.cuda.synchronize()
    assert codes == golden["dit_io"]["error_codes"].tolist()
    assert L.s2_timestep_embedding(gpu_ctx.handle, s2lib._floats([1.0]), 0, out.data_ptr()) == -1


def test_timestep_embedding_golden(gpu_ctx, s2lib, golden):
    import torch

    g = golden["dit_io"]
    got = s2lib.timestep_embedding(gpu_ctx, g["timesteps"].tolist())
    torch.cuda.synchronize()
    assert np.abs(got.cpu().numpy() - g["timestep_embedding"]).max() <= 5e-7


def _frontend_case(gpu_ctx, s2lib, port, *, D, heads, shapes, text_lengths, timesteps, seed):
    import torch

    rng = np.random.default_rng(seed)
    io = make_io_weights(rng, port, D)
    dit = s2lib.Dit(gpu_ctx, num_blocks=1, hidden=D, heads=heads, head_dim=128, mlp_hidden=4 * D, rope_pairs=21,
                    window=(1, 8, 8), window_mode=s2lib.S2_WINDOW_EXTENT)
    dit.set_io_weights(io)
    tokens = sum(t * h * w for t, h, w in shapes)
    video = rng.standard_normal((tokens, 33)).astype(np.float32)
    text = rng.standard_normal((sum(text_lengths), 5120)).astype(np.float32)
    v, t, mod = dit.forward_frontend(shapes, text_lengths, timesteps, torch.from_numpy(video).cuda(),
                                     torch.from_numpy(text).cuda())
    torch.cuda.synchronize()
    rv, rt, rmod = port.frontend_forward(io, shapes, timesteps, video, text, emulate_bf16=True)
    return dit, io, (v, t, mod), (rv, rt, rmod), rng, (video, text)


def test_frontend_and_tail_full_width(gpu_ctx, s2lib, port):
    """BASELINE 720p latents (6 x 90 x 160 x 33 -> 21600 patches), D = 2560, T = 58."""
    import torch

    shapes, tl, ts = [[6, 90, 160]], [58], [437.0]
    dit, io, (v, t, mod), (rv, rt, rmod), rng, (vin, tin) = _frontend_case(
        gpu_ctx, s2lib, port, D=2560, heads=20, shapes=shapes, text_lengths=tl, timesteps=ts, seed=21)
    assert rel_maxabs(v.cpu().numpy(), rv) <= 1e-3
    assert rel_maxabs(t.cpu().numpy(), rt) <= 1e-3
    assert rel_maxabs(mod.cpu().numpy(), rmod) <= 1e-4
    # and against the plain fp32 reference (no bf16 rounding anywhere) at the north-star gate
    fv, ft, _ = port.frontend_forward(io, shapes, ts, vin, tin, emulate_bf16=False)
    for got, ref in ((v.cpu().numpy(), fv), (t.cpu().numpy(), ft)):
        assert cosine(got, ref) >= 0.9995 and rel_maxabs(got, ref) <= 2e-2
    # tail on perturbed block output
    x = (rv + rng.standard_normal(rv.shape).astype(np.float32)).astype(np.float32)
    pred = dit.forward_tail(shapes, torch.from_numpy(x).cuda(), mod)
    torch.cuda.synchronize()
    ref = port.tail_forward(io, shapes, x, mod.cpu().numpy(), emulate_bf16=True)
    got = pred.cpu().numpy()
    assert cosine(got, ref) >= 0.99999
    assert rel_maxabs(got, ref) <= 1e-2
    ref32 = port.tail_forward(io, shapes, x, mod.cpu().numpy(), emulate_bf16=False)
    assert cosine(got, ref32) >= 0.9995 and rel_maxabs(got, ref32) <= 2e-2
    dit.close()


def test_frontend_batch_two(gpu_ctx, s2lib, port):
    dit, io, (v, t, mod), (rv, rt, rmod), _, _ = _frontend_case(gpu_ctx, s2lib, port, D=512, heads=4,
                                                             shapes=[[2, 6, 8], [1, 4, 10]], text_lengths=[5, 9],
                                                             timesteps=[999.0, 3.5], seed=22)
    assert rel_maxabs(v.cpu().numpy(), rv) <= 1e-3
    assert rel_maxabs(t.cpu().numpy(), rt) <= 1e-3
    assert rel_maxabs(mod.cpu().numpy(), rmod) <= 1e-4
    dit.close()


def test_step_requires_io_weights_and_valid_inputs(gpu_ctx, s2lib):
    import torch

    L = s2lib.lib()
    dit = s2lib.Dit(gpu_ctx, num_blocks=1, hidden=256, heads=2, head_dim=128, mlp_hidden=1024,
                    window=(1, 8, 8), window_mode=s2lib.S2_WINDOW_EXTENT)
    v = torch.zeros((64, 33), device="cuda")
    t = torch.zeros((4, 5120), device="cuda")
    p = torch.zeros((64, 16), device="cuda")
    o = torch.zeros((4, 256), device="cuda")

    def step(shapes, tl, ts, rows=64, trows=4):
        return L.s2_dit_forward_step(dit.handle, s2lib._ints([x for s in shapes for x in s]), s2lib._ints(tl),
                                     s2lib._floats(ts), len(shapes), v.data_ptr(), rows, t.data_ptr(), trows,
                                     p.data_ptr(), o.data_ptr())

    assert step([[1, 8, 8]], [4], [1.0]) == -1  # frontend / tail not loaded
    dit.init_random(3)
    assert step([[1, 8, 8]], [4], [float("nan")]) == -1  # non-finite timestep
    assert step([[1, 7, 8]], [4], [1.0], rows=56) == -1  # odd height
    assert step([[1, 8, 8]], [4], [1.0], rows=63) == -1  # row count mismatch
    assert step([[1, 8, 8]], [3], [1.0]) == -1  # text rows mismatch
    assert step([[1, 8, 8]], [4], [1.0]) == 0
    torch.cuda.synchronize()
    dit.close()


def test_dit_step_vs_oracle_chain(gpu_ctx, s2lib, port):
    """Frontend, two blocks (unshifted, shifted), tail for a 2-sample batch at reduced width, against
    the oracle's frontend -> block -> block -> tail chain in fp32; the host-buffer call matches the
    device call bit for bit."""
    import torch

    from tests.test_gpu_block import make_block_weights

    D, heads, F, pairs = 256, 2, 1024, 21
    shapes, tl, ts = [[2, 24, 32], [1, 16, 16]], [7, 5], [900.0, 12.0]
    rng = np.random.default_rng(31)
    io = make_io_weights(rng, port, D)
    ws = [make_block_weights(rng, D, F, 128, pairs) for _ in range(2)]
    dit = s2lib.Dit(gpu_ctx, num_blocks=2, hidden=D, heads=heads, head_dim=128, mlp_hidden=F, rope_pairs=pairs,
                    window=(1, 8, 8), window_mode=s2lib.S2_WINDOW_EXTENT)
    dit.set_io_weights(io)
    for b, w in enumerate(ws):
        dit.set_block_weights(b, w)
    tokens = sum(t * h * w for t, h, w in shapes)
    video = rng.standard_normal((tokens, 33)).astype(np.float32)
    text = rng.standard_normal((sum(tl), 5120)).astype(np.float32)
    pred, tout = dit.forward_step(shapes, tl, ts, torch.from_numpy(video).cuda(), torch.from_numpy(text).cuda())
    torch.cuda.synchronize()
    assert gpu_ctx.status() == 0
    hp = np.zeros((tokens, 16), np.float32)
    ht = np.zeros((sum(tl), D), np.float32)
    dit.forward_step_host(shapes, tl, ts, video, text, hp, ht)
    assert np.array_equal(_bits(hp), _bits(pred.cpu().numpy()))
    assert np.array_equal(_bits(ht), _bits(tout.cpu().numpy()))

    rv, rt, rmod = port.frontend_forward(io, shapes, ts, video, text)
    preds, texts = [], []
    v_off = t_off = 0
    for s, ((T, H, W), nt) in enumerate(zip(shapes, tl)):
        pshape = [T, H // 2, W // 2]
        npch = int(np.prod(pshape))
        xv, xt = rv[v_off:v_off + npch], rt[t_off:t_off + nt]
        for b, w in enumerate(ws):
            wo = dict(w)
            wo["freqs"] = wo.pop("rope_freqs")
            dims = [D, heads, 128, F, pairs, s2lib.S2_WINDOW_EXTENT, 1, 8, 8, b & 1]
            xv, xt = port.block_forward(dims=dims, eps_norm=1e-5, eps_qk=1e-5, weights=wo,
                                        modulation=rmod[:, s][None], shapes=[pshape], text_lengths=[nt],
                                        x_video=xv, x_text=xt)
        preds.append(port.tail_forward(io, [[T, H, W]], xv, rmod[:, s:s + 1]))
        texts.append(xt)
        v_off += npch
        t_off += nt
    ref_p, ref_t = np.concatenate(preds), np.concatenate(texts)
    got_p, got_t = pred.cpu().numpy(), tout.cpu().numpy()
    assert cosine(got_p, ref_p) >= 0.9995 and rel_maxabs(got_p, ref_p) <= 2e-2
    assert cosine(got_t, ref_t) >= 0.9995 and rel_maxabs(got_t, ref_t) <= 2e-2
    dit.close()


# ---- denoise loop (SeedVR2Pipeline::denoise / predict / apply_cfg) ----
def test_apply_cfg_golden(gpu_ctx, s2lib, golden):
    """The combine is bit-exact; with rescale the factor's double sums run in a different order than
    the reference's sequential loop, so allow 2 ulp."""
    import torch

    from tests.golden.gen_golden import CFG_CASES

    g = golden["dit_io"]
    for i, (_, scale, rescale) in enumerate(CFG_CASES):
        got = s2lib.apply_cfg(gpu_ctx, torch.from_numpy(g[f"cfg{i}__pos"]).cuda(),
                              torch.from_numpy(g[f"cfg{i}__neg"]).cuda(), scale, rescale)
        torch.cuda.synchronize()
        got, ref = got.cpu().numpy(), g[f"cfg{i}__out"]
        if rescale == 0.0:
            assert np.array_equal(_bits(got), _bits(ref)), i
        else:
            assert (np.abs(got - ref) <= 2 * np.spacing(np.abs(ref))).all(), i


def _oracle_predict(port, io, ws, shape, texts, D, heads, F, window):
    def predict(rows, t, positive):
        text = texts[0] if positive else texts[1]
        rv, rt, rmod = port.frontend_forward(io, [shape], [t], rows, text)
        pshape = [shape[0], shape[1] // 2, shape[2] // 2]
        xv, xt = rv, rt
        for b, w in enumerate(ws):
            wo = dict(w)
            wo["freqs"] = wo.pop("rope_freqs")
            dims = [D, heads, 128, F, 21, 1, window[0], window[1], window[2], b & 1]
            xv, xt = port.block_forward(dims=dims, eps_norm=1e-5, eps_qk=1e-5, weights=wo, modulation=rmod[:, 0][None],
                                        shapes=[pshape], text_lengths=[text.shape[0]], x_video=xv, x_text=xt)
        return port.tail_forward(io, [shape], xv, rmod)

    return predict


@pytest.mark.parametrize("steps,cfg_scale,cfg_rescale", [(2, 3.0, 0.5), (1, 1.0, 0.0)])
def test_denoise_vs_oracle(gpu_ctx, s2lib, port, steps, cfg_scale, cfg_rescale):
    """Whole denoise loop at reduced width (D = 256, 2 blocks) on padded channel planes (cstep > t*h*w,
    the ncnn Mat layout): the latent update matches the oracle's loop (the block gate on the change),
    the padding is untouched, and the host-buffer call matches the device call bit for bit."""
    import torch

    from tests.test_gpu_block import make_block_weights

    D, heads, F, window = 256, 2, 1024, (1, 8, 8)
    shape = [2, 16, 24]
    tokens = int(np.prod(shape))
    cstep = tokens + 8
    rng = np.random.default_rng(41)
    io = make_io_weights(rng, port, D)
    ws = [make_block_weights(rng, D, F, 128, 21) for _ in range(2)]
    dit = s2lib.Dit(gpu_ctx, num_blocks=2, hidden=D, heads=heads, head_dim=128, mlp_hidden=F, rope_pairs=21,
                    window=window, window_mode=s2lib.S2_WINDOW_EXTENT)
    dit.set_io_weights(io)
    for b, w in enumerate(ws):
        dit.set_block_weights(b, w)
    latent = rng.standard_normal((16, cstep)).astype(np.float32)
    cond = rng.standard_normal((16, cstep)).astype(np.float32)
    ptext = rng.standard_normal((7, 5120)).astype(np.float32)
    ntext = rng.standard_normal((5, 5120)).astype(np.float32)
    use_neg = cfg_scale != 1.0
    dl = torch.from_numpy(latent).cuda()
    dit.denoise(shape, dl, torch.from_numpy(cond).cuda(), torch.from_numpy(ptext).cuda(),
                torch.from_numpy(ntext).cuda() if use_neg else None, steps=steps, cfg_scale=cfg_scale,
                cfg_rescale=cfg_rescale)
    torch.cuda.synchronize()
    assert gpu_ctx.status() == 0
    got = dl.cpu().numpy()
    host = latent.copy()
    dit.denoise_host(shape, host, cond, ptext, ntext if use_neg else None, steps=steps, cfg_scale=cfg_scale,
                     cfg_rescale=cfg_rescale)
    assert np.array_equal(_bits(host), _bits(got))
    assert np.array_equal(_bits(got[:, tokens:]), _bits(latent[:, tokens:]))

    predict = _oracle_predict(port, io, ws, shape, (ptext, ntext), D, heads, F, window)
    ref = port.denoise(predict, latent[:, :tokens], cond[:, :tokens], steps, cfg_scale, cfg_rescale)
    d_got, d_ref = got[:, :tokens] - latent[:, :tokens], ref - latent[:, :tokens]
    assert cosine(d_got, d_ref) >= 0.9995 and rel_maxabs(d_got, d_ref) <= 2e-2
    dit.close()


def test_denoise_rejects_bad_options(gpu_ctx, s2lib):
    import torch

    dit = s2lib.Dit(gpu_ctx, num_blocks=1, hidden=256, heads=2, head_dim=128, mlp_hidden=1024,
                    window=(1, 8, 8), window_mode=s2lib.S2_WINDOW_EXTENT)
    dit.init_random(5)
    lat = torch.zeros((16, 64), device="cuda")
    txt = torch.zeros((3, 5120), device="cuda")
    L = s2lib.lib()

    def call(shape, steps, scale, neg=None, cstep=64):
        import ctypes

        opt = s2lib.DenoiseOptions(steps, scale, 0.0)
        return L.s2_dit_denoise(dit.handle, s2lib._ints(shape), lat.data_ptr(), cstep, lat.data_ptr(), cstep,
                                txt.data_ptr(), 3, None if neg is None else neg.data_ptr(),
                                0 if neg is None else 3, ctypes.byref(opt))

    assert call([1, 8, 8], 0, 1.0) == -1          # steps <= 0 (restore)
    assert call([1, 8, 8], 1, 2.0) == -1          # guidance without a negative text
    assert call([1, 7, 8], 1, 1.0, cstep=56) == -1  # odd height (is_latent)
    assert call([1, 8, 8], 1, 1.0, cstep=63) == -1  # plane stride below t*h*w
    assert call([1, 8, 8], 1, 1.0) == 0
    torch.cuda.synchronize()
    dit.close()
