"""GPU parity of whole DiT blocks (s2_dit, through the C ABI) against the CPU
oracle's fp32 block restatement on identical seeded inputs and weights.

Gate per block (north star): cosine >= 0.9995 and
max|gpu - ref| / max|ref| <= 2e-2 on the block output; the block's update
(output - input) must also agree (cosine >= 0.999) so the residual stream
cannot hide an error in the block itself.
"""
import numpy as np
import pytest

from tests.conftest import cosine, rel_maxabs

pytestmark = pytest.mark.gpu


def make_block_weights(rng, D, F, hd, pairs, bias=True):
    n = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731
    ada = n(6, D) / np.sqrt(D)
    ada[1] += 1.0
    ada[4] += 1.0
    return dict(ada=ada, w_qkv=0.02 * n(3 * D, D), b_qkv=(0.02 * n(3 * D)) if bias else None,
                w_out=0.02 * n(D, D), b_out=(0.02 * n(D)) if bias else None, w_up=0.02 * n(F, D),
                b_up=(0.02 * n(F)) if bias else None, w_down=0.02 * n(D, F), b_down=(0.02 * n(D)) if bias else None,
                qk_norm=1 + 0.02 * n(4, hd), rope_freqs=(1.0 / 10000 ** (np.arange(pairs) * 2 / (2 * pairs))))


def run_case(gpu_ctx, s2lib, port, *, D, heads, F, shape, T, window, mode, blocks, seed, bias=True, layer=()):
    import torch

    hd, pairs = 128, 21
    rng = np.random.default_rng(seed)
    ws = [make_block_weights(rng, D, F, hd, pairs, bias) for _ in range(blocks)]
    mod = rng.standard_normal((6, D)).astype(np.float32)
    nv = int(np.prod(shape))
    xv = rng.standard_normal((nv, D)).astype(np.float32)
    xt = rng.standard_normal((T, D)).astype(np.float32)

    dit = s2lib.Dit(gpu_ctx, num_blocks=blocks, hidden=D, heads=heads, head_dim=hd, mlp_hidden=F, rope_pairs=pairs,
                    window=window, window_mode=mode, bias=bias)
    for b, w in enumerate(ws):
        dit.set_block_weights(b, w)
        if b in layer:
            dit.set_block_norm(b, True)
    x = torch.from_numpy(np.concatenate([xv, xt])).cuda()
    dit.forward(shape, T, x, torch.from_numpy(mod).cuda())
    torch.cuda.synchronize()
    assert gpu_ctx.status() == 0
    got = x.cpu().numpy()

    ref_v, ref_t = xv, xt
    for b, w in enumerate(ws):
        dims = [D, heads, hd, F, pairs, mode, window[0], window[1], window[2], b & 1, int(b in layer)]
        wo = dict(w)
        wo["freqs"] = wo.pop("rope_freqs")
        prev = np.concatenate([ref_v, ref_t])
        ref_v, ref_t = port.block_forward(dims=dims, eps_norm=1e-5, eps_qk=1e-5, weights=wo, modulation=mod[None],
                                          shapes=[shape], text_lengths=[T], x_video=ref_v, x_text=ref_t)
    ref = np.concatenate([ref_v, ref_t])
    dit.close()
    return got, ref, prev, np.concatenate([xv, xt])


def check(got, ref, prev):
    assert cosine(got, ref) >= 0.9995
    assert rel_maxabs(got, ref) <= 2e-2
    assert cosine(got - prev, ref - prev) >= 0.999


def test_block_reduced_width_two_blocks(gpu_ctx, s2lib, port):
    """Block 0 (unshifted) then block 1 (shifted) at D=512, ragged shifted windows."""
    got, ref, prev, x0 = run_case(gpu_ctx, s2lib, port, D=512, heads=4, F=2048, shape=[2, 12, 20], T=58,
                                  window=[1, 8, 8], mode=1, blocks=2, seed=3)
    check(got, ref, prev)


def test_block_full_width_one_block(gpu_ctx, s2lib, port):
    """BASELINE widths (D=2560, 20x128 heads, MLP 10240), one 720p-shaped window slab."""
    got, ref, prev, x0 = run_case(gpu_ctx, s2lib, port, D=2560, heads=20, F=10240, shape=[2, 15, 20], T=58,
                                  window=[4, 3, 4], mode=0, blocks=1, seed=4)
    check(got, ref, x0)


def test_block_layernorm_then_rmsnorm(gpu_ctx, s2lib, port):
    """Per-block norm choice: block 0 with LayerNorm AdaLN passes, block 1 with RMSNorm, at D=512."""
    got, ref, prev, x0 = run_case(gpu_ctx, s2lib, port, D=512, heads=4, F=2048, shape=[2, 12, 20], T=58,
                                  window=[1, 8, 8], mode=1, blocks=2, seed=8, layer=(0,))
    check(got, ref, prev)


def test_block_no_bias_target_windows(gpu_ctx, s2lib, port):
    got, ref, prev, x0 = run_case(gpu_ctx, s2lib, port, D=256, heads=2, F=1024, shape=[3, 9, 14], T=7,
                                  window=[2, 2, 3], mode=0, blocks=2, seed=5, bias=False)
    check(got, ref, prev)


def test_block_odd_head_count(gpu_ctx, s2lib, port):
    """3 heads (D=384): the QKV projection cannot pack whole heads per 256-column tile, so the block runs the
    projection into a buffer and the separate prepare kernel."""
    got, ref, prev, x0 = run_case(gpu_ctx, s2lib, port, D=384, heads=3, F=1536, shape=[2, 8, 12], T=9,
                                  window=[1, 4, 6], mode=1, blocks=2, seed=6)
    check(got, ref, prev)


def test_forward_host_matches_device(gpu_ctx, s2lib):
    """s2_dit_forward_host (host buffers, 2 samples run one after another) == per-sample s2_dit_forward."""
    import torch

    D, heads, F = 256, 2, 1024
    dit = s2lib.Dit(gpu_ctx, num_blocks=2, hidden=D, heads=heads, head_dim=128, mlp_hidden=F, window=[1, 4, 4],
                    window_mode=1)
    dit.init_random(9)
    rng = np.random.default_rng(0)
    shapes, tls = [[1, 6, 8], [2, 4, 4]], [5, 3]
    nv = [48, 32]
    video = rng.standard_normal((sum(nv), D)).astype(np.float32)
    text = rng.standard_normal((sum(tls), D)).astype(np.float32)
    mod = rng.standard_normal((6, 2, D)).astype(np.float32)
    vo = np.zeros_like(video)
    to = np.zeros_like(text)
    dit.forward_host(shapes, tls, video, text, mod, vo, to)
    voff = toff = 0
    for s in range(2):
        x = torch.from_numpy(np.concatenate([video[voff:voff + nv[s]], text[toff:toff + tls[s]]])).cuda()
        dit.forward(shapes[s], tls[s], x, torch.from_numpy(np.ascontiguousarray(mod[:, s])).cuda())
        x = x.cpu().numpy()
        np.testing.assert_array_equal(x[:nv[s]], vo[voff:voff + nv[s]])
        np.testing.assert_array_equal(x[nv[s]:], to[toff:toff + tls[s]])
        voff += nv[s]
        toff += tls[s]
    dit.close()


def test_forward_host_async_pipeline(gpu_ctx, s2lib):
    """s2_dit_forward_host_async: five calls back to back (pinned buffers, each a batch of two samples, the
    staging buffers used in turn and one grown on the way) give what s2_dit_forward_host gives for each."""
    import torch

    D, heads, F = 256, 2, 1024
    dit = s2lib.Dit(gpu_ctx, num_blocks=2, hidden=D, heads=heads, head_dim=128, mlp_hidden=F, window=[1, 4, 4],
                    window_mode=1)
    dit.init_random(11)
    g = torch.Generator().manual_seed(3)
    calls = []
    for i in range(5):
        shapes = [[1, 6, 8], [2, 4, 4]] if i != 3 else [[2, 8, 8], [1, 4, 4]]
        tls = [5, 3]
        nvt = sum(a * b * c for a, b, c in shapes)
        pin = lambda *sz: torch.randn(*sz, generator=g).pin_memory()
        calls.append((shapes, tls, pin(nvt, D), pin(sum(tls), D), pin(6, 2, D),
                      torch.zeros(nvt, D).pin_memory(), torch.zeros(sum(tls), D).pin_memory()))
    for shapes, tls, v, t, m, vo, to in calls:
        dit.forward_host_async(shapes, tls, v, t, m, vo, to)
    dit.host_wait()
    for shapes, tls, v, t, m, vo, to in calls:
        rv, rt = torch.zeros_like(vo), torch.zeros_like(to)
        dit.forward_host(shapes, tls, v, t, m, rv, rt)
        assert torch.equal(vo, rv) and torch.equal(to, rt)
        assert not torch.equal(vo, v)
    assert gpu_ctx.status() == 0
    dit.close()


def test_block_checkpoints(gpu_ctx, s2lib):
    """s2_dit_set_checkpoints: block 0's copy equals a one-block stack's output bit for bit, the last block's
    equals the final rows, s2_dit_forward_host writes each sample at its rows, and a block outside the stack
    is -1 (the reference's range check)."""
    import torch

    D, heads, F = 256, 2, 1024
    rng = np.random.default_rng(21)
    ws = [make_block_weights(rng, D, F, 128, 21) for _ in range(2)]

    def stack(n):
        dit = s2lib.Dit(gpu_ctx, num_blocks=n, hidden=D, heads=heads, head_dim=128, mlp_hidden=F, window=[1, 4, 4],
                        window_mode=1)
        for b in range(n):
            dit.set_block_weights(b, ws[b])
        return dit

    # one sample on the device
    shape, T = [2, 6, 8], 5
    nv = int(np.prod(shape))
    x0 = rng.standard_normal((nv + T, D)).astype(np.float32)
    mod = rng.standard_normal((6, D)).astype(np.float32)
    two, one = stack(2), stack(1)
    cv = [torch.empty((nv, D), device="cuda") for _ in range(2)]
    ct = [torch.empty((T, D), device="cuda") for _ in range(2)]
    two.set_checkpoints([0, 1], cv, ct)
    x = torch.from_numpy(x0).cuda()
    two.forward(shape, T, x, torch.from_numpy(mod).cuda())
    y = torch.from_numpy(x0).cuda()
    one.forward(shape, T, y, torch.from_numpy(mod).cuda())
    torch.cuda.synchronize()
    assert torch.equal(cv[0], y[:nv]) and torch.equal(ct[0], y[nv:])
    assert torch.equal(cv[1], x[:nv]) and torch.equal(ct[1], x[nv:])

    # two samples through the host entry point: checkpoints at the samples' rows
    shapes, tls = [[1, 6, 8], [2, 4, 4]], [5, 3]
    nvs = [48, 32]
    video = rng.standard_normal((sum(nvs), D)).astype(np.float32)
    text = rng.standard_normal((sum(tls), D)).astype(np.float32)
    mods = rng.standard_normal((6, 2, D)).astype(np.float32)
    cv = [torch.full((sum(nvs), D), float("nan"), device="cuda") for _ in range(2)]
    ct = [torch.full((sum(tls), D), float("nan"), device="cuda") for _ in range(2)]
    two.set_checkpoints([1, 0], [cv[1], cv[0]], [ct[1], ct[0]])
    vo, to = np.zeros_like(video), np.zeros_like(text)
    two.forward_host(shapes, tls, video, text, mods, vo, to)
    v1, t1 = np.zeros_like(video), np.zeros_like(text)
    one.forward_host(shapes, tls, video, text, mods, v1, t1)
    np.testing.assert_array_equal(cv[1].cpu().numpy(), vo)
    np.testing.assert_array_equal(ct[1].cpu().numpy(), to)
    np.testing.assert_array_equal(cv[0].cpu().numpy(), v1)
    np.testing.assert_array_equal(ct[0].cpu().numpy(), t1)

    for bad in ([2], [-1]):
        with pytest.raises(s2lib.S2Error) as e:
            two.set_checkpoints(bad, cv[:1], ct[:1])
        assert e.value.code == -1
    two.set_checkpoints([], [], [])
    torch.cuda.synchronize()
    assert gpu_ctx.status() == 0
    two.close()
    one.close()
