"""GPU: the finite checks (the reference's SEEDVR2_DIT_CHECK_FINITE,
seedvr2_dit.cpp:33-54, :651-716, :1068-1071).

s2_count_nonfinite must equal numpy's count of ~isfinite exactly, for fp32
and bf16, at every 16-byte misalignment of the start and ragged lengths.  A
DiT forward with the check on returns -1 (the reference's code) when the
block stack's input or any block's output holds a NaN / Inf, names the first
such point, and leaves finite results bit-identical to an unchecked forward.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _plant(rng, a, k):
    """k non-finite values (NaN, +Inf, -Inf) at random positions, always including the first and last."""
    n = a.size
    idx = np.unique(np.concatenate([[0, n - 1], rng.integers(0, n, size=max(k - 2, 0))])) if n else np.zeros(0, int)
    vals = np.asarray([np.nan, np.inf, -np.inf], np.float32)
    a[idx] = vals[rng.integers(0, 3, size=idx.size)]
    return a


@pytest.mark.parametrize("n", [1, 3, 7, 9, 17, 1000, (1 << 20) + 5])
def test_count_nonfinite_matches_numpy(gpu_ctx, s2lib, n):
    import torch

    rng = np.random.default_rng(n)
    for dtype in (torch.float32, torch.bfloat16):
        buf = rng.standard_normal(n + 8).astype(np.float32)
        buf[8:] = _plant(rng, buf[8:].copy(), 1 + n // 97)
        dev = torch.from_numpy(buf).cuda().to(dtype)
        for off in range(8):  # every start alignment within 16 bytes
            view = dev[off:off + n]
            want = int((~torch.isfinite(view.float())).sum().item())
            assert s2lib.count_nonfinite(gpu_ctx, view) == want, (n, dtype, off)
    clean = torch.randn(n, device="cuda")
    assert s2lib.count_nonfinite(gpu_ctx, clean) == 0
    assert s2lib.count_nonfinite(gpu_ctx, clean[:0]) == 0


def _dit(s2lib, gpu_ctx, ws=None):
    from tests.test_gpu_block import make_block_weights

    D, heads, F = 256, 2, 1024
    dit = s2lib.Dit(gpu_ctx, num_blocks=2, hidden=D, heads=heads, head_dim=128, mlp_hidden=F, window=[1, 4, 4],
                    window_mode=1)
    rng = np.random.default_rng(17)
    ws = ws or [make_block_weights(rng, D, F, 128, 21) for _ in range(2)]
    for b, w in enumerate(ws):
        dit.set_block_weights(b, w)
    return dit, ws


def test_dit_check_finite(gpu_ctx, s2lib):
    import torch

    shape, T, D = [2, 6, 8], 5, 256
    nv = int(np.prod(shape))
    rng = np.random.default_rng(2)
    x0 = rng.standard_normal((nv + T, D)).astype(np.float32)
    mod = torch.from_numpy(rng.standard_normal((6, D)).astype(np.float32)).cuda()
    dit, ws = _dit(s2lib, gpu_ctx)

    # finite: same bits as an unchecked forward, report "all finite"
    plain = torch.from_numpy(x0).cuda()
    dit.forward(shape, T, plain, mod)
    dit.set_check_finite(True)
    checked = torch.from_numpy(x0).cuda()
    dit.forward(shape, T, checked, mod)
    assert torch.equal(plain, checked)
    assert dit.nonfinite_report() == (2, 0, 0)

    # a NaN in one video row and an Inf in one text row of the input: block -1
    bad = x0.copy()
    bad[3, 7] = np.nan
    bad[nv + 1, 0] = np.inf
    with pytest.raises(s2lib.S2Error) as e:
        dit.forward(shape, T, torch.from_numpy(bad).cuda(), mod)
    assert e.value.code == -1
    assert dit.nonfinite_report() == (-1, 1, 1)

    # block 1's MLP gate is NaN: block 0's output is finite, block 1's is not anywhere
    dit.close()
    ws[1] = dict(ws[1])
    ws[1]["ada"] = ws[1]["ada"].copy()
    ws[1]["ada"][5] = np.nan
    dit, _ = _dit(s2lib, gpu_ctx, ws)
    dit.set_check_finite(True)
    with pytest.raises(s2lib.S2Error) as e:
        dit.forward(shape, T, torch.from_numpy(x0).cuda(), mod)
    assert e.value.code == -1
    assert dit.nonfinite_report() == (1, nv * D, T * D)

    # check off: the same forward returns 0
    dit.set_check_finite(False)
    dit.forward(shape, T, torch.from_numpy(x0).cuda(), mod)
    torch.cuda.synchronize()
    assert gpu_ctx.status() == 0
    dit.close()
