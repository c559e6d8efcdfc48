"""Bit-exact window indexing on the device.

The host window plan is bit-exact with the reference's build_adaptive_window_plan
(tests/test_abi_host.py).  These tests check what the kernels actually read:
the attention schedule tables copied back from the device
(s2_plan_schedule_copy) must reproduce, bit for bit, the reference's own
video_indices, inverse_video_indices and local_positions
(adaptive_window_attention.cpp:446-473 build them; :886-915 gathers rows with
them and forms the RoPE positions (t + text_len, h, w) and (i, i, i); :954-961
scatters back) for every golden plan -- every BASELINE shape, shifted and
unshifted, ragged shapes and a 2-sample batch (SHA-256 for the large ones).

And an attention case whose scattered rows are exact: one-token windows
(extent 1x1x1), one text token with V = 0, Q = 0 so every score is 0 and P is
uniform: each video token's context is exactly its own V row / 2, which must
land at its own source row bit for bit (bf16 values that halve exactly).
"""
import hashlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a, np.int32).tobytes()).hexdigest()


def test_device_schedule_tables_match_reference_plans(gpu_ctx, s2lib, golden):
    g = golden["plans"]
    cases = sorted({k.split("__")[0] for k in g.files})
    assert len(cases) >= 20
    for case in cases:
        shapes = g[f"{case}__shapes"].tolist()
        target = g[f"{case}__target"].tolist()
        shifted = case.endswith("_s1")
        plan = s2lib.Plan(shapes, target, s2lib.S2_WINDOW_TARGET, shifted)
        tls = [5 + 3 * i for i in range(len(shapes))]
        d = plan.schedule(gpu_ctx, tls)
        windows = g[f"{case}__windows"]
        n = int(sum(int(np.prod(s)) for s in shapes))
        # partition order: the device's video_indices and the rows the windows pack
        vi, rs, pos, wi = d["video_indices"], d["row_src"], d["row_pos"], d["win_info"]
        assert wi.shape[0] == windows.shape[0], case
        text0 = np.concatenate([[0], np.cumsum(tls)])
        packed_vi = np.empty(n, np.int32)
        packed_pos = np.empty((n, 3), np.int32)
        inverse = np.full(n, -1, np.int32)
        for k, (seq, L, T, part) in enumerate(wi.tolist()):
            sample, count = int(windows[k, 0]), int(windows[k, 8])
            assert (L, T, part) == (count, tls[sample], int(windows[k, 7])), case
            packed_vi[part:part + L] = rs[seq:seq + L]
            packed_pos[part:part + L] = pos[seq:seq + L] - np.array([T, 0, 0], np.int32)
            # text rows: -1 - global text row, RoPE position (j, j, j)
            j = np.arange(T, dtype=np.int32)
            np.testing.assert_array_equal(rs[seq + L:seq + L + T], -1 - (text0[sample] + j), err_msg=case)
            np.testing.assert_array_equal(pos[seq + L:seq + L + T], np.stack([j, j, j], 1), err_msg=case)
            # pack_dst (source token -> packed row) read back as the partition slot of each token
            toks = rs[seq:seq + L]
            np.testing.assert_array_equal(d["pack_dst"][toks], seq + np.arange(L), err_msg=case)
            inverse[toks] = part + np.arange(L)
        np.testing.assert_array_equal(packed_vi, vi, err_msg=case)
        for name, arr in (("video_indices", vi), ("inverse_video_indices", inverse),
                          ("local_positions", packed_pos)):
            key = f"{case}__{name}"
            if key in g.files:
                np.testing.assert_array_equal(arr, g[key], err_msg=f"{case} {name}")
            assert _sha(arr) == bytes(g[f"{case}__sha_{name}"]).decode(), (case, name)


def test_one_token_windows_scatter_is_exact(gpu_ctx, s2lib):
    import torch

    heads, hd = 2, 128
    inner = heads * hd
    shapes = [[2, 5, 7], [1, 3, 4]]
    n = sum(int(np.prod(s)) for s in shapes)
    T = 1
    tok = np.arange(n)
    # V row of token t: small integers that identify it (exact in bf16, and their halves too)
    v = np.stack([(tok * 7 + c) % 127 for c in range(inner)], 1).astype(np.float32)
    v[:, 0] = tok % 128
    v[:, 1] = tok // 128
    video = np.zeros((n, 3 * inner), np.float32)
    video[:, inner:2 * inner] = np.random.default_rng(0).standard_normal((n, inner))  # any K
    video[:, 2 * inner:] = v
    text = np.zeros((T * len(shapes), 3 * inner), np.float32)
    text[:, inner:2 * inner] = 1.0
    norms = torch.ones(4, hd, device="cuda")
    freqs = torch.from_numpy((1.0 / 10000 ** (np.arange(21) * 2 / 42)).astype(np.float32)).cuda()
    out_v, _ = s2lib.awa_forward(gpu_ctx, heads=heads, head_dim=hd, window=[1, 1, 1],
                                 window_mode=s2lib.S2_WINDOW_EXTENT, shifted=0, eps=1e-5, rope_pairs=21, norms=norms,
                                 freqs=freqs, shapes=shapes, text_lengths=[T] * len(shapes),
                                 video_qkv=torch.from_numpy(video).cuda(), text_qkv=torch.from_numpy(text).cuda(),
                                 out_dtype=s2lib.S2_DTYPE_BF16, official_bf16=1)
    torch.cuda.synchronize()
    got = out_v.float().cpu().numpy()
    np.testing.assert_array_equal(got, v / 2)
