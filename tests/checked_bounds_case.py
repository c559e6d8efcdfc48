"""Runs in a process of its own, against the index-checked library (S2_CUDA_LIB points at
libseedvr2_cuda_checked.so, the S2_DEBUG_BOUNDS build), and prints one JSON line.

A small shifted AdaptiveWindowAttention case runs once on a clean schedule; then, on a fresh plan
each time, one entry of a device schedule table is overwritten with an index far outside its
target (the gather source of a video row, of a text row, the scatter target of a video row, and
a scatter target with a negative peer field) and the forward runs over it: every table index the
kernels read is checked in this build, so each such run must end with s2_status = -1 and no
memory access through the bad index; a clean run afterwards on the same context must reproduce
the first run bit for bit (the context and the GPU are still fine).
"""
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

from seedvr2_ncnn_b200 import abi  # noqa: E402


def main():
    assert os.path.basename(abi.LIB_PATH) == "libseedvr2_cuda_checked.so", abi.LIB_PATH
    ctx = abi.Context(0)
    shape, window, heads, hd, T, pairs = [3, 7, 11], [2, 3, 4], 3, 128, 9, 21
    rng = np.random.default_rng(11)
    inner = heads * hd
    nv = int(np.prod(shape))
    dev = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    kw = dict(heads=heads, head_dim=hd, window=window, window_mode=abi.S2_WINDOW_EXTENT, shifted=1, eps=1e-5,
              rope_pairs=pairs, norms=dev((1 + 0.02 * rng.standard_normal((4, hd))).astype(np.float32)),
              freqs=dev((1.0 / 10000 ** (np.arange(pairs) * 2 / 42)).astype(np.float32)), shapes=[shape],
              text_lengths=[T], video_qkv=dev(rng.standard_normal((nv, 3 * inner)).astype(np.float32)),
              text_qkv=dev(rng.standard_normal((T, 3 * inner)).astype(np.float32)))

    def plan():
        return abi.Plan([shape], window, abi.S2_WINDOW_EXTENT, True)

    def run(p):
        vo, to = abi.awa_forward(ctx, plan=p, **kw)
        torch.cuda.synchronize()
        return vo.cpu().numpy(), to.cpu().numpy(), ctx.status()

    v0, t0, st0 = run(plan())
    out = {"clean_status": st0, "clean_finite": bool(np.isfinite(v0).all() and np.isfinite(t0).all())}
    probe = plan()
    tables = probe.schedule(ctx, [T])
    row_src = tables["row_src"]
    video_row = int(np.flatnonzero(row_src >= 0)[0])
    text_row = int(np.flatnonzero(row_src < 0)[0])
    cases = {
        "gather_video": (0, video_row, 1 << 27),
        "gather_text": (0, text_row, -(1 << 27)),
        "scatter_row": (1, 3, (1 << 26) - 1),  # peer field 0, row far past the outputs
        "scatter_peer": (1, 4, -5),  # negative peer field
    }
    for name, (table, index, value) in cases.items():
        p = plan()
        p.schedule(ctx, [T])
        rc = p.debug_poke(ctx, table, index, value)
        _, _, st = run(p)
        out[name] = [rc, st]
    v1, t1, st1 = run(plan())
    out["after_status"] = st1
    out["after_equal"] = bool(np.array_equal(v0, v1) and np.array_equal(t0, t1))
    print(json.dumps(out))


if __name__ == "__main__":
    main()
