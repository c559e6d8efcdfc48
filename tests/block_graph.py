"""Writes a synthetic DiT block graph as an ncnn .param / .bin pair.

The exported SeedVR2 block graph (blocks/seedvr2_blocks.ncnn.param, a download)
is not in the reference tree, so this script builds one from the block
restatement the oracle and the GPU stack share: per block,

    mod_k = in{4+k} + ada_k                       (k = 0..5; MemoryData + BinaryOp)
    h     = norm(x) * mod_1 + mod_0               (RMSNorm or LayerNorm, no affine)
    (qv, qt) = SharedLinear_qkv(h)
    (cv, ct) = AdaptiveWindowAttention(qv, qt, in2, in3)
    x    += SharedLinear_out(c) * mod_2
    h     = norm(x) * mod_4 + mod_3
    x    += SharedLinear_down(GELU_tanh(SharedLinear_up(h))) * mod_5

with the graph I/O names of seedvr2_dit.cpp:730-738 / :832-833: in0 video
rows, in1 text rows, in2 video shapes, in3 text lengths, in4..in9 the six
shared modulation vectors; out0 / out1 the video / text rows after the last
block.  Every blob with more than one consumer goes through a Split, as ncnn
requires; weights follow each layer's load_model order (SharedLinear weight
[num_output][num_input] then bias, raw fp32; AdaptiveWindowAttention
video_norm_q, video_norm_k, text_norm_q, text_norm_k, rope_freqs).
"""
from __future__ import annotations

import numpy as np


class _Graph:
    def __init__(self):
        self.layers: list[str] = []
        self.blobs = 0
        self.weights: list[np.ndarray] = []
        self.uses: dict[str, list[str]] = {}

    def layer(self, ltype, name, bottoms, tops, params=None, weights=()):
        p = " ".join(f"{k}={v:.9e}" if isinstance(v, float) else f"{k}={v}" for k, v in (params or {}).items())
        self.layers.append(f"{ltype:<24} {name:<20} {len(bottoms)} {len(tops)} {' '.join(bottoms)} {' '.join(tops)} "
                           f"{p}".rstrip())
        self.blobs += len(tops)
        self.weights.extend(np.ascontiguousarray(w, np.float32).ravel() for w in weights)

    def fan_out(self, blob, consumers, tag):
        """Split `blob` into one copy per consumer (ncnn's multi-consumer rule)."""
        if consumers == 1:
            return [blob]
        outs = [f"{blob}_{tag}{i}" for i in range(consumers)]
        self.layer("Split", f"split_{blob}_{tag}", [blob], outs)
        return outs


def write_block_graph(param_path, bin_path, blocks, *, D, heads, F, window, window_mode, eps_norm=1e-5, eps_qk=1e-5,
                      rope_pairs=21, layer_norm=(), bias=True):
    """blocks: list of weight dicts (ada [6][D], w_qkv, b_qkv, w_out, b_out, w_up, b_up, w_down, b_down,
    qk_norm [4][128], rope_freqs); block b is shifted when b is odd; its norm is LayerNorm when b in
    layer_norm."""
    g = _Graph()
    nb = len(blocks)
    for i in range(10):
        g.layer("Input", f"in{i}", [], [f"in{i}"], {0: D if i in (0, 1) or i >= 4 else (3 if i == 2 else 1)})
    shapes = g.fan_out("in2", nb, "b")
    texts = g.fan_out("in3", nb, "b")
    mods_in = [g.fan_out(f"in{4 + k}", nb, "b") for k in range(6)]
    xv, xt = "in0", "in1"
    for b, w in enumerate(blocks):
        p = f"b{b}_"
        norm = "LayerNorm" if b in layer_norm else "RMSNorm"
        mod_v, mod_t = [], []
        for k in range(6):
            g.layer("MemoryData", f"{p}ada{k}", [], [f"{p}ada{k}"], {0: D, 1: 1}, [w["ada"][k]])
            g.layer("BinaryOp", f"{p}mod{k}", [mods_in[k][b], f"{p}ada{k}"], [f"{p}mod{k}"], {0: 0})
            a, c = g.fan_out(f"{p}mod{k}", 2, "s")
            mod_v.append(a)
            mod_t.append(c)

        def half_in(x, stream, mods, kk, tag):
            xa, xr = g.fan_out(x, 2, f"{tag}")
            n = f"{p}{tag}_n"
            g.layer(norm, n, [xa], [n], {0: D, 1: float(eps_norm), 2: 0})
            g.layer("BinaryOp", f"{p}{tag}_sc", [n, mods[kk + 1]], [f"{p}{tag}_sc"], {0: 2})
            g.layer("BinaryOp", f"{p}{tag}_h", [f"{p}{tag}_sc", mods[kk]], [f"{p}{tag}_h"], {0: 0})
            return f"{p}{tag}_h", xr

        def residual(xr, y, mods, kk, tag):
            g.layer("BinaryOp", f"{p}{tag}_g", [y, mods[kk]], [f"{p}{tag}_g"], {0: 2})
            g.layer("BinaryOp", f"{p}{tag}_x", [xr, f"{p}{tag}_g"], [f"{p}{tag}_x"], {0: 0})
            return f"{p}{tag}_x"

        def linear(name, ins, outs, wk, bk, n_out, n_in):
            g.layer("SharedLinear", f"{p}{name}", ins, outs, {0: n_out, 1: n_in, 2: int(bias)},
                    [w[wk]] + ([w[bk]] if bias else []))

        hv, xv_r = half_in(xv, "v", mod_v, 0, "av")
        ht, xt_r = half_in(xt, "t", mod_t, 0, "at")
        linear("qkv", [hv, ht], [f"{p}qv", f"{p}qt"], "w_qkv", "b_qkv", 3 * D, D)
        qn = np.asarray(w["qk_norm"], np.float32).reshape(4, -1)
        g.layer("AdaptiveWindowAttention", f"{p}awa", [f"{p}qv", f"{p}qt", shapes[b], texts[b]],
                [f"{p}cv", f"{p}ct"],
                {0: heads, 1: D // heads, 2: window[0], 3: window[1], 4: window[2], 5: b & 1, 6: float(eps_qk),
                 7: rope_pairs, 8: 0, 9: 0, 10: 0, 11: window_mode},
                [qn[0], qn[1], qn[2], qn[3], w["rope_freqs"]])
        linear("out", [f"{p}cv", f"{p}ct"], [f"{p}ov", f"{p}ot"], "w_out", "b_out", D, D)
        xv = residual(xv_r, f"{p}ov", mod_v, 2, "rv")
        xt = residual(xt_r, f"{p}ot", mod_t, 2, "rt")
        hv, xv_r = half_in(xv, "v", mod_v, 3, "mv")
        ht, xt_r = half_in(xt, "t", mod_t, 3, "mt")
        linear("up", [hv, ht], [f"{p}uv", f"{p}ut"], "w_up", "b_up", F, D)
        g.layer("GELU", f"{p}gv", [f"{p}uv"], [f"{p}gv"], {0: 1})
        g.layer("GELU", f"{p}gt", [f"{p}ut"], [f"{p}gt"], {0: 1})
        linear("down", [f"{p}gv", f"{p}gt"], [f"{p}dv", f"{p}dt"], "w_down", "b_down", D, F)
        last = b == nb - 1
        g.layer("BinaryOp", f"{p}dv_g", [f"{p}dv", mod_v[5]], [f"{p}dv_g"], {0: 2})
        g.layer("BinaryOp", f"{p}xv_out", [xv_r, f"{p}dv_g"], ["out0" if last else f"{p}xv_out"], {0: 0})
        g.layer("BinaryOp", f"{p}dt_g", [f"{p}dt", mod_t[5]], [f"{p}dt_g"], {0: 2})
        g.layer("BinaryOp", f"{p}xt_out", [xt_r, f"{p}dt_g"], ["out1" if last else f"{p}xt_out"], {0: 0})
        xv, xt = f"{p}xv_out", f"{p}xt_out"
    with open(param_path, "w") as f:
        f.write("7767517\n")
        f.write(f"{len(g.layers)} {g.blobs}\n")
        f.write("\n".join(g.layers) + "\n")
    with open(bin_path, "wb") as f:
        for a in g.weights:
            f.write(a.tobytes())
    return len(g.layers), g.blobs
