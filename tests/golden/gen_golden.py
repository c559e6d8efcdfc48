"""Generates the golden fixtures in tests/golden/ from the reference's OWN
layer code (oracle/_ref/libs2_ref.so: src/seedvr2/adaptive_window_attention.cpp
and src/seedvr2/shared_linear.cpp compiled unmodified against the clean-room
ncnn API shim).  Run from the repository root where the reference tree is
available:

    python tests/golden/gen_golden.py [--reference-tree PATH]

Outputs:
  plans.npz   -- build_adaptive_window_plan for every BASELINE shape, both
                 shift states, several target tuples, a 2-sample batch and a
                 set of ragged shapes.  Small plans store every array; large
                 plans store the window table plus SHA-256 digests of the
                 index/position arrays.
  awa.npz     -- AdaptiveWindowAttention::forward (CPU) on a seeded 2-sample
                 batch, fused-QKV input, shifted/unshifted x bf16 on/off.
  linear.npz  -- SharedLinear::forward on seeded inputs, with and without bias.
  vae_conv.npz -- DecomposedConv3D::forward (oracle/_ref/libs2_ref_vae.so:
                 src/seedvr2/decomposed_conv3d.cpp compiled unmodified) on seeded
                 inputs: memory disabled, and three chunks with the temporal
                 memory (initializing, then active).
  dit_io.npz  -- patchify_video / unpatchify_prediction / make_timestep_embedding
                 (oracle/_ref/libs2_ref_dit_io.so: src/seedvr2/seedvr2_dit.cpp:167-326
                 compiled unmodified) on seeded inputs, plus the return codes of
                 a set of invalid / empty calls.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))

# (name, shapes, target, shifted)
PLAN_CASES = [
    ("c1_default", [[1, 32, 32]], (4, 3, 3)),
    ("c2_default", [[1, 64, 64]], (4, 3, 3)),
    ("c3_default", [[6, 45, 80]], (4, 3, 3)),
    ("c3_434", [[6, 45, 80]], (4, 3, 4)),
    ("c5_default", [[12, 68, 120]], (4, 3, 3)),
    ("c5_433_21f", [[21, 90, 160]], (4, 3, 3)),
    ("batch2", [[2, 6, 8], [1, 4, 4]], (2, 2, 2)),
    ("ragged_a", [[3, 7, 11]], (2, 3, 2)),
    ("ragged_b", [[1, 1, 1]], (4, 3, 3)),
    ("ragged_c", [[5, 13, 9]], (5, 1, 7)),
    ("ragged_d", [[31, 17, 29]], (4, 3, 3)),
    ("wide", [[1, 9, 400]], (1, 2, 9)),
]
FULL_ARRAYS_MAX_TOKENS = 4096


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a, dtype=np.int32).tobytes()).hexdigest()


def gen_plans(ref: oracle.Ref) -> None:
    out = {}
    for name, shapes, target in PLAN_CASES:
        for shifted in (0, 1):
            key = f"{name}_s{shifted}"
            p = ref.plan(shapes, target, shifted)
            out[f"{key}__shapes"] = np.asarray(shapes, np.int32)
            out[f"{key}__target"] = np.asarray(target, np.int32)
            out[f"{key}__windows"] = p.windows
            out[f"{key}__sample_window_count"] = p.sample_window_count
            for arr_name in ("video_indices", "inverse_video_indices", "local_positions"):
                arr = getattr(p, arr_name)
                out[f"{key}__sha_{arr_name}"] = np.frombuffer(digest(arr).encode(), np.uint8)
                if len(p.video_indices) <= FULL_ARRAYS_MAX_TOKENS:
                    out[f"{key}__{arr_name}"] = arr
    np.savez_compressed(os.path.join(OUT, "plans.npz"), **out)


AWA_SEED = 1234


def awa_inputs():
    rng = np.random.default_rng(AWA_SEED)
    heads, hd = 2, 128
    shapes = np.asarray([[1, 6, 8], [2, 2, 3]], np.int32)
    text_lengths = np.asarray([5, 3], np.int32)
    nv = int(np.prod(shapes, axis=1).sum())
    nt = int(text_lengths.sum())
    inner = heads * hd
    video_qkv = rng.standard_normal((nv, 3 * inner)).astype(np.float32)
    text_qkv = rng.standard_normal((nt, 3 * inner)).astype(np.float32)
    norms = (1.0 + 0.02 * rng.standard_normal((4, hd))).astype(np.float32)
    freqs = (1.0 / 10000.0 ** (np.arange(21) * 2.0 / 42.0)).astype(np.float32)
    return dict(heads=heads, head_dim=hd, shapes=shapes, text_lengths=text_lengths, video_qkv=video_qkv,
                text_qkv=text_qkv, norms=norms, freqs=freqs, target=np.asarray([2, 2, 2], np.int32),
                eps=np.float32(1e-5), rope_pairs=21)


def gen_awa(ref: oracle.Ref) -> None:
    inp = awa_inputs()
    out = {k: np.asarray(v) for k, v in inp.items()}
    for shifted in (0, 1):
        for bf16 in (0, 1):
            vo, to = ref.awa_forward(heads=inp["heads"], head_dim=inp["head_dim"], target=inp["target"],
                                     shifted=shifted, eps=float(inp["eps"]), rope_pairs=inp["rope_pairs"],
                                     norms=inp["norms"], freqs=inp["freqs"], shapes=inp["shapes"],
                                     text_lengths=inp["text_lengths"], video_qkv=inp["video_qkv"],
                                     text_qkv=inp["text_qkv"], bf16=bool(bf16))
            out[f"video_out_s{shifted}_b{bf16}"] = vo
            out[f"text_out_s{shifted}_b{bf16}"] = to
    np.savez_compressed(os.path.join(OUT, "awa.npz"), **out)


def gen_linear(ref: oracle.Ref) -> None:
    rng = np.random.default_rng(99)
    k, n = 96, 80
    video = rng.standard_normal((37, k)).astype(np.float32)
    text = rng.standard_normal((5, k)).astype(np.float32)
    weight = (0.02 * rng.standard_normal((n, k))).astype(np.float32)
    bias = (0.02 * rng.standard_normal(n)).astype(np.float32)
    vo_b, to_b = ref.shared_linear(video, text, weight, bias)
    vo_n, to_n = ref.shared_linear(video, text, weight, None)
    np.savez_compressed(os.path.join(OUT, "linear.npz"), video=video, text=text, weight=weight, bias=bias,
                        video_out_bias=vo_b, text_out_bias=to_b, video_out_nobias=vo_n, text_out_nobias=to_n)


DIT_IO_CASES = [("one", [[2, 6, 8]]), ("batch2", [[1, 2, 2], [3, 4, 10]]), ("frames", [[3, 8, 10]])]
# (function, shapes, rows): rows are the input blob's height
DIT_IO_ERRORS = [
    ("patchify", [[1, 3, 4]], 12), ("patchify", [[1, 4, 4]], 15), ("patchify", [], 0), ("patchify", [], 5),
    ("patchify", [[0, 4, 4]], 0), ("patchify", [[-1, 4, 4]], 16), ("patchify", [[2, 4, 4]], 32),
    ("unpatchify", [[1, 3, 4]], 3), ("unpatchify", [], 0), ("unpatchify", [], 3), ("unpatchify", [[0, 4, 4]], 0),
    ("unpatchify", [[0, 4, 4], [1, 2, 2]], 1), ("unpatchify", [[2, 4, 4]], 7), ("unpatchify", [[2, 4, 4]], 8),
]


# apply_cfg cases: (rows of 16, scale, rescale)
CFG_CASES = [(96, 6.5, 0.0), (96, 6.5, 0.7), (1, 3.0, 1.0), (500, 1.5, 0.3)]


def _code(fn) -> int:
    try:
        fn()
        return 0
    except ValueError as e:
        return int(e.args[0])


def gen_dit_io(refio: oracle.RefIO) -> None:
    rng = np.random.default_rng(4321)
    out = {}
    for name, shapes in DIT_IO_CASES:
        tokens = sum(t * h * w for t, h, w in shapes)
        video = rng.standard_normal((tokens, 33)).astype(np.float32)
        patches = refio.patchify_video(video, shapes)
        pred = rng.standard_normal((patches.shape[0], 64)).astype(np.float32)
        out[f"{name}__shapes"] = np.asarray(shapes, np.int32)
        out[f"{name}__video"] = video
        out[f"{name}__patches"] = patches
        out[f"{name}__pred"] = pred
        out[f"{name}__unpatched"] = refio.unpatchify_prediction(pred, shapes)
    t = np.asarray([0.0, 1.0, 0.5, 999.0, 1000.0, 437.25, -3.0, 1e-3, 250.0, 12345.5], np.float32)
    out["timesteps"] = t
    out["timestep_embedding"] = refio.timestep_embedding(t)
    codes = []
    for fn, shapes, rows in DIT_IO_ERRORS:
        if fn == "patchify":
            codes.append(_code(lambda: refio.patchify_video(np.zeros((max(rows, 1), 33), np.float32), shapes, rows)))
        else:
            codes.append(_code(lambda: refio.unpatchify_prediction(np.zeros((max(rows, 1), 64), np.float32), shapes,
                                                                    rows)))
    out["error_codes"] = np.asarray(codes, np.int32)
    # apply_cfg (seedvr2_pipeline.cpp:171-210) on [tokens][16] predictions
    for i, (rows, scale, rescale) in enumerate(CFG_CASES):
        pos = rng.standard_normal((rows, 16)).astype(np.float32)
        neg = (0.5 * pos + rng.standard_normal((rows, 16))).astype(np.float32)
        out[f"cfg{i}__pos"] = pos
        out[f"cfg{i}__neg"] = neg
        out[f"cfg{i}__out"] = refio.apply_cfg(pos, neg, scale, rescale)
    np.savez_compressed(os.path.join(OUT, "dit_io.npz"), **out)


# DecomposedConv3D cases: (name, cfg (16 values), input (c, d, h, w), chunks)
CONV_CASES = [
    ("k333", [16, 8, 3, 3, 3, 1, 1, 2, 1, 1, 1, 1, 1, 1, 1, 1], (8, 5, 10, 12), 1),
    ("k333_mem", [16, 8, 3, 3, 3, 1, 1, 2, 1, 1, 1, 1, 1, 1, 1, 1], (8, 4, 10, 12), 3),
    ("st2_nobias", [7, 5, 3, 3, 3, 2, 1, 2, 1, 1, 1, 1, 1, 1, 1, 0], (5, 5, 8, 9), 2),
    ("k111", [6, 4, 1, 1, 1, 1, 1, 0, 1, 1, 1, 1, 0, 0, 1, 1], (4, 3, 6, 6), 1),
    ("dil2", [6, 4, 3, 3, 3, 1, 2, 4, 1, 1, 2, 2, 2, 2, 1, 1], (4, 3, 7, 11), 2),
]


def conv_blob(rng, co, ci, k, kt, st, head, sw, pad, bias):
    """One DecomposedConv3D's load_model blob: config, bias, kernels."""
    cfg = [co, ci, k, k, kt, st, 1, head, sw, sw, 1, 1, pad, pad, 1, int(bias)]
    parts = [np.asarray(cfg, np.float32)]
    if bias:
        parts.append((0.1 * rng.standard_normal(co)).astype(np.float32))
    parts.append((0.1 * rng.standard_normal(kt * co * ci * k * k)).astype(np.float32))
    return np.concatenate(parts)


def resample_blob(rng, kind, head):
    """VAEDownsample3D (0): 8 channels, pad right / bottom 1, 3x3 spatial stride 2 over 3 frames.
    VAEUpsample3D (1): 4 channels, temporal and spatial ratio 2 (head frame removed), 3x3x3 post and
    upscale convs."""
    if kind == 0:
        return np.concatenate([np.asarray([8, 1, 1], np.float32), conv_blob(rng, 8, 8, 3, 3, 1, head, 2, 0, True)])
    return np.concatenate([np.asarray([4, 2, 2, 1], np.float32), conv_blob(rng, 4, 4, 3, 3, 1, head, 1, 1, True),
                           conv_blob(rng, 32, 4, 3, 3, 1, head, 1, 1, True)])


# VAEChunkedMHA cases: (name, embed_dim, tokens), one head
MHA_CASES = [("mha16", 16, 20), ("mha64", 64, 100)]


def mha_weights(rng, E):
    """q w, q b, k w, k b, v w, v b, out w, out b (load_model order), flat fp32."""
    sizes = [E * E, E] * 4
    return np.concatenate([(0.1 * rng.standard_normal(n)).astype(np.float32) for n in sizes])


# (name, kind, head frames, input (c, d, h, w), memory states per chunk)
RESAMPLE_CASES = [
    ("down", 0, 2, (8, 3, 9, 12), [1, 2, 2]),
    ("down_off", 0, 2, (8, 4, 10, 10), [0]),
    ("up", 1, 2, (4, 2, 5, 6), [1, 2, 2]),
    ("up_off", 1, 2, (4, 3, 4, 4), [0]),
]


def conv_weights(rng, cfg):
    co, ci, kw, kh, kt = cfg[0], cfg[1], cfg[2], cfg[3], cfg[4]
    w = (0.1 * rng.standard_normal((kt, co, ci, kh, kw))).astype(np.float32)
    b = (0.1 * rng.standard_normal(co)).astype(np.float32) if cfg[15] else None
    return b, w


def gen_vae_conv() -> None:
    rng = np.random.default_rng(777)
    out = {}
    for name, cfg, (c, d, h, w), chunks in CONV_CASES:
        b, wt = conv_weights(rng, cfg)
        layer = oracle.RefConv3d(cfg, b, wt)
        out[f"{name}__cfg"] = np.asarray(cfg, np.int32)
        out[f"{name}__w"] = wt
        if b is not None:
            out[f"{name}__b"] = b
        for i in range(chunks):
            x = rng.standard_normal((c, d, h, w)).astype(np.float32)
            state = (oracle.VAE_MEMORY_DISABLED if chunks == 1 else
                     oracle.VAE_MEMORY_INITIALIZING if i == 0 else oracle.VAE_MEMORY_ACTIVE)
            out[f"{name}__x{i}"] = x
            out[f"{name}__state{i}"] = np.asarray(state, np.int32)
            out[f"{name}__y{i}"] = layer.forward(x, state)
    for name, kind, head, (c, d, h, w), states in RESAMPLE_CASES:
        blob = resample_blob(rng, kind, head)
        layer = oracle.RefResample(kind, blob)
        out[f"{name}__blob"] = blob
        out[f"{name}__kind"] = np.asarray(kind, np.int32)
        for i, st in enumerate(states):
            x = rng.standard_normal((c, d, h, w)).astype(np.float32)
            out[f"{name}__x{i}"] = x
            out[f"{name}__state{i}"] = np.asarray(st, np.int32)
            out[f"{name}__y{i}"] = layer.forward(x, st)
    # VAEChunkedMHA on its CPU path
    for name, E, T in MHA_CASES:
        w = mha_weights(rng, E)
        x = rng.standard_normal((T, E)).astype(np.float32)
        out[f"{name}__w"] = w
        out[f"{name}__x"] = x
        out[f"{name}__y"] = oracle.ref_mha_forward(E, 1, float(1.0 / np.sqrt(E)), w, x)
    np.savez_compressed(os.path.join(OUT, "vae_conv.npz"), **out)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-tree", default=oracle.reference_tree(),
                    help="reference checkout (default: $S2_REFERENCE_TREE or ../reference beside the repository)")
    args = ap.parse_args()
    if not args.reference_tree:
        ap.error("the reference checkout was not found: pass --reference-tree or set S2_REFERENCE_TREE")
    oracle.build(args.reference_tree)
    ref = oracle.Ref()
    gen_plans(ref)
    gen_awa(ref)
    gen_linear(ref)
    gen_dit_io(oracle.RefIO())
    gen_vae_conv()
    for f in ("plans.npz", "awa.npz", "linear.npz", "dit_io.npz", "vae_conv.npz"):
        print(f, os.path.getsize(os.path.join(OUT, f)), "bytes")


if __name__ == "__main__":
    main()
