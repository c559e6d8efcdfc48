"""ctypes front-end for the CPU checkers (TEST INFRASTRUCTURE ONLY).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline /
reference arm import this module, and only as the checker or the timed CPU
baseline; the shipped package never imports it.

* :class:`Port` wraps ``oracle/libs2_oracle.so`` -- our C restatement of the
  reference's hot path (``s2_oracle.c``).
* :class:`Ref` wraps ``oracle/_ref/libs2_ref.so`` -- the reference's OWN
  ``adaptive_window_attention.cpp`` / ``shared_linear.cpp`` compiled against
  the clean-room ncnn API shim (built only where the reference tree exists).
* :class:`RefIO` wraps ``oracle/_ref/libs2_ref_dit_io.so`` -- the reference's
  own ``patchify_video`` / ``make_timestep_embedding`` /
  ``unpatchify_prediction`` (``src/seedvr2/seedvr2_dit.cpp:167-326``).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "libs2_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libs2_ref.so")
REF_IO_SO = os.path.join(HERE, "_ref", "libs2_ref_dit_io.so")
REF_VAE_SO = os.path.join(HERE, "_ref", "libs2_ref_vae.so")
REF_VAE_RT_SO = os.path.join(HERE, "_ref", "libs2_ref_vae_rt.so")

# DecomposedConv3D memory states (seedvr2::MemoryState)
VAE_MEMORY_DISABLED = 0
VAE_MEMORY_INITIALIZING = 1
VAE_MEMORY_ACTIVE = 2

WINDOW_TARGET = 0
WINDOW_EXTENT = 1

_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")


def reference_tree() -> str | None:
    """The reference checkout (Chisato623/seedvr2_ncnn) to build the checkers from: $S2_REFERENCE_TREE, else a
    checkout named `reference` beside this repository's directory; None when neither holds its sources (as on
    a GPU box, which uses the checkers built beforehand)."""
    repo_parent = os.path.dirname(os.path.dirname(HERE))
    for tree in (os.environ.get("S2_REFERENCE_TREE"), os.path.join(repo_parent, "reference")):
        if tree and os.path.isdir(os.path.join(tree, "src", "seedvr2")):
            return tree
    return None


def build(ref_tree: str | None = None) -> None:
    """Compile the port (always) and the reference build (when its tree exists)."""
    subprocess.run(["make", "-s", "-C", HERE, "port"], check=True)
    tree = ref_tree or reference_tree()
    if tree and os.path.isdir(os.path.join(tree, "src", "seedvr2")):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={tree}"], check=True)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int32)


class Plan:
    """Window plan arrays (AdaptiveWindowPlan, adaptive_window_attention.h:29-36)."""

    def __init__(self, windows, sample_window_count, video_indices, inverse, local_positions):
        self.windows = windows  # [nw, 9]
        self.sample_window_count = sample_window_count
        self.video_indices = video_indices
        self.inverse_video_indices = inverse
        self.local_positions = local_positions  # [n, 3]

    def as_dict(self):
        return {
            "windows": self.windows,
            "sample_window_count": self.sample_window_count,
            "video_indices": self.video_indices,
            "inverse_video_indices": self.inverse_video_indices,
            "local_positions": self.local_positions,
        }


class Port:
    """Our C restatement (oracle/s2_oracle.c)."""

    def __init__(self, path: str = PORT_SO):
        if not os.path.exists(path):
            build()
        lib = C.CDLL(path)
        lib.s2o_plan_sizes.argtypes = [_i32p, C.c_int, C.c_int, _i32p, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int)]
        lib.s2o_plan_build.argtypes = [_i32p, C.c_int, C.c_int, _i32p, C.c_int, _i32p, _i32p, _i32p, _i32p, _i32p]
        lib.s2o_round_bf16.argtypes = [C.c_float]
        lib.s2o_round_bf16.restype = C.c_float
        lib.s2o_awa_forward.argtypes = [_i32p, C.c_float, _f32p, _f32p, _i32p, _i32p, C.c_int,
                                        C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                        C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, _f32p, _f32p]
        lib.s2o_linear.argtypes = [_f32p, C.c_int, C.c_int, _f32p, C.c_void_p, C.c_int, _f32p]
        lib.s2o_block_forward.argtypes = [_i32p, C.c_float, C.c_float, C.c_void_p, _f32p, _i32p, _i32p, C.c_int,
                                          _f32p, _f32p, C.c_int]
        lib.s2o_patchify_video.argtypes = [C.c_void_p, C.c_int, _i32p, C.c_int, C.c_void_p]
        lib.s2o_unpatchify_prediction.argtypes = [C.c_void_p, C.c_int, _i32p, C.c_int, C.c_void_p]
        lib.s2o_timestep_embedding.argtypes = [_f32p, C.c_int, _f32p]
        lib.s2o_assemble_dit_input.argtypes = [_f32p, C.c_long, _f32p, C.c_long, C.c_long, _f32p]
        lib.s2o_apply_cfg.argtypes = [_f32p, _f32p, C.c_long, C.c_float, C.c_float, _f32p]
        lib.s2o_euler_update.argtypes = [_f32p, C.c_long, C.c_long, _f32p, C.c_float]
        lib.s2o_denoise_schedule.argtypes = [C.c_int, C.c_int, C.POINTER(C.c_float), C.POINTER(C.c_float)]
        lib.s2o_conv3d_dims.argtypes = [_i32p, C.c_int, C.c_int, C.c_int, C.c_int, _i32p]
        lib.s2o_conv3d_forward.argtypes = [_i32p, C.c_void_p, _f32p, _f32p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                           C.c_int, _f32p, C.c_void_p]
        lib.s2o_mha_forward.argtypes = [C.c_int, C.c_int, C.c_float, _f32p, _f32p, C.c_int, _f32p]
        self.lib = lib

    def mha_forward(self, E, heads, scale, weights, x):
        """VAEChunkedMHA's CPU path: x [T][E] -> [T][E] (weights in load_model order, flat)."""
        x = _f32(x)
        out = np.zeros_like(x)
        r = self.lib.s2o_mha_forward(E, heads, scale, _f32(weights), x, x.shape[0], out)
        if r != 0:
            raise ValueError(r)
        return out

    def plan(self, shapes, window, shifted, mode=WINDOW_TARGET) -> Plan:
        shapes = _i32(shapes).reshape(-1, 3)
        win = _i32(window)
        nw, nt = C.c_int(), C.c_int()
        r = self.lib.s2o_plan_sizes(shapes, len(shapes), mode, win, int(shifted), C.byref(nw), C.byref(nt))
        if r != 0:
            raise ValueError(f"s2o_plan_sizes returned {r}")
        windows = np.zeros((nw.value, 9), np.int32)
        swc = np.zeros(len(shapes), np.int32)
        vi = np.zeros(nt.value, np.int32)
        inv = np.zeros(nt.value, np.int32)
        pos = np.zeros((nt.value, 3), np.int32)
        r = self.lib.s2o_plan_build(shapes, len(shapes), mode, win, int(shifted), windows, swc, vi, inv, pos)
        if r != 0:
            raise ValueError(f"s2o_plan_build returned {r}")
        return Plan(windows, swc, vi, inv, pos)

    def round_bf16(self, x):
        x = _f32(x)
        # vectorised restatement of the same rule, checked against the C one
        b = x.view(np.uint32).astype(np.uint64)
        finite = (b & 0x7F800000) != 0x7F800000
        b = np.where(finite, b + 0x7FFF + ((b >> 16) & 1), b) & 0xFFFF0000
        return b.astype(np.uint32).view(np.float32)

    def awa_forward(self, *, heads, head_dim, window, shifted, eps, rope_pairs, norms, freqs, shapes,
                    text_lengths, video_qkv=None, text_qkv=None, split=None, mode=WINDOW_TARGET,
                    bf16=False):
        """norms: [4, head_dim]; video_qkv [Nv, 3*inner] or split=(vq,vk,vv,tq,tk,tv)."""
        inner = heads * head_dim
        shapes = _i32(shapes).reshape(-1, 3)
        tl = _i32(text_lengths)
        nv = int(np.prod(shapes, axis=1).sum())
        nt = int(tl.sum())
        keep = []
        if split is None:
            v = _f32(video_qkv)
            t = _f32(text_qkv)
            keep += [v, t]
            vb, tb = v.ctypes.data, t.ctypes.data
            ptrs = [vb, vb + inner * 4, vb + 2 * inner * 4, tb, tb + inner * 4, tb + 2 * inner * 4]
            vld = tld = 3 * inner
        else:
            arrs = [_f32(a) for a in split]
            keep += arrs
            ptrs = [a.ctypes.data for a in arrs]
            vld = tld = inner
        ip = _i32([heads, head_dim, window[0], window[1], window[2], int(shifted), rope_pairs, mode, int(bf16)])
        vo = np.zeros((nv, inner), np.float32)
        to = np.zeros((nt, inner), np.float32)
        r = self.lib.s2o_awa_forward(ip, eps, _f32(norms).reshape(-1), _f32(freqs), shapes, tl, len(shapes),
                                     ptrs[0], ptrs[1], ptrs[2], vld, ptrs[3], ptrs[4], ptrs[5], tld, vo, to)
        if r != 0:
            raise ValueError(f"s2o_awa_forward returned {r}")
        return vo, to

    def linear(self, a, w, bias=None):
        a = _f32(a)
        w = _f32(w)
        out = np.zeros((a.shape[0], w.shape[0]), np.float32)
        b = _f32(bias) if bias is not None else None
        self.lib.s2o_linear(a, a.shape[0], a.shape[1], w, b.ctypes.data if b is not None else None,
                            w.shape[0], out)
        return out

    def block_forward(self, *, dims, eps_norm, eps_qk, weights: dict, modulation, shapes, text_lengths,
                      x_video, x_text, emulate_bf16=False):
        """weights: dict of fp32 arrays keyed like s2o_block_weights; returns updated (xv, xt).
        dims: D, heads, head_dim, F, rope_pairs, window_mode, window0..2, shifted[, norm: 0 RMS, 1 Layer]."""

        class W(C.Structure):
            _fields_ = [(n, C.c_void_p) for n in
                        ("ada", "w_qkv", "b_qkv", "w_out", "b_out", "w_up", "b_up", "w_down", "b_down",
                         "qk_norm", "freqs")]

        keep = {k: (_f32(v) if v is not None else None) for k, v in weights.items()}
        w = W(*[(keep[n].ctypes.data if keep.get(n) is not None else None) for n, _ in W._fields_])
        xv = _f32(x_video).copy()
        xt = _f32(x_text).copy()
        shapes = _i32(shapes).reshape(-1, 3)
        dims = list(dims) + [0] * (11 - len(dims))  # norm type defaults to RMSNorm
        r = self.lib.s2o_block_forward(_i32(dims), eps_norm, eps_qk, C.addressof(w), _f32(modulation).reshape(-1),
                                       shapes, _i32(text_lengths), len(shapes), xv, xt, int(emulate_bf16))
        if r != 0:
            raise ValueError(f"s2o_block_forward returned {r}")
        return xv, xt


    # ---- token formats and the frontend / tail nets (seedvr2_dit.cpp) ----
    def patchify_video(self, video, shapes, rows=None):
        """[tokens, 33] -> [patches, 132]; raises ValueError(code) like the reference's return code."""
        video = _f32(video)
        shapes = _i32(shapes).reshape(-1, 3)
        rows = video.shape[0] if rows is None else rows
        patches = int(sum(max(t, 0) * (max(h, 0) // 2) * (max(w, 0) // 2) for t, h, w in shapes.tolist()))
        out = np.zeros((max(patches, 1), 132), np.float32)
        r = self.lib.s2o_patchify_video(video.ctypes.data, rows, shapes, len(shapes), out.ctypes.data)
        if r != 0:
            raise ValueError(r)
        return out[:patches]

    def unpatchify_prediction(self, pred, shapes, rows=None):
        """[patches, 64] -> [tokens, 16] (latent shapes)."""
        pred = _f32(pred)
        shapes = _i32(shapes).reshape(-1, 3)
        rows = pred.shape[0] if rows is None else rows
        tokens = int(sum(max(t, 0) * max(h, 0) * max(w, 0) for t, h, w in shapes.tolist()))
        out = np.zeros((max(tokens, 1), 16), np.float32)
        r = self.lib.s2o_unpatchify_prediction(pred.ctypes.data, rows, shapes, len(shapes), out.ctypes.data)
        if r != 0:
            raise ValueError(r)
        return out[:tokens]

    def timestep_embedding(self, timesteps):
        t = _f32(timesteps)
        out = np.zeros((len(t), 256), np.float32)
        r = self.lib.s2o_timestep_embedding(t, len(t), out)
        if r != 0:
            raise ValueError(r)
        return out

    def frontend_forward(self, io: dict, shapes, timesteps, video, text, emulate_bf16=False):
        """The frontend net (in0..in2 -> out0..out7 of forward_frontend, seedvr2_dit.cpp:1183-1295) as this
        build restates it (the exported graph is not in the reference tree):
          video = patchify(latents) W_vid_in^T + b;  text = text W_txt_in^T + b
          e = silu(temb W_emb0^T + b0); e = silu(e W_emb1^T + b1); modulation = e W_emb2^T + b2 -> [6][batch][D]
        emulate_bf16 rounds the GEMM activations the device path stores in bf16 (patches, text)."""
        rnd = self.round_bf16 if emulate_bf16 else _f32
        p = self.patchify_video(video, shapes)
        v = rnd(p) @ _f32(io["w_vid_in"]).T + _bias(io.get("b_vid_in"))
        t = rnd(text) @ _f32(io["w_txt_in"]).T + _bias(io.get("b_txt_in"))
        temb = self.timestep_embedding(timesteps).astype(np.float64)
        e = _silu(temb @ _f64(io["w_emb0"]).T + _bias(io.get("b_emb0")))
        e = _silu(e @ _f64(io["w_emb1"]).T + _bias(io.get("b_emb1")))
        emb = e @ _f64(io["w_emb2"]).T + _bias(io.get("b_emb2"))
        B = len(timesteps)
        D = emb.shape[1] // 6
        mod = emb.reshape(B, 6, D).transpose(1, 0, 2)
        return _f32(v), _f32(t), _f32(mod)

    def tail_forward(self, io: dict, shapes, video, modulation, eps=1e-5, emulate_bf16=False):
        """The tail net + unpatchify: per sample h = rmsnorm(x) * (mod[1] + tail_ada[1]) + (mod[0] + tail_ada[0]),
        prediction patches = h W_out^T + b_out [patches][64] -> tokens [tokens][16]."""
        rnd = self.round_bf16 if emulate_bf16 else _f32
        video = _f32(video)
        mod = _f32(modulation)
        ada = _f32(io["tail_ada"])
        out = []
        off = 0
        for s, (t, h, w) in enumerate(_i32(shapes).reshape(-1, 3).tolist()):
            n = t * (h // 2) * (w // 2)
            x = video[off:off + n]
            off += n
            ss = np.concatenate([np.square(x[i:i + 4096], dtype=np.float64).mean(axis=1)
                                 for i in range(0, len(x), 4096)])[:, None]
            inv = (1.0 / np.sqrt(ss.astype(np.float32) + np.float32(eps))).astype(np.float32)
            hh = x * inv * (mod[1, s] + ada[1]) + (mod[0, s] + ada[0])
            pp = rnd(hh) @ _f32(io["w_out"]).T + _bias(io.get("b_out"))
            out.append(self.unpatchify_prediction(_f32(pp), [[t, h, w]]))
        return np.concatenate(out)


    # ---- denoise loop (seedvr2_pipeline.cpp) ----
    def assemble_dit_input(self, latent, condition):
        """latent, condition: [16][tokens] planes -> [tokens][33] rows (predict, :296-318)."""
        latent = _f32(latent)
        condition = _f32(condition)
        tokens = latent.shape[1]
        out = np.zeros((tokens, 33), np.float32)
        self.lib.s2o_assemble_dit_input(latent, tokens, condition, tokens, tokens, out)
        return out

    def apply_cfg(self, pos, neg, scale, rescale):
        pos = _f32(pos)
        out = np.zeros_like(pos)
        self.lib.s2o_apply_cfg(pos, _f32(neg), pos.size, scale, rescale, out)
        return out

    def denoise_schedule(self, steps, step):
        t, d = C.c_float(), C.c_float()
        self.lib.s2o_denoise_schedule(steps, step, C.byref(t), C.byref(d))
        return t.value, d.value

    def euler_update(self, latent, pred, delta):
        """latent [16][tokens] (returned updated copy), pred [tokens][16]."""
        lat = _f32(latent).copy()
        self.lib.s2o_euler_update(lat, lat.shape[1], lat.shape[1], _f32(pred), delta)
        return lat

    def denoise(self, predict, latent, condition, steps, cfg_scale=1.0, cfg_rescale=0.0):
        """SeedVR2Pipeline::denoise (seedvr2_pipeline.cpp:536-588) with predict(video_rows [tokens][33],
        timestep, positive: bool) -> prediction [tokens][16] supplied by the caller."""
        lat = _f32(latent).copy()
        for step in range(steps):
            t, delta = self.denoise_schedule(steps, step)
            rows = self.assemble_dit_input(lat, condition)
            pred = predict(rows, t, True)
            if cfg_scale != 1.0:
                neg = predict(rows, t, False)
                pred = self.apply_cfg(pred, neg, cfg_scale, cfg_rescale)
            lat = self.euler_update(lat, pred, delta)
        return lat


    # ---- VAE DecomposedConv3D (decomposed_conv3d.cpp) ----
    def conv3d_forward(self, cfg, bias, weights, x, mem=None, keep_memory=True):
        """x [c][d][h][w]; mem [c][m][h][w] cached frames or None (head = copies of frame 0).
        Returns (out [co][t][oh][ow], next memory [c][kernel_t - stride_t][h][w] or None)."""
        cfg = _i32(cfg)
        x = _f32(x)
        c, d, h, w = x.shape
        m = 0 if mem is None else mem.shape[1]
        dims = np.zeros(4, np.int32)
        if self.lib.s2o_conv3d_dims(cfg, w, h, d, m if m else int(cfg[7]), dims) != 0:
            raise ValueError(-1)
        out = np.zeros((dims[3], dims[2], dims[1], dims[0]), np.float32)
        cache = int(cfg[4] - cfg[5])
        nm = np.zeros((c, cache, h, w), np.float32) if (keep_memory and cache > 0) else None
        b = _f32(bias) if bias is not None else None
        memf = _f32(mem) if mem is not None else None
        r = self.lib.s2o_conv3d_forward(cfg, b.ctypes.data if b is not None else None, _f32(weights), x, w, h, d,
                                        memf.ctypes.data if memf is not None else None, m, out,
                                        nm.ctypes.data if nm is not None else None)
        if r != 0:
            raise ValueError(r)
        return out, nm


class PortConv3dLayer:
    """DecomposedConv3D with its temporal memory (decomposed_conv3d.cpp:605-765) on top of the stateless
    C restatement Port.conv3d_forward."""

    def __init__(self, port: Port, cfg, bias, weights, emulate_bf16=False):
        self.port, self.cfg, self.bias = port, list(cfg), bias
        self.emulate = emulate_bf16
        self.weights = port.round_bf16(weights) if emulate_bf16 else weights
        self.memory = None

    def forward(self, x, state):
        if state != VAE_MEMORY_ACTIVE:
            self.memory = None
        x = self.port.round_bf16(x) if self.emulate else _f32(x)
        mem = self.memory if (state == VAE_MEMORY_ACTIVE and self.memory is not None) else None
        if mem is not None and mem.shape[2:] != x.shape[2:]:
            raise ValueError(-1)
        y, nm = self.port.conv3d_forward(self.cfg, self.bias, self.weights, x, mem,
                                         keep_memory=state != VAE_MEMORY_DISABLED)
        if state != VAE_MEMORY_DISABLED and nm is not None:
            self.memory = nm
        return y


def split_conv_blob(blob, offset=0):
    """(cfg, bias, weights, next offset) of one DecomposedConv3D in a weight blob (its load_model order)."""
    cfg = [int(v) for v in blob[offset:offset + 16]]
    co, ci, kw, kh, kt = cfg[:5]
    o = offset + 16
    bias = None
    if cfg[15]:
        bias = _f32(blob[o:o + co])
        o += co
    n = kt * co * ci * kh * kw
    w = _f32(blob[o:o + n]).reshape(kt, co, ci, kh, kw)
    return cfg, bias, w, o + n


class PortDownsample:
    """VAEDownsample3D::forward (vae_downsample3d.cpp:145-173): zero padding on the right / bottom, then
    its DecomposedConv3D.  blob: its load_model sequence (channels, pad_right, pad_bottom, conv blob)."""

    def __init__(self, port: Port, blob, emulate_bf16=False):
        blob = _f32(blob)
        self.channels, self.pad_right, self.pad_bottom = (int(v) for v in blob[:3])
        cfg, b, w, _ = split_conv_blob(blob, 3)
        self.conv = PortConv3dLayer(port, cfg, b, w, emulate_bf16)

    def forward(self, x, state):
        x = _f32(x)
        c, d, h, w = x.shape
        if c != self.channels:
            raise ValueError(-1)
        padded = np.zeros((c, d, h + self.pad_bottom, w + self.pad_right), np.float32)
        padded[:, :, :h, :w] = x
        return self.conv.forward(padded, state)


class PortUpsample:
    """VAEUpsample3D::forward (vae_upsample3d.cpp:258-320): upscale conv to channels * tr * sr^2, the
    pixel / temporal shuffle (dropping frame 1 unless the memory is active, when tr = 2), then the post
    conv.  blob: config (channels, temporal_ratio, spatial_ratio, remove_temporal_head), post conv blob,
    upscale conv blob."""

    def __init__(self, port: Port, blob, emulate_bf16=False):
        blob = _f32(blob)
        self.channels, self.tr, self.sr, self.remove_head = (int(v) for v in blob[:4])
        cfg, b, w, o = split_conv_blob(blob, 4)
        self.post = PortConv3dLayer(port, cfg, b, w, emulate_bf16)
        cfg, b, w, _ = split_conv_blob(blob, o)
        self.upscale = PortConv3dLayer(port, cfg, b, w, emulate_bf16)

    def forward(self, x, state):
        x = _f32(x)
        if x.shape[0] != self.channels:
            raise ValueError(-1)
        packed = self.upscale.forward(x, state)
        ch, tr, sr = self.channels, self.tr, self.sr
        _, pd, ph, pw = packed.shape
        # packed channel ((yo * sr + xo) * tr + z) * ch + c -> frame * tr + z, pixel (y * sr + yo, x * sr + xo)
        p = packed.reshape(sr, sr, tr, ch, pd, ph, pw)
        sh = np.transpose(p, (3, 4, 2, 5, 0, 6, 1)).reshape(ch, pd * tr, ph * sr, pw * sr)
        if self.remove_head and state != VAE_MEMORY_ACTIVE:
            sh = np.concatenate([sh[:, :1], sh[:, 2:]], axis=1)
        return self.post.forward(np.ascontiguousarray(sh), state)


def ref_mha_forward(E, heads, scale, weights, x, chunk=128, path: str = REF_VAE_SO):
    """The reference's own VAEChunkedMHA (oracle/_ref/libs2_ref_vae.so) on its CPU path."""
    lib = C.CDLL(path)
    lib.s2ref_mha_forward.argtypes = [_i32p, C.c_float, _f32p, C.c_size_t, _f32p, C.c_int, _f32p]
    x = _f32(x)
    w = _f32(weights)
    out = np.zeros_like(x)
    r = lib.s2ref_mha_forward(_i32([E, heads, E * E, E, E, chunk]), scale, w, w.size, x, x.shape[0], out)
    if r != 0:
        raise ValueError(r)
    return out


def ref_moments_to_latent(moments, sample_posterior=True, seed=666, path: str = REF_VAE_RT_SO):
    """The reference's own moments_to_latent (seedvr2_vae.cpp:454-478): moments fp32 [32, d, h, w] ->
    latent fp32 [16, d, h, w], posterior noise from its own generator."""
    if not os.path.exists(path):
        raise FileNotFoundError(path)
    lib = C.CDLL(path)
    lib.ref_vae_moments_to_latent.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_uint64, _f32p]
    m = _f32(moments)
    _, d, h, w = m.shape
    out = np.zeros((16, d, h, w), dtype=np.float32)
    r = lib.ref_vae_moments_to_latent(m, w, h, d, int(bool(sample_posterior)), int(seed), out)
    if r != 0:
        raise ValueError(r)
    return out


def ref_vae_load(kind, blob, path: str = REF_VAE_SO) -> int:
    """Load-time code (first nonzero of load_param / load_model / create_pipeline) of the reference's own
    DecomposedConv3D (kind 0; the blob's 16 config values also go through load_param), VAEDownsample3D (1)
    or VAEUpsample3D (2) given the floats its load_model reads."""
    lib = C.CDLL(path)
    lib.s2ref_vae_load.argtypes = [C.c_int, _f32p, C.c_size_t]
    n = len(blob)
    return int(lib.s2ref_vae_load(kind, _f32(blob) if n else np.zeros(1, np.float32), n))


def ref_mha_code(ip, scale, weights, x, path: str = REF_VAE_SO) -> int:
    """Return code of the reference's own VAEChunkedMHA built from params ip = (embed_dim, num_heads,
    weight_data_size, kdim, vdim, chunk_size) and scale, then run on x [tokens][weight_data_size / embed_dim]
    when it loaded."""
    lib = C.CDLL(path)
    lib.s2ref_mha_forward.argtypes = [_i32p, C.c_float, _f32p, C.c_size_t, _f32p, C.c_int, _f32p]
    x = _f32(x)
    w = _f32(weights) if len(weights) else np.zeros(1, np.float32)
    out = np.zeros_like(x)
    return int(lib.s2ref_mha_forward(_i32(ip), scale, w, len(weights), x, x.shape[0], out))


class RefResample:
    """The reference's own VAEDownsample3D (kind 0) / VAEUpsample3D (kind 1) (oracle/_ref/libs2_ref_vae.so)."""

    def __init__(self, kind, blob, path: str = REF_VAE_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        lib = C.CDLL(path)
        lib.s2ref_resample_create.argtypes = [C.c_int, _f32p, C.c_size_t]
        lib.s2ref_resample_create.restype = C.c_void_p
        lib.s2ref_resample_forward.argtypes = [C.c_void_p, C.c_int, _f32p, C.c_int, C.c_int, C.c_int, C.c_int, _f32p,
                                               C.c_size_t, _i32p]
        lib.s2ref_resample_free.argtypes = [C.c_void_p]
        self.lib = lib
        blob = _f32(blob)
        self.handle = lib.s2ref_resample_create(kind, blob, blob.size)
        if not self.handle:
            raise ValueError("load failed")

    def forward(self, x, memory_state):
        x = _f32(x)
        c, d, h, w = x.shape
        cap = 64 * max(c, 8) * (2 * d + 8) * (2 * h + 8) * (2 * w + 8)
        out = np.zeros(cap, np.float32)
        dims = np.zeros(4, np.int32)
        r = self.lib.s2ref_resample_forward(self.handle, memory_state, x, w, h, d, c, out, cap, dims)
        if r != 0:
            raise ValueError(r)
        ow, oh, od, oc = dims.tolist()
        return out[:ow * oh * od * oc].reshape(oc, od, oh, ow).copy()

    def __del__(self):
        if getattr(self, "handle", None):
            self.lib.s2ref_resample_free(self.handle)
            self.handle = None


def _f64(a) -> np.ndarray:
    return np.asarray(a, dtype=np.float64)


def _bias(b):
    return 0.0 if b is None else np.asarray(b, dtype=np.float64)


def _silu(x):
    return x / (1.0 + np.exp(-x))


class RefIO:
    """The reference's own patchify_video / make_timestep_embedding / unpatchify_prediction
    (oracle/_ref/libs2_ref_dit_io.so; seedvr2_dit.cpp:167-326 compiled unmodified)."""

    def __init__(self, path: str = REF_IO_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        lib = C.CDLL(path)
        lib.s2ref_patchify_video.argtypes = [C.c_void_p, C.c_int, _i32p, C.c_int, C.c_void_p, C.c_void_p]
        lib.s2ref_unpatchify_prediction.argtypes = [C.c_void_p, C.c_int, _i32p, C.c_int, C.c_void_p]
        lib.s2ref_timestep_embedding.argtypes = [_f32p, C.c_int, C.c_void_p]
        lib.s2ref_apply_cfg.argtypes = [_f32p, _f32p, C.c_int, C.c_int, C.c_float, C.c_float, _f32p]
        self.lib = lib

    def apply_cfg(self, pos, neg, scale, rescale):
        pos = _f32(pos)
        out = np.zeros_like(pos)
        w = pos.shape[-1] if pos.ndim > 1 else pos.size
        self.lib.s2ref_apply_cfg(pos, _f32(neg), w, pos.size // w, scale, rescale, out)
        return out

    def patchify_video(self, video, shapes, rows=None):
        video = _f32(video)
        shapes = _i32(shapes).reshape(-1, 3)
        rows = video.shape[0] if rows is None else rows
        patches = int(sum(max(t, 0) * (max(h, 0) // 2) * (max(w, 0) // 2) for t, h, w in shapes.tolist()))
        out = np.zeros((max(patches, 1), 132), np.float32)
        oshapes = np.zeros((max(len(shapes), 1), 3), np.int32)
        r = self.lib.s2ref_patchify_video(video.ctypes.data, rows, shapes, len(shapes), out.ctypes.data,
                                          oshapes.ctypes.data)
        if r != 0:
            raise ValueError(r)
        return out[:patches]

    def unpatchify_prediction(self, pred, shapes, rows=None):
        pred = _f32(pred)
        shapes = _i32(shapes).reshape(-1, 3)
        rows = pred.shape[0] if rows is None else rows
        tokens = int(sum(max(t, 0) * max(h, 0) * max(w, 0) for t, h, w in shapes.tolist()))
        out = np.zeros((max(tokens, 1), 16), np.float32)
        r = self.lib.s2ref_unpatchify_prediction(pred.ctypes.data, rows, shapes, len(shapes), out.ctypes.data)
        if r != 0:
            raise ValueError(r)
        return out[:tokens]

    def timestep_embedding(self, timesteps):
        t = _f32(timesteps)
        out = np.zeros((max(len(t), 1), 256), np.float32)
        r = self.lib.s2ref_timestep_embedding(t if len(t) else np.zeros(1, np.float32), len(t), out.ctypes.data)
        if r != 0:
            raise ValueError(r)
        return out[:len(t)]


class RefConv3d:
    """The reference's own DecomposedConv3D layer (oracle/_ref/libs2_ref_vae.so), one layer instance
    with its temporal memory."""

    def __init__(self, cfg, bias, weights, path: str = REF_VAE_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        lib = C.CDLL(path)
        lib.s2ref_conv3d_create.argtypes = [_f32p, _f32p, C.c_size_t]
        lib.s2ref_conv3d_create.restype = C.c_void_p
        lib.s2ref_conv3d_forward.argtypes = [C.c_void_p, C.c_int, _f32p, C.c_int, C.c_int, C.c_int, C.c_int, _f32p,
                                             C.c_size_t, _i32p]
        lib.s2ref_conv3d_free.argtypes = [C.c_void_p]
        self.lib = lib
        self.cfg = _i32(cfg)
        parts = ([] if bias is None else [_f32(bias).ravel()]) + [_f32(weights).ravel()]
        blob = np.concatenate(parts).astype(np.float32)
        self.handle = lib.s2ref_conv3d_create(_f32(self.cfg.astype(np.float32)), blob, blob.size)
        if not self.handle:
            raise ValueError("DecomposedConv3D load failed")

    def forward(self, x, memory_state):
        x = _f32(x)
        c, d, h, w = x.shape
        cap = int(self.cfg[0]) * (d + 64) * (h + 2 * int(self.cfg[13]) + 8) * (w + 2 * int(self.cfg[12]) + 8)
        out = np.zeros(cap, np.float32)
        dims = np.zeros(4, np.int32)
        r = self.lib.s2ref_conv3d_forward(self.handle, memory_state, x, w, h, d, c, out, cap, dims)
        if r != 0:
            raise ValueError(r)
        ow, oh, od, oc = dims.tolist()
        return out[:ow * oh * od * oc].reshape(oc, od, oh, ow).copy()

    def __del__(self):
        if getattr(self, "handle", None):
            self.lib.s2ref_conv3d_free(self.handle)
            self.handle = None


class Ref:
    """The reference's own layer code (oracle/_ref/libs2_ref.so)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        lib = C.CDLL(path)
        lib.s2ref_plan_build.argtypes = [_i32p, C.c_int, _i32p, C.c_int, C.POINTER(C.c_void_p)]
        lib.s2ref_plan_sizes.argtypes = [C.c_void_p, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int)]
        lib.s2ref_plan_copy.argtypes = [C.c_void_p, _i32p, _i32p, _i32p, _i32p, _i32p]
        lib.s2ref_plan_free.argtypes = [C.c_void_p]
        lib.s2ref_awa_forward.argtypes = [_i32p, C.c_float, _f32p, C.c_int, C.c_int, C.POINTER(C.c_void_p),
                                          C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_int, _f32p, _f32p]
        lib.s2ref_shared_linear_forward.argtypes = [C.c_int, C.c_int, C.c_int, _f32p, _f32p, C.c_int, _f32p,
                                                    C.c_int, _f32p, _f32p]
        self.lib = lib

    def plan(self, shapes, target, shifted) -> Plan:
        shapes = _i32(shapes).reshape(-1, 3)
        h = C.c_void_p()
        r = self.lib.s2ref_plan_build(shapes, len(shapes), _i32(target), int(shifted), C.byref(h))
        if r != 0:
            raise ValueError(f"build_adaptive_window_plan returned {r}")
        nw, nt, ns = C.c_int(), C.c_int(), C.c_int()
        self.lib.s2ref_plan_sizes(h, C.byref(nw), C.byref(nt), C.byref(ns))
        windows = np.zeros((nw.value, 9), np.int32)
        swc = np.zeros(ns.value, np.int32)
        vi = np.zeros(nt.value, np.int32)
        inv = np.zeros(nt.value, np.int32)
        pos = np.zeros((nt.value, 3), np.int32)
        self.lib.s2ref_plan_copy(h, windows, swc, vi, inv, pos)
        self.lib.s2ref_plan_free(h)
        return Plan(windows, swc, vi, inv, pos)

    def awa_forward(self, *, heads, head_dim, target, shifted, eps, rope_pairs, norms, freqs, shapes,
                    text_lengths, video_qkv=None, text_qkv=None, split=None, shared_norm=False,
                    shape_int32=False, bf16=False):
        inner = heads * head_dim
        shapes = _i32(shapes).reshape(-1, 3)
        tl = _i32(text_lengths)
        nv = int(np.prod(shapes, axis=1).sum())
        nt = int(tl.sum())
        norms = _f32(norms).reshape(4, head_dim)
        wts = [norms[0], norms[1]] + ([] if shared_norm else [norms[2], norms[3]]) + [_f32(freqs)]
        wflat = np.concatenate(wts).astype(np.float32)
        if split is None:
            arrs = [_f32(video_qkv), _f32(text_qkv)]
            nv, nt = arrs[0].shape[0], arrs[1].shape[0]  # blob heights as given (the layer validates them)
        else:
            arrs = [_f32(a) for a in split]
            nv, nt = arrs[0].shape[0], arrs[3].shape[0]
        ptrs = (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])
        if shape_int32:
            sb = shapes.astype(np.int32)
            tb = tl.astype(np.int32)
        else:
            sb = shapes.astype(np.float32)
            tb = tl.astype(np.float32)
        sb = np.ascontiguousarray(sb)
        tb = np.ascontiguousarray(tb)
        ip = _i32([heads, head_dim, target[0], target[1], target[2], int(shifted), rope_pairs, int(shared_norm),
                   int(shape_int32), int(bf16)])
        vo = np.zeros((nv, inner), np.float32)
        to = np.zeros((nt, inner), np.float32)
        r = self.lib.s2ref_awa_forward(ip, eps, wflat, len(wflat), 0 if split is None else 1, ptrs, nv, nt,
                                       sb.ctypes.data, tb.ctypes.data, len(shapes), vo, to)
        if r != 0:
            raise ValueError(f"AdaptiveWindowAttention::forward returned {r}")
        return vo, to

    def shared_linear(self, video, text, weight, bias=None):
        video = _f32(video)
        text = _f32(text)
        n, k = weight.shape
        flat = _f32(weight).reshape(-1) if bias is None else np.concatenate([_f32(weight).reshape(-1), _f32(bias)])
        vo = np.zeros((video.shape[0], n), np.float32)
        to = np.zeros((text.shape[0], n), np.float32)
        r = self.lib.s2ref_shared_linear_forward(n, k, int(bias is not None), _f32(flat), video, video.shape[0],
                                                 text, text.shape[0], vo, to)
        if r != 0:
            raise ValueError(f"SharedLinear::forward returned {r}")
        return vo, to
