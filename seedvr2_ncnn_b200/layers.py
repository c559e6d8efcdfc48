"""ctypes driver of the ncnn-surface layer classes (libseedvr2_ncnn.so).

The C++ classes ``seedvr2::AdaptiveWindowAttention``, ``seedvr2::SharedLinear``
and the VAE's ``DecomposedConv3D``, ``VAEDownsample3D``, ``VAEUpsample3D`` and
``VAEChunkedMHA`` keep the reference's ncnn custom-layer surface (creator,
ParamDict ids, ModelBin weight order, blob arity, error codes); their
``forward`` runs on libseedvr2_cuda.  This module drives them through
the library's small extern "C" driver with host fp32 arrays, the way ncnn's
Net would: create -> load_param -> load_model -> forward.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import LIB_PATH

LAYER_LIB_PATH = os.path.join(os.path.dirname(LIB_PATH), "libseedvr2_ncnn.so")
_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LAYER_LIB_PATH):
            raise ImportError(f"{LAYER_LIB_PATH} is missing: build it with `python -m seedvr2_ncnn_b200.build`")
        L = C.CDLL(LAYER_LIB_PATH)
        f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
        i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
        L.s2layer_awa_forward.argtypes = [i32p, C.c_float, f32p, C.c_int, C.c_int, C.POINTER(C.c_void_p), C.c_int,
                                          C.c_int, C.c_void_p, C.c_void_p, C.c_int, f32p, f32p]
        L.s2layer_shared_linear_forward.argtypes = [C.c_int, C.c_int, C.c_int, f32p, f32p, C.c_int, f32p, C.c_int,
                                                    f32p, f32p]
        L.s2layer_vae_create.argtypes = [C.c_int, f32p, C.c_size_t, C.POINTER(C.c_void_p)]
        L.s2layer_vae_output_shape.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, i32p]
        L.s2layer_vae_forward.argtypes = [C.c_void_p, C.c_int, f32p, C.c_int, C.c_int, C.c_int, C.c_int, f32p,
                                          C.c_size_t, i32p]
        L.s2layer_vae_reset.argtypes = [C.c_void_p]
        L.s2layer_vae_free.argtypes = [C.c_void_p]
        L.s2layer_mha_create.argtypes = [i32p, C.c_float, f32p, C.c_size_t, C.POINTER(C.c_void_p)]
        L.s2layer_mha_forward.argtypes = [C.c_void_p, f32p, C.c_int, C.c_int, f32p]
        L.s2layer_vae_free.restype = None
        vp = C.c_void_p
        L.s2net_create.restype = vp
        L.s2net_create.argtypes = []
        L.s2net_destroy.argtypes = [vp]
        L.s2net_destroy.restype = None
        L.s2net_load.argtypes = [vp, C.c_char_p, C.c_char_p]
        L.s2net_info.argtypes = [vp, C.POINTER(C.c_int), C.POINTER(C.c_int)]
        L.s2net_set_runtime.argtypes = [vp, i32p, i32p, C.c_int]
        L.s2net_extract_cuda.argtypes = [vp, C.c_int, C.POINTER(C.c_char_p), C.POINTER(vp), i32p, i32p, C.c_int,
                                         C.POINTER(C.c_char_p), C.POINTER(vp), i32p, i32p]
        L.s2layer_vae_reset.restype = None
        _lib = L
    return _lib


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def awa_forward(*, heads, head_dim, target, shifted, eps, rope_pairs, norms, freqs, shapes, text_lengths,
                video_qkv=None, text_qkv=None, split=None, shared_norm=False, shape_int32=False, bf16=False):
    """AdaptiveWindowAttention::forward through the layer surface; returns (code, video_out, text_out)."""
    inner = heads * head_dim
    shapes = np.ascontiguousarray(np.asarray(shapes, np.int32).reshape(-1, 3))
    tl = np.ascontiguousarray(np.asarray(text_lengths, np.int32))
    norms = _f32(norms).reshape(4, head_dim)
    w = np.concatenate(([norms[0], norms[1]] + ([] if shared_norm else [norms[2], norms[3]])) + [_f32(freqs)])
    w = _f32(w)
    if split is None:
        arrs = [_f32(video_qkv), _f32(text_qkv)]
        nv, nt = arrs[0].shape[0], arrs[1].shape[0]
    else:
        arrs = [_f32(a) for a in split]
        nv, nt = arrs[0].shape[0], arrs[3].shape[0]
    ptrs = (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])
    sb = np.ascontiguousarray(shapes if shape_int32 else shapes.astype(np.float32))
    tb = np.ascontiguousarray(tl if shape_int32 else tl.astype(np.float32))
    ip = np.asarray([heads, head_dim, target[0], target[1], target[2], int(shifted), rope_pairs, int(shared_norm),
                     int(shape_int32), int(bf16)], np.int32)
    vo = np.zeros((nv, inner), np.float32)
    to = np.zeros((nt, inner), np.float32)
    r = lib().s2layer_awa_forward(ip, eps, w, len(w), 0 if split is None else 1, ptrs, nv, nt, sb.ctypes.data,
                                  tb.ctypes.data, len(shapes), vo, to)
    return r, vo, to


def shared_linear(video, text, weight, bias=None):
    """SharedLinear::forward through the layer surface; returns (code, video_out, text_out)."""
    video, text = _f32(video), _f32(text)
    n, k = weight.shape
    flat = _f32(weight).reshape(-1) if bias is None else np.concatenate([_f32(weight).reshape(-1), _f32(bias)])
    vo = np.zeros((video.shape[0], n), np.float32)
    to = np.zeros((text.shape[0], n), np.float32)
    r = lib().s2layer_shared_linear_forward(n, k, int(bias is not None), _f32(flat), video, video.shape[0], text,
                                            text.shape[0], vo, to)
    return r, vo, to


class LayerError(RuntimeError):
    """A layer call returned a nonzero code (the reference's codes: -1 invalid, -100 allocation; plus the
    library's -3 CUDA, -5 no device)."""

    def __init__(self, what, code):
        super().__init__(f"{what} returned {code}")
        self.code = code


# VAE layer kinds of s2layer_vae_create
DECOMPOSED_CONV3D, VAE_DOWNSAMPLE3D, VAE_UPSAMPLE3D = 0, 1, 2


def _blob(a):
    a = _f32(np.asarray(a).ravel())
    return (a if a.size else np.zeros(1, np.float32)), int(a.size)


def vae_load_code(kind, blob):
    """First nonzero code of load_param / load_model / create_pipeline for a VAE layer, else 0."""
    arr, n = _blob(blob)
    h = C.c_void_p()
    r = lib().s2layer_vae_create(kind, arr, n, C.byref(h))
    if r == 0:
        lib().s2layer_vae_free(h)
    return r


class VaeLayer:
    """DecomposedConv3D / VAEDownsample3D / VAEUpsample3D through the layer surface, built from the floats
    its load_model reads (for DecomposedConv3D the 16 config values also go through load_param)."""

    def __init__(self, kind, blob):
        arr, n = _blob(blob)
        self.handle = C.c_void_p()
        r = lib().s2layer_vae_create(kind, arr, n, C.byref(self.handle))
        if r != 0:
            self.handle = None
            raise LayerError("load", r)

    def output_shape(self, w, h, d, memory_state):
        dims = np.zeros(4, np.int32)
        r = lib().s2layer_vae_output_shape(self.handle, memory_state, w, h, d, dims)
        if r != 0:
            raise LayerError("output_shape", r)
        return dims.tolist()

    def forward(self, x, memory_state):
        """x [c][d][h][w] fp32 (host) under the VAE memory state -> [c'][d'][h'][w']."""
        x = _f32(x)
        c, d, h, w = x.shape
        try:
            ow, oh, od, oc = self.output_shape(w, h, d, memory_state)
            cap = ow * oh * od * oc
        except LayerError:
            cap = 1  # forward reports the same rejection (and drops the cached frames as it does)
        out = np.zeros(max(cap, 1), np.float32)
        dims = np.zeros(4, np.int32)
        r = lib().s2layer_vae_forward(self.handle, memory_state, x, w, h, d, c, out, out.size, dims)
        if r != 0:
            raise LayerError("forward", r)
        ow, oh, od, oc = dims.tolist()
        return out[:ow * oh * od * oc].reshape(oc, od, oh, ow).copy()

    def reset_temporal_memory(self):
        lib().s2layer_vae_reset(self.handle)

    def close(self):
        if self.handle:
            lib().s2layer_vae_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _mha_params(E, heads, wds, kdim, vdim, chunk):
    return np.asarray([E, heads, E * E if wds is None else wds, E if kdim is None else kdim,
                       E if vdim is None else vdim, chunk], np.int32)


def mha_load_code(E, heads, scale, weights, *, wds=None, kdim=None, vdim=None, chunk=128):
    """First nonzero code of VAEChunkedMHA's load_param / load_model / create_pipeline, else 0."""
    arr, n = _blob(weights)
    h = C.c_void_p()
    r = lib().s2layer_mha_create(_mha_params(E, heads, wds, kdim, vdim, chunk), scale, arr, n, C.byref(h))
    if r == 0:
        lib().s2layer_vae_free(h)
    return r


class VaeMhaLayer:
    """VAEChunkedMHA through the layer surface: x [tokens][E] (host) -> [tokens][E]."""

    def __init__(self, E, heads, scale, weights, chunk=128):
        arr, n = _blob(weights)
        self.E = E
        self.handle = C.c_void_p()
        r = lib().s2layer_mha_create(_mha_params(E, heads, None, None, None, chunk), scale, arr, n,
                                     C.byref(self.handle))
        if r != 0:
            self.handle = None
            raise LayerError("load", r)

    def forward(self, x):
        x = _f32(x)
        out = np.zeros_like(x)
        r = lib().s2layer_mha_forward(self.handle, x, x.shape[0], x.shape[1], out)
        if r != 0:
            raise LayerError("forward", r)
        return out

    def close(self):
        if self.handle:
            lib().s2layer_vae_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Net:
    """A block graph from ncnn .param / .bin files (seedvr2::Net) with SeedVR2's AdaptiveWindowAttention and
    SharedLinear registered; blobs by name on the device."""

    def __init__(self, param_path, bin_path):
        self.handle = C.c_void_p(lib().s2net_create())
        r = lib().s2net_load(self.handle, str(param_path).encode(), str(bin_path).encode())
        if r != 0:
            self.close()
            raise LayerError("Net load", r)

    def info(self):
        n, b = C.c_int(), C.c_int()
        lib().s2net_info(self.handle, C.byref(n), C.byref(b))
        return n.value, b.value

    def set_runtime(self, shapes, text_lengths):
        sh = np.ascontiguousarray(np.asarray(shapes, np.int32).reshape(-1, 3))
        tl = np.ascontiguousarray(np.asarray(text_lengths, np.int32))
        r = lib().s2net_set_runtime(self.handle, sh, tl, len(tl))
        if r != 0:
            raise LayerError("Net set_runtime", r)

    def extract(self, inputs: dict, outputs: dict):
        """inputs / outputs: name -> contiguous fp32 CUDA tensor [rows][cols] (outputs are written)."""
        def arr(d):
            names = (C.c_char_p * len(d))(*[k.encode() for k in d])
            ptrs = (C.c_void_p * len(d))(*[t.data_ptr() for t in d.values()])
            rows = np.ascontiguousarray([t.shape[0] for t in d.values()], np.int32)
            cols = np.ascontiguousarray([t.shape[1] for t in d.values()], np.int32)
            return names, ptrs, rows, cols
        i, o = arr(inputs), arr(outputs)
        r = lib().s2net_extract_cuda(self.handle, len(inputs), *i, len(outputs), *o)
        if r != 0:
            raise LayerError("Net extract", r)

    def close(self):
        if self.handle:
            lib().s2net_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
