"""ctypes driver of the ncnn-surface layer classes (libseedvr2_ncnn.so).

The C++ classes ``seedvr2::AdaptiveWindowAttention`` and
``seedvr2::SharedLinear`` keep the reference's ncnn custom-layer surface
(creator, ParamDict ids, ModelBin weight order, blob arity, error codes);
their ``forward`` runs on libseedvr2_cuda.  This module drives them through
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
