"""ctypes bindings of libseedvr2_cuda (include/seedvr2_cuda.h).

Device buffers are passed as raw pointers; the helpers here accept torch
tensors for convenience (torch is used only for device memory and streams).
Every entry point returns the library's integer status; :func:`check` turns a
non-zero status into :class:`S2Error`.
"""
from __future__ import annotations

import ctypes as C
import os

from . import LIB_PATH

S2_OK = 0
S2_ERR_INVALID = -1
S2_ERR_PLAN = -2
S2_ERR_CUDA = -3
S2_ERR_TIMEOUT = -4
S2_ERR_DEVICE = -5
S2_ERR_TOO_LARGE = -6
S2_ERR_ALLOC = -100

S2_DTYPE_F32 = 0
S2_DTYPE_BF16 = 1

S2_WINDOW_TARGET = 0
S2_WINDOW_EXTENT = 1

S2_KERNEL_SHARED_LINEAR = 0
S2_KERNEL_WINDOW_ATTENTION = 1
S2_KERNEL_PREPARE_QKV = 2
S2_KERNEL_ADA_RMSNORM = 3
S2_KERNEL_TEXT_POOL = 4
S2_KERNEL_OTHER = 5
S2_KERNEL_COMM = 6
S2_KERNEL_HOST_WAIT = 7
KERNEL_NAMES = ["shared_linear", "window_attention", "prepare_qkv", "ada_rmsnorm", "text_pool", "other", "comm",
                "host_wait"]

S2_EPI_STORE = 0
S2_EPI_GELU_TANH = 1
S2_EPI_GATE_RESIDUAL = 2

# Every symbol include/seedvr2_cuda.h declares.
EXPORTED = [
    "s2_init", "s2_destroy", "s2_set_stream", "s2_status", "s2_error_string", "s2_version", "s2_launch_count",
    "s2_profile_enable", "s2_profile_read",
    "s2_plan_build", "s2_plan_info", "s2_plan_copy", "s2_plan_free", "s2_plan_schedule_copy", "s2_debug_poke_schedule",
    "s2_awa_forward", "s2_awa_forward_static", "s2_awa_static_status", "s2_shared_linear", "s2_ada_rmsnorm", "s2_ada_layernorm",
    "s2_convert_f32_bf16",
    "s2_count_nonfinite", "s2_binary_op", "s2_norm_f32", "s2_gelu_f32",
    "s2_dit_create", "s2_dit_free", "s2_dit_set_block_weights", "s2_dit_set_block_norm", "s2_dit_init_random",
    "s2_dit_forward",
    "s2_dit_set_check_finite", "s2_dit_nonfinite_report", "s2_dit_set_checkpoints",
    "s2_dit_forward_host", "s2_dit_forward_host_async", "s2_dit_host_wait", "s2_vae_temporal_segments",
    "s2_vae_encode_frames", "s2_vae_decode_frames", "s2_vae_posterior_noise", "s2_vae_moments_to_latent",
    "s2_vae_unscale_latent", "s2_shard_build", "s2_shard_counts", "s2_shard_lists", "s2_shard_windows", "s2_shard_free",
    "s2_dist_unique_id", "s2_dist_init", "s2_dist_sync", "s2_dist_destroy", "s2_peer_barrier",
    "s2_dit_forward_sharded",
    "s2_patchify_video", "s2_unpatchify_prediction", "s2_timestep_embedding", "s2_dit_set_io_weights",
    "s2_dit_forward_frontend", "s2_dit_forward_tail", "s2_dit_forward_step", "s2_dit_forward_step_host",
    "s2_dit_denoise", "s2_dit_denoise_host", "s2_apply_cfg",
    "s2_conv3d_create", "s2_conv3d_output_shape", "s2_conv3d_forward", "s2_conv3d_reset_memory", "s2_conv3d_free",
    "s2_vae_resample_create", "s2_vae_resample_output_shape", "s2_vae_resample_forward",
    "s2_vae_resample_reset_memory", "s2_vae_resample_free",
    "s2_vae_mha_create", "s2_vae_mha_forward", "s2_vae_mha_free",
]

S2_VAE_DOWNSAMPLE = 0
S2_VAE_UPSAMPLE = 1

S2_VAE_MEMORY_DISABLED = 0
S2_VAE_MEMORY_INITIALIZING = 1
S2_VAE_MEMORY_ACTIVE = 2

# Widths fixed by the reference's DiT input/output formats.
S2_LATENT_CHANNELS = 33
S2_PATCH_FEATURES = 132
S2_PRED_CHANNELS = 16
S2_PRED_FEATURES = 64
S2_TEXT_CHANNELS = 5120
S2_TIME_FEATURES = 256


class S2Error(RuntimeError):
    def __init__(self, code: int, what: str):
        super().__init__(f"{what} failed: {code} ({error_string(code)})")
        self.code = code


class AwaParams(C.Structure):
    _fields_ = [
        ("heads", C.c_int), ("head_dim", C.c_int), ("window", C.c_int * 3), ("window_mode", C.c_int),
        ("shifted", C.c_int), ("epsilon", C.c_float), ("rope_pairs", C.c_int),
        ("official_bf16_attention", C.c_int), ("norm_weights", C.c_void_p), ("rope_freqs", C.c_void_p),
    ]


class DitConfig(C.Structure):
    _fields_ = [
        ("num_blocks", C.c_int), ("hidden", C.c_int), ("heads", C.c_int), ("head_dim", C.c_int),
        ("mlp_hidden", C.c_int), ("rope_pairs", C.c_int), ("window", C.c_int * 3), ("window_mode", C.c_int),
        ("norm_eps", C.c_float), ("qk_eps", C.c_float), ("qkv_bias", C.c_int), ("out_bias", C.c_int),
        ("mlp_bias", C.c_int),
    ]


class BlockHostWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("ada", "w_qkv", "b_qkv", "w_out", "b_out", "w_up", "b_up", "w_down",
                                          "b_down", "qk_norm", "rope_freqs")]


class DenoiseOptions(C.Structure):
    _fields_ = [("steps", C.c_int), ("cfg_scale", C.c_float), ("cfg_rescale", C.c_float)]


class IoHostWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("w_vid_in", "b_vid_in", "w_txt_in", "b_txt_in", "w_emb0", "b_emb0",
                                          "w_emb1", "b_emb1", "w_emb2", "b_emb2", "tail_ada", "w_out", "b_out")]


_lib = None


def lib() -> C.CDLL:
    """Loads libseedvr2_cuda.so (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python -m seedvr2_ncnn_b200.build` "
                          "(there is no fallback implementation)")
    L = C.CDLL(LIB_PATH)
    vp, ip, i64 = C.c_void_p, C.c_int, C.c_int64
    pint = C.POINTER(C.c_int)
    L.s2_init.argtypes = [ip, vp, C.POINTER(vp)]
    L.s2_destroy.argtypes = [vp]
    L.s2_destroy.restype = None
    L.s2_set_stream.argtypes = [vp, vp]
    L.s2_status.argtypes = [vp]
    L.s2_error_string.argtypes = [ip]
    L.s2_error_string.restype = C.c_char_p
    L.s2_version.argtypes = []
    L.s2_launch_count.argtypes = [vp]
    L.s2_launch_count.restype = C.c_uint64
    L.s2_profile_enable.argtypes = [vp, ip]
    L.s2_profile_read.argtypes = [vp, ip, C.POINTER(C.c_int64), C.POINTER(C.c_double), C.POINTER(C.c_double),
                                  C.POINTER(C.c_double)]
    L.s2_plan_build.argtypes = [pint, ip, pint, ip, ip, C.POINTER(vp)]
    L.s2_plan_info.argtypes = [vp, pint, pint, pint]
    L.s2_plan_copy.argtypes = [vp, pint, pint, pint, pint, pint]
    L.s2_plan_free.argtypes = [vp]
    L.s2_plan_free.restype = None
    L.s2_plan_schedule_copy.argtypes = [vp, vp, pint, pint, vp, vp, vp, vp, vp]
    L.s2_debug_poke_schedule.argtypes = [vp, vp, ip, ip, ip]
    L.s2_awa_forward.argtypes = [vp, C.POINTER(AwaParams), vp, pint, pint, ip, ip, vp, vp, vp, i64, vp, vp, vp, i64,
                                 ip, vp, vp]
    L.s2_awa_forward_static.argtypes = [C.POINTER(AwaParams), pint, pint, ip, ip, vp, vp, vp, i64, vp, vp, vp, i64,
                                        ip, vp, vp, vp]
    L.s2_awa_static_status.argtypes = [vp]
    L.s2_shared_linear.argtypes = [vp, ip, ip, ip, ip, vp, vp, vp, vp, ip, vp, ip, vp, vp]
    L.s2_ada_rmsnorm.argtypes = [vp, ip, ip, vp, C.c_float, vp, vp, vp]
    L.s2_ada_layernorm.argtypes = [vp, ip, ip, vp, C.c_float, vp, vp, vp]
    L.s2_binary_op.argtypes = [vp, ip, ip, ip, vp, vp, ip, vp]
    L.s2_norm_f32.argtypes = [vp, ip, ip, ip, vp, C.c_float, vp, vp, vp]
    L.s2_gelu_f32.argtypes = [vp, ip, i64, vp, vp]
    L.s2_dit_set_block_norm.argtypes = [vp, ip, ip]
    L.s2_convert_f32_bf16.argtypes = [vp, vp, vp, i64]
    L.s2_dit_create.argtypes = [vp, C.POINTER(DitConfig), C.POINTER(vp)]
    L.s2_dit_free.argtypes = [vp]
    L.s2_dit_free.restype = None
    L.s2_dit_set_block_weights.argtypes = [vp, ip, C.POINTER(BlockHostWeights)]
    L.s2_dit_init_random.argtypes = [vp, C.c_uint64]
    L.s2_count_nonfinite.argtypes = [vp, vp, i64, C.c_int, C.POINTER(C.c_int64)]
    L.s2_dit_set_check_finite.argtypes = [vp, C.c_int]
    L.s2_dit_set_checkpoints.argtypes = [vp, vp, C.c_int, vp, vp]
    L.s2_dit_nonfinite_report.argtypes = [vp, C.POINTER(C.c_int), C.POINTER(C.c_int64), C.POINTER(C.c_int64)]
    L.s2_dit_forward.argtypes = [vp, pint, ip, vp, vp]
    L.s2_dit_forward_host.argtypes = [vp, pint, pint, ip, vp, vp, vp, vp, vp]
    L.s2_dit_forward_host_async.argtypes = [vp, pint, pint, ip, vp, vp, vp, vp, vp]
    L.s2_dit_host_wait.argtypes = [vp]
    L.s2_vae_temporal_segments.argtypes = [ip, ip, ip, ip, pint]
    L.s2_vae_encode_frames.argtypes = [ip]
    L.s2_vae_decode_frames.argtypes = [ip]
    L.s2_vae_posterior_noise.argtypes = [C.c_uint64, C.c_int64, vp]
    L.s2_vae_moments_to_latent.argtypes = [vp, vp, ip, ip, ip, vp, vp]
    L.s2_vae_unscale_latent.argtypes = [vp, vp, C.c_int64]
    L.s2_shard_build.argtypes = [pint, ip, pint, ip, ip, ip, C.POINTER(vp)]
    L.s2_shard_counts.argtypes = [vp, ip, pint, pint, pint]
    L.s2_shard_lists.argtypes = [vp, ip, pint, pint, pint]
    L.s2_shard_windows.argtypes = [vp, ip, pint, pint]
    L.s2_shard_free.argtypes = [vp]
    L.s2_shard_free.restype = None
    L.s2_dist_unique_id.argtypes = [vp]
    L.s2_dist_init.argtypes = [vp, vp, ip, ip, ip]
    L.s2_dist_sync.argtypes = [vp]
    L.s2_dist_destroy.argtypes = [vp]
    L.s2_dit_forward_sharded.argtypes = [vp, pint, ip, vp, vp]
    L.s2_peer_barrier.argtypes = [vp, vp, vp, ip, ip, C.c_uint32]
    L.s2_patchify_video.argtypes = [vp, vp, ip, pint, ip, vp]
    L.s2_unpatchify_prediction.argtypes = [vp, vp, ip, pint, ip, vp]
    L.s2_timestep_embedding.argtypes = [vp, C.POINTER(C.c_float), ip, vp]
    L.s2_dit_set_io_weights.argtypes = [vp, C.POINTER(IoHostWeights)]
    L.s2_dit_forward_frontend.argtypes = [vp, pint, pint, C.POINTER(C.c_float), ip, vp, ip, vp, ip, vp, vp, vp]
    L.s2_dit_forward_tail.argtypes = [vp, pint, ip, vp, ip, vp, vp]
    L.s2_dit_forward_step.argtypes = [vp, pint, pint, C.POINTER(C.c_float), ip, vp, ip, vp, ip, vp, vp]
    L.s2_dit_forward_step_host.argtypes = [vp, pint, pint, C.POINTER(C.c_float), ip, vp, ip, vp, ip, vp, vp]
    L.s2_dit_denoise.argtypes = [vp, pint, vp, i64, vp, i64, vp, ip, vp, ip, C.POINTER(DenoiseOptions)]
    L.s2_dit_denoise_host.argtypes = [vp, pint, vp, i64, vp, i64, vp, ip, vp, ip, C.POINTER(DenoiseOptions)]
    L.s2_apply_cfg.argtypes = [vp, vp, vp, i64, C.c_float, C.c_float, vp]
    L.s2_conv3d_create.argtypes = [vp, pint, vp, vp, C.POINTER(vp)]
    L.s2_conv3d_output_shape.argtypes = [vp, ip, ip, ip, ip, pint]
    L.s2_conv3d_forward.argtypes = [vp, vp, i64, ip, ip, ip, ip, ip, vp, i64]
    L.s2_conv3d_free.argtypes = [vp]
    L.s2_conv3d_reset_memory.argtypes = [vp]
    L.s2_conv3d_reset_memory.restype = None
    L.s2_vae_resample_create.argtypes = [vp, ip, vp, C.c_size_t, C.POINTER(vp)]
    L.s2_vae_resample_output_shape.argtypes = [vp, ip, ip, ip, ip, pint]
    L.s2_vae_resample_forward.argtypes = [vp, vp, i64, ip, ip, ip, ip, ip, vp, i64]
    L.s2_vae_resample_free.argtypes = [vp]
    L.s2_vae_resample_reset_memory.argtypes = [vp]
    L.s2_vae_resample_reset_memory.restype = None
    L.s2_vae_mha_create.argtypes = [vp, ip, ip, C.c_float, vp, C.POINTER(vp)]
    L.s2_vae_mha_forward.argtypes = [vp, vp, ip, vp]
    L.s2_vae_mha_free.argtypes = [vp]
    _lib = L
    return L


def error_string(code: int) -> str:
    try:
        return lib().s2_error_string(code).decode()
    except ImportError:
        return "library not loaded"


def check(code: int, what: str) -> None:
    if code != S2_OK:
        raise S2Error(code, what)


def count_nonfinite(ctx, t) -> int:
    """NaN / Inf elements of a contiguous fp32 or bf16 CUDA tensor (s2_count_nonfinite; synchronises)."""
    import torch

    dtype = {torch.float32: S2_DTYPE_F32, torch.bfloat16: S2_DTYPE_BF16}[t.dtype]
    n = C.c_int64()
    check(lib().s2_count_nonfinite(ctx.handle, t.data_ptr(), t.numel(), dtype, C.byref(n)), "s2_count_nonfinite")
    return n.value


def _ints(values) -> C.Array:
    values = [int(v) for v in values]
    return (C.c_int * len(values))(*values)


def ptr(t) -> int | None:
    """Device (or host) address of a torch tensor / numpy array, or None."""
    if t is None:
        return None
    if hasattr(t, "data_ptr"):
        return t.data_ptr()
    return t.ctypes.data


class Context:
    """An s2_context on one device and stream (torch's current stream by default)."""

    def __init__(self, device: int = 0, stream=None):
        import torch

        self.device = device
        if stream is None:
            stream = torch.cuda.current_stream(device)
        self.stream = stream
        h = C.c_void_p()
        check(lib().s2_init(device, C.c_void_p(stream.cuda_stream), C.byref(h)), "s2_init")
        self.handle = h

    def close(self):
        if self.handle:
            lib().s2_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def status(self) -> int:
        return lib().s2_status(self.handle)

    def launches(self) -> int:
        return int(lib().s2_launch_count(self.handle))

    def profile(self, enable: bool) -> None:
        check(lib().s2_profile_enable(self.handle, int(bool(enable))), "s2_profile_enable")

    def counters(self) -> dict:
        """{kernel name: {launches, ms, flops, bytes}} since profiling was enabled."""
        out = {}
        for k, name in enumerate(KERNEL_NAMES):
            n, ms, fl, by = C.c_int64(), C.c_double(), C.c_double(), C.c_double()
            check(lib().s2_profile_read(self.handle, k, C.byref(n), C.byref(ms), C.byref(fl), C.byref(by)),
                  "s2_profile_read")
            out[name] = {"launches": n.value, "ms": ms.value, "flops": fl.value, "bytes": by.value}
        return out


class Plan:
    """A window plan (s2_plan) -- AdaptiveWindowPlan of the reference."""

    def __init__(self, shapes, window, window_mode=S2_WINDOW_TARGET, shifted=False):
        flat = [int(v) for s in shapes for v in s]
        self.batch = len(flat) // 3
        h = C.c_void_p()
        check(lib().s2_plan_build(_ints(flat), self.batch, _ints(window), window_mode, int(bool(shifted)),
                                  C.byref(h)), "s2_plan_build")
        self.handle = h

    def __del__(self):
        try:
            if self.handle:
                lib().s2_plan_free(self.handle)
                self.handle = None
        except Exception:
            pass

    def arrays(self) -> dict:
        import numpy as np

        nw, nt, mx = C.c_int(), C.c_int(), C.c_int()
        check(lib().s2_plan_info(self.handle, C.byref(nw), C.byref(nt), C.byref(mx)), "s2_plan_info")
        windows = np.zeros((nw.value, 9), np.int32)
        swc = np.zeros(self.batch, np.int32)
        vi = np.zeros(nt.value, np.int32)
        inv = np.zeros(nt.value, np.int32)
        pos = np.zeros((nt.value, 3), np.int32)
        P = lambda a: a.ctypes.data_as(C.POINTER(C.c_int))  # noqa: E731
        check(lib().s2_plan_copy(self.handle, P(windows), P(swc), P(vi), P(inv), P(pos)), "s2_plan_copy")
        return {"windows": windows, "sample_window_count": swc, "video_indices": vi,
                "inverse_video_indices": inv, "local_positions": pos, "max_window_tokens": mx.value}

    def schedule(self, ctx, text_lengths) -> dict:
        """The attention schedule tables as they sit on the device (s2_plan_schedule_copy)."""
        import numpy as np

        tl = _ints(text_lengths)
        sizes = (C.c_int * 4)()
        check(lib().s2_plan_schedule_copy(ctx.handle, self.handle, tl, sizes, None, None, None, None, None),
              "s2_plan_schedule_copy")
        R, nw, n, npd = list(sizes)
        out = {"row_src": np.zeros(R, np.int32), "row_pos": np.zeros((R, 3), np.int32),
               "win_info": np.zeros((nw, 4), np.int32), "video_indices": np.zeros(n, np.int32),
               "pack_dst": np.zeros(npd, np.int32)}
        check(lib().s2_plan_schedule_copy(ctx.handle, self.handle, tl, sizes,
                                          *[out[k].ctypes.data for k in ("row_src", "row_pos", "win_info",
                                                                         "video_indices", "pack_dst")]),
              "s2_plan_schedule_copy")
        return out

    def debug_poke(self, ctx, table: int, index: int, value: int) -> int:
        """Overwrites one entry of the device schedule (table 0 row_src, 1 video_indices): checked
        build only (libseedvr2_cuda_checked.so); any other build returns S2_ERR_INVALID untouched."""
        return lib().s2_debug_poke_schedule(ctx.handle, self.handle, int(table), int(index), int(value))


def awa_forward(ctx: Context, *, heads, head_dim, window, window_mode, shifted, eps, rope_pairs, norms, freqs,
                shapes, text_lengths, video_qkv=None, text_qkv=None, split=None, out_dtype=S2_DTYPE_F32,
                official_bf16=False, video_out=None, text_out=None, plan: Plan | None = None):
    """AdaptiveWindowAttention forward on torch CUDA tensors (fp32 or bf16)."""
    import torch

    inner = heads * head_dim
    nv = sum(int(s[0]) * int(s[1]) * int(s[2]) for s in shapes)
    nt = sum(int(t) for t in text_lengths)
    if split is None:
        vq, tq = video_qkv, text_qkv
        esz = vq.element_size()
        ptrs = [vq.data_ptr(), vq.data_ptr() + inner * esz, vq.data_ptr() + 2 * inner * esz,
                tq.data_ptr(), tq.data_ptr() + inner * esz, tq.data_ptr() + 2 * inner * esz]
        vld, tld = vq.stride(0), tq.stride(0)
        dt = vq.dtype
    else:
        ptrs = [t.data_ptr() for t in split]
        vld, tld = split[0].stride(0), split[3].stride(0)
        dt = split[0].dtype
    in_dtype = S2_DTYPE_BF16 if dt == torch.bfloat16 else S2_DTYPE_F32
    tdt = torch.float32 if out_dtype == S2_DTYPE_F32 else torch.bfloat16
    dev = torch.device("cuda", ctx.device)
    if video_out is None:
        video_out = torch.empty((nv, inner), dtype=tdt, device=dev)
    if text_out is None:
        text_out = torch.empty((nt, inner), dtype=tdt, device=dev)
    p = AwaParams()
    p.heads, p.head_dim = heads, head_dim
    p.window[:] = [int(w) for w in window]
    p.window_mode, p.shifted, p.epsilon, p.rope_pairs = window_mode, int(bool(shifted)), float(eps), rope_pairs
    p.official_bf16_attention = int(bool(official_bf16))
    p.norm_weights, p.rope_freqs = norms.data_ptr(), freqs.data_ptr()
    flat = [int(v) for s in shapes for v in s]
    r = lib().s2_awa_forward(ctx.handle, C.byref(p), plan.handle if plan is not None else None, _ints(flat),
                             _ints(text_lengths), len(shapes), in_dtype, ptrs[0], ptrs[1], ptrs[2], vld, ptrs[3],
                             ptrs[4], ptrs[5], tld, out_dtype, video_out.data_ptr(), text_out.data_ptr())
    check(r, "s2_awa_forward")
    return video_out, text_out


def shared_linear(ctx: Context, a0, weight, bias=None, *, a1=None, epilogue=S2_EPI_STORE, gate=None,
                  out_dtype=S2_DTYPE_BF16, out0=None, out1=None):
    """out_s = a_s @ weight.T + bias (+ epilogue); a_s, weight bf16 CUDA tensors."""
    import torch

    M0, K = a0.shape
    M1 = a1.shape[0] if a1 is not None else 0
    N = weight.shape[0]
    tdt = torch.float32 if out_dtype == S2_DTYPE_F32 else torch.bfloat16
    if out0 is None:
        out0 = torch.empty((M0, N), dtype=tdt, device=a0.device)
    if a1 is not None and out1 is None:
        out1 = torch.empty((M1, N), dtype=tdt, device=a0.device)
    r = lib().s2_shared_linear(ctx.handle, M0, M1, N, K, a0.data_ptr(), ptr(a1), weight.data_ptr(), ptr(bias),
                               epilogue, ptr(gate), out_dtype, out0.data_ptr(), ptr(out1))
    check(r, "s2_shared_linear")
    return out0, out1


def ada_rmsnorm(ctx: Context, x, eps, shift, scale, out=None):
    import torch

    rows, D = x.shape
    if out is None:
        out = torch.empty((rows, D), dtype=torch.bfloat16, device=x.device)
    check(lib().s2_ada_rmsnorm(ctx.handle, rows, D, x.data_ptr(), float(eps), shift.data_ptr(), scale.data_ptr(),
                               out.data_ptr()), "s2_ada_rmsnorm")
    return out


def ada_layernorm(ctx: Context, x, eps, shift, scale, out=None):
    import torch

    rows, D = x.shape
    if out is None:
        out = torch.empty((rows, D), dtype=torch.bfloat16, device=x.device)
    check(lib().s2_ada_layernorm(ctx.handle, rows, D, x.data_ptr(), float(eps), shift.data_ptr(), scale.data_ptr(),
                                 out.data_ptr()), "s2_ada_layernorm")
    return out


def _floats(values) -> C.Array:
    values = [float(v) for v in values]
    return (C.c_float * len(values))(*values)


def _flat_shapes(shapes):
    return [int(v) for s in shapes for v in s]


def patch_rows(shapes) -> tuple[int, int]:
    """(latent tokens, 1x2x2 patches) of a batch of latent shapes."""
    tokens = sum(int(t) * int(h) * int(w) for t, h, w in shapes)
    patches = sum(int(t) * (int(h) // 2) * (int(w) // 2) for t, h, w in shapes)
    return tokens, patches


def patchify_video(ctx: Context, video, shapes, rows=None, out=None):
    """patchify_video: fp32 CUDA [tokens, 33] -> [patches, 132]."""
    import torch

    rows = video.shape[0] if rows is None else rows
    if out is None:
        out = torch.empty((max(patch_rows(shapes)[1], 1), S2_PATCH_FEATURES), dtype=torch.float32,
                          device=video.device)
    check(lib().s2_patchify_video(ctx.handle, video.data_ptr(), int(rows), _ints(_flat_shapes(shapes)), len(shapes),
                                  out.data_ptr()), "s2_patchify_video")
    return out


def unpatchify_prediction(ctx: Context, pred, shapes, rows=None, out=None):
    """unpatchify_prediction: fp32 CUDA [patches, 64] -> [tokens, 16]."""
    import torch

    rows = pred.shape[0] if rows is None else rows
    if out is None:
        out = torch.empty((max(patch_rows(shapes)[0], 1), S2_PRED_CHANNELS), dtype=torch.float32, device=pred.device)
    check(lib().s2_unpatchify_prediction(ctx.handle, pred.data_ptr(), int(rows), _ints(_flat_shapes(shapes)),
                                         len(shapes), out.data_ptr()), "s2_unpatchify_prediction")
    return out


def timestep_embedding(ctx: Context, timesteps, out=None, device="cuda"):
    """make_timestep_embedding: host timesteps -> fp32 CUDA [batch, 256]."""
    import torch

    n = len(timesteps)
    if out is None:
        out = torch.empty((max(n, 1), S2_TIME_FEATURES), dtype=torch.float32, device=device)
    check(lib().s2_timestep_embedding(ctx.handle, _floats(timesteps), n, out.data_ptr()), "s2_timestep_embedding")
    return out


def apply_cfg(ctx: Context, pos, neg, scale, rescale, out=None):
    """apply_cfg on fp32 CUDA tensors of the same shape."""
    import torch

    if out is None:
        out = torch.empty_like(pos)
    check(lib().s2_apply_cfg(ctx.handle, pos.data_ptr(), neg.data_ptr(), pos.numel(), float(scale), float(rescale),
                             out.data_ptr()), "s2_apply_cfg")
    return out


class Dit:
    """s2_dit: the block stack (SeedVR2DiTBlocks' block graph) and its frontend / tail nets."""

    def __init__(self, ctx: Context, *, num_blocks=32, hidden=2560, heads=20, head_dim=128, mlp_hidden=10240,
                 rope_pairs=21, window=(4, 3, 3), window_mode=S2_WINDOW_TARGET, norm_eps=1e-5, qk_eps=1e-5,
                 bias=True):
        cfg = DitConfig()
        cfg.num_blocks, cfg.hidden, cfg.heads, cfg.head_dim = num_blocks, hidden, heads, head_dim
        cfg.mlp_hidden, cfg.rope_pairs = mlp_hidden, rope_pairs
        cfg.window[:] = [int(w) for w in window]
        cfg.window_mode, cfg.norm_eps, cfg.qk_eps = window_mode, norm_eps, qk_eps
        cfg.qkv_bias = cfg.out_bias = cfg.mlp_bias = int(bool(bias))
        self.cfg = cfg
        self.ctx = ctx
        h = C.c_void_p()
        check(lib().s2_dit_create(ctx.handle, C.byref(cfg), C.byref(h)), "s2_dit_create")
        self.handle = h

    def close(self):
        if self.handle:
            lib().s2_dit_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def init_random(self, seed: int):
        check(lib().s2_dit_init_random(self.handle, seed), "s2_dit_init_random")

    def set_check_finite(self, enable: bool = True):
        """Count the NaN / Inf values of the video and text rows at the block stack's input and after every
        block; a forward that finds any fails with code -1 (see nonfinite_report)."""
        check(lib().s2_dit_set_check_finite(self.handle, int(bool(enable))), "s2_dit_set_check_finite")

    def set_block_norm(self, block: int, layer: bool):
        """The block's AdaLN norms: LayerNorm (layer=True) or RMSNorm (the default)."""
        check(lib().s2_dit_set_block_norm(self.handle, block, 1 if layer else 0), "s2_dit_set_block_norm")

    def set_checkpoints(self, blocks, videos, texts):
        """After block blocks[i] of every following forward, copy its video rows into videos[i] and its text
        rows into texts[i] (contiguous fp32 CUDA tensors kept alive by this object); [] clears them."""
        n = len(blocks)
        bl = _ints(blocks)
        vp_ = (C.c_void_p * max(n, 1))(*[v.data_ptr() for v in videos])
        tp_ = (C.c_void_p * max(n, 1))(*[t.data_ptr() for t in texts])
        check(lib().s2_dit_set_checkpoints(self.handle, bl, n, vp_, tp_), "s2_dit_set_checkpoints")
        self._checkpoints = (list(videos), list(texts))  # the library keeps the pointers

    def nonfinite_report(self):
        """(block, video_count, text_count) of the last checked forward's first non-finite point: block -1 =
        the input, b = block b's output, num_blocks = all finite."""
        b, v, t = C.c_int(), C.c_int64(), C.c_int64()
        check(lib().s2_dit_nonfinite_report(self.handle, C.byref(b), C.byref(v), C.byref(t)),
              "s2_dit_nonfinite_report")
        return b.value, v.value, t.value

    def set_block_weights(self, block: int, w: dict):
        """w: dict of contiguous fp32 numpy arrays (keys of BlockHostWeights; biases may be None)."""
        import numpy as np

        keep = {k: (np.ascontiguousarray(v, dtype=np.float32) if v is not None else None) for k, v in w.items()}
        hw = BlockHostWeights(*[(keep[n].ctypes.data if keep.get(n) is not None else None)
                                for n, _ in BlockHostWeights._fields_])
        check(lib().s2_dit_set_block_weights(self.handle, block, C.byref(hw)), "s2_dit_set_block_weights")

    def forward(self, video_shape, text_length, x, modulation):
        """x: fp32 CUDA [Nv+Nt, D] (updated in place); modulation fp32 CUDA [6, D]."""
        check(lib().s2_dit_forward(self.handle, _ints(video_shape), int(text_length), x.data_ptr(),
                                   modulation.data_ptr()), "s2_dit_forward")
        return x

    def forward_sharded(self, video_shape, text_length, x_local, modulation):
        """x_local: fp32 CUDA [n_local + Nt, D] (this rank's rows, see shard()), updated in place."""
        check(lib().s2_dit_forward_sharded(self.handle, _ints(video_shape), int(text_length), x_local.data_ptr(),
                                           modulation.data_ptr()), "s2_dit_forward_sharded")
        return x_local

    def forward_host(self, video_shapes, text_lengths, video, text, modulation, video_out, text_out):
        """Host buffers (numpy or pinned torch CPU tensors, fp32)."""
        flat = [int(v) for s in video_shapes for v in s]
        check(lib().s2_dit_forward_host(self.handle, _ints(flat), _ints(text_lengths), len(video_shapes),
                                        ptr(video), ptr(text), ptr(modulation), ptr(video_out), ptr(text_out)),
              "s2_dit_forward_host")

    def forward_host_async(self, video_shapes, text_lengths, video, text, modulation, video_out, text_out):
        """Pipelined forward_host: enqueues and returns; the buffers (pinned for overlap) must
        stay alive and untouched until host_wait()."""
        flat = [int(v) for s in video_shapes for v in s]
        check(lib().s2_dit_forward_host_async(self.handle, _ints(flat), _ints(text_lengths), len(video_shapes),
                                              ptr(video), ptr(text), ptr(modulation), ptr(video_out),
                                              ptr(text_out)),
              "s2_dit_forward_host_async")

    def host_wait(self):
        check(lib().s2_dit_host_wait(self.handle), "s2_dit_host_wait")


    def set_io_weights(self, w: dict):
        """w: dict of fp32 numpy arrays keyed like IoHostWeights (biases may be None)."""
        import numpy as np

        keep = {k: (np.ascontiguousarray(v, dtype=np.float32) if v is not None else None) for k, v in w.items()}
        hw = IoHostWeights(*[(keep[n].ctypes.data if keep.get(n) is not None else None)
                             for n, _ in IoHostWeights._fields_])
        check(lib().s2_dit_set_io_weights(self.handle, C.byref(hw)), "s2_dit_set_io_weights")

    def forward_frontend(self, video_shapes, text_lengths, timesteps, video, text, video_out=None, text_out=None,
                         modulation=None):
        """DiTInputs -> DiTBlockInputs on the device: returns (video [patches, D], text [T, D],
        modulation [6, batch, D]), fp32 CUDA."""
        import torch

        D, B = self.cfg.hidden, len(video_shapes)
        dev = video.device
        _, np_ = patch_rows(video_shapes)
        if video_out is None:
            video_out = torch.empty((np_, D), dtype=torch.float32, device=dev)
        if text_out is None:
            text_out = torch.empty((text.shape[0], D), dtype=torch.float32, device=dev)
        if modulation is None:
            modulation = torch.empty((6, B, D), dtype=torch.float32, device=dev)
        check(lib().s2_dit_forward_frontend(self.handle, _ints(_flat_shapes(video_shapes)), _ints(text_lengths),
                                            _floats(timesteps), B, video.data_ptr(), video.shape[0], text.data_ptr(),
                                            text.shape[0], video_out.data_ptr(), text_out.data_ptr(),
                                            modulation.data_ptr()), "s2_dit_forward_frontend")
        return video_out, text_out, modulation

    def forward_tail(self, video_shapes, video, modulation, prediction=None):
        """Block-stack video rows [patches, D] + modulation [6, batch, D] -> prediction [tokens, 16]."""
        import torch

        tokens, _ = patch_rows(video_shapes)
        if prediction is None:
            prediction = torch.empty((tokens, S2_PRED_CHANNELS), dtype=torch.float32, device=video.device)
        check(lib().s2_dit_forward_tail(self.handle, _ints(_flat_shapes(video_shapes)), len(video_shapes),
                                        video.data_ptr(), video.shape[0], modulation.data_ptr(),
                                        prediction.data_ptr()), "s2_dit_forward_tail")
        return prediction

    def forward_step(self, video_shapes, text_lengths, timesteps, video, text, prediction=None, text_out=None):
        """The whole DiT on device buffers: latents [tokens, 33] + text [T, 5120] -> (prediction [tokens, 16],
        text [T, D])."""
        import torch

        dev = video.device
        if prediction is None:
            prediction = torch.empty((video.shape[0], S2_PRED_CHANNELS), dtype=torch.float32, device=dev)
        if text_out is None:
            text_out = torch.empty((text.shape[0], self.cfg.hidden), dtype=torch.float32, device=dev)
        check(lib().s2_dit_forward_step(self.handle, _ints(_flat_shapes(video_shapes)), _ints(text_lengths),
                                        _floats(timesteps), len(video_shapes), video.data_ptr(), video.shape[0],
                                        text.data_ptr(), text.shape[0], prediction.data_ptr(), text_out.data_ptr()),
              "s2_dit_forward_step")
        return prediction, text_out

    def forward_step_host(self, video_shapes, text_lengths, timesteps, video, text, prediction, text_out):
        """Same, host buffers (numpy or pinned torch CPU tensors, fp32); synchronises."""
        check(lib().s2_dit_forward_step_host(self.handle, _ints(_flat_shapes(video_shapes)), _ints(text_lengths),
                                             _floats(timesteps), len(video_shapes), ptr(video), video.shape[0],
                                             ptr(text), text.shape[0], ptr(prediction), ptr(text_out)),
              "s2_dit_forward_step_host")


    def denoise(self, latent_shape, latent, condition, positive_text, negative_text=None, *, steps=1, cfg_scale=1.0,
                cfg_rescale=0.0, latent_cstep=None, condition_cstep=None):
        """SeedVR2Pipeline::denoise on the device: latent / condition fp32 CUDA [16, >= t*h*w] planes (latent
        updated in place), texts fp32 CUDA [rows, 5120]."""
        opt = DenoiseOptions(int(steps), float(cfg_scale), float(cfg_rescale))
        check(lib().s2_dit_denoise(self.handle, _ints(latent_shape), latent.data_ptr(),
                                   latent.stride(0) if latent_cstep is None else latent_cstep, condition.data_ptr(),
                                   condition.stride(0) if condition_cstep is None else condition_cstep,
                                   positive_text.data_ptr(), positive_text.shape[0], ptr(negative_text),
                                   0 if negative_text is None else negative_text.shape[0], C.byref(opt)),
              "s2_dit_denoise")
        return latent

    def denoise_host(self, latent_shape, latent, condition, positive_text, negative_text=None, *, steps=1,
                     cfg_scale=1.0, cfg_rescale=0.0):
        """Same with host numpy planes [16, cstep] (latent updated in place)."""
        opt = DenoiseOptions(int(steps), float(cfg_scale), float(cfg_rescale))
        check(lib().s2_dit_denoise_host(self.handle, _ints(latent_shape), ptr(latent), latent.shape[1],
                                        ptr(condition), condition.shape[1], ptr(positive_text),
                                        positive_text.shape[0], ptr(negative_text),
                                        0 if negative_text is None else negative_text.shape[0], C.byref(opt)),
              "s2_dit_denoise_host")
        return latent


class Conv3d:
    """s2_conv3d: the VAE's DecomposedConv3D layer (cfg = its 16-value config blob; host fp32 bias and
    kernel_t x [co][ci][kh][kw] weights)."""

    def __init__(self, ctx: Context, cfg, bias, weights):
        import numpy as np

        self.ctx = ctx
        self.cfg = [int(v) for v in cfg]
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        w = np.ascontiguousarray(weights, dtype=np.float32)
        h = C.c_void_p()
        check(lib().s2_conv3d_create(ctx.handle, _ints(self.cfg), ptr(b), ptr(w), C.byref(h)), "s2_conv3d_create")
        self.handle = h

    def output_shape(self, w, h, d, memory_state):
        out = (C.c_int * 4)()
        check(lib().s2_conv3d_output_shape(self.handle, w, h, d, memory_state, out), "s2_conv3d_output_shape")
        return list(out)

    def forward(self, x, memory_state=S2_VAE_MEMORY_DISABLED, out=None):
        """x: fp32 CUDA [c, d, h, w] -> fp32 CUDA [co, t, oh, ow]."""
        import torch

        c, d, h, w = x.shape
        ow, oh, od, oc = self.output_shape(w, h, d, memory_state)
        if out is None:
            out = torch.empty((oc, od, oh, ow), dtype=torch.float32, device=x.device)
        check(lib().s2_conv3d_forward(self.handle, x.data_ptr(), d * h * w, w, h, d, c, memory_state,
                                      out.data_ptr(), od * oh * ow), "s2_conv3d_forward")
        return out

    def reset_temporal_memory(self):
        lib().s2_conv3d_reset_memory(self.handle)

    def close(self):
        if self.handle:
            lib().s2_conv3d_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class VaeResample:
    """s2_vae_resample: VAEDownsample3D (kind S2_VAE_DOWNSAMPLE) or VAEUpsample3D (S2_VAE_UPSAMPLE) from the
    weight-blob sequence its load_model reads (host fp32)."""

    def __init__(self, ctx: Context, kind, blob):
        import numpy as np

        self.ctx = ctx
        b = np.ascontiguousarray(blob, dtype=np.float32)
        h = C.c_void_p()
        check(lib().s2_vae_resample_create(ctx.handle, int(kind), ptr(b), b.size, C.byref(h)),
              "s2_vae_resample_create")
        self.handle = h

    def output_shape(self, w, h, d, memory_state):
        out = (C.c_int * 4)()
        check(lib().s2_vae_resample_output_shape(self.handle, w, h, d, memory_state, out),
              "s2_vae_resample_output_shape")
        return list(out)

    def forward(self, x, memory_state=S2_VAE_MEMORY_DISABLED, out=None):
        """x: fp32 CUDA [c, d, h, w] -> fp32 CUDA [c', t, oh, ow]."""
        import torch

        c, d, h, w = x.shape
        ow, oh, od, oc = self.output_shape(w, h, d, memory_state)
        if out is None:
            out = torch.empty((oc, od, oh, ow), dtype=torch.float32, device=x.device)
        check(lib().s2_vae_resample_forward(self.handle, x.data_ptr(), d * h * w, w, h, d, c, memory_state,
                                            out.data_ptr(), od * oh * ow), "s2_vae_resample_forward")
        return out

    def reset_temporal_memory(self):
        lib().s2_vae_resample_reset_memory(self.handle)

    def close(self):
        if self.handle:
            lib().s2_vae_resample_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class VaeMha:
    """s2_vae_mha: VAEChunkedMHA (one head); weights host fp32 in load_model order."""

    def __init__(self, ctx: Context, embed_dim, num_heads, scale, weights):
        import numpy as np

        self.ctx = ctx
        w = np.ascontiguousarray(weights, dtype=np.float32)
        h = C.c_void_p()
        check(lib().s2_vae_mha_create(ctx.handle, int(embed_dim), int(num_heads), float(scale), ptr(w), C.byref(h)),
              "s2_vae_mha_create")
        self.handle = h

    def forward(self, x, out=None):
        """x: fp32 CUDA [tokens, E] -> fp32 CUDA [tokens, E]."""
        import torch

        if out is None:
            out = torch.empty_like(x)
        check(lib().s2_vae_mha_forward(self.handle, x.data_ptr(), x.shape[0], out.data_ptr()), "s2_vae_mha_forward")
        return out

    def close(self):
        if self.handle:
            lib().s2_vae_mha_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


VAE_SCALING_FACTOR = 0.9152


def vae_temporal_segments(frames, first, active):
    """The VAE runtime's graph runs over a video or latent: list of (start, count, memory_state)."""
    n = lib().s2_vae_temporal_segments(int(frames), int(first), int(active), 0, None)
    if n < 0:
        raise S2Error(n, "s2_vae_temporal_segments")
    buf = (C.c_int * (3 * n))()
    lib().s2_vae_temporal_segments(int(frames), int(first), int(active), n, buf)
    return [tuple(buf[3 * i:3 * i + 3]) for i in range(n)]


def vae_encode_frames(frames) -> int:
    return lib().s2_vae_encode_frames(int(frames))


def vae_decode_frames(latent_frames) -> int:
    return lib().s2_vae_decode_frames(int(latent_frames))


def vae_posterior_noise(seed, count):
    """The reference's posterior noise sequence (host fp32 numpy)."""
    import numpy as np

    out = np.empty(int(count), dtype=np.float32)
    check(lib().s2_vae_posterior_noise(C.c_uint64(int(seed)), int(count), out.ctypes.data), "s2_vae_posterior_noise")
    return out


def vae_moments_to_latent(ctx: Context, moments, noise=None, latent=None):
    """moments: fp32 CUDA [32, d, h, w] -> latent fp32 CUDA [16, d, h, w]; noise fp32 CUDA [16, d, h, w]
    (None: no posterior sample)."""
    import torch

    _, d, h, w = moments.shape
    if latent is None:
        latent = torch.empty((16, d, h, w), dtype=torch.float32, device=moments.device)
    check(lib().s2_vae_moments_to_latent(ctx.handle, moments.data_ptr(), w, h, d, ptr(noise), latent.data_ptr()),
          "s2_vae_moments_to_latent")
    return latent


def vae_unscale_latent(ctx: Context, latent):
    """latent /= 0.9152 in place (fp32 CUDA)."""
    check(lib().s2_vae_unscale_latent(ctx.handle, latent.data_ptr(), latent.numel()), "s2_vae_unscale_latent")
    return latent


def shard(video_shape, text_length, window, window_mode, rank, world, shifted=1) -> dict:
    """Token ownership of a sharded forward (host only): local tokens, the exchange lists and the
    owned windows (plan window indices) of window plan `shifted` (0 = unshifted, 1 = shifted)."""
    import numpy as np

    h = C.c_void_p()
    check(lib().s2_shard_build(_ints(video_shape), int(text_length), _ints(window), int(window_mode), int(rank),
                               int(world), C.byref(h)), "s2_shard_build")
    try:
        n = C.c_int()
        sc = np.zeros(world, np.int32)
        rc = np.zeros(world, np.int32)
        P = lambda a: a.ctypes.data_as(C.POINTER(C.c_int))  # noqa: E731
        check(lib().s2_shard_counts(h, int(shifted), C.byref(n), P(sc), P(rc)), "s2_shard_counts")
        local = np.zeros(n.value, np.int32)
        st = np.zeros(int(sc.sum()), np.int32)
        rt = np.zeros(int(rc.sum()), np.int32)
        check(lib().s2_shard_lists(h, int(shifted), P(local), P(st), P(rt)), "s2_shard_lists")
        nw = C.c_int()
        check(lib().s2_shard_windows(h, int(shifted), C.byref(nw), None), "s2_shard_windows")
        wins = np.zeros(nw.value, np.int32)
        check(lib().s2_shard_windows(h, int(shifted), C.byref(nw), P(wins)), "s2_shard_windows")
    finally:
        lib().s2_shard_free(h)
    return {"local_tokens": local, "send_counts": sc, "recv_counts": rc, "send_tokens": st, "recv_tokens": rt,
            "windows": wins}


def dist_unique_id() -> bytes:
    buf = (C.c_char * 128)()
    check(lib().s2_dist_unique_id(buf), "s2_dist_unique_id")
    return bytes(buf)


def dist_init(ctx: Context, uid: bytes, rank: int, world: int, timeout_ms: int = 60000) -> None:
    buf = (C.c_char * 128).from_buffer_copy(uid)
    check(lib().s2_dist_init(ctx.handle, buf, rank, world, timeout_ms), "s2_dist_init")


def dist_sync(ctx: Context) -> None:
    check(lib().s2_dist_sync(ctx.handle), "s2_dist_sync")


def dist_destroy(ctx: Context) -> None:
    check(lib().s2_dist_destroy(ctx.handle), "s2_dist_destroy")
