"""Benchmark of the SeedVR2 DiT block hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c3] [--impl ours|reference]

One step = one full 32-block DiT forward (one denoising step's block stack)
over one sample of the chosen configuration, synthetic seeded inputs and
random-init weights of the BASELINE architecture (hidden 2560, 20x128 heads,
MLP 10240 GELU-tanh, 58 text tokens).  Default workload: BASELINE config 3,
720p x 21 frames -> 6x45x80 = 21600 video tokens, windows 2x15x20 (the
reference's own target-count rule with target (4,3,4)), half-shifted in odd
blocks.

Prints one JSON line (rank 0).  ``value`` = tokens/s of the device-resident
forward; ``e2e`` = the same metric through s2_dit_forward_host with host
buffers (H2D + D2H inside the timed region); ``roofline`` = the dominant
kernel from the library's own per-kernel counters (CUDA events inside the
timed region); ``window_attention`` = the same for the attention kernel;
``cpu_baseline`` = the reference's CPU layer code (oracle/_ref) or the oracle
port on a bounded sample of the same workload.

``--impl reference`` times the reference's CPU implementation (oracle/_ref,
the reference's own AdaptiveWindowAttention/SharedLinear sources built
against a clean-room ncnn API shim; the oracle port when that build is
absent) with all host threads, on the same config and metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

D, HEADS, HD, F, TEXT, PAIRS, BLOCKS = 2560, 20, 128, 10240, 58, 21, 32

# name -> (video shape t,h,w ; window tuple ; window mode 0=target count (reference) 1=extent ; description)
# DRAM bytes per launch of each kernel class on the C3 workload (single GPU), from
# `ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum` over one 720p block; the command
# and per-launch table are in profiles/traffic_c3_one_block.md.  shared_linear is the mean of the
# block's four projections.
NCU_TRAFFIC_C3 = {
    "shared_linear": 996.2e6,
    "window_attention": 474.2e6,
    "ada_rmsnorm": 302.0e6,
    "text_pool": 21.4e6,
}

CONFIGS = {
    "c1": ([1, 32, 32], [1, 16, 16], 1, "BASELINE config 1 geometry: 1x32x32 tokens, windows 16x16"),
    "c2": ([1, 64, 64], [1, 16, 16], 1, "BASELINE config 2: 1024x1024 image, 64x64 tokens, windows 1x16x16"),
    "c3": ([6, 45, 80], [4, 3, 4], 0, "BASELINE config 3: 720p x 21 frames, 6x45x80 tokens, windows 2x15x20"),
    "c5": ([12, 68, 120], [4, 17, 30], 1, "BASELINE config 5: 1080p x 45 frames, 12x68x120 tokens, windows 4x17x30"),
    # window-length sweep over ~65k video tokens (explicit extents that tile the
    # token grid; L = 600 uses the 720p window on a 16x60x60 grid, 57600 tokens)
    "c4_l64": ([16, 64, 64], [1, 8, 8], 1, "BASELINE config 4, L=64: 16x64x64 tokens, windows 1x8x8"),
    "c4_l256": ([16, 64, 64], [1, 16, 16], 1, "BASELINE config 4, L=256: 16x64x64 tokens, windows 1x16x16"),
    "c4_l600": ([16, 60, 60], [2, 15, 20], 1, "BASELINE config 4, L=600: 16x60x60 tokens, windows 2x15x20"),
    "c4_l1024": ([16, 64, 64], [1, 32, 32], 1, "BASELINE config 4, L=1024: 16x64x64 tokens, windows 1x32x32"),
    "c4_l2048": ([16, 64, 64], [2, 32, 32], 1, "BASELINE config 4, L=2048: 16x64x64 tokens, windows 2x32x32"),
}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return {"hbm_gbs": j["hbm_gbs"], "bf16_tflops": j["bf16_tflops"],
                "bf16_tflops_sustained": j.get("bf16_tflops_sustained", j["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown," \
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown," \
             "clocks_event_reasons.sw_power_cap"

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "50"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        t0 = time.time()
        while not self.lines and time.time() - t0 < 5.0:  # sampler is up before the timed region starts
            time.sleep(0.01)
        self.skip = len(self.lines)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines[getattr(self, "skip", 0):]:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "samples": len(sm),
                "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------- CPU baseline
def cpu_sample(kind_pref: str = "reference", threads: int | None = None):
    """Times one window-block of the config-3 workload on the host: the reference's
    AdaptiveWindowAttention (one 2x15x20 window + 58 text tokens) and its four
    SharedLinear projections (QKV, out, MLP up, MLP down) over those 658 tokens.
    Returns (seconds, kind, cores)."""
    import numpy as np

    from oracle import oracle

    if threads:
        os.environ["OMP_NUM_THREADS"] = str(threads)
    cores = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    rng = np.random.default_rng(0)
    shape, T = [2, 15, 20], TEXT
    nv = 600
    inner = HEADS * HD
    x = rng.standard_normal((nv, D)).astype(np.float32)
    xt = rng.standard_normal((T, D)).astype(np.float32)
    w_qkv = (0.02 * rng.standard_normal((3 * D, D))).astype(np.float32)
    w_out = (0.02 * rng.standard_normal((D, D))).astype(np.float32)
    w_up = (0.02 * rng.standard_normal((F, D))).astype(np.float32)
    w_down = (0.02 * rng.standard_normal((D, F))).astype(np.float32)
    b = lambda n: (0.02 * rng.standard_normal(n)).astype(np.float32)  # noqa: E731
    norms = (1 + 0.02 * rng.standard_normal((4, HD))).astype(np.float32)
    freqs = (1.0 / 10000 ** (np.arange(PAIRS) * 2 / 42)).astype(np.float32)
    use_ref = kind_pref == "reference" and os.path.exists(oracle.REF_SO)
    if use_ref:
        lib = oracle.Ref()
        t0 = time.perf_counter()
        qv, qt = lib.shared_linear(x, xt, w_qkv, b(3 * D))
        # one window covering the slab: target (1,1,1) -> a single 2x15x20 window
        cv, ct = lib.awa_forward(heads=HEADS, head_dim=HD, target=[1, 1, 1], shifted=0, eps=1e-5, rope_pairs=PAIRS,
                                 norms=norms, freqs=freqs, shapes=[shape], text_lengths=[T], video_qkv=qv,
                                 text_qkv=qt)
        ov, ot = lib.shared_linear(cv, ct, w_out, b(D))
        uv, ut = lib.shared_linear(ov, ot, w_up, b(F))
        lib.shared_linear(uv, ut, w_down, b(D))
        dt = time.perf_counter() - t0
        return dt, "reference", cores
    lib = oracle.Port()
    t0 = time.perf_counter()
    a = np.concatenate([x, xt])
    qkv = lib.linear(a, w_qkv, b(3 * D))
    cv, ct = lib.awa_forward(heads=HEADS, head_dim=HD, window=[2, 15, 20], shifted=0, eps=1e-5, rope_pairs=PAIRS,
                             norms=norms, freqs=freqs, shapes=[shape], text_lengths=[T], video_qkv=qkv[:nv],
                             text_qkv=qkv[nv:], mode=oracle.WINDOW_EXTENT)
    o = lib.linear(np.concatenate([cv, ct]), w_out, b(D))
    u = lib.linear(o, w_up, b(F))
    lib.linear(u, w_down, b(D))
    dt = time.perf_counter() - t0
    return dt, "port", cores


def cpu_tokens_per_s(sample_s: float, cfg_name: str) -> float:
    """Extrapolates one window-block (600 video + 58 text tokens) to a full 32-block step:
    step time = 32 blocks x (video tokens / 600) window-blocks x sample time."""
    shape = CONFIGS[cfg_name][0]
    nv = shape[0] * shape[1] * shape[2]
    step_s = BLOCKS * (nv / 600.0) * sample_s
    return (nv + TEXT) / step_s


# ---------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="c3", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer pass (profiling runs)")
    ap.add_argument("--blocks", type=int, default=BLOCKS, help="fewer blocks for small profiling captures only")
    ap.add_argument("--no-dit-step", action="store_true", help="skip the whole-DiT pass (frontend, blocks, tail)")
    args = ap.parse_args()

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    shape, window, mode, desc = CONFIGS[args.config]
    nv = shape[0] * shape[1] * shape[2]
    M = nv + TEXT

    if args.impl == "reference":
        if rank != 0:
            return
        for _ in range(args.warmup):
            cpu_sample("reference")
        samples = []
        kind = cores = None
        for _ in range(args.steps):
            dt, kind, cores = cpu_sample("reference")
            samples.append(dt)
        sample_s = statistics.median(samples)
        v = cpu_tokens_per_s(sample_s, args.config)
        step_ms = BLOCKS * (nv / 600.0) * sample_s * 1000.0
        print(json.dumps({
            "impl": "reference", "metric": "DiT tokens/sec/GPU (32-block step)", "value": v, "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": desc, "config": args.config, "tokens": M},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": kind,
                             "sample": "one 2x15x20 window + 58 text tokens through AWA and the 4 SharedLinear "
                                       "projections of one block (fp32), extrapolated x32 blocks x windows"},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }))
        return

    import torch

    from seedvr2_ncnn_b200 import abi

    torch.cuda.set_device(local_rank)
    if world > 1:
        from datetime import timedelta

        import torch.distributed as dist

        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local_rank))
    ctx = abi.Context(local_rank)
    sharded = world > 1
    if sharded:
        # NCCL communicator of the library (its own, next to torch's process group)
        uid = [abi.dist_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        abi.dist_init(ctx, uid[0], rank, world, 120000)
    dit = abi.Dit(ctx, num_blocks=args.blocks, hidden=D, heads=HEADS, head_dim=HD, mlp_hidden=F, rope_pairs=PAIRS,
                  window=window, window_mode=mode)
    dit.init_random(1234)
    g = torch.Generator(device="cuda").manual_seed(100)
    x_global = torch.randn(M, D, device="cuda", generator=g)
    mod = torch.randn(6, D, device="cuda", generator=g)
    if sharded:
        sh = abi.shard(shape, TEXT, window, mode, rank, world)
        local = torch.from_numpy(sh["local_tokens"].astype("int64")).cuda()
        x0 = torch.cat([x_global[local], x_global[nv:]]).contiguous()
        n_local = int(local.numel())
    else:
        x0 = x_global
        n_local = nv
    del x_global
    x = torch.empty_like(x0)
    stream = torch.cuda.current_stream()

    def forward(buf):
        if sharded:
            dit.forward_sharded(shape, TEXT, buf, mod)
        else:
            dit.forward(shape, TEXT, buf, mod)

    def step():
        x.copy_(x0)
        forward(x)

    def barrier():
        if sharded:
            abi.dist_sync(ctx)  # bounded wait; aborts the communicator on expiry
            torch.distributed.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    barrier()
    status = ctx.status()
    if status != 0:
        raise RuntimeError(f"device status {status} after warm-up")

    clocks = ClockSampler(local_rank)
    clocks.start()

    def timed(instrumented):
        """K steps between a barrier + synchronize on both sides, timed with CUDA events."""
        ctx.profile(instrumented)
        launches0 = ctx.launches()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        barrier()
        t_ms = e0.elapsed_time(e1) / args.steps
        n = ctx.launches() - launches0
        cnt = ctx.counters() if instrumented else None
        ctx.profile(False)
        if sharded:
            t = torch.tensor([t_ms], device="cuda")
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            t_ms = float(t.item())
        return t_ms, n, cnt

    # The step time comes from a pass without per-launch events (recording two
    # events around every launch adds 1-2 % to the step); the per-kernel
    # durations behind the roofline figures come from an identical instrumented
    # pass right after it.
    ms, launches, _ = timed(False)
    ms_instr, _, counters = timed(True)
    clk = clocks.stop()
    value = M / (ms / 1000.0)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)

    # end to end with host buffers (pinned): H2D of this rank's rows and the
    # modulation, the forward, D2H of the result -- inside the timed region
    e2e_ms = float("nan")
    if not args.no_e2e:
        hx = x0.cpu().pin_memory()
        hm = mod.cpu().pin_memory()
        hout = torch.empty_like(hx).pin_memory()
        if sharded:
            dx = torch.empty_like(x0)
            dm = torch.empty_like(mod)

            def e2e_step():
                dx.copy_(hx, non_blocking=True)
                dm.copy_(hm, non_blocking=True)
                forward(dx)
                hout.copy_(dx, non_blocking=True)
        else:
            hv, ht = hx[:nv], hx[nv:]
            ov, ot = hout[:nv], hout[nv:]
            hm3 = hm.reshape(6, 1, D)

            def e2e_step():
                dit.forward_host([shape], [TEXT], hv, ht, hm3, ov, ot)

        e2e_step()
        barrier()
        e2e_steps = max(1, min(args.steps, 5))
        e0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        e1.record(stream)
        barrier()
        e2e_ms = e0.elapsed_time(e1) / e2e_steps
        if sharded:
            t = torch.tensor([e2e_ms], device="cuda")
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            e2e_ms = float(t.item())
    # The whole DiT (SeedVR2DiTBlocks::forward(DiTInputs)): 1x2x2-patchified
    # latents of the same video (33 channels) + 58 text embeddings (5120) +
    # one timestep -> frontend, the blocks, tail -> prediction (16 channels),
    # on device buffers, then through the host-buffer entry point.
    dit_step = None
    if not sharded and not args.no_dit_step:
        lat = [shape[0], 2 * shape[1], 2 * shape[2]]
        ntok = lat[0] * lat[1] * lat[2]
        gl = torch.Generator(device="cuda").manual_seed(7)
        lv = torch.randn(ntok, abi.S2_LATENT_CHANNELS, device="cuda", generator=gl)
        lt = torch.randn(TEXT, abi.S2_TEXT_CHANNELS, device="cuda", generator=gl)
        pred = torch.empty(ntok, abi.S2_PRED_CHANNELS, device="cuda")
        tout = torch.empty(TEXT, D, device="cuda")

        def full_step():
            dit.forward_step([lat], [TEXT], [500.0], lv, lt, pred, tout)

        for _ in range(args.warmup):
            full_step()
        barrier()
        launches0 = ctx.launches()
        e0.record(stream)
        for _ in range(args.steps):
            full_step()
        e1.record(stream)
        barrier()
        st_ms = e0.elapsed_time(e1) / args.steps
        st_launches = ctx.launches() - launches0

        # the frontend and the tail alone (same inputs), K calls each
        fv = torch.empty(M - TEXT, D, device="cuda")
        ft = torch.empty(TEXT, D, device="cuda")
        fm = torch.empty(6, 1, D, device="cuda")
        dit.forward_frontend([lat], [TEXT], [500.0], lv, lt, fv, ft, fm)
        barrier()
        e0.record(stream)
        for _ in range(args.steps):
            dit.forward_frontend([lat], [TEXT], [500.0], lv, lt, fv, ft, fm)
        e1.record(stream)
        barrier()
        fe_ms = e0.elapsed_time(e1) / args.steps
        e0.record(stream)
        for _ in range(args.steps):
            dit.forward_tail([lat], fv, fm, pred)
        e1.record(stream)
        barrier()
        tail_ms = e0.elapsed_time(e1) / args.steps
        del fv, ft, fm
        hlv, hlt = lv.cpu().pin_memory(), lt.cpu().pin_memory()
        hpred, htout = torch.empty_like(pred, device="cpu").pin_memory(), torch.empty_like(tout, device="cpu").pin_memory()
        dit.forward_step_host([lat], [TEXT], [500.0], hlv, hlt, hpred, htout)
        barrier()
        st_e2e_steps = max(1, min(args.steps, 5))
        e0.record(stream)
        for _ in range(st_e2e_steps):
            dit.forward_step_host([lat], [TEXT], [500.0], hlv, hlt, hpred, htout)
        e1.record(stream)
        barrier()
        st_e2e_ms = e0.elapsed_time(e1) / st_e2e_steps
        dit_step = {"value": M / (st_ms / 1000.0), "unit": "tokens/s", "ms_per_step": st_ms,
                    "frontend_ms": fe_ms, "tail_ms": tail_ms, "gpu_launches": st_launches,
                    "workload": f"latents {lat[0]}x{lat[1]}x{lat[2]}x33 + {TEXT}x5120 text + 1 timestep -> "
                                f"prediction {lat[0]}x{lat[1]}x{lat[2]}x16 (frontend, {args.blocks} blocks, tail)",
                    "entry_point": "s2_dit_forward_step",
                    "e2e": {"value": M / (st_e2e_ms / 1000.0), "unit": "tokens/s", "ms_per_step": st_e2e_ms,
                            "h2d_bytes_per_step": int(ntok * 33 * 4 + TEXT * 5120 * 4),
                            "d2h_bytes_per_step": int(ntok * 16 * 4 + TEXT * D * 4),
                            "entry_point": "s2_dit_forward_step_host"}}
        del lv, lt, pred, tout, hlv, hlt, hpred, htout

        # SeedVR2Pipeline::denoise on the device: 2 Euler steps with
        # classifier-free guidance (two whole-DiT passes per step + apply_cfg
        # with rescale + the update), latent / condition as 16 channel planes.
        planes = torch.randn(2, abi.S2_PRED_CHANNELS, ntok, device="cuda", generator=gl)
        neg_text = torch.randn(TEXT, abi.S2_TEXT_CHANNELS, device="cuda", generator=gl)
        pos_text = torch.randn(TEXT, abi.S2_TEXT_CHANNELS, device="cuda", generator=gl)
        lat0 = planes[0].clone()

        def denoise():
            planes[0].copy_(lat0)
            dit.denoise(lat, planes[0], planes[1], pos_text, neg_text, steps=2, cfg_scale=6.5, cfg_rescale=0.7)

        denoise()
        barrier()
        e0.record(stream)
        denoise()
        e1.record(stream)
        barrier()
        dn_ms = e0.elapsed_time(e1)
        dit_step["denoise"] = {"steps": 2, "cfg_scale": 6.5, "cfg_rescale": 0.7, "ms": dn_ms,
                               "ms_per_dit_pass": dn_ms / 4, "entry_point": "s2_dit_denoise",
                               "host_round_trips_between_steps": 0}
        del planes, neg_text, pos_text, lat0

    # VAE DecomposedConv3D (implicit GEMM on the tensor cores) on the shapes the
    # 720p decoder runs: 512 -> 512 channels at the latent size (6 frames of
    # 90 x 160) and 128 -> 128 at full resolution (720 x 1280), 3 x 3 x 3
    # causal kernels (two head frames).
    vae_conv = None
    if not sharded and not args.no_dit_step:
        vae_conv = []
        gv = torch.Generator(device="cpu").manual_seed(11)
        for ci, frames, hh, ww in ((512, 6, 90, 160), (128, 6, 720, 1280)):
            cfg = [ci, ci, 3, 3, 3, 1, 1, 2, 1, 1, 1, 1, 1, 1, 1, 1]
            wts = (0.02 * torch.randn(3, ci, ci, 3, 3, generator=gv)).numpy()
            bias = (0.02 * torch.randn(ci, generator=gv)).numpy()
            layer = abi.Conv3d(ctx, cfg, bias, wts)
            xin = torch.randn(ci, frames, hh, ww, device="cuda")
            yout = layer.forward(xin, abi.S2_VAE_MEMORY_DISABLED)
            barrier()
            ctx.profile(True)
            e0.record(stream)
            for _ in range(args.steps):
                layer.forward(xin, abi.S2_VAE_MEMORY_DISABLED, out=yout)
            e1.record(stream)
            barrier()
            cc = ctx.counters()
            ctx.profile(False)
            call_ms = e0.elapsed_time(e1) / args.steps
            flops = 2.0 * frames * hh * ww * ci * 27 * ci
            gemm = cc["shared_linear"]
            vae_conv.append({"shape": f"{ci}->{ci} ch, {frames}x{hh}x{ww}, 3x3x3", "ms_per_call": call_ms,
                             "tflops_per_call": flops / call_ms / 1e9,
                             "conv_kernel_ms": gemm["ms"] / gemm["launches"],
                             "conv_kernel_tflops": flops / (gemm["ms"] / gemm["launches"]) / 1e9,
                             "conv_kernel_frac_of_burst_peak": flops / (gemm["ms"] / gemm["launches"]) / 1e9
                             / load_peaks()["bf16_tflops"],
                             "pack_ms": cc["other"]["ms"] / max(cc["other"]["launches"], 1)})
            layer.close()
            del xin, yout
        # VAEChunkedMHA at the mid block: one 512-wide head over a 90 x 160 latent frame
        E, T = 512, 90 * 160
        mw = (0.02 * torch.randn(4 * (E * E + E), generator=gv)).numpy()
        mha = abi.VaeMha(ctx, E, 1, 1.0 / E ** 0.5, mw)
        xin = torch.randn(T, E, device="cuda")
        yout = mha.forward(xin)
        barrier()
        e0.record(stream)
        for _ in range(args.steps):
            mha.forward(xin, out=yout)
        e1.record(stream)
        barrier()
        mha_ms = e0.elapsed_time(e1) / args.steps
        mha_flops = 2.0 * T * E * E * 4 + 4.0 * T * T * E
        vae_conv.append({"shape": f"VAEChunkedMHA, {T} tokens x {E}, one head", "ms_per_call": mha_ms,
                         "tflops_per_call": mha_flops / mha_ms / 1e9})
        mha.close()
        del xin, yout
    status = ctx.status()

    peaks = load_peaks()

    def traffic_of(name):
        """DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) from the committed ncu
        capture of one 720p block (profiles/traffic_c3_one_block.md); the single-GPU C3 workload only."""
        if args.config != "c3" or world != 1:
            return None
        t = NCU_TRAFFIC_C3.get(name)
        return None if t is None else {"bytes_per_launch": t, "source": "profiles/traffic_c3_one_block.md"}

    def roof(name, bound):
        c = counters[name]
        per_launch_ms = c["ms"] / max(c["launches"], 1)
        if bound == "tensor":
            achieved = c["flops"] / (c["ms"] / 1000.0) / 1e12
            peak = peaks["bf16_tflops_sustained"]
            unit = "TFLOP/s"
        else:
            achieved = c["bytes"] / (c["ms"] / 1000.0) / 1e9
            peak = peaks["hbm_gbs"]
            unit = "GB/s"
        return {"kernel": name, "bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
                "frac": achieved / peak, "peak_source": f"{peaks['source']} "
                + ("bf16 sustained (kernel timed inside a long step)" if bound == "tensor" else "HBM copy"),
                "launches_per_step": c["launches"] / args.steps, "ms_per_launch": per_launch_ms,
                "share_of_step": c["ms"] / args.steps / ms_instr, "traffic": traffic_of(name),
                "kernel_times": "CUDA events around every launch in an instrumented pass of the same steps"}

    kinds = {"shared_linear": "tensor", "window_attention": "tensor", "prepare_qkv": "hbm", "ada_rmsnorm": "hbm",
             "text_pool": "hbm"}
    dominant = max(kinds, key=lambda k: counters[k]["ms"])
    result = {
        "metric": "DiT tokens/sec/GPU (32-block step)", "value": value, "unit": "tokens/s", "n_gpus": world,
        "value_per_gpu": value / world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "ms_per_step_instrumented": ms_instr,
        "higher_is_better": True,
        "scaling": "strong" if sharded else "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) tokens and "
        "modulation, N(0,0.02) random-init weights)",
        "config": {"workload": desc, "config": args.config, "video_tokens": nv, "text_tokens": TEXT,
                   "blocks": args.blocks, "hidden": D, "heads": HEADS, "mlp": F, "window": window,
                   "window_mode": "target-count" if mode == 0 else "extent", "global_batch": 1,
                   "parallelism": (f"window sharding x{world} (rank 0 owns {n_local} video tokens; qkv rows "
                                   "pushed to window owners and context rows stored back over NVLink peer memory, "
                                   "text partials summed over peers; no NCCL in the block loop)")
                   if sharded else "single GPU",
                   "l2": "inputs larger than L2 (5 GB of weights + 222 MB residual per step)"},
        "roofline": roof(dominant, kinds[dominant]),
        # window attention against the burst bf16 peak (the BASELINE metric's denominator) too
        "window_attention": dict(roof("window_attention", "tensor"), frac_of_burst_peak=(
            counters["window_attention"]["flops"] / (counters["window_attention"]["ms"] / 1000.0) / 1e12
            / peaks["bf16_tflops"]) if counters["window_attention"]["ms"] > 0 else None,
            burst_peak=peaks["bf16_tflops"]),
        # prepare_qkv runs only when the QKV projection cannot pack whole heads per tile
        "hbm_passes": {k: roof(k, "hbm") for k in ("prepare_qkv", "ada_rmsnorm", "text_pool")
                       if counters[k]["launches"]},
        # cross-GPU kernels (NVLink peer pushes, flag barriers, text reduce)
        "comm": {"peer_kernels_ms_per_step": counters["comm"]["ms"] / args.steps,
                 "peer_bytes_per_step": counters["comm"]["bytes"] / args.steps,
                 "host_wait_ms_per_step": counters["host_wait"]["ms"] / args.steps,
                 "other_kernels_ms_per_step": counters["other"]["ms"] / args.steps},
        "e2e": {"value": None if args.no_e2e else M / (e2e_ms / 1000.0), "unit": "tokens/s",
                "h2d_bytes_per_step": int((n_local + TEXT) * D * 4 + 6 * D * 4),
                "d2h_bytes_per_step": int((n_local + TEXT) * D * 4), "ms_per_step": None if args.no_e2e else e2e_ms,
                "entry_point": "s2_dit_forward_sharded + pinned H2D/D2H" if sharded else "s2_dit_forward_host"},
        "gpu_launches": launches,
        "dit_step": dit_step,
        "vae_conv": vae_conv,
        "clocks": clk,
        "device_status": status,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        dt, kind, cores = cpu_sample("reference")
        v = cpu_tokens_per_s(dt, args.config)
        result["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": cores, "kind": kind,
                                  "sample": "one 2x15x20 window + 58 text tokens through AWA and the 4 SharedLinear "
                                            "projections of one block (fp32), extrapolated x32 blocks x windows",
                                  "sample_seconds": dt}
    if rank == 0:
        print(json.dumps(result))
    dit.close()
    if sharded:
        abi.dist_destroy(ctx)
    ctx.close()
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
