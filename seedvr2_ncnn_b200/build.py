"""Builds libseedvr2_cuda.so in-tree for sm_100a with nvcc.

    python -m seedvr2_ncnn_b200.build          # or: python seedvr2_ncnn_b200/build.py

Objects go to seedvr2_ncnn_b200/_build/, the library to
seedvr2_ncnn_b200/libseedvr2_cuda.so (next to this file, so it travels with
the source tree).  The CUDA runtime is linked statically; the driver entry
point for TMA descriptors is resolved at run time.
"""
from __future__ import annotations

import concurrent.futures as cf
import hashlib
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libseedvr2_cuda.so")
# The checked build: the same sources with S2_DEBUG_BOUNDS, whose kernels test
# every index read from a schedule table before it addresses memory (a bad one
# records an error status instead of faulting).  Tests load it by setting
# S2_CUDA_LIB to its path; nothing else uses it.
BUILD_CHECKED = os.path.join(HERE, "_build_checked")
LIB_CHECKED = os.path.join(HERE, "libseedvr2_cuda_checked.so")
LAYER_LIB = os.path.join(HERE, "libseedvr2_ncnn.so")
LAYER_SOURCES = ["adaptive_window_attention.cpp", "shared_linear.cpp", "vae_layers.cpp", "net.cpp", "layer_capi.cpp"]
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
ROOT = os.path.dirname(HERE)

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I" + os.path.join(ROOT, "include"),
          "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills", "-Wno-deprecated-gpu-targets"]

SOURCES = ["s2_api.cu", "dit.cu", "gemm_sm100.cu", "attention_sm100.cu", "elementwise.cu", "plan.cpp", "awa_static.cu", "dist.cpp", "peer.cu", "dit_io.cu", "conv_sm100.cu", "vae_mha.cu", "graph_ops.cu", "vae_runtime.cu"]


def _headers_digest() -> str:
    h = hashlib.sha256()
    for d in (CSRC, os.path.join(ROOT, "include")):
        for f in sorted(os.listdir(d)):
            if f.endswith((".h", ".cuh")):
                with open(os.path.join(d, f), "rb") as fh:
                    h.update(fh.read())
    return h.hexdigest()[:16]


def _compile(src: str, extra: list[str], hdr: str, build_dir: str = BUILD) -> str:
    obj = os.path.join(build_dir, os.path.splitext(src)[0] + ".o")
    stamp = obj + ".hdr"
    path = os.path.join(CSRC, src)
    fresh = (os.path.exists(obj) and os.path.getmtime(obj) >= os.path.getmtime(path) and os.path.exists(stamp)
             and open(stamp).read() == hdr + " ".join(extra))
    if fresh:
        return obj
    cmd = [NVCC] + ARCH + COMMON + extra + ["-c", path, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [NVCC] + COMMON + extra + ["-x", "c++", "-c", path, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip():
        sys.stderr.write(r.stderr)
    with open(stamp, "w") as fh:
        fh.write(hdr + " ".join(extra))
    return obj


def _build_lib(lib: str, build_dir: str, extra: list[str]) -> str:
    os.makedirs(build_dir, exist_ok=True)
    hdr = _headers_digest()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 2)) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra, hdr, build_dir), SOURCES))
    if not os.path.exists(lib) or any(os.path.getmtime(o) > os.path.getmtime(lib) for o in objs):
        cmd = [NVCC] + ARCH + ["-shared", "-o", lib] + objs + ["-cudart", "static", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return lib


def build(verbose: bool = False, extra: list[str] | None = None) -> str:
    _build_lib(LIB, BUILD, list(extra or []))
    build_layers(verbose)
    build_checked(verbose)
    if verbose:
        print(LIB)
    return LIB


def build_checked(verbose: bool = False) -> str:
    """libseedvr2_cuda_checked.so: the S2_DEBUG_BOUNDS build (index checks in the table-driven kernels)."""
    _build_lib(LIB_CHECKED, BUILD_CHECKED, ["-DS2_DEBUG_BOUNDS"])
    if verbose:
        print(LIB_CHECKED)
    return LIB_CHECKED


def build_layers(verbose: bool = False) -> str:
    """The ncnn-surface layer classes (C++, host) over libseedvr2_cuda.so."""
    srcs = [os.path.join(CSRC, "layers", f) for f in LAYER_SOURCES]
    deps = srcs + [os.path.join(CSRC, "layers", f) for f in os.listdir(os.path.join(CSRC, "layers")) if f.endswith(".h")]
    deps.append(os.path.join(ROOT, "include", "seedvr2_cuda.h"))
    if os.path.exists(LAYER_LIB) and all(os.path.getmtime(d) <= os.path.getmtime(LAYER_LIB) for d in deps) and \
            os.path.getmtime(LIB) <= os.path.getmtime(LAYER_LIB):
        return LAYER_LIB
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-o", LAYER_LIB] + srcs + [
        "-I" + os.path.join(CUDA_HOME, "include"), "-L" + HERE, "-lseedvr2_cuda", "-L" + os.path.join(CUDA_HOME, "lib64"),
        "-lcudart", "-Wl,-rpath,$ORIGIN", "-Wl,-rpath," + os.path.join(CUDA_HOME, "lib64")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"layer library build failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(LAYER_LIB)
    return LAYER_LIB


if __name__ == "__main__":
    build(verbose=True, extra=sys.argv[1:])
