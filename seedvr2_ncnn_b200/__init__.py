"""seedvr2_ncnn_b200: B200 (sm_100a) implementation of the SeedVR2 DiT block
hot path -- the AdaptiveWindowAttention and SharedLinear custom layers of
Chisato623/seedvr2_ncnn and the block arithmetic around them.

The compute lives in ``libseedvr2_cuda.so`` (C ABI, ``include/seedvr2_cuda.h``).
This package only loads it and exposes thin ctypes bindings
(:mod:`seedvr2_ncnn_b200.abi`) and the ncnn-style layer surface
(:mod:`seedvr2_ncnn_b200.layers`).  There is no CPU or eager fallback: if the
library is missing, importing :mod:`seedvr2_ncnn_b200.abi` raises.
"""

import os

# S2_CUDA_LIB selects another build of the same library (the tests use it to load the
# index-checked libseedvr2_cuda_checked.so in a separate process).
LIB_PATH = os.environ.get("S2_CUDA_LIB") or os.path.join(os.path.dirname(os.path.abspath(__file__)),
                                                         "libseedvr2_cuda.so")

__all__ = ["LIB_PATH"]
