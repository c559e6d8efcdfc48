"""Failure detection on one GPU, without a fault: a bounded device wait that
runs out.

The sharded forward's cross-GPU barrier (s2_peer_barrier) is run with a world
of 2 on one GPU: rank 0's own flag array stands for its own slot, and a plain
local buffer stands for the absent peer, whose flag nothing ever sets.  The
barrier's wait must give up after its limit (2 s of device time), the context
must report S2_ERR_TIMEOUT through s2_status, and the context must stay
usable: the same barrier with every flag present passes, and an
AdaptiveWindowAttention call on the same context afterwards matches the one
made before the timeout bit for bit.
"""
import ctypes as C
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _awa(s2lib, ctx, vq, tq, norms, freqs):
    return s2lib.awa_forward(ctx, heads=2, head_dim=128, window=[1, 4, 4], window_mode=s2lib.S2_WINDOW_EXTENT,
                             shifted=1, eps=1e-5, rope_pairs=21, norms=norms, freqs=freqs, shapes=[[2, 6, 8]],
                             text_lengths=[5], video_qkv=vq, text_qkv=tq)


def test_peer_barrier_timeout_is_reported_and_context_recovers(s2lib):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ctx = s2lib.Context(0)
    rng = np.random.default_rng(1)
    vq = torch.from_numpy(rng.standard_normal((96, 3 * 256)).astype(np.float32)).cuda()
    tq = torch.from_numpy(rng.standard_normal((5, 3 * 256)).astype(np.float32)).cuda()
    norms = torch.ones(4, 128, device="cuda")
    freqs = torch.from_numpy((1.0 / 10000 ** (np.arange(21) * 2 / 42)).astype(np.float32)).cuda()
    before_v, before_t = _awa(s2lib, ctx, vq, tq, norms, freqs)
    torch.cuda.synchronize()
    assert ctx.status() == s2lib.S2_OK

    own = torch.zeros(8, dtype=torch.int32, device="cuda")     # rank 0's flags: slot i = peer i's epoch
    absent = torch.zeros(8, dtype=torch.int32, device="cuda")  # the missing peer's flags (nobody waits on them)
    peers = (C.c_void_p * 2)(own.data_ptr(), absent.data_ptr())
    t0 = time.time()
    r = s2lib.lib().s2_peer_barrier(ctx.handle, peers, own.data_ptr(), 0, 2, 1)
    assert r == s2lib.S2_OK  # only enqueued
    assert ctx.status() == s2lib.S2_ERR_TIMEOUT  # synchronises: the wait ran out on the device
    waited = time.time() - t0
    assert 1.5 < waited < 30.0, waited
    # rank 0 stored its epoch into its own slot and into the absent peer's
    assert own[0].item() == 1 and absent[0].item() == 1 and own[1].item() == 0
    assert ctx.status() == s2lib.S2_OK  # the status word was cleared by the read

    # the peer's flag arrives: the same barrier passes
    own[1] = 1
    r = s2lib.lib().s2_peer_barrier(ctx.handle, peers, own.data_ptr(), 0, 2, 1)
    assert r == s2lib.S2_OK and ctx.status() == s2lib.S2_OK

    # the context still runs kernels, with the same results as before
    after_v, after_t = _awa(s2lib, ctx, vq, tq, norms, freqs)
    torch.cuda.synchronize()
    assert ctx.status() == s2lib.S2_OK
    assert torch.equal(after_v, before_v) and torch.equal(after_t, before_t)

    # invalid arguments are refused on the host
    assert s2lib.lib().s2_peer_barrier(ctx.handle, peers, own.data_ptr(), 2, 2, 1) == s2lib.S2_ERR_INVALID
    assert s2lib.lib().s2_peer_barrier(ctx.handle, peers, own.data_ptr() + 2, 0, 2, 1) == s2lib.S2_ERR_INVALID
    ctx.close()
