"""CPU: the token ownership of the sharded forward and its exchange volume.

Ranks own equal contiguous runs of the unshifted window plan's token order
(window after window, the plan walks w outermost -- adaptive_window_attention.cpp
:600-630 -- so a rank owns a W-slab of whole windows).  Sharding along T/H
instead (windows ordered t, h outermost) is the alternative the multi-GPU
design was weighed against.  Per block, a window's tokens that live on another
rank than the window's owner (the rank holding most of them) are exchanged;
this counts them for both orders on the 720p (config 3) and 1080p (config 5)
plans at 2, 4 and 8 ranks and checks that the W-slab order the library uses
moves no more tokens than T/H slabs (C3) and at most a few percent more (C5).
"""
import numpy as np
import pytest


def _plans(abi, shape, window, mode):
    return [abi.Plan([shape], window, mode, s).arrays() for s in (0, 1)]


def _moved(plans, world, order):
    p0 = plans[0]
    W0 = p0["windows"]
    worder = list(range(len(W0))) if order == "plan" else sorted(range(len(W0)),
                                                                 key=lambda w: (W0[w, 1], W0[w, 3], W0[w, 5]))
    toks = np.concatenate([p0["video_indices"][W0[w, 7]:W0[w, 7] + W0[w, 8]] for w in worder])
    owner = np.empty(len(toks), np.int64)
    owner[toks] = (np.arange(len(toks)) * world) // len(toks)
    total = 0
    for p in plans:
        W = p["windows"]
        for w in range(len(W)):
            counts = np.bincount(owner[p["video_indices"][W[w, 7]:W[w, 7] + W[w, 8]]], minlength=world)
            total += int(counts.sum() - counts.max())
    return total, owner


@pytest.mark.parametrize("name,shape,window,mode,slack", [
    ("C3", [6, 45, 80], [4, 3, 4], 0, 1.0),
    ("C5", [12, 68, 120], [4, 17, 30], 1, 1.02),
])
def test_w_slab_ownership_moves_no_more_than_th_slabs(s2lib, name, shape, window, mode, slack):
    plans = _plans(s2lib, shape, window, mode)
    for world in (2, 4, 8):
        mine, owner = _moved(plans, world, "plan")
        th, _ = _moved(plans, world, "th")
        assert mine <= slack * th, (name, world, mine, th)
        # the library's own ownership is that contiguous plan-order split
        for rank in (0, world - 1):
            local = s2lib.shard(shape, 58, window, mode, rank, world)["local_tokens"]
            assert np.all(owner[local] == rank) and len(local) == np.count_nonzero(owner == rank)


def _unit_costs(sizes, heads=20):
    """The attention kernel's units for windows of `sizes` (L + T rows): per head, one unit per pair of
    128-row query tiles, costing its key tiles plus about one key tile of set-up and epilogue."""
    out = []
    for S in sizes:
        out += [(S + 127) // 128 + 1] * (heads * ((S + 255) // 256))
    return out


def _makespan(costs, ctas=148):
    """Longest-first units dealt round-robin over the persistent grid (the schedule's own order)."""
    load = np.zeros(ctas)
    for i, c in enumerate(sorted(costs, reverse=True)):
        load[i % ctas] += c
    return load.max()


@pytest.mark.parametrize("name,shape,window,mode,bound", [
    # simulated slowest-rank kernel time (key-tile steps) with (L+T)^2 as the window cost, in comments
    ("C3", [6, 45, 80], [4, 3, 4], 0, {(2, 1): 46, (8, 0): 21, (8, 1): 15}),  # 49, 21, 15
    ("C5", [12, 68, 120], [4, 17, 30], 1, {(2, 1): 386, (4, 1): 201, (8, 1): 105}),  # 400, 211, 112
])
def test_window_owners_balance_attention_work(s2lib, name, shape, window, mode, bound):
    """Every window has exactly one owner, and the owners even out the attention kernel's work: per
    rank within 12 % of the mean (whole windows: 36 equal 720p windows over 8 ranks are 5 or 4 each,
    11 % apart), and the slowest rank's simulated kernel time no worse than it is today."""
    T = 58
    for world in (2, 4, 8):
        for shifted in (0, 1):
            W = s2lib.Plan([shape], window, mode, shifted).arrays()["windows"]
            sizes = W[:, 8] + T
            owned = [s2lib.shard(shape, T, window, mode, r, world, shifted)["windows"] for r in range(world)]
            allw = np.concatenate(owned)
            assert len(allw) == len(W) and np.array_equal(np.sort(allw), np.arange(len(W))), (name, world, shifted)
            work = np.array([sum(_unit_costs(sizes[o])) for o in owned], float)
            assert work.max() <= 1.12 * work.mean(), (name, world, shifted, work.tolist())
            if (world, shifted) in bound:
                span = max(_makespan(_unit_costs(sizes[o])) for o in owned)
                assert span <= bound[(world, shifted)], (name, world, shifted, span)
