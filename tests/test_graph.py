"""The drop-in path at graph level: an ncnn .param / .bin block graph (written by
tests/block_graph.py from the block restatement) loaded by the ncnn-surface
library's Net with the two custom layers registered as seedvr2_dit.cpp:614-618
does, inputs bound by name (in0..in9) and out0 / out1 extracted
(seedvr2_dit.cpp:724-738, :832-833).

CPU: the files parse (layer / blob counts), custom layers are created through
their creators and load their weights; malformed files are refused with -1.
GPU: the graph's outputs against the block stack (s2_dit_forward, same
weights) and against the fp32 oracle block restatement, with an RMSNorm and a
LayerNorm block and a shifted second block.
"""
import numpy as np
import pytest

from tests.block_graph import write_block_graph
from tests.conftest import cosine, rel_maxabs
from tests.test_gpu_block import make_block_weights

D, HEADS, F, HD, PAIRS = 256, 2, 1024, 128, 21
SHAPE, T, WINDOW, MODE = [2, 8, 12], 9, [1, 4, 6], 1


def _weights(seed, blocks):
    rng = np.random.default_rng(seed)
    ws = [make_block_weights(rng, D, F, HD, PAIRS) for _ in range(blocks)]
    for w in ws:
        w["rope_freqs"] = np.asarray(w["rope_freqs"], np.float32)
    return ws


def _files(tmp_path, ws, layer_norm=()):
    p, b = tmp_path / "blocks.param", tmp_path / "blocks.bin"
    counts = write_block_graph(p, b, ws, D=D, heads=HEADS, F=F, window=WINDOW, window_mode=MODE,
                               layer_norm=layer_norm)
    return p, b, counts


def test_graph_files_load(tmp_path):
    from seedvr2_ncnn_b200 import build, layers

    build.build()
    ws = _weights(1, 2)
    p, b, (n_layers, n_blobs) = _files(tmp_path, ws, layer_norm=(0,))
    net = layers.Net(p, b)
    assert net.info() == (n_layers, n_blobs)
    net.close()
    # a truncated .bin: the last SharedLinear cannot read its bias
    data = b.read_bytes()
    (tmp_path / "short.bin").write_bytes(data[:-16])
    with pytest.raises(layers.LayerError) as e:
        layers.Net(p, tmp_path / "short.bin")
    assert e.value.args[0].endswith("-100")
    # an unknown layer type, a bad magic, a blob consumed before it is produced
    text = p.read_text()
    for bad in (text.replace("GELU", "Swish", 1), text.replace("7767517", "7767518", 1),
                text.replace(" in2 in2_b0", " in2x in2_b0", 1)):
        (tmp_path / "bad.param").write_text(bad)
        with pytest.raises(layers.LayerError) as e:
            layers.Net(tmp_path / "bad.param", b)
        assert e.value.args[0].endswith("-1")


@pytest.mark.gpu
def test_graph_matches_block_stack_and_oracle(tmp_path, gpu_ctx, s2lib, port):
    import torch

    from seedvr2_ncnn_b200 import layers

    ws = _weights(2, 2)
    p, b, _ = _files(tmp_path, ws, layer_norm=(0,))
    rng = np.random.default_rng(3)
    nv = int(np.prod(SHAPE))
    xv = rng.standard_normal((nv, D)).astype(np.float32)
    xt = rng.standard_normal((T, D)).astype(np.float32)
    mod = rng.standard_normal((6, D)).astype(np.float32)

    net = layers.Net(p, b)
    net.set_runtime([SHAPE], [T])
    ins = {"in0": torch.from_numpy(xv).cuda(), "in1": torch.from_numpy(xt).cuda()}
    for k in range(6):
        ins[f"in{4 + k}"] = torch.from_numpy(mod[k:k + 1].copy()).cuda()
    outs = {"out0": torch.empty(nv, D, device="cuda"), "out1": torch.empty(T, D, device="cuda")}
    net.extract(ins, outs)
    gv, gt = outs["out0"].cpu().numpy(), outs["out1"].cpu().numpy()
    net.close()

    # the block stack with the same weights (its fused epilogues round at other points: close, not equal)
    dit = s2lib.Dit(gpu_ctx, num_blocks=2, hidden=D, heads=HEADS, head_dim=HD, mlp_hidden=F, rope_pairs=PAIRS,
                    window=WINDOW, window_mode=MODE)
    for i, w in enumerate(ws):
        dit.set_block_weights(i, w)
    dit.set_block_norm(0, True)
    x = torch.from_numpy(np.concatenate([xv, xt])).cuda()
    dit.forward(SHAPE, T, x, torch.from_numpy(mod).cuda())
    sx = x.cpu().numpy()
    dit.close()
    g = np.concatenate([gv, gt])
    assert cosine(g, sx) >= 0.9999 and rel_maxabs(g, sx) <= 1e-2

    # the fp32 oracle
    rv, rt = xv, xt
    for i, w in enumerate(ws):
        wo = dict(w)
        wo["freqs"] = wo.pop("rope_freqs")
        rv, rt = port.block_forward(dims=[D, HEADS, HD, F, PAIRS, MODE, *WINDOW, i & 1, int(i == 0)], eps_norm=1e-5,
                                    eps_qk=1e-5, weights=wo, modulation=mod[None], shapes=[SHAPE], text_lengths=[T],
                                    x_video=rv, x_text=rt)
    ref = np.concatenate([rv, rt])
    assert cosine(g, ref) >= 0.9995 and rel_maxabs(g, ref) <= 2e-2
    assert gpu_ctx.status() == 0
