"""CPU: bench.py's reference arm keeps the driver's JSON contract.

`bench.py --impl reference` times the reference's own CPU layer code on the
host (no GPU): whole blocks, each once, and a one-thread sample.  Rank 0
prints one JSON line with the arm's metric, the same config dict as the GPU
arm, a cpu_baseline describing the run, the extrapolation it made and an e2e
of zero copied bytes; other ranks of a torchrun launch exit 0 without output.
Run on the small config-1 geometry so the CPU suite stays short.
"""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(extra_env=None):
    env = dict(os.environ)
    env.update(extra_env or {})
    return subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0",
                           "--config", "c1"],
                          cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_json_line():
    from oracle import oracle

    if not os.path.exists(oracle.REF_SO):
        pytest.skip("oracle/_ref not built (reference tree absent)")
    r = _run()
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    import bench

    assert d["metric"] == bench.METRIC and d["unit"] == "tokens/s"
    assert d["value"] > 0 and d["higher_is_better"] is True and d["steps"] == 1 and d["warmup"] == 0
    args = type("A", (), {"config": "c1", "blocks": bench.BLOCKS})
    assert d["config"] == json.loads(json.dumps(bench.config_dict(args, 1)))
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    ex = d["extrapolated"]
    assert ex["measured_blocks"] == 2 and ex["scale"] == 16
    assert abs(d["ms_per_step"] - 16e3 * (ex["unshifted_block_s"] + ex["shifted_block_s"])) < 1e-6 * d["ms_per_step"]
    st = d["single_thread"]
    assert st["cores"] == 1 and st["value"] > 0
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    r = _run({"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
