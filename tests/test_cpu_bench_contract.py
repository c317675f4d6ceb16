"""The reference arm of bench.py: one JSON line from rank 0, nothing from the others.

The arm times the reference's own CPU library (built from the reference
sources into oracle/_ref) on the benchmark workload, B=64 T=32 K=8 V=32000.
It needs no GPU, so its output contract is checked here.
"""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libdbs_ref.so")


def _run(extra_env):
    env = dict(os.environ)
    env.update(extra_env)
    return subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"],
                          cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


@pytest.mark.skipif(not os.path.exists(REF_LIB), reason="reference library not built (oracle/Makefile)")
def test_reference_arm_prints_one_line_with_the_contract_keys():
    out = _run({"RANK": "0", "WORLD_SIZE": "1"})
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, out.stdout
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    assert "unavailable" not in line
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["unit"] == "elem/s" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["steps"] == 1 and line["warmup"] == 3
    cfg = line["config"]
    assert (cfg["global_batch"], cfg["seq_len"], cfg["beam_size"], cfg["vocab"]) == (64, 32, 8, 32000)
    base = line["cpu_baseline"]
    assert base["kind"] == "reference" and base["cores"] >= 1 and base["value"] == line["value"]
    assert base["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_exit_without_work():
    out = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert out.returncode == 0, out.stderr[-2000:]
    assert out.stdout.strip() == ""


def test_port_baseline_when_the_reference_library_is_absent():
    """Without oracle/_ref the arm times the oracle's C restatement instead."""
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import torch
    import bench
    x = bench.make_inputs(torch, 2, 4, 8, 32000, 0, "cpu").numpy()
    value, cores, kind, sample = bench._oracle_port_run(x, 0.0)
    assert value > 0 and cores == 1 and kind == "port"
    assert "B=2,T=4,K=8,V=32000" in sample
