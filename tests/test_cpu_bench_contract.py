"""The reference arm of bench.py: one JSON line from rank 0, nothing from the others.

The arm times the reference's own CPU library (built from the reference
sources into oracle/_ref) on the benchmark workloads: by default the
large-beam batch (B=256 T=64 K=32 V=50257; a seeded sample of examples per
step), with --config 2 the torch final_scores batch (B=64 T=32 K=8 V=32000).
It needs no GPU, so its output contract is checked here.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libdbs_ref.so")


def _run(extra_env, *args):
    env = dict(os.environ)
    env.update(extra_env)
    return subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3", *args],
                          cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)


def _check_line(out):
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, out.stdout
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    assert "unavailable" not in line
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e", "kind"):
        assert key in line, key
    assert line["unit"] == "elem/s" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["steps"] == 1 and line["warmup"] == 3
    base = line["cpu_baseline"]
    assert base["kind"] == "reference" == line["kind"] and base["cores"] >= 1 and base["value"] == line["value"]
    assert base["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    return line


@pytest.mark.skipif(not os.path.exists(REF_LIB), reason="reference library not built (oracle/Makefile)")
def test_reference_arm_default_config_is_the_large_beam_batch():
    line = _check_line(_run({"RANK": "0", "WORLD_SIZE": "1"}, "--ref-sample", "1"))
    cfg = line["config"]
    assert (cfg["global_batch"], cfg["seq_len"], cfg["beam_size"], cfg["vocab"]) == (256, 64, 32, 50257)
    assert line["scaling"] == "strong"
    assert "1 examples" in line["cpu_baseline"]["sample"]


@pytest.mark.skipif(not os.path.exists(REF_LIB), reason="reference library not built (oracle/Makefile)")
def test_reference_arm_config2():
    line = _check_line(_run({"RANK": "0", "WORLD_SIZE": "1"}, "--config", "2"))
    cfg = line["config"]
    assert (cfg["global_batch"], cfg["seq_len"], cfg["beam_size"], cfg["vocab"]) == (64, 32, 8, 32000)


@pytest.mark.skipif(not os.path.exists(REF_LIB), reason="reference library not built (oracle/Makefile)")
def test_reference_arm_config1():
    line = _check_line(_run({"RANK": "0", "WORLD_SIZE": "1"}, "--config", "1"))
    cfg = line["config"]
    assert (cfg["global_batch"], cfg["seq_len"], cfg["beam_size"], cfg["vocab"]) == (4, 4, 4, 32000)
    assert "20 x 4 examples" in line["cpu_baseline"]["sample"]


def test_config1_inputs_are_the_seeded_cpu_tensor():
    """Config 1's log-probs come from the CPU generator seeded 0, so the GPU
    arm and the reference arm decode the same tensor on any host."""
    sys.path.insert(0, ROOT)
    import torch
    import bench
    a = bench.make_inputs1(torch, "cpu")
    g = torch.Generator().manual_seed(0)
    want = torch.log_softmax(1.5 * torch.randn((4, 4, 4, 32000), generator=g), dim=-1)
    assert a.shape == (4, 4, 4, 32000) and torch.equal(a, want)


def test_reference_arm_other_ranks_exit_without_work():
    out = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert out.returncode == 0, out.stderr[-2000:]
    assert out.stdout.strip() == ""


def test_port_baseline_when_the_reference_library_is_absent():
    """Without oracle/_ref the config-2 arm times the oracle's C restatement instead."""
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import torch
    import bench
    x = bench.make_inputs(torch, 2, 4, 8, 32000, 0, "cpu").numpy()
    value, cores, kind, sample = bench._oracle_port_run(x, 0.0)
    assert value > 0 and cores == 1 and kind == "port"
    assert "B=2,T=4,K=8,V=32000" in sample


def test_scatter_add_keeps_duplicate_indices():
    """The CPU arms build the dense gradient with np.add.at: a selected slot and
    a pool entry can name one index, and both contributions must count."""
    g = np.zeros(4, dtype=np.float32)
    np.add.at(g, np.array([1, 1, 3]), np.array([0.5, 0.25, 1.0], dtype=np.float32))
    assert g.tolist() == [0.0, 0.75, 0.0, 1.0]


@pytest.mark.parametrize("content,want", [
    ('{"hbm_gbs": 6538.9, "bf16_tflops": 1500.0}', (6538.9, "measured")),
    ('{"b200": {"hbm_gbs": 6500}}', (6500.0, "measured")),
    ('{"bf16_tflops": 1500.0}', (6650.0, "fallback")),
    ("not json", (6650.0, "fallback")),
    (None, (6650.0, "fallback")),
])
def test_roofline_peak_from_the_measured_peaks_file(tmp_path, monkeypatch, content, want):
    """The roofline's denominator: the measured copy bandwidth when the peaks
    file holds one, the fallback figure (and says so) when it is absent or
    unreadable, never an exception that would lose the bench line."""
    sys.path.insert(0, ROOT)
    import bench
    if content is not None:
        (tmp_path / "MEASURED_PEAKS.json").write_text(content)
    monkeypatch.setattr(bench, "ROOT", str(tmp_path))
    assert bench.measured_peaks() == want


def test_compare_with_reference_flags_a_difference():
    """The bench's parity check of its sample against the reference's outputs."""
    sys.path.insert(0, ROOT)
    import bench
    T, K, P = 2, 2, 4
    base = {f: np.zeros(T * K, np.int32) for f in ("parents", "tokens", "lengths")}
    base.update({f: np.zeros(T * P, np.int32) for f in ("pool_parents", "pool_tokens", "pool_lengths")})
    base.update({f: np.full(T * K, -1.5, np.float32) for f in ("raw_scores", "scores", "weights")})
    base.update({f: np.full(T * P, -1.5, np.float32) for f in ("pool_raw_scores", "pool_scores", "relaxed_weights")})
    base.update({f: np.full(K, -3.0, np.float32) for f in ("final_scores", "final_raw_scores")})
    ours = dict(base, sparse_indices=np.array([3, 9]), sparse_values=np.array([1.0, 1.0], np.float32),
                grad_initial=np.array([1.0, 0.0], np.float32))
    ref = dict(base, backward={"indices": np.array([3, 9]), "values": np.array([1.0, 1.0], np.float32),
                               "grad_initial": np.array([1.0, 0.0], np.float32)})
    assert bench.compare_with_reference(ours, ref, "ex") is None
    bad = dict(ours, tokens=ours["tokens"].copy())
    bad["tokens"][1] = 7
    assert "tokens" in bench.compare_with_reference(bad, ref, "ex")
    bad = dict(ours, sparse_values=np.array([1.0, 1.001], np.float32))
    assert "sparse values" in bench.compare_with_reference(bad, ref, "ex")


def _warm_up_worker(rank, world, port, path):
    # ranks whose steps take different times must still run the same number
    # of warm-up steps: each step holds a collective, so a rank that stopped
    # early would leave the others waiting in it
    import time
    import types
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        sys.path.insert(0, ROOT)
        import bench
        count = [0]
        buf = torch.zeros(4)
        out = torch.zeros(4 * world)

        def step():
            time.sleep(0.002 if rank == 0 else 0.02)
            dist.all_gather_into_tensor(out, buf)
            count[0] += 1

        args = types.SimpleNamespace(warmup=3, warmup_seconds=0.3)
        if rank == 1:
            time.sleep(0.2)   # its warm-up clock starts later than rank 0's
        n = bench.warm_up(step, args, world, torch.device("cpu"), 5, sync=lambda: None)
        counts = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(counts, torch.tensor([count[0]], dtype=torch.int64))
        if rank == 0:
            with open(path, "w") as f:
                f.write(json.dumps({"n": n, "counts": [int(c.item()) for c in counts]}))
    finally:
        dist.destroy_process_group()


def test_warm_up_runs_the_same_steps_on_every_rank(tmp_path):
    import torch.multiprocessing as mp
    path = tmp_path / "warm.json"
    mp.start_processes(_warm_up_worker, args=(2, 29637, str(path)), nprocs=2, start_method="spawn")
    got = json.loads(path.read_text())
    assert got["counts"][0] == got["counts"][1] == got["n"] >= 3
