#!/usr/bin/env python
"""Benchmark of the differentiable beam search hot path on B200.

Workload (one "step"): the PyTorch `final_scores` autograd path on a batch of
B=64 examples, T=32 steps, K=8 beams, V=32000 fp32 log-probs (2.1 GB per GPU,
larger than L2), options eos_token=2, length_penalty_alpha=0.2,
selected_temperature=0.7: y = final_scores(x); y.sum().backward().
Logits are 2*N(0,1) plus a Zipf rank bias -1.1*ln(v+1), log_softmax over V,
generated on the device per example with seed 1_000_003*seed + example.

Metric: log-prob elements per second, B*T*K*V / (forward + backward time).

  * value  -- device-resident inputs, timed with CUDA events, max over ranks.
  * e2e    -- the same call with the inputs copied from pinned host memory
              every step and the loss read back (two input buffers: the next
              step's copy overlaps this step's decode and backward).
  * roofline -- the row scan kernel (the pass that streams every log-prob
              once) timed live with CUDA events around its launches; its
              algorithmic bytes are 4*B*(T*K - (K-1))*V per launch (every
              row but those of beams 1..K-1 at step 0, which no live beam
              extends).
  * cpu_baseline -- the reference's CPU library (compiled from its source into
              oracle/_ref) on the same workload, all host threads; the
              oracle's C restatement on one thread when that library is not
              built.

Warm-up: at least --warmup steps and at least --warmup-seconds (5 s) of
steps, since a freshly started GPU runs the first seconds measurably slower;
the line's "warmup" is the number of warm-up steps run.

`--impl reference` times only the reference CPU arm (rank 0).
Multi-GPU (torchrun): every rank runs its own batch (weak scaling, no
collective on the data path); value = all ranks' elements / max rank time.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import re
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "differentiable-beam-search-cuda_b200")
sys.path.insert(0, os.path.join(PKG, "python"))

METRIC = "log-prob elems/s (B·T·K·V) fwd+sparse bwd; % B200 HBM BW; 1/2/4/8 GPU"
WORKLOAD = dict(B=64, T=32, K=8, V=32000)
OPTIONS = dict(beam_size=8, eos_token=2, length_penalty_alpha=0.2, selected_temperature=0.7)
SEED = 0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--warmup-seconds", type=float, default=5.0,
                    help="untimed warm-up lasts at least this long (and at least --warmup steps)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=None,
                    help="override B (profiling a smaller case only; bench lines use the default 64)")
    ap.add_argument("--pool-decode", type=int, default=None, metavar="MULT",
                    help="profiling only: run the relaxed-pool device decode (relaxed_pool_multiplier MULT) "
                         "--steps times on the workload and print no bench line")
    ap.add_argument("--shape", default=None, metavar="T,K,V",
                    help="profiling only (--pool-decode): steps, beams and vocabulary instead of the workload's")
    ap.add_argument("--constrained", type=int, default=None, metavar="EXAMPLES",
                    help="profiling only: run the constrained variable-batch device decode (V=128256, K_b in "
                         "{1,2,4,8,16}, T_b in [8,128], 256 banned ids, forced first token, minimum length 8 before "
                         "EOS 2, repetition penalty 1.2, no repeated 3-gram) on its first EXAMPLES examples, "
                         "--steps times, and print no bench line")
    ap.add_argument("--rows", choices=("zipf", "normal"), default="zipf",
                    help="profiling only (--pool-decode): the workload's Zipf-biased rows, or "
                         "log_softmax(N(0,1)) rows as in the 256-example V=50257 configuration")
    return ap.parse_args()


def pool_decode_loop(args):
    """Device decode with the relaxed pool and weights (the ABI's work per
    call), for profiling the long-list row scan and the merge."""
    import torch
    import torch_dbs_extension as ext
    B, T, K, V = (WORKLOAD[k] for k in "BTKV")
    B = args.batch or B
    if args.shape:
        T, K, V = (int(v) for v in args.shape.split(","))
    device = torch.device("cuda", 0)
    if args.rows == "zipf":
        x = make_inputs(torch, B, T, K, V, 0, device)
    else:
        x = torch.empty((B, T, K, V), dtype=torch.float32, device=device)
        g = torch.Generator(device=device)
        for b in range(B):
            g.manual_seed(SEED * 1_000_003 + b)
            x[b].normal_(generator=g)
            x[b] = torch.log_softmax(x[b], dim=-1)
    opts = ext.DBSOptions(**dict(OPTIONS, beam_size=K, relaxed_pool_multiplier=args.pool_decode))
    for _ in range(args.steps):
        ext.device_decode(x, opts, with_pool=True, with_weights=True)
    torch.cuda.synchronize()
    print(f"pool decode x{args.steps} done")


def constrained_loop(args):
    """Device decode of the 512-example constrained variable batch's first
    slice (padded [n, 128, 16, 128256] layout, live rows only written), for
    profiling the constrained row scan and merge."""
    import numpy as np
    import torch
    import dbs_ctypes as dc
    import torch_dbs_extension as ext
    rng = np.random.default_rng(4)
    B, maxT, maxK, V = 512, 128, 16, 128256
    steps_all = rng.integers(8, maxT + 1, B).astype(np.int32)
    beams_all = rng.choice(np.array([1, 2, 4, 8, 16], np.int32), B).astype(np.int32)
    banned_row = np.zeros(V, np.uint8)
    banned_row[rng.choice(V, 256, replace=False)] = 1
    nb = min(B, args.constrained)
    steps = np.ascontiguousarray(steps_all[:nb])
    beams = np.ascontiguousarray(beams_all[:nb])
    dev = torch.device("cuda", 0)
    x = torch.zeros((nb, maxT, maxK, V), dtype=torch.float32, device=dev)
    g = torch.Generator(device=dev)
    for b in range(nb):
        g.manual_seed(4 * 1_000_003 + b)
        T, K = int(steps[b]), int(beams[b])
        z = torch.empty((T, K, V), device=dev)
        z.normal_(generator=g)
        x[b, :T, :K] = torch.log_softmax(1.5 * z, dim=-1)
    eos = np.full(nb, 2, np.int32)
    minl = np.full(nb, 8, np.int32)
    banned = torch.tensor(np.tile(banned_row, (nb, 1)), device=dev)
    forced_np = np.full((nb, maxT), -1, np.int32)
    forced_np[:, 0] = 1
    forced = torch.tensor(forced_np, device=dev)
    sel = int((steps.astype(np.int64) * beams).sum())
    fin = int(beams.sum())
    sel_names = ("parents", "tokens", "lengths", "from_logprob", "raw_scores", "scores", "weights")
    out = {}
    s = dc.DBSDeviceDecodeOutputs()
    for name, _ in dc.DBSDeviceDecodeOutputs._fields_:
        n = sel if name in sel_names else (fin if name.startswith("final") else 8 * sel)
        dt = torch.uint8 if "from_logprob" in name else (
            torch.int32 if name.split("_")[-1] in ("parents", "tokens", "lengths") else torch.float32)
        out[name] = torch.empty(n, dtype=dt, device=dev)
        setattr(s, name, out[name].data_ptr())
    opts = ext.DBSOptions(beam_size=maxK, eos_token=2, min_length=8)
    h = ext._handle(opts)
    lib = ext._library()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(args.steps):
        rc = lib.dbs_device_decode_batch_variable_ex(
            h, ext._vp(x), nb, maxT, maxK, V, steps.ctypes.data_as(ctypes.c_void_p),
            beams.ctypes.data_as(ctypes.c_void_p), eos.ctypes.data_as(ctypes.c_void_p),
            minl.ctypes.data_as(ctypes.c_void_p), ext._vp(banned), ext._vp(forced), ctypes.c_float(1.2), 3,
            ctypes.byref(s), stream)
        if rc != 0:
            raise RuntimeError(lib.dbs_last_error(h).decode())
    torch.cuda.synchronize()
    print(f"constrained decode of {nb} examples ({sel} live rows) x{args.steps} done")


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_traffic_per_launch():
    """DRAM bytes per row-scan launch from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "row_scan_config2.md")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        m = re.search(r"dram_bytes_per_launch:\s*([0-9.eE+]+)", f.read())
    return float(m.group(1)) if m else None


def make_inputs(torch, B, T, K, V, first_example, device):
    x = torch.empty((B, T, K, V), dtype=torch.float32, device=device)
    bias = -1.1 * torch.log(torch.arange(V, dtype=torch.float32, device=device) + 1.0)
    g = torch.Generator(device=device)
    for b in range(B):
        g.manual_seed(SEED * 1_000_003 + first_example + b)
        x[b].normal_(generator=g)
        x[b].mul_(2.0).add_(bias)
        x[b] = torch.log_softmax(x[b], dim=-1)
    return x


class ClockSampler:
    """nvidia-smi clock / throttle sampling while the timed region runs."""

    def __init__(self, uuid: str):
        self.uuid = uuid
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.uuid, f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        # nvidia-smi's start-up contends with this process's CUDA calls: let it
        # settle (three samples delivered) before the timed region begins
        t0 = time.time()
        while len(self.lines) < 3 and time.time() - t0 < 10.0 and self.proc.poll() is None:
            time.sleep(0.05)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for name, val in zip(names, parts[3:7]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def reference_cpu_run(x_host, steps_budget_s=20.0):
    """Time the reference CPU library on the workload (all host threads).

    Mirrors the reference's CPU path for final_scores forward + backward:
    dbs_decode_batch over the batch, then per example the sparse backward of
    grad_final = ones and the scatter into a zero dense gradient
    (python/torch_extension.cpp:128-188). Returns (elems/s, cores, kind, sample).
    """
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import dbs_ctypes as dc
    from oracle import reference_library_path
    path = reference_library_path()
    cores = os.cpu_count() or 1
    B, T, K, V = x_host.shape
    x = np.ascontiguousarray(x_host)
    if path is None:
        return _oracle_port_run(x, steps_budget_s)
    lib = dc.load_library(path, device_api=False)
    dec = dc.Decoder(lib, dc.Options(**OPTIONS))
    gf = np.ones(K, dtype=np.float32)
    elems = 0
    t0 = time.perf_counter()
    reps = 0
    while True:
        br = dec.decode_batch(x, B, T, V, cores)
        grad = np.zeros((B, T * K * V), dtype=np.float32)
        for b in range(B):
            r = lib.dbs_batch_result_at(br, b)
            bw = dec.backward(r, None, None, gf, mode="default")
            out = dc.read_backward(lib, bw, K=K)
            grad[b, out["indices"]] += out["values"]
            lib.dbs_free_backward(bw)
        lib.dbs_free_batch_result(br)
        del grad
        elems += B * T * K * V
        reps += 1
        if time.perf_counter() - t0 >= steps_budget_s or reps >= 50:
            break
    dt = time.perf_counter() - t0
    dec.close()
    sample = (f"{reps} x full batch B={B},T={T},K={K},V={V} via dbs_decode_batch({cores} threads) + per-example "
              f"dbs_backward + dense scatter; kernel={lib.dbs_selected_kernel_name().decode()}")
    return elems / dt, cores, "reference", sample


def _oracle_port_run(x, steps_budget_s):
    """The CPU restatement in oracle/ on one host thread, for when the reference
    library could not be built: per example the decode, the sparse backward of
    grad_final = ones and the scatter into a zero dense gradient. Returns
    (elems/s, 1, "port", sample), or None when the oracle is not built either."""
    import numpy as np
    from oracle import ORACLE_SO, OracleLib
    if not os.path.exists(ORACLE_SO):
        return None
    ol = OracleLib()
    opts = ol.options(**OPTIONS)
    B, T, K, V = x.shape
    gf = np.ones(K, dtype=np.float32)
    elems = 0
    reps = 0
    t0 = time.perf_counter()
    while True:
        grad = np.zeros((B, T * K * V), dtype=np.float32)
        for b in range(B):
            fwd = ol.decode(opts, x[b], T, V)
            out = ol.backward_sparse(fwd, grad_final=gf)
            grad[b, out["indices"]] += out["values"]
        del grad
        elems += B * T * K * V
        reps += 1
        if time.perf_counter() - t0 >= steps_budget_s or reps >= 50:
            break
    dt = time.perf_counter() - t0
    sample = (f"{reps} x full batch B={B},T={T},K={K},V={V} through the oracle's C restatement (1 thread) "
              f"+ sparse backward + dense scatter")
    return elems / dt, 1, "port", sample


def bench_config(B, T, K, V, world):
    return {"workload": f"torch final_scores fwd + y.sum().backward(), B={B} T={T} K={K} V={V}, eos_token=2, "
                        "length_penalty_alpha=0.2, selected_temperature=0.7 (per GPU)",
            "global_batch": B * world, "seq_len": T, "beam_size": K, "vocab": V,
            "parallelism": f"batch-sharded x{world}, no data-path collective",
            "l2": f"inputs larger than L2 ({4 * B * T * K * V / 1e9:.1f} GB per GPU); no flush needed"}


def run_reference_arm(args, rank, world):
    """The reference's own CPU implementation of the path on the host cores.

    One step = one full batch (decode + sparse backward + dense scatter, all
    host threads); rank 0 alone runs and prints."""
    if rank != 0:
        return
    B, T, K, V = (WORKLOAD[k] for k in "BTKV")
    # the GPU arm's recipe on the CPU generator (same distribution; the CUDA
    # generator's stream differs)
    import torch
    x = make_inputs(torch, B, T, K, V, 0, "cpu").numpy()
    vals = []
    res = None
    for i in range(max(3, args.warmup) + args.steps):
        res = reference_cpu_run(x, steps_budget_s=0.0)
        if res is None:
            print(json.dumps({"impl": "reference", "unavailable": "neither oracle/_ref/libdbs_ref.so nor the oracle port was built"}))
            return
        if i >= max(3, args.warmup):
            vals.append(res[0])
    value = statistics.median(vals)
    elems = B * T * K * V
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "elem/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * elems / value, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: 2*N(0,1) logits + Zipf bias -1.1*ln(v+1), log_softmax over V (CPU generator)",
        "config": bench_config(B, T, K, V, 1),
        "cpu_baseline": {"value": value, "unit": "elem/s", "cores": res[1], "kind": res[2],
                         "sample": res[3] + "; median over steps"},
        "e2e": {"value": value, "unit": "elem/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    if args.pool_decode:
        pool_decode_loop(args)
        return
    if args.constrained:
        constrained_loop(args)
        return

    import numpy as np
    import torch
    import torch.distributed as dist
    import torch_dbs_extension as ext
    import dbs_ctypes

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)

    B, T, K, V = (WORKLOAD[k] for k in "BTKV")
    if args.batch:
        B = args.batch
    elems = B * T * K * V
    opts = ext.DBSOptions(**OPTIONS)
    lib = ext._library()

    x = make_inputs(torch, B, T, K, V, rank * B, device)
    x.requires_grad_(True)

    def step():
        x.grad = None
        y = ext.final_scores(x, opts)
        y.sum().backward()

    # at least W steps and at least a few seconds: a freshly started GPU runs
    # the first seconds of this workload measurably slower
    warm_steps = 0
    t_warm = time.perf_counter()
    while warm_steps < max(3, args.warmup) or time.perf_counter() - t_warm < args.warmup_seconds:
        step()
        warm_steps += 1
        if warm_steps % 50 == 0:
            torch.cuda.synchronize()
    torch.cuda.synchronize()
    if world > 1:   # every rank ran the same number of steps before the timed region
        wt = torch.tensor([warm_steps], dtype=torch.int64, device=device)
        dist.all_reduce(wt, op=dist.ReduceOp.MAX)
        for _ in range(int(wt.item()) - warm_steps):
            step()
        warm_steps = int(wt.item())
        torch.cuda.synchronize()

    uuid = str(torch.cuda.get_device_properties(device).uuid)
    sampler = ClockSampler(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
    sampler.start()
    time.sleep(0.3)
    # inside the timed region only the row scan (the roofline kernel) is
    # bracketed by events, on the stream it is launched on
    lib.dbs_device_profile(-1)
    lib.dbs_device_profile_kernels(1 << dbs_ctypes.PROFILED_KERNELS.index("row_scan"))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        step()
    end.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    lib.dbs_device_profile(0)
    clocks = sampler.stop()
    ms = start.elapsed_time(end)

    def read_profile():
        out = {}
        for i, name in enumerate(dbs_ctypes.PROFILED_KERNELS):
            tot = ctypes.c_double()
            n = ctypes.c_int64()
            lib.dbs_device_profile_read(i, ctypes.byref(tot), ctypes.byref(n))
            out[name] = {"total_ms": tot.value, "launches": n.value}
        return out

    rs_live = read_profile()["row_scan"]
    # per-kernel breakdown from a short separate pass with every kernel timed
    # (events between launches cost a little, so it stays out of the timed region)
    prof_steps = min(args.steps, 20)
    lib.dbs_device_profile(-1)
    lib.dbs_device_profile(1)
    for _ in range(prof_steps):
        step()
    torch.cuda.synchronize()
    lib.dbs_device_profile(0)
    kern = read_profile()
    for v in kern.values():
        v["avg_ms"] = v["total_ms"] / v["launches"] if v["launches"] else None
        v["launches_per_step"] = v["launches"] / prof_steps
    launches = int(round(sum(v["launches"] for v in kern.values()) / prof_steps * args.steps))
    t = torch.tensor([ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    ms_per_step = ms_max / args.steps
    value = world * elems / (ms_per_step / 1e3)

    # live roofline of the row scan
    rs = rs_live
    peak, peak_kind = measured_peaks()
    rs_ms = rs["total_ms"] / max(1, rs["launches"])
    # every row but the K-1 rows of step 0 that no live beam extends
    alg_bytes = 4.0 * B * (T * K - (K - 1)) * V
    achieved = alg_bytes / (rs_ms / 1e3) / 1e9 if rs_ms > 0 else None
    traffic = ncu_traffic_per_launch()
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": (achieved / peak) if achieved else None, "traffic": traffic,
                "peak_kind": peak_kind, "kernel": "row_scan_kernel",
                "algorithmic_bytes_per_launch": alg_bytes, "avg_launch_ms": rs_ms}
    step_bytes = alg_bytes + 4.0 * elems  # log-prob read + dense gradient write
    whole = {"achieved_gbs": step_bytes / (ms_per_step / 1e3) / 1e9,
             "frac": step_bytes / (ms_per_step / 1e3) / 1e9 / peak}

    # end to end from pinned host memory: every step copies its inputs from
    # pinned host memory and reads its loss back; two device input buffers
    # let the next step's copy (a side stream) run beside this step's decode
    # and backward. A buffer is refilled only after the loss read-back of
    # the step that used it, and every copy lies inside the timed region.
    x_host = x.detach().cpu().pin_memory()
    bufs = [torch.empty_like(x.detach()).requires_grad_(True) for _ in range(2)]
    copy_stream = torch.cuda.Stream(device=device)
    ready = [torch.cuda.Event(), torch.cuda.Event()]
    main_stream = torch.cuda.current_stream(device)

    def issue_copy(i, after=None):
        with torch.cuda.stream(copy_stream):
            if after is not None:
                copy_stream.wait_event(after)
            with torch.no_grad():
                bufs[i % 2].copy_(x_host, non_blocking=True)
            ready[i % 2].record(copy_stream)

    def e2e_run(n, start=None):
        issue_copy(0, start)
        for i in range(n):
            if i + 1 < n:
                issue_copy(i + 1)
            main_stream.wait_event(ready[i % 2])
            xd = bufs[i % 2]
            xd.grad = None
            y = ext.final_scores(xd, opts)
            loss = y.sum()
            loss.backward()
            loss.item()

    e2e_run(2)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    e2e_run(args.e2e_steps, start=e0)
    e1.record()
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms = float(te.item()) / args.e2e_steps
    e2e = {"value": world * elems / (e2e_ms / 1e3), "unit": "elem/s", "h2d_bytes_per_step": 4 * elems,
           "d2h_bytes_per_step": 4, "ms_per_step": e2e_ms}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        r = reference_cpu_run(x_host.numpy(), steps_budget_s=10.0)
        if r is not None:
            cpu = {"value": r[0], "unit": "elem/s", "cores": r[1], "kind": r[2], "sample": r[3]}
    rescans = (ctypes.c_int64(), ctypes.c_int64())
    lib.dbs_device_last_rescan_counts(ext._handle(opts), ctypes.byref(rescans[0]), ctypes.byref(rescans[1]))

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": value, "unit": "elem/s", "n_gpus": world, "steps": args.steps,
        "warmup": warm_steps, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: 2*N(0,1) logits + Zipf bias -1.1*ln(v+1), log_softmax over V, seeded per example",
        "config": bench_config(B, T, K, V, world),
        "roofline": roofline,
        "step_hbm": whole,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": launches,
        "kernels": {"source": f"separate {prof_steps}-step pass, every kernel bracketed by events", **kern},
        "rescans": {"row_scan": rescans[0].value, "step_merge": rescans[1].value},
        "clocks": clocks,
    }
    print(json.dumps(line))


if __name__ == "__main__":
    main()
