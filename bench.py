#!/usr/bin/env python
"""Benchmark of the differentiable beam search hot path on B200.

Default workload (one "step", `--config 3`): the large-beam batch of
B=256 examples, T=64 steps, K=32 beams, V=50257 fp32 log-probs (105 GB),
log_softmax over V of N(0,1) logits generated on the device per example
(seed 1_000_003*seed + example), default decoder options (so every step also
selects the relaxed pool of P=256 candidates and its weights). A step is the
C ABI's work for that batch on the device:

  dbs_device_decode_batch (pool + weights)  ->  dbs_device_backward_batch
  (sparse, grad_final = e_0 per example)    ->  NCCL all-gather of the
  results ([B,K] final scores, [B,T,K] tokens and parents, sparse counts and
  the sparse gradient entries) when there is more than one rank.

Strong scaling: the 256 examples are split contiguously over the ranks
(256/N each); every rank decodes its share and the all-gather gives every
rank the whole batch's results.

Metric: log-prob elements per second, B*T*K*V / (forward + backward time).

  * value  -- device-resident inputs, timed with CUDA events around the
              steps, max over ranks.
  * e2e    -- the same batch through the reference-facing C ABI with HOST
              buffers: dbs_decode_batch on pinned host log-probs, then
              dbs_backward per example, every result read into host memory
              (the library stages the inputs to the device inside the call).
  * roofline -- the row scan (the pass that streams every log-prob once),
              timed live with CUDA events inside the timed region: one event
              pair per decode call around all of its row-scan launches;
              algorithmic bytes 4*B*(T*K - (K-1))*V per call (every row but
              those of beams 1..K-1 at step 0, which no live beam extends).
  * cpu_baseline -- the reference's CPU library (compiled from its source
              into oracle/_ref) on a seeded 16-example sample of the same
              workload with all host threads; its outputs for those examples
              are also compared with this run's ("parity").

`--config 2`: the PyTorch final_scores autograd path on B=64, T=32, K=8,
V=32000 (Zipf-biased logits, eos 2, length penalty 0.2, selected
temperature 0.7; forward + y.sum().backward() with the dense gradient),
64 examples per GPU (weak scaling, no collective on the data path).

Warm-up: at least --warmup steps and at least --warmup-seconds of steps,
since a freshly started GPU runs the first seconds measurably slower; the
line's "warmup" is the number of warm-up steps run.

`--config 4`: the 512-example constrained variable batch (V=128256, all
sequence constraints) on one GPU, decoded in eight 64-example slices whose
decodes are timed with the slice resident; its CPU arm is the reference
library's dbs_decode_constrained_ex on a 16-example sample (see
run_config4).

`--impl reference` times only the reference CPU arm (rank 0 prints; other
ranks exit without work).
"""
from __future__ import annotations

import argparse
import ctypes
import json
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
METRIC4 = "log-prob elems/s (sum of T_b*K_b*V) constrained variable batch"
SEED = 0
# config 1 (the reference's own small case: four examples, launch-bound; one GPU)
WORKLOAD1 = dict(B=4, T=4, K=4, V=32000)
OPTIONS1 = dict(beam_size=4)
# config 2 (torch final_scores, per GPU)
WORKLOAD = dict(B=64, T=32, K=8, V=32000)
OPTIONS = dict(beam_size=8, eos_token=2, length_penalty_alpha=0.2, selected_temperature=0.7)
# config 3 (whole batch, split over the ranks)
WORKLOAD3 = dict(B=256, T=64, K=32, V=50257)
OPTIONS3 = dict(beam_size=32)
REF_SAMPLE3 = 16
# config 5 (one long huge-vocabulary example; one GPU)
WORKLOAD5 = dict(B=1, T=256, K=16, V=256000)
OPTIONS5 = dict(beam_size=16)


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=3, choices=(1, 2, 3, 4, 5),
                    help="3: the large-beam batch (default, the bench line); 1: the B=4 T=4 K=4 V=32000 case "
                         "(one GPU, L2 flushed between steps); 2: the torch final_scores batch; 4: the constrained "
                         "variable batch; 5: the single B=1 T=256 K=16 V=256000 example (one GPU)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=None,
                    help="end-to-end steps (default 20 for config 2, 2 for config 3)")
    ap.add_argument("--warmup-seconds", type=float, default=5.0,
                    help="untimed warm-up lasts at least this long (and at least --warmup steps)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ref-sample", type=int, default=REF_SAMPLE3,
                    help="config 3: examples in the reference CPU library's timed sample")
    ap.add_argument("--batch", type=int, default=None,
                    help="profiling only: examples per GPU instead of the workload's (the line says so)")
    ap.add_argument("--pool-decode", type=int, default=None, metavar="MULT",
                    help="profiling only: run the relaxed-pool device decode (relaxed_pool_multiplier MULT) "
                         "--steps times on the config-2 inputs and print no bench line")
    ap.add_argument("--shape", default=None, metavar="T,K,V",
                    help="profiling only (--pool-decode): steps, beams and vocabulary instead of the workload's")
    ap.add_argument("--constrained", type=int, default=None, metavar="EXAMPLES",
                    help="profiling only: run the constrained variable-batch device decode (V=128256, K_b in "
                         "{1,2,4,8,16}, T_b in [8,128], 256 banned ids, forced first token, minimum length 8 before "
                         "EOS 2, repetition penalty 1.2, no repeated 3-gram) on its first EXAMPLES examples, "
                         "--steps times, and print no bench line")
    ap.add_argument("--rows", choices=("zipf", "normal"), default="zipf",
                    help="profiling only (--pool-decode): the Zipf-biased rows of config 2, or "
                         "log_softmax(N(0,1)) rows as in config 3")
    ap.add_argument("--default-options", action="store_true",
                    help="profiling only (--pool-decode): the default options (beam_size K, eos -1, no length "
                         "penalty) as in config 3, instead of config 2's")
    return ap.parse_args(argv)


# ---------------------------------------------------------------------------
# inputs
# ---------------------------------------------------------------------------
def make_inputs(torch, B, T, K, V, first_example, device):
    """Config 2: 2*N(0,1) logits plus the Zipf rank bias -1.1*ln(v+1), log_softmax over V."""
    x = torch.empty((B, T, K, V), dtype=torch.float32, device=device)
    bias = -1.1 * torch.log(torch.arange(V, dtype=torch.float32, device=device) + 1.0)
    g = torch.Generator(device=device)
    for b in range(B):
        g.manual_seed(SEED * 1_000_003 + first_example + b)
        x[b].normal_(generator=g)
        x[b].mul_(2.0).add_(bias)
        x[b] = torch.log_softmax(x[b], dim=-1)
    return x


def make_inputs3(torch, B, T, K, V, first_example, device):
    """Config 3: log_softmax over V of N(0,1) logits, one generator seed per example."""
    x = torch.empty((B, T, K, V), dtype=torch.float32, device=device)
    g = torch.Generator(device=device)
    for b in range(B):
        g.manual_seed(SEED * 1_000_003 + first_example + b)
        x[b].normal_(generator=g)
        x[b] = torch.log_softmax(x[b], dim=-1)
    return x


def make_inputs1(torch, device):
    """Config 1: log_softmax over V of 1.5*N(0,1) logits, [4,4,4,32000], from
    the CPU generator seeded 0 (the same tensor on every host)."""
    B, T, K, V = (WORKLOAD1[k] for k in "BTKV")
    g = torch.Generator().manual_seed(SEED)
    x = torch.log_softmax(1.5 * torch.randn((B, T, K, V), generator=g), dim=-1)
    return x.to(device)


def make_inputs5(torch, T, K, V, device):
    """Config 5: log_softmax over V of N(0,1) logits plus +8 on 64 seeded ids of
    each step (the same ids in every row of the step), one example."""
    x = torch.empty((1, T, K, V), dtype=torch.float32, device=device)
    g = torch.Generator(device=device)
    g.manual_seed(SEED * 1_000_003)
    x[0].normal_(generator=g)
    for t in range(T):
        ids = torch.randint(0, V, (64,), generator=g, device=device)
        x[0, t, :, ids] += 8.0
    x[0] = torch.log_softmax(x[0], dim=-1)
    return x


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
        x = make_inputs3(torch, B, T, K, V, 0, device)
    base = {} if args.default_options else OPTIONS
    opts = ext.DBSOptions(**dict(base, beam_size=K, relaxed_pool_multiplier=args.pool_decode))
    for _ in range(args.steps):
        ext.device_decode(x, opts, with_pool=True, with_weights=True)
    torch.cuda.synchronize()
    print(f"pool decode x{args.steps} done")


def constrained_batch4():
    """Config 4: steps, beams and the banned row of the 512-example
    constrained variable batch (seeded)."""
    import numpy as np
    rng = np.random.default_rng(4)
    B, maxT, V = 512, 128, 128256
    steps_all = rng.integers(8, maxT + 1, B).astype(np.int32)
    beams_all = rng.choice(np.array([1, 2, 4, 8, 16], np.int32), B).astype(np.int32)
    banned_row = np.zeros(V, np.uint8)
    banned_row[rng.choice(V, 256, replace=False)] = 1
    return steps_all, beams_all, banned_row


def run_config4(args, rank, world, local):
    """Config 4: the 512-example constrained variable batch (T_b in [8, 128],
    K_b in {1, 2, 4, 8, 16}, V = 128256; 256 banned ids, forced token 1 at
    step 0, minimum length 8 before EOS 2, repetition penalty 1.2, no
    repeated 3-gram) through dbs_device_decode_batch_variable_ex, in eight
    64-example slices of the padded [64, 128, 16, 128256] layout (67 GB
    each; the whole padded batch would be 538 GB). Each slice's log-probs
    are generated on the device, then its decode is timed --steps times
    with CUDA events; a step is one decode of every slice, so ms_per_step is
    the sum of the slices' mean times. The CPU arm is the reference
    library's dbs_decode_constrained_ex on a sample of slice 0's examples,
    16 at a time on host threads; its outputs are compared with this run's."""
    import numpy as np
    import torch
    import dbs_ctypes as dc
    import torch_dbs_extension as ext
    if world > 1:
        raise SystemExit("--config 4 runs on one GPU (its slices would split by examples like config 3)")
    steps_all, beams_all, banned_row = constrained_batch4()
    B, maxT, maxK, V, SL = 512, 128, 16, 128256, 64
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    lib = ext._library()
    opts = ext.DBSOptions(beam_size=maxK, eos_token=2, min_length=8)
    h = ext._handle(opts)
    n_ref = 0 if args.no_cpu_baseline else min(args.ref_sample, SL)
    elems = int((steps_all.astype(np.int64) * beams_all).sum()) * V
    alg = int(((steps_all.astype(np.int64) * beams_all) - (beams_all - 1)).sum()) * V * 4
    slice_ms, scan_ms, launches, t_gen = [], [], 0, 0.0
    sample = None
    uuid = str(torch.cuda.get_device_properties(dev).uuid)
    sampler = ClockSampler(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
    for s0 in range(0, B, SL):
        steps = np.ascontiguousarray(steps_all[s0:s0 + SL])
        beams = np.ascontiguousarray(beams_all[s0:s0 + SL])
        nb = len(steps)
        t0 = time.perf_counter()
        x = torch.zeros((nb, maxT, maxK, V), dtype=torch.float32, device=dev)
        g = torch.Generator(device=dev)
        for b in range(nb):
            g.manual_seed(4 * 1_000_003 + s0 + b)
            T, K = int(steps[b]), int(beams[b])
            z = torch.empty((T, K, V), device=dev)
            z.normal_(generator=g)
            x[b, :T, :K] = torch.log_softmax(1.5 * z, dim=-1)
            del z
        eos = np.full(nb, 2, np.int32)
        minl = np.full(nb, 8, np.int32)
        banned = torch.tensor(np.tile(banned_row, (nb, 1)), device=dev)
        forced_np = np.full((nb, maxT), -1, np.int32)
        forced_np[:, 0] = 1
        forced = torch.tensor(forced_np, device=dev)
        torch.cuda.synchronize()
        t_gen += time.perf_counter() - t0
        sel = int((steps.astype(np.int64) * beams).sum())
        fin = int(beams.sum())
        sel_names = ("parents", "tokens", "lengths", "from_logprob", "raw_scores", "scores", "weights")
        out = {}
        so = dc.DBSDeviceDecodeOutputs()
        for name, _ in dc.DBSDeviceDecodeOutputs._fields_:
            n = sel if name in sel_names else (fin if name.startswith("final") else 8 * sel)
            dt = torch.uint8 if "from_logprob" in name else (
                torch.int32 if name.split("_")[-1] in ("parents", "tokens", "lengths") else torch.float32)
            out[name] = torch.empty(n, dtype=dt, device=dev)
            setattr(so, name, out[name].data_ptr())

        def step():
            rc = lib.dbs_device_decode_batch_variable_ex(
                h, ext._vp(x), nb, maxT, maxK, V, steps.ctypes.data_as(ctypes.c_void_p),
                beams.ctypes.data_as(ctypes.c_void_p), eos.ctypes.data_as(ctypes.c_void_p),
                minl.ctypes.data_as(ctypes.c_void_p), ext._vp(banned), ext._vp(forced), ctypes.c_float(1.2), 3,
                ctypes.byref(so), ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
            if rc != 0:
                raise RuntimeError("dbs_device_decode_batch_variable_ex: " + lib.dbs_last_error(h).decode())

        for _ in range(max(3, args.warmup) if s0 == 0 else 1):
            step()
        torch.cuda.synchronize()
        if s0 == 0:
            sampler.start()
            time.sleep(0.3)
        lib.dbs_device_profile(-1)
        lib.dbs_device_profile_kernels(1 << dbs_ctypes_index(dc, "row_scan"))
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        n0 = kernel_launches(lib)
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
        launches += kernel_launches(lib) - n0
        lib.dbs_device_profile(0)
        slice_ms.append(e0.elapsed_time(e1) / args.steps)
        scan_ms.append(read_profile(lib, dc)["row_scan"]["total_ms"] / args.steps)
        if s0 == 0 and n_ref:
            # this run's results for the CPU arm's sample
            sel_off = np.concatenate([[0], np.cumsum(steps.astype(np.int64) * beams)])
            fin_off = np.concatenate([[0], np.cumsum(beams.astype(np.int64))])
            tok = out["tokens"].cpu().numpy()
            fs = out["final_scores"].cpu().numpy()
            sample = []
            for b in range(n_ref):
                T, K = int(steps[b]), int(beams[b])
                sample.append({"x": np.ascontiguousarray(x[b, :T, :K].cpu().numpy()), "T": T, "K": K,
                               "tokens": tok[sel_off[b]:sel_off[b + 1]].copy(),
                               "final": fs[fin_off[b]:fin_off[b + 1]].copy()})
        del x, banned, forced, out
        torch.cuda.empty_cache()
    clocks = sampler.stop()
    ms = float(sum(slice_ms))
    rs = float(sum(scan_ms))
    peak, peak_kind = measured_peaks()
    achieved = alg / (rs / 1e3) / 1e9 if rs > 0 else None
    cpu, parity = None, "not run: no CPU baseline requested" if not n_ref else None
    if n_ref:
        r = reference_run4(sample, banned_row, V)
        if r is None:
            parity = "not run: the reference library is not built"
        else:
            cpu = {"value": r[0], "unit": "elem/s", "cores": r[1], "kind": "reference", "sample": r[2]}
            bad = [b for b, (want, got) in enumerate(zip(r[3], sample))
                   if not (np.array_equal(want["tokens"], got["tokens"]) and
                           np.array_equal(want["final"], got["final"]))]
            parity = (f"ok: {n_ref} examples identical to the reference library (tokens, final scores)" if not bad
                      else f"MISMATCH in examples {bad}")
    line = {
        "metric": METRIC4, "value": elems / (ms / 1e3),
        "unit": "elem/s", "n_gpus": 1, "steps": args.steps, "warmup": max(3, args.warmup),
        "ms_per_step": ms, "higher_is_better": True, "scaling": "none (one GPU)", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic: log_softmax(1.5 N(0,1)) over V per live row, generated on the device (seeded)",
        "config": {"workload": "dbs_device_decode_batch_variable_ex, B=512 T_b in [8,128] K_b in {1,2,4,8,16} "
                               "V=128256, 256 banned ids, forced token 1 at step 0, min length 8 before EOS 2, "
                               "repetition penalty 1.2, no repeated 3-gram", "global_batch": 512, "seq_len": 128,
                   "vocab": V, "slices": "8 x 64 examples, padded [64,128,16,128256] (67 GB each), decodes timed "
                                          "per slice with the slice resident",
                   "l2": "inputs larger than L2; no flush needed"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": (achieved / peak) if achieved else None, "traffic": None, "peak_kind": peak_kind,
                     "kernel": "row_scan_kernel", "algorithmic_bytes_per_launch": alg,
                     "unit_of_launch": "all eight slices' row scans", "avg_launch_ms": rs},
        "cpu_baseline": cpu, "parity": parity,
        "e2e": {"value": None, "unit": "elem/s", "h2d_bytes_per_step": None, "d2h_bytes_per_step": None,
                "note": "not measured: the padded host layout of the batch is 538 GB"},
        "gpu_launches": launches, "slice_ms": slice_ms, "clocks": clocks, "input_generation_s": t_gen,
    }
    print(json.dumps(line), flush=True)


def dbs_ctypes_index(dc, name):
    return dc.PROFILED_KERNELS.index(name)


def reference_run4(sample, banned_row, V, budget_s=10.0):
    """Config 4's CPU arm: the reference library's dbs_decode_constrained_ex
    per example (src/differentiable_beam.cpp:3438-3482), the sample's
    examples 16 at a time on host threads (the call takes one example).
    Returns (elems/s, threads, sample text, outputs) or None when the
    reference library is not built."""
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import dbs_ctypes as dc
    from oracle import reference_library_path
    path = reference_library_path()
    if not path or not os.path.exists(path):
        return None
    lib = dc.load_library(path, device_api=False)
    threads = min(16, os.cpu_count() or 1)
    decs = {}
    for ex in sample:
        if ex["K"] not in decs:
            decs[ex["K"]] = [dc.Decoder(lib, dc.Options(beam_size=ex["K"], eos_token=2, min_length=8))
                             for _ in range(threads)]

    def one(i):
        ex = sample[i]
        dec = decs[ex["K"]][i % threads]
        forced = np.full(ex["T"], -1, np.int32)
        forced[0] = 1
        r = dec.decode_constrained_ex(ex["x"], ex["T"], V, banned=banned_row, forced=forced, min_length=8,
                                      repetition_penalty=1.2, no_repeat_ngram_size=3)
        res = dc.read_result(lib, r)
        lib.dbs_free_result(r)
        return {"tokens": res["tokens"].ravel(), "final": res["final_scores"].ravel()}

    outs = None
    reps = 0
    t0 = time.perf_counter()
    with ThreadPoolExecutor(max_workers=threads) as pool:
        while True:
            outs = list(pool.map(one, range(len(sample))))
            reps += 1
            if time.perf_counter() - t0 >= budget_s or reps >= 20:
                break
    dt = time.perf_counter() - t0
    el = sum(ex["T"] * ex["K"] for ex in sample) * V * reps
    for ds in decs.values():
        for d in ds:
            d.close()
    return (el / dt, threads, f"{reps} x {len(sample)} examples of slice 0 via dbs_decode_constrained_ex "
                             f"({threads} host threads, one example per call)", outs)


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


# ---------------------------------------------------------------------------
# shared measurement helpers
# ---------------------------------------------------------------------------
def warm_up(step, args, world, device, sync_every, sync=None):
    """Run the warm-up steps: at least max(3, --warmup), then as many more as
    --warmup-seconds asks for, estimated from the first ones. Every rank runs
    the same number of steps (a step may hold a collective, so the ranks
    agree on the count, by one all-reduce after the fixed steps, before any
    rank runs more). `sync` waits for the device (default: CUDA). Returns
    the number of steps run."""
    import torch
    import torch.distributed as dist
    if sync is None:
        sync = torch.cuda.synchronize
    n_min = max(3, args.warmup)
    t0 = time.perf_counter()
    for i in range(n_min):
        step()
        if (i + 1) % sync_every == 0:
            sync()
    sync()
    elapsed = time.perf_counter() - t0
    extra = 0
    if elapsed < args.warmup_seconds:
        per_step = max(elapsed / n_min, 1e-6)
        extra = min(100000, int((args.warmup_seconds - elapsed) / per_step) + 1)
    if world > 1:
        t = torch.tensor([extra], dtype=torch.int64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        extra = int(t.item())
    for i in range(extra):
        step()
        if (i + 1) % sync_every == 0:
            sync()
    sync()
    return n_min + extra


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        v = d.get("hbm_gbs")
        if v is None:   # a nested layout: the first "hbm_gbs" one level down
            v = next((x["hbm_gbs"] for x in d.values() if isinstance(x, dict) and "hbm_gbs" in x), None)
        if v is not None and float(v) > 0:
            return float(v), "measured"
    except (OSError, ValueError, TypeError, AttributeError):
        pass
    return 6650.0, "fallback"


def ncu_traffic_per_launch(config):
    """DRAM bytes per row-scan launch (config 2) or per decode call's scan
    (config 3) from the committed ncu summary, if any."""
    name = "row_scan_config2.md" if config == 2 else "row_scan_config3.md"
    p = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(p):
        return None
    with open(p) as f:
        m = re.search(r"dram_bytes_per_launch:\s*([0-9.eE+]+)", f.read())
    return float(m.group(1)) if m else None


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


def kernel_launches(lib):
    """Kernel launches the library has queued so far in this process."""
    n = ctypes.c_int64()
    lib.dbs_device_kernel_launches(ctypes.byref(n))
    return n.value


def read_profile(lib, dbs_ctypes):
    out = {}
    for i, name in enumerate(dbs_ctypes.PROFILED_KERNELS):
        tot = ctypes.c_double()
        n = ctypes.c_int64()
        lib.dbs_device_profile_read(i, ctypes.byref(tot), ctypes.byref(n))
        out[name] = {"total_ms": tot.value, "launches": n.value}
    return out


# ---------------------------------------------------------------------------
# CPU arms (the reference's library; the oracle's C port when it is absent)
# ---------------------------------------------------------------------------
def reference_cpu_run(x_host, steps_budget_s=20.0):
    """Config 2: time the reference CPU library on the workload (all host threads).

    Mirrors the reference's CPU path for final_scores forward + backward:
    dbs_decode_batch over the batch, then per example the sparse backward of
    grad_final = ones and the scatter-add into a zero dense gradient
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
            np.add.at(grad[b], out["indices"], out["values"])
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
              f"dbs_backward + dense scatter-add; kernel={lib.dbs_selected_kernel_name().decode()}")
    return elems / dt, cores, "reference", sample


def _oracle_port_run(x, steps_budget_s):
    """The CPU restatement in oracle/ on one host thread, for when the reference
    library could not be built: per example the decode, the sparse backward of
    grad_final = ones and the scatter-add into a zero dense gradient. Returns
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
            np.add.at(grad[b], out["indices"], out["values"])
        del grad
        elems += B * T * K * V
        reps += 1
        if time.perf_counter() - t0 >= steps_budget_s or reps >= 50:
            break
    dt = time.perf_counter() - t0
    sample = (f"{reps} x full batch B={B},T={T},K={K},V={V} through the oracle's C restatement (1 thread) "
              f"+ sparse backward + dense scatter-add")
    return elems / dt, 1, "port", sample


def reference_run3(x_host, reps_min=1, budget_s=10.0, keep_outputs=False, options=None, threads=None):
    """Config 3: time the reference CPU library on a sample of examples.

    One repetition = dbs_decode_batch over the sample (all host threads) and
    per example dbs_backward(grad_final = e_0) with its sparse result read,
    the reference's C ABI route for this configuration
    (src/differentiable_beam.cpp:3588-3673, :3782-3798). Returns
    (elems/s, cores, kind, sample, outputs) where outputs (keep_outputs) holds
    the last repetition's decode and backward results per example; None when
    neither the reference library nor the oracle port is built. `threads`:
    dbs_decode_batch's thread count (default: every host core)."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import dbs_ctypes as dc
    from oracle import ORACLE_SO, OracleLib, reference_library_path
    n, T, K, V = x_host.shape
    x = np.ascontiguousarray(x_host)
    gf = np.zeros(K, dtype=np.float32)
    gf[0] = 1.0
    path = reference_library_path()
    outs = None
    reps = 0
    t0 = time.perf_counter()
    if path is not None:
        cores = threads or os.cpu_count() or 1
        lib = dc.load_library(path, device_api=False)
        dec = dc.Decoder(lib, dc.Options(**(options or OPTIONS3)))
        while True:
            br = dec.decode_batch(x, n, T, V, cores)
            cur = []
            for b in range(n):
                r = lib.dbs_batch_result_at(br, b)
                bw = dec.backward(r, None, None, gf, mode="default")
                bk = dc.read_backward(lib, bw, K=K)
                lib.dbs_free_backward(bw)
                if keep_outputs:
                    fwd = dc.read_result(lib, r)
                    fwd["backward"] = bk
                    cur.append(fwd)
            lib.dbs_free_batch_result(br)
            outs = cur
            reps += 1
            if reps >= reps_min and time.perf_counter() - t0 >= budget_s:
                break
        dt = time.perf_counter() - t0
        dec.close()
        kind = "reference"
        sample = (f"{reps} x {n} examples (T={T},K={K},V={V}) via dbs_decode_batch({cores} threads) + per-example "
                  f"dbs_backward(grad_final=e_0); kernel={lib.dbs_selected_kernel_name().decode()}")
    else:
        if not os.path.exists(ORACLE_SO):
            return None
        cores = 1
        ol = OracleLib()
        opts = ol.options(**(options or OPTIONS3))
        while True:
            cur = []
            for b in range(n):
                fwd = ol.decode(opts, x[b], T, V)
                bk = ol.backward_sparse(fwd, grad_final=gf)
                if keep_outputs:
                    fwd["backward"] = bk
                    cur.append(fwd)
            outs = cur
            reps += 1
            if reps >= reps_min and time.perf_counter() - t0 >= budget_s:
                break
        dt = time.perf_counter() - t0
        kind = "port"
        sample = (f"{reps} x {n} examples (T={T},K={K},V={V}) through the oracle's C restatement (1 thread) "
                  f"+ sparse backward(grad_final=e_0)")
    return reps * n * T * K * V / dt, cores, kind, sample, outs


def bench_config2(B, T, K, V, world):
    return {"workload": f"torch final_scores fwd + y.sum().backward(), B={B} T={T} K={K} V={V}, eos_token=2, "
                        "length_penalty_alpha=0.2, selected_temperature=0.7 (per GPU)",
            "global_batch": B * world, "seq_len": T, "beam_size": K, "vocab": V,
            "parallelism": f"batch-sharded x{world}, no data-path collective",
            "l2": f"inputs larger than L2 ({4 * B * T * K * V / 1e9:.1f} GB per GPU); no flush needed"}


def bench_config3(B, T, K, V, world, per_rank):
    return {"workload": f"C ABI device decode (pool P={8 * K} + weights) + sparse backward (grad_final=e_0), "
                        f"B={B} T={T} K={K} V={V}, log_softmax(N(0,1)), default options",
            "global_batch": B, "seq_len": T, "beam_size": K, "vocab": V, "examples_per_gpu": per_rank,
            "parallelism": (f"batch split {per_rank} examples x {world} ranks; NCCL all-gather of final scores, "
                            f"tokens, parents and sparse gradients each step" if world > 1 else
                            "one GPU, whole batch"),
            "l2": f"inputs larger than L2 ({4 * per_rank * T * K * V / 1e9:.1f} GB per GPU); no flush needed"}


def bench_config1(B, T, K, V):
    return {"workload": f"C ABI device decode (pool P={8 * K} + weights) + sparse backward (grad_final=e_0), "
                        f"B={B} T={T} K={K} V={V}, log_softmax(1.5 N(0,1)) (CPU generator, seed 0), default options",
            "global_batch": B, "seq_len": T, "beam_size": K, "vocab": V, "examples_per_gpu": B,
            "parallelism": "one GPU",
            "l2": (f"inputs smaller than L2 ({4 * B * T * K * V / 1e6:.1f} MB): a 256 MB buffer is written "
                   "between timed steps, outside each step's event pair")}


def bench_config5(T, K, V):
    return {"workload": f"C ABI device decode (pool P={8 * K} + weights) + sparse backward (grad_final=e_0), "
                        f"B=1 T={T} K={K} V={V}, log_softmax(N(0,1) + 8 on 64 ids per step), default options",
            "global_batch": 1, "seq_len": T, "beam_size": K, "vocab": V, "examples_per_gpu": 1,
            "parallelism": "one GPU",
            "l2": f"inputs larger than L2 ({4 * T * K * V / 1e9:.1f} GB); no flush needed"}


def bench_bytes_bound(B, T, K, V):
    """Algorithmic bytes of one decode call's row scan: every live row once."""
    return 4.0 * B * (T * K - (K - 1)) * V


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------
def run_reference_arm(args, rank, world):
    """The reference's own CPU implementation of the path on the host cores.

    Config 3: one step = the reference library on a seeded sample of
    --ref-sample examples (dbs_decode_batch with all host threads + per-example
    dbs_backward). Config 2: one full batch (decode + sparse backward + dense
    scatter, all host threads). Config 4: dbs_decode_constrained_ex on a
    sample of the constrained batch's first examples (16 host threads).
    Config 5: the one example, decode + sparse backward. Config 1: twenty
    repetitions of its four examples per step (dbs_decode_batch with all
    host threads + per-example dbs_backward). Rank 0 alone runs and prints."""
    if rank != 0:
        return
    import torch
    if args.config == 2:
        B, T, K, V = (WORKLOAD[k] for k in "BTKV")
        # the GPU arm's recipe on the CPU generator (same distribution; the CUDA
        # generator's stream differs)
        x = make_inputs(torch, B, T, K, V, 0, "cpu").numpy()
        vals, res = [], None
        for i in range(max(3, args.warmup) + args.steps):
            res = reference_cpu_run(x, steps_budget_s=0.0)
            if res is None:
                print(json.dumps({"impl": "reference", "unavailable":
                                  "neither oracle/_ref/libdbs_ref.so nor the oracle port was built"}))
                return
            if i >= max(3, args.warmup):
                vals.append(res[0])
        value = statistics.median(vals)
        elems = B * T * K * V
        config = bench_config2(B, T, K, V, 1)
        data = "synthetic: 2*N(0,1) logits + Zipf bias -1.1*ln(v+1), log_softmax over V (CPU generator)"
        scaling = "weak"
    elif args.config == 4:
        steps_all, beams_all, banned_row = constrained_batch4()
        V = 128256
        n = max(1, min(64, args.ref_sample))
        g = torch.Generator()
        sample = []
        for b in range(n):
            g.manual_seed(4 * 1_000_003 + b)
            T, K = int(steps_all[b]), int(beams_all[b])
            z = torch.empty((T, K, V)).normal_(generator=g)
            sample.append({"x": torch.log_softmax(1.5 * z, dim=-1).numpy(), "T": T, "K": K})
        vals, res = [], None
        for i in range(max(3, args.warmup) + args.steps):
            r = reference_run4(sample, banned_row, V, budget_s=0.0)
            if r is None:
                print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libdbs_ref.so was not built"}))
                return
            res = (r[0], r[1], "reference", r[2])
            if i >= max(3, args.warmup):
                vals.append(r[0])
        value = statistics.median(vals)
        elems = int(sum(ex["T"] * ex["K"] for ex in sample)) * V
        config = {"workload": "dbs_decode_constrained_ex per example, constrained variable batch (B=512, "
                              "T_b in [8,128], K_b in {1,2,4,8,16}, V=128256)", "global_batch": 512, "seq_len": 128,
                  "vocab": V, "sample": f"the first {n} examples"}
        data = "synthetic: log_softmax(1.5 N(0,1)) over V (CPU generator), seeded per example"
        scaling = "none (one GPU)"
    elif args.config == 1:
        B, T, K, V = (WORKLOAD1[k] for k in "BTKV")
        x = make_inputs1(torch, "cpu").numpy()
        reps = 20
        vals, res = [], None
        for i in range(max(3, args.warmup) + args.steps):
            res = reference_run3(x, reps_min=reps, budget_s=0.0, options=OPTIONS1)
            if res is None:
                print(json.dumps({"impl": "reference", "unavailable":
                                  "neither oracle/_ref/libdbs_ref.so nor the oracle port was built"}))
                return
            if i >= max(3, args.warmup):
                vals.append(res[0])
        value = statistics.median(vals)
        elems = reps * B * T * K * V
        config = bench_config1(B, T, K, V)
        data = "synthetic: log_softmax(1.5 N(0,1)) over V (CPU generator, seed 0)"
        scaling = "none (one GPU)"
    elif args.config == 5:
        T, K, V = (WORKLOAD5[k] for k in "TKV")
        x = make_inputs5(torch, T, K, V, "cpu").numpy()
        vals, res = [], None
        for i in range(max(3, args.warmup) + args.steps):
            res = reference_run3(x, reps_min=1, budget_s=0.0, options=OPTIONS5)
            if res is None:
                print(json.dumps({"impl": "reference", "unavailable":
                                  "neither oracle/_ref/libdbs_ref.so nor the oracle port was built"}))
                return
            if i >= max(3, args.warmup):
                vals.append(res[0])
        value = statistics.median(vals)
        elems = T * K * V
        config = {"workload": "one example, decode (pool) + sparse backward", "global_batch": 1, "seq_len": T,
                  "beam_size": K, "vocab": V}
        data = "synthetic: log_softmax(N(0,1)) + 8 on 64 seeded ids per step (CPU generator)"
        scaling = "none (one GPU)"
    else:
        B, T, K, V = (WORKLOAD3[k] for k in "BTKV")
        n = max(1, min(B, args.ref_sample))
        x = make_inputs3(torch, n, T, K, V, 0, "cpu").numpy()
        vals, res = [], None
        for i in range(max(3, args.warmup) + args.steps):
            res = reference_run3(x, reps_min=1, budget_s=0.0)
            if res is None:
                print(json.dumps({"impl": "reference", "unavailable":
                                  "neither oracle/_ref/libdbs_ref.so nor the oracle port was built"}))
                return
            if i >= max(3, args.warmup):
                vals.append(res[0])
        value = statistics.median(vals)
        elems = n * T * K * V
        config = bench_config3(B, T, K, V, 1, B)
        data = "synthetic: log_softmax(N(0,1)) over V (CPU generator), seeded per example"
        scaling = "strong"
    kind = res[2]
    line = {
        "impl": "reference", "kind": kind, "metric": METRIC4 if args.config == 4 else METRIC, "value": value,
        "unit": "elem/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * elems / value, "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None, "dtype": "f32", "data": data, "config": config,
        "cpu_baseline": {"value": value, "unit": "elem/s", "cores": res[1], "kind": kind,
                         "sample": res[3] + "; median over steps"},
        "e2e": {"value": value, "unit": "elem/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if kind == "port":
        line["note"] = ("the reference library is not built here: this is the oracle's one-thread C restatement, "
                        "not the reference's multi-threaded library")
    print(json.dumps(line))


# ---------------------------------------------------------------------------
# config 3: device decode + sparse backward, strong-scaled, all-gather
# ---------------------------------------------------------------------------
def compare_with_reference(ours, ref, label):
    """Our device results for one example against the reference library's:
    ints and scores bit-exact, weights within the reference's own SIMD
    tolerances (3e-3 / 5e-3), sparse indices exact and values within 1e-5
    relative. Returns None when they agree, else the first difference."""
    import numpy as np
    for f in ("parents", "tokens", "lengths", "pool_parents", "pool_tokens", "pool_lengths"):
        if not np.array_equal(ours[f], ref[f]):
            return f"{label} {f} differs"
    for f in ("raw_scores", "scores", "pool_raw_scores", "pool_scores", "final_scores", "final_raw_scores"):
        g, w = ours[f], ref[f]
        if not (((g == w) | (np.isnan(g) & np.isnan(w))).all()):
            return f"{label} {f} differs"
    for f, tol in (("weights", 3e-3), ("relaxed_weights", 5e-3)):
        if float(np.max(np.abs(ours[f] - ref[f]))) > tol:
            return f"{label} {f} beyond {tol}"
    rb = ref["backward"]
    if not np.array_equal(ours["sparse_indices"], rb["indices"]):
        return f"{label} sparse indices differ"
    for a, b, name in ((ours["sparse_values"], rb["values"], "sparse values"),
                       (ours["grad_initial"], rb["grad_initial"], "grad_initial")):
        a = np.asarray(a, np.float64)
        b = np.asarray(b, np.float64)
        if not (np.abs(a - b) <= 1e-5 * np.maximum(np.abs(b), 1.0)).all():
            return f"{label} {name} beyond 1e-5"
    return None


def run_config3(args, rank, world, local):
    """Configs 3, 5 and 1: device decode (pool + weights) + sparse backward of
    grad_final = e_0 through the C ABI's device entry points; config 3's
    batch is split over the ranks with an all-gather of the results. Config
    1's inputs fit in L2, so L2 is flushed before each timed step."""
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

    five = args.config == 5
    one = args.config == 1
    W, O = (WORKLOAD5, OPTIONS5) if five else (WORKLOAD1, OPTIONS1) if one else (WORKLOAD3, OPTIONS3)
    Bg, T, K, V = (W[k] for k in "BTKV")
    if Bg % world:
        raise SystemExit(f"the {Bg}-example batch does not split over {world} ranks")
    Bl = args.batch or Bg // world
    first = rank * Bl
    P = 8 * K
    elems = Bl * T * K * V
    opts = ext.DBSOptions(**O)
    lib = ext._library()
    h = ext._handle(opts)

    t_gen = time.perf_counter()
    if five:
        x = make_inputs5(torch, T, K, V, device)
    elif one:
        x = make_inputs1(torch, device)
    else:
        x = make_inputs3(torch, Bl, T, K, V, first, device)
    torch.cuda.synchronize()
    t_gen = time.perf_counter() - t_gen

    # device outputs; final scores, tokens and parents live in one byte
    # packet with the sparse counts and entries, which the all-gather moves
    i32 = dict(dtype=torch.int32, device=device)
    f32 = dict(dtype=torch.float32, device=device)
    SK = T * K   # sparse entries gathered per example (grad_final only: at most K per step)
    sizes = [("final_scores", 4 * Bl * K), ("tokens", 4 * Bl * T * K), ("parents", 4 * Bl * T * K),
             ("sparse_counts", 8 * Bl), ("sparse_indices", 8 * Bl * SK), ("sparse_values", 4 * Bl * SK)]
    offs, off = {}, 0
    for name, nb in sizes:
        off = (off + 15) & ~15
        offs[name] = (off, nb)
        off += nb
    packet = torch.zeros(off, dtype=torch.uint8, device=device)

    def pk(name, dtype):
        o, nb = offs[name]
        return packet[o:o + nb].view(dtype)

    fin = pk("final_scores", torch.float32)
    tok = pk("tokens", torch.int32)
    par = pk("parents", torch.int32)
    cnt = pk("sparse_counts", torch.int64)
    pk_idx = pk("sparse_indices", torch.int64).view(Bl, SK)
    pk_val = pk("sparse_values", torch.float32).view(Bl, SK)
    trace = dict(
        parents=par, tokens=tok, lengths=torch.empty(Bl * T * K, **i32),
        from_logprob=torch.empty(Bl * T * K, dtype=torch.uint8, device=device),
        raw_scores=torch.empty(Bl * T * K, **f32), scores=torch.empty(Bl * T * K, **f32),
        weights=torch.empty(Bl * T * K, **f32),
        pool_parents=torch.empty(Bl * T * P, **i32), pool_tokens=torch.empty(Bl * T * P, **i32),
        pool_lengths=torch.empty(Bl * T * P, **i32),
        pool_from_logprob=torch.empty(Bl * T * P, dtype=torch.uint8, device=device),
        pool_raw_scores=torch.empty(Bl * T * P, **f32), pool_scores=torch.empty(Bl * T * P, **f32),
        relaxed_weights=torch.empty(Bl * T * P, **f32),
        final_raw_scores=torch.empty(Bl * K, **f32), final_scores=fin)
    outs = dbs_ctypes.DBSDeviceDecodeOutputs()
    for name, _ in dbs_ctypes.DBSDeviceDecodeOutputs._fields_:
        setattr(outs, name, trace[name].data_ptr())
    cap = T * (K + P)
    sp_idx = torch.empty((Bl, cap), dtype=torch.int64, device=device)
    sp_val = torch.empty((Bl, cap), **f32)
    gfin = torch.zeros((Bl, K), **f32)
    gfin[:, 0] = 1.0
    ginit = torch.empty((Bl, K), **f32)
    gathered = torch.empty(world * off, dtype=torch.uint8, device=device) if world > 1 else None

    def stream_ptr():
        return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)

    def step():
        s = stream_ptr()
        rc = lib.dbs_device_decode_batch(h, ext._vp(x), Bl, T, V, ctypes.byref(outs), s)
        if rc != 0:
            raise RuntimeError("dbs_device_decode_batch: " + lib.dbs_last_error(h).decode())
        rc = lib.dbs_device_backward_batch(h, Bl, T, V, ctypes.byref(outs), None, None, ext._vp(gfin), None,
                                           ext._vp(sp_idx), ext._vp(sp_val), ext._vp(cnt), ext._vp(ginit), s)
        if rc != 0:
            raise RuntimeError("dbs_device_backward_batch: " + lib.dbs_last_error(h).decode())
        if world > 1:
            pk_idx.copy_(sp_idx[:, :SK])
            pk_val.copy_(sp_val[:, :SK])
            dist.all_gather_into_tensor(gathered, packet)

    warm_steps = warm_up(step, args, world, device, 20)
    # the gathered counts bound the gathered entries (grad_final only)
    if world > 1:
        gc = torch.stack([gathered[r * off + offs["sparse_counts"][0]:
                                   r * off + offs["sparse_counts"][0] + 8 * Bl].view(torch.int64)
                          for r in range(world)])
        assert int(gc.max().item()) <= SK, "sparse entries beyond the gathered bound"
        assert torch.equal(gathered[rank * off:(rank + 1) * off], packet), "all-gather lost this rank's results"
    else:
        assert int(cnt.max().item()) <= SK

    uuid = str(torch.cuda.get_device_properties(device).uuid)
    sampler = ClockSampler(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
    sampler.start()
    time.sleep(0.3)
    lib.dbs_device_profile(-1)
    lib.dbs_device_profile_kernels(1 << dbs_ctypes.PROFILED_KERNELS.index("row_scan"))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    n_launch0 = kernel_launches(lib)
    if not one:
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            step()
        end.record()
        torch.cuda.synchronize()
    else:
        # inputs smaller than L2: a 256 MB write before each step evicts them,
        # and each step is timed by its own event pair (the write is outside)
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
        pairs = []
        for i in range(args.steps):
            flush.fill_(i & 0xFF)
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            step()
            b.record()
            pairs.append((a, b))
        torch.cuda.synchronize()
    launches = kernel_launches(lib) - n_launch0
    if world > 1:
        dist.barrier()
    lib.dbs_device_profile(0)
    clocks = sampler.stop()
    ms = start.elapsed_time(end) if not one else sum(a.elapsed_time(b) for a, b in pairs)
    rs = read_profile(lib, dbs_ctypes)["row_scan"]

    # per-kernel breakdown from a short separate pass with every kernel timed
    prof_steps = min(args.steps, 5)
    lib.dbs_device_profile(-1)
    lib.dbs_device_profile(1)
    for _ in range(prof_steps):
        step()
    torch.cuda.synchronize()
    lib.dbs_device_profile(0)
    kern = read_profile(lib, dbs_ctypes)
    for v in kern.values():
        v["avg_ms"] = v["total_ms"] / v["launches"] if v["launches"] else None
        v["launches_per_step"] = v["launches"] / prof_steps
    t = torch.tensor([ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    ms_per_step = ms_max / args.steps
    value = world * elems / (ms_per_step / 1e3)

    peak, peak_kind = measured_peaks()
    rs_ms = rs["total_ms"] / max(1, rs["launches"])
    alg_bytes = bench_bytes_bound(Bl, T, K, V)
    achieved = alg_bytes / (rs_ms / 1e3) / 1e9 if rs_ms > 0 else None
    traffic = ncu_traffic_per_launch(3) if not (five or one) else None
    if traffic is not None and args.batch is None:
        traffic = traffic * Bl / 32.0   # the committed capture covers 32 examples
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": (achieved / peak) if achieved else None, "traffic": traffic,
                "peak_kind": peak_kind, "kernel": "row_scan_kernel",
                "unit_of_launch": "one decode call's row scan (all its row-scan launches, one event pair)",
                "algorithmic_bytes_per_launch": alg_bytes, "avg_launch_ms": rs_ms}
    whole = {"achieved_gbs": alg_bytes / (ms_per_step / 1e3) / 1e9,
             "frac": alg_bytes / (ms_per_step / 1e3) / 1e9 / peak}
    rescans = (ctypes.c_int64(), ctypes.c_int64())
    lib.dbs_device_last_rescan_counts(h, ctypes.byref(rescans[0]), ctypes.byref(rescans[1]))

    # results of this rank's sample examples, for the parity check below
    n_ref = max(1, min(Bl, args.ref_sample))
    want_cpu = rank == 0 and world == 1 and not args.no_cpu_baseline
    ours = None
    x_sample = None
    if want_cpu:
        step()
        torch.cuda.synchronize()
        def host(name, shape):
            return trace[name].view(Bl, *shape)[:n_ref].cpu().numpy()
        ours = []
        for b in range(n_ref):
            d = {}
            for name in ("parents", "tokens", "lengths", "raw_scores", "scores", "weights"):
                d[name] = trace[name].view(Bl, T * K)[b].cpu().numpy()
            for name in ("pool_parents", "pool_tokens", "pool_lengths", "pool_raw_scores", "pool_scores",
                         "relaxed_weights"):
                d[name] = trace[name].view(Bl, T * P)[b].cpu().numpy()
            for name in ("final_scores", "final_raw_scores"):
                d[name] = trace[name].view(Bl, K)[b].cpu().numpy()
            c = int(cnt[b].item())
            d["sparse_indices"] = sp_idx[b, :c].cpu().numpy()
            d["sparse_values"] = sp_val[b, :c].cpu().numpy()
            d["grad_initial"] = ginit[b].cpu().numpy()
            ours.append(d)
        x_sample = x[:n_ref].cpu().numpy()

    # end to end through the C ABI with host buffers: dbs_decode_batch on
    # pinned host log-probs (the library stages them to the device inside the
    # call), dbs_backward per example, every result read on the host
    e2e_steps = args.e2e_steps if args.e2e_steps is not None else (20 if one else 2)
    x_host = torch.empty((Bl if e2e_steps > 0 else 1, T, K, V), dtype=torch.float32, pin_memory=True)
    if e2e_steps > 0:
        for b0 in range(0, Bl, 16):
            x_host[b0:b0 + 16].copy_(x[b0:b0 + 16])
    del x
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    import dbs_ctypes as dc
    gf_host = np.zeros(K, dtype=np.float32)
    gf_host[0] = 1.0
    dec = dc.Decoder(lib, dc.Options(**O))
    xh = x_host.numpy()
    nnz_total = [0]
    split_s = [0.0, 0.0]   # host time in dbs_decode_batch, in the backward calls

    def e2e_step():
        t0 = time.perf_counter()
        br = dec.decode_batch(xh, Bl, T, V, 0)
        t1 = time.perf_counter()
        nnz = 0
        fs = []
        for b in range(Bl):
            r = lib.dbs_batch_result_at(br, b)
            bw = dec.backward(r, None, None, gf_host, mode="default")
            nnz += lib.dbs_backward_sparse_logprob_count(bw)
            fs.append(lib.dbs_result_final_scores(r))
            lib.dbs_free_backward(bw)
        lib.dbs_free_batch_result(br)
        split_s[0] += t1 - t0
        split_s[1] += time.perf_counter() - t1
        nnz_total[0] = nnz

    e2e_ms = float("nan")
    if e2e_steps > 0:   # (0: profiling runs without the end-to-end part)
        e2e_step()   # warm-up: the library's staging pools
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        split_s[0] = split_s[1] = 0.0
        e0 = time.perf_counter()
        for _ in range(e2e_steps):
            e2e_step()
        torch.cuda.synchronize()
        e2e_s = time.perf_counter() - e0
        te = torch.tensor([e2e_s], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_ms = float(te.item()) * 1e3 / e2e_steps
    dec.close()
    # bytes the library moves per step: the log-probs, and for each
    # example's backward the trace it stages (parents, tokens, lengths,
    # from_logprob) and grad_final; back: every decode result array
    # (selected 6 x 4 B + 1 B per [T,K] entry, pool likewise per [T,P],
    # 2 x 4 B per beam of finals), grad_initial, the count and the entries
    h2d = 4 * Bl * T * K * V + Bl * (13 * T * K + 4 * K)
    d2h = Bl * (25 * T * K + 25 * T * P + 8 * K) + Bl * (4 * K + 8) + 12 * nnz_total[0]
    e2e = {"value": world * elems / (e2e_ms / 1e3), "unit": "elem/s", "h2d_bytes_per_step": h2d,
           "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
           "path": "dbs_decode_batch(pinned host log-probs) + dbs_backward per example, results read on the host",
           "timing": "host wall clock around the steps (the calls synchronise), max over ranks",
           "rank0_decode_ms_per_step": split_s[0] * 1e3 / max(1, e2e_steps),
           "rank0_backward_ms_per_step": split_s[1] * 1e3 / max(1, e2e_steps)}

    cpu = None
    parity = "not run: the CPU baseline leg runs on rank 0 at one GPU only" if not want_cpu else None
    if want_cpu:
        r = reference_run3(x_sample, reps_min=1, budget_s=10.0, keep_outputs=True, options=O)
        if r is None:
            parity = "not run: neither the reference library nor the oracle is built"
        else:
            cpu = {"value": r[0], "unit": "elem/s", "cores": r[1], "kind": r[2], "sample": r[3]}
            if one and r[2] == "reference":   # the small case also on one host thread
                r1 = reference_run3(x_sample, reps_min=1, budget_s=5.0, options=O, threads=1)
                cpu["one_thread"] = {"value": r1[0], "unit": "elem/s", "cores": 1, "sample": r1[3]}
            bad = None
            for b in range(n_ref):
                bad = compare_with_reference(ours[b], r[4][b], f"example {first + b}")
                if bad:
                    break
            who = "reference library" if r[2] == "reference" else "oracle port"
            parity = (f"ok: {n_ref} examples identical to the {who} (ints, scores, sparse indices exact; "
                      f"weights within 3e-3/5e-3; gradients within 1e-5)") if bad is None else f"FAILED: {bad}"

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": value, "unit": "elem/s", "n_gpus": world, "steps": args.steps,
        "warmup": warm_steps, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32",
        "data": ("synthetic: log_softmax(N(0,1) + 8 on 64 seeded ids per step) over V, generated on the device"
                 if five else "synthetic: log_softmax(1.5 N(0,1)) over V (CPU generator, seed 0), copied to the device"
                 if one else "synthetic: log_softmax(N(0,1)) over V, generated on the device per example (seeded)"),
        "config": (bench_config5(T, K, V) if five else bench_config1(Bg, T, K, V) if one
                   else bench_config3(Bg, T, K, V, world, Bl)),
        "roofline": roofline,
        "step_hbm": whole,
        "cpu_baseline": cpu,
        "parity": parity,
        "e2e": e2e,
        "gpu_launches": launches,
        "kernels": {"source": f"separate {prof_steps}-step pass, every kernel bracketed by events", **kern},
        "rescans": {"row_scan": rescans[0].value, "step_merge": rescans[1].value},
        "clocks": clocks,
        "input_generation_s": t_gen,
    }
    if args.batch is not None:
        line["profiling_override"] = f"--batch {args.batch}: not the configuration's split"
    print(json.dumps(line))


# ---------------------------------------------------------------------------
# config 2: torch final_scores autograd, weak scaling
# ---------------------------------------------------------------------------
def run_config2(args, rank, world, local):
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

    warm_steps = warm_up(step, args, world, device, 50)

    uuid = str(torch.cuda.get_device_properties(device).uuid)
    sampler = ClockSampler(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
    sampler.start()
    time.sleep(0.3)
    lib.dbs_device_profile(-1)
    lib.dbs_device_profile_kernels(1 << dbs_ctypes.PROFILED_KERNELS.index("row_scan"))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    n_launch0 = kernel_launches(lib)
    start.record()
    for _ in range(args.steps):
        step()
    end.record()
    torch.cuda.synchronize()
    launches = kernel_launches(lib) - n_launch0
    if world > 1:
        dist.barrier()
    lib.dbs_device_profile(0)
    clocks = sampler.stop()
    ms = start.elapsed_time(end)
    rs = read_profile(lib, dbs_ctypes)["row_scan"]
    prof_steps = min(args.steps, 20)
    lib.dbs_device_profile(-1)
    lib.dbs_device_profile(1)
    for _ in range(prof_steps):
        step()
    torch.cuda.synchronize()
    lib.dbs_device_profile(0)
    kern = read_profile(lib, dbs_ctypes)
    for v in kern.values():
        v["avg_ms"] = v["total_ms"] / v["launches"] if v["launches"] else None
        v["launches_per_step"] = v["launches"] / prof_steps
    t = torch.tensor([ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    ms_per_step = ms_max / args.steps
    value = world * elems / (ms_per_step / 1e3)

    peak, peak_kind = measured_peaks()
    rs_ms = rs["total_ms"] / max(1, rs["launches"])
    alg_bytes = bench_bytes_bound(B, T, K, V)
    achieved = alg_bytes / (rs_ms / 1e3) / 1e9 if rs_ms > 0 else None
    traffic = ncu_traffic_per_launch(2)
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
    e2e_steps = args.e2e_steps if args.e2e_steps is not None else 20
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
    e2e_run(e2e_steps, start=e0)
    e1.record()
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms = float(te.item()) / e2e_steps
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
        "config": bench_config2(B, T, K, V, world),
        "roofline": roofline,
        "step_hbm": whole,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": launches,
        "kernels": {"source": f"separate {prof_steps}-step pass, every kernel bracketed by events", **kern},
        "rescans": {"row_scan": rescans[0].value, "step_merge": rescans[1].value},
        "clocks": clocks,
    }
    if args.batch is not None:
        line["profiling_override"] = f"--batch {args.batch}: not the configuration's batch"
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
    if args.config == 2:
        run_config2(args, rank, world, local)
    elif args.config == 4:
        run_config4(args, rank, world, local)
    else:
        if args.config == 5 and world > 1:
            raise SystemExit("--config 5 runs on one GPU (its one example does not split by examples)")
        if args.config == 1 and world > 1:
            raise SystemExit("--config 1 runs on one GPU (four examples: a launch-bound parity case)")
        run_config3(args, rank, world, local)


if __name__ == "__main__":
    main()
