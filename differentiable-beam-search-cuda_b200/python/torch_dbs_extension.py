"""PyTorch interface of the B200 differentiable beam search.

Mirrors the reference's public tensor API (maged15/differentiable-beam-search-
cuda, python/torch_dbs_extension.py): `DBSOptions`, `final_scores` (autograd
Function over [T,K,V] -> [K] and [B,T,K,V] -> [B,K]) and `decode`, with the
same argument meaning, validation messages and error types. It also registers
`torch.ops.dbs.final_scores_forward / final_scores_backward` with the
reference's schemas (python/torch_extension.cpp:191-194).

Every forward and backward runs as sm_100a kernels through the device entry
points of lib/libdbs.so (include/dbs_device.h) on the current CUDA stream:
the forward saves the device trace (backpointers, tokens, lengths) and the
backward turns it into the dense gradient on the device -- no re-decode, no
host round trip. CPU tensors are moved to the current CUDA device and the
results moved back. There is no CPU implementation: without a CUDA device or
without the built library every call raises.
"""

from __future__ import annotations

import ctypes
import math
import threading
from dataclasses import dataclass, fields
from typing import Dict, Optional, Tuple

import torch

import dbs_ctypes

_INT_MAX = 2_147_483_647


@dataclass(frozen=True)
class DBSOptions:
    beam_size: int
    eos_token: int = -1
    selected_temperature: float = 1.0
    soft_topk_temperature: float = 0.25
    relaxed_pool_multiplier: int = 8
    vocab_block: int = 4096
    length_penalty_alpha: float = 0.0
    soft_topk_tolerance: float = 1.0e-4
    soft_topk_max_iters: int = 48
    min_length: int = 0
    validate_inputs: int = 1
    max_dense_gradient_elements: int = 100_000_000

    def args(self) -> Tuple[object, ...]:
        return tuple(getattr(self, f.name) for f in fields(self))


# ---------------------------------------------------------------------------
# Public validation (python/torch_dbs_extension.py:73-140 of the reference)
# ---------------------------------------------------------------------------
def _validate_positive_int_dim(value: int, name: str) -> None:
    if value <= 0:
        raise ValueError(f"{name} must be positive")
    if value > _INT_MAX:
        raise ValueError(f"{name} exceeds INT_MAX")


def _validate_finite_float(value: float, name: str) -> None:
    if not math.isfinite(float(value)):
        raise ValueError(f"{name} must be finite")


def _validate_public_options(options: DBSOptions) -> None:
    _validate_finite_float(options.selected_temperature, "selected_temperature")
    if not options.selected_temperature > 0.0:
        raise ValueError("selected_temperature must be positive")
    _validate_finite_float(options.soft_topk_temperature, "soft_topk_temperature")
    if not options.soft_topk_temperature > 0.0:
        raise ValueError("soft_topk_temperature must be positive")
    if options.relaxed_pool_multiplier <= 0:
        raise ValueError("relaxed_pool_multiplier must be positive")
    if options.vocab_block <= 0:
        raise ValueError("vocab_block must be positive")
    _validate_finite_float(options.length_penalty_alpha, "length_penalty_alpha")
    if options.length_penalty_alpha < 0.0:
        raise ValueError("length_penalty_alpha cannot be negative")
    _validate_finite_float(options.soft_topk_tolerance, "soft_topk_tolerance")
    if not options.soft_topk_tolerance > 0.0:
        raise ValueError("soft_topk_tolerance must be positive")
    if options.soft_topk_max_iters <= 0:
        raise ValueError("soft_topk_max_iters must be positive")
    if options.min_length < 0:
        raise ValueError("min_length cannot be negative")
    if options.validate_inputs not in (0, 1):
        raise ValueError("validate_inputs must be 0 or 1")
    if options.max_dense_gradient_elements <= 0:
        raise ValueError("max_dense_gradient_elements must be positive")


def _validate_eos_token(options: DBSOptions, vocab_size: int) -> None:
    if options.eos_token < -1:
        raise ValueError("eos_token must be -1 or non-negative")
    if options.eos_token >= vocab_size:
        raise ValueError(f"eos_token={options.eos_token} must be < vocab_size={vocab_size}")


def _validate_public_shape(log_probs: torch.Tensor, options: DBSOptions) -> bool:
    """Validate the public shape; True when the input is unbatched [T,K,V]."""
    _validate_positive_int_dim(options.beam_size, "beam_size")
    _validate_public_options(options)
    if log_probs.dim() == 3:
        _validate_positive_int_dim(log_probs.size(0), "T")
        _validate_positive_int_dim(log_probs.size(1), "K")
        _validate_positive_int_dim(log_probs.size(2), "V")
        if log_probs.size(1) != options.beam_size:
            raise ValueError(f"beam_size={options.beam_size} must equal log_probs.shape[1]={log_probs.size(1)}")
        _validate_eos_token(options, log_probs.size(2))
        return True
    if log_probs.dim() == 4:
        _validate_positive_int_dim(log_probs.size(0), "B")
        _validate_positive_int_dim(log_probs.size(1), "T")
        _validate_positive_int_dim(log_probs.size(2), "K")
        _validate_positive_int_dim(log_probs.size(3), "V")
        if log_probs.size(2) != options.beam_size:
            raise ValueError(f"beam_size={options.beam_size} must equal log_probs.shape[2]={log_probs.size(2)}")
        _validate_eos_token(options, log_probs.size(3))
        return False
    raise ValueError("log_probs must have shape [T,K,V] or [B,T,K,V]")


# ---------------------------------------------------------------------------
# Library and decoder handles
# ---------------------------------------------------------------------------
_LOCK = threading.Lock()
_LIB = None
_HANDLES: Dict[Tuple[object, ...], ctypes.c_void_p] = {}


def _library():
    global _LIB
    with _LOCK:
        if _LIB is None:
            _LIB = dbs_ctypes.load_library()
        return _LIB


def _handle(options: DBSOptions) -> ctypes.c_void_p:
    key = options.args()
    with _LOCK:
        h = _HANDLES.get(key)
    if h is not None:
        return h
    lib = _library()
    c = dbs_ctypes.Options(*options.args()).to_c()
    h = ctypes.c_void_p()
    rc = lib.dbs_create_ex(c, ctypes.byref(h))
    if rc != 0:
        raise RuntimeError(f"dbs_create_ex failed: {lib.dbs_last_global_error().decode()}")
    with _LOCK:
        _HANDLES.setdefault(key, h)
        return _HANDLES[key]


def _check(rc: int, h, what: str) -> None:
    if rc != 0:
        msg = _library().dbs_last_error(h).decode()
        raise RuntimeError(f"{what} failed" + (f": {msg}" if msg else ""))


def _cuda_device_for(t: torch.Tensor) -> torch.device:
    if t.is_cuda:
        return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("differentiable beam search runs on CUDA devices only; no CUDA device is available")
    return torch.device("cuda", torch.cuda.current_device())


def _vp(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream_ptr(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


class DeviceTrace:
    """Device arrays of one batched decode (tight [B,T,K] layout)."""

    def __init__(self, B: int, T: int, K: int, device: torch.device, with_pool: bool = False,
                 P: int = 0, with_weights: bool = False):
        i32 = dict(dtype=torch.int32, device=device)
        f32 = dict(dtype=torch.float32, device=device)
        self.parents = torch.empty((B, T, K), **i32)
        self.tokens = torch.empty((B, T, K), **i32)
        self.lengths = torch.empty((B, T, K), **i32)
        self.from_logprob = torch.empty((B, T, K), dtype=torch.uint8, device=device)
        self.raw_scores = torch.empty((B, T, K), **f32)
        self.scores = torch.empty((B, T, K), **f32)
        self.weights = torch.empty((B, T, K), **f32) if with_weights else None
        self.final_raw_scores = torch.empty((B, K), **f32)
        self.final_scores = torch.empty((B, K), **f32)
        if with_pool:
            self.pool_parents = torch.empty((B, T, P), **i32)
            self.pool_tokens = torch.empty((B, T, P), **i32)
            self.pool_lengths = torch.empty((B, T, P), **i32)
            self.pool_from_logprob = torch.empty((B, T, P), dtype=torch.uint8, device=device)
            self.pool_raw_scores = torch.empty((B, T, P), **f32)
            self.pool_scores = torch.empty((B, T, P), **f32)
            self.relaxed_weights = torch.empty((B, T, P), **f32)
        else:
            self.pool_parents = self.pool_tokens = self.pool_lengths = None
            self.pool_from_logprob = self.pool_raw_scores = self.pool_scores = self.relaxed_weights = None

    def struct(self) -> dbs_ctypes.DBSDeviceDecodeOutputs:
        s = dbs_ctypes.DBSDeviceDecodeOutputs()
        for name, _ in dbs_ctypes.DBSDeviceDecodeOutputs._fields_:
            t = getattr(self, name)
            setattr(s, name, None if t is None else t.data_ptr())
        return s


def device_decode(x4: torch.Tensor, options: DBSOptions, with_pool: bool = False,
                  with_weights: bool = False, zero_fill: Optional[torch.Tensor] = None) -> DeviceTrace:
    """Decode a contiguous fp32 CUDA tensor [B,T,K,V] on its device.

    `zero_fill`, when given, is a float32 tensor the call zeroes beside the
    step merge (the autograd path passes the gradient its backward fills).
    """
    B, T, K, V = (int(s) for s in x4.shape)
    P = max(K, K * options.relaxed_pool_multiplier)
    trace = DeviceTrace(B, T, K, x4.device, with_pool=with_pool, P=P, with_weights=with_weights)
    lib = _library()
    h = _handle(options)
    outs = trace.struct()
    zf = None if zero_fill is None else _vp(zero_fill)
    zn = 0 if zero_fill is None else int(zero_fill.numel())
    with torch.cuda.device(x4.device):
        rc = lib.dbs_device_decode_batch_ex(h, _vp(x4), B, T, V, ctypes.byref(outs), zf, zn, _stream_ptr(x4.device))
    _check(rc, h, "dbs_decode")
    return trace


def row_shards(rows: int, world: int):
    """Contiguous row ranges of a row-sharded decode: rank r scans
    [r * per, min(rows, (r + 1) * per)); every rank's range is padded to `per`
    rows so the all-gather moves equal chunks."""
    if world < 1:
        raise ValueError("world size must be positive")
    per = max(1, -(-rows // world))
    return per, [(min(rows, r * per), min(rows, (r + 1) * per)) for r in range(world)]


def decode_row_sharded(x4: torch.Tensor, options: DBSOptions, with_pool: bool = False, with_weights: bool = False,
                       group=None) -> DeviceTrace:
    """Decode a uniform batch whose log-probs every rank holds, with the row
    scan split across the ranks of `group` (NCCL): each rank scans its
    contiguous share of the B*T*K rows, one all-gather assembles every row's
    candidate list on every rank, and each rank runs the (sequential, small)
    step merge itself. Every rank returns the trace dbs_device_decode_batch
    would produce."""
    import torch.distributed as dist
    B, T, K, V = (int(s) for s in x4.shape)
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    lib = _library()
    h = _handle(options)
    cap = ctypes.c_int()
    _check(lib.dbs_device_row_list_capacity(h, 1 if with_pool else 0, ctypes.byref(cap)), h, "dbs_decode")
    C = int(cap.value)
    rows = B * T * K
    per, ranges = row_shards(rows, world)
    dev = x4.device
    lists = torch.empty((world * per, C), dtype=torch.int64, device=dev)
    counts = torch.empty((world * per,), dtype=torch.int32, device=dev)
    bounds = torch.empty((world * per,), dtype=torch.float32, device=dev)
    begin, end = ranges[rank]
    stream = _stream_ptr(dev)
    with torch.cuda.device(dev):
        rc = lib.dbs_device_scan_rows(h, _vp(x4), B, T, V, 1 if with_pool else 0, begin, end, _vp(lists), _vp(counts),
                                      _vp(bounds), stream)
    _check(rc, h, "dbs_decode")
    sl = slice(rank * per, (rank + 1) * per)
    for t in (lists, counts, bounds):
        dist.all_gather_into_tensor(t, t[sl].clone(), group=group)
    P = max(K, K * options.relaxed_pool_multiplier)
    trace = DeviceTrace(B, T, K, dev, with_pool=with_pool, P=P, with_weights=with_weights)
    outs = trace.struct()
    with torch.cuda.device(dev):
        rc = lib.dbs_device_merge_rows(h, _vp(x4), B, T, V, _vp(lists), _vp(counts), _vp(bounds), ctypes.byref(outs),
                                       stream)
    _check(rc, h, "dbs_decode")
    return trace


def gather_examples(arrays: Dict[str, torch.Tensor], group=None) -> Dict[str, torch.Tensor]:
    """Every rank's per-example arrays, in rank order, on every rank of `group`.

    The first dimension of each tensor is this rank's examples (the same
    count for every tensor; the other dimensions and the dtypes equal on every
    rank). Two collectives whatever the number of arrays: an all-gather of
    the example counts, then one all_gather_into_tensor of a packed byte
    buffer in which each rank's share is padded to the largest share. Works
    on NCCL (CUDA tensors) and on gloo (CPU tensors)."""
    import torch.distributed as dist
    if not arrays:
        return {}
    world = dist.get_world_size(group)
    names = list(arrays)
    n = int(arrays[names[0]].shape[0])
    dev = arrays[names[0]].device
    for name in names:
        t = arrays[name]
        if t.dim() < 1 or int(t.shape[0]) != n or t.device != dev:
            raise ValueError(f"gather_examples: '{name}' must have {n} examples on {dev}")
    counts = torch.empty(world, dtype=torch.int64, device=dev)
    dist.all_gather_into_tensor(counts, torch.tensor([n], dtype=torch.int64, device=dev), group=group)
    counts = [int(c) for c in counts.tolist()]
    per = max(counts)
    layout, off = [], 0
    for name in names:
        t = arrays[name]
        tail = tuple(int(s) for s in t.shape[1:])
        ex_bytes = math.prod(tail) * t.element_size()
        off = (off + 15) & ~15   # every array starts 16-byte aligned, so the views below hold
        layout.append((name, off, ex_bytes, t.dtype, tail))
        off += per * ex_bytes
    size = (off + 15) & ~15
    packet = torch.zeros(size, dtype=torch.uint8, device=dev)
    for name, o, ex_bytes, _, _ in layout:
        if n and ex_bytes:
            packet[o:o + n * ex_bytes].copy_(arrays[name].contiguous().reshape(-1).view(torch.uint8))
    gathered = torch.empty(world * size, dtype=torch.uint8, device=dev)
    dist.all_gather_into_tensor(gathered, packet, group=group)
    out = {}
    for name, o, ex_bytes, dtype, tail in layout:
        parts = [gathered[r * size + o:r * size + o + counts[r] * ex_bytes].view(dtype).view(counts[r], *tail)
                 for r in range(world)]
        out[name] = torch.cat(parts)
    return out


def decode_batch_sharded(x_local: torch.Tensor, options: DBSOptions, grad_final: Optional[torch.Tensor] = None,
                         with_pool: bool = False, with_weights: bool = False, group=None):
    """Batch-sharded decode: each rank decodes its own share of a global
    batch of examples on its own GPU, then every rank holds every example's
    results.

    `x_local` is this rank's contiguous share [B_r,T,K,V] of the examples
    (fp32 on this rank's GPU; shares follow rank order and may differ in
    size). The share is decoded with dbs_device_decode_batch and, with
    `grad_final` ([B_r,K]), its sparse surrogate backward runs with
    dbs_device_backward_batch; gather_examples then gives every rank of
    `group` the whole batch's final_scores [B,K], tokens and parents [B,T,K]
    and, with grad_final, each example's sparse gradient: sparse_counts [B],
    sparse_indices / sparse_values [B,T*K] (grad_final alone gives at most K
    entries per step; entries beyond an example's count are unspecified;
    indices are local to the example's [T*K*V]) and grad_initial [B,K].
    Returns (the gathered dict, this rank's DeviceTrace)."""
    B, T, K, V = (int(s) for s in x_local.shape)
    trace = device_decode(x_local, options, with_pool=with_pool, with_weights=with_weights)
    arrays = {"final_scores": trace.final_scores, "tokens": trace.tokens, "parents": trace.parents}
    if grad_final is not None:
        sp = device_backward_sparse(trace, grad_final, options, V)
        arrays["sparse_counts"] = sp["counts"]
        arrays["sparse_indices"] = sp["indices"][:, :T * K]
        arrays["sparse_values"] = sp["values"][:, :T * K]
        arrays["grad_initial"] = sp["grad_initial"]
    return gather_examples(arrays, group), trace


def device_backward_sparse(trace: DeviceTrace, grad_final: torch.Tensor, options: DBSOptions,
                           V: int) -> Dict[str, torch.Tensor]:
    """Sparse surrogate gradient of the final scores, per example, on the
    device: counts [B] (int64), indices [B,T*(K+P)] (int64, local to the
    example's [T*K*V], ascending) and values [B,T*(K+P)] (fp32), entries
    beyond an example's count unspecified, and grad_initial [B,K]."""
    B, T, K = (int(s) for s in trace.parents.shape)
    P = max(K, K * options.relaxed_pool_multiplier)
    cap = T * (K + P)
    device = trace.parents.device
    indices = torch.empty((B, cap), dtype=torch.int64, device=device)
    values = torch.empty((B, cap), dtype=torch.float32, device=device)
    counts = torch.empty((B,), dtype=torch.int64, device=device)
    grad_initial = torch.empty((B, K), dtype=torch.float32, device=device)
    g = grad_final.detach().to(device=device, dtype=torch.float32).contiguous()
    lib = _library()
    h = _handle(options)
    tr = trace.struct()
    with torch.cuda.device(device):
        rc = lib.dbs_device_backward_batch(h, B, T, V, ctypes.byref(tr), None, None, _vp(g), None, _vp(indices),
                                           _vp(values), _vp(counts), _vp(grad_initial), _stream_ptr(device))
    _check(rc, h, "dbs_backward")
    return {"counts": counts, "indices": indices, "values": values, "grad_initial": grad_initial}


def device_backward_dense(trace: DeviceTrace, grad_final: torch.Tensor, options: DBSOptions, V: int,
                          out: Optional[torch.Tensor] = None, prezeroed: bool = False) -> torch.Tensor:
    """Dense surrogate gradient [B,T,K,V] of the final scores, on the device.

    With `prezeroed`, `out` already holds zeros and only its non-zero
    entries are written.
    """
    B, T, K = (int(s) for s in trace.parents.shape)
    device = trace.parents.device
    if out is None:
        out = torch.empty((B, T, K, V), dtype=torch.float32, device=device)
        prezeroed = False
    g = grad_final.detach().to(device=device, dtype=torch.float32).contiguous()
    lib = _library()
    h = _handle(options)
    tr = trace.struct()
    flags = dbs_ctypes.DBS_DEVICE_GRAD_PREZEROED if prezeroed else 0
    with torch.cuda.device(device):
        rc = lib.dbs_device_backward_batch_ex(h, B, T, V, ctypes.byref(tr), None, None, _vp(g), _vp(out), None, None,
                                              None, None, flags, _stream_ptr(device))
    _check(rc, h, "dbs_backward")
    return out


class _DBSFinalScores(torch.autograd.Function):
    @staticmethod
    def forward(ctx, log_probs: torch.Tensor, options: DBSOptions):
        unbatched = _validate_public_shape(log_probs, options)
        device = _cuda_device_for(log_probs)
        ctx.options = options
        ctx.input_dtype = log_probs.dtype
        ctx.input_device = log_probs.device
        ctx.unbatched = unbatched
        ctx.needs_log_probs_grad = bool(ctx.needs_input_grad[0])
        # fp16 / bf16 inputs are promoted to fp32 like the reference
        # (python/torch_dbs_extension.py:244-245).
        x = log_probs.detach().to(device=device, dtype=torch.float32).contiguous()
        x4 = x.unsqueeze(0) if unbatched else x
        # The dense gradient is allocated here and zeroed beside the step
        # merge, so the backward only writes its non-zero entries.
        grad = torch.empty_like(x4) if ctx.needs_log_probs_grad else None
        trace = device_decode(x4, options, zero_fill=grad)
        ctx.V = int(x4.size(3))
        if ctx.needs_log_probs_grad:
            ctx.trace = trace
            ctx.grad = grad
        scores = trace.final_scores
        if unbatched:
            scores = scores.squeeze(0)
        return scores.to(log_probs.device)

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        if not ctx.needs_log_probs_grad:
            return None, None
        trace: DeviceTrace = ctx.trace
        g = grad_output
        if g.dim() == 1:
            g = g.unsqueeze(0)
        # the pre-zeroed buffer serves the first backward; a repeated backward
        # (retain_graph) gets a fresh, zero-filled one
        pre = getattr(ctx, "grad", None)
        grad = device_backward_dense(trace, g, ctx.options, ctx.V, out=pre, prezeroed=pre is not None)
        ctx.grad = None
        if ctx.unbatched:
            grad = grad.squeeze(0)
        return grad.to(device=ctx.input_device, dtype=ctx.input_dtype), None


def final_scores(log_probs: torch.Tensor, options: DBSOptions) -> torch.Tensor:
    """Final beam scores for [T,K,V] or [B,T,K,V] log-probs, with surrogate autograd."""
    return _DBSFinalScores.apply(log_probs, options)


def decode(log_probs: torch.Tensor, options: DBSOptions) -> Tuple[torch.Tensor, torch.Tensor]:
    """Hard-decode token traces and final scores: ([T,K] or [B,T,K] int32, [K] or [B,K]).

    Unlike the reference (python/torch_dbs_extension.py:306-326), which serves
    only CUDA inputs with default decoder-shaping options, every option is
    decoded here, for CUDA and CPU tensors alike (results on the input device).
    """
    unbatched = _validate_public_shape(log_probs, options)
    device = _cuda_device_for(log_probs)
    x = log_probs.detach().to(device=device, dtype=torch.float32).contiguous()
    x4 = x.unsqueeze(0) if unbatched else x
    trace = device_decode(x4, options)
    tokens, scores = trace.tokens, trace.final_scores
    if unbatched:
        tokens, scores = tokens.squeeze(0), scores.squeeze(0)
    return tokens.to(log_probs.device), scores.to(log_probs.device)


# ---------------------------------------------------------------------------
# torch.ops.dbs.* with the reference's schemas (python/torch_extension.cpp:191-194)
# ---------------------------------------------------------------------------
def _op_options(*args) -> DBSOptions:
    return DBSOptions(*args)


def _op_forward(log_probs, *args):
    opts = _op_options(*args)
    if log_probs.dim() != 3:
        raise RuntimeError("log_probs must have shape [T, K, V]")
    return final_scores(log_probs.detach(), opts)


def _op_backward(log_probs, grad_final_scores, *args):
    opts = _op_options(*args)
    if log_probs.dim() != 3:
        raise RuntimeError("log_probs must have shape [T, K, V]")
    if grad_final_scores.dim() != 1 or grad_final_scores.size(0) != opts.beam_size:
        raise RuntimeError("grad_final_scores must have shape [K]")
    _validate_public_shape(log_probs, opts)
    device = _cuda_device_for(log_probs)
    x4 = log_probs.detach().to(device=device, dtype=torch.float32).contiguous().unsqueeze(0)
    trace = device_decode(x4, opts)
    grad = device_backward_dense(trace, grad_final_scores.reshape(1, -1), opts, int(x4.size(3)))
    return grad.squeeze(0).to(log_probs.device)


_SCHEMA_ARGS = ("int beam_size, int eos_token, float selected_temperature, float soft_topk_temperature, "
                "int relaxed_pool_multiplier, int vocab_block, float length_penalty_alpha, "
                "float soft_topk_tolerance, int soft_topk_max_iters, int min_length, int validate_inputs, "
                "int max_dense_gradient_elements")

try:
    _OPS = torch.library.Library("dbs", "DEF")
    _OPS.define(f"final_scores_forward(Tensor log_probs, {_SCHEMA_ARGS}) -> Tensor")
    _OPS.define(f"final_scores_backward(Tensor log_probs, Tensor grad_final_scores, {_SCHEMA_ARGS}) -> Tensor")
    for _key in ("CPU", "CUDA"):
        _OPS.impl("final_scores_forward", _op_forward, _key)
        _OPS.impl("final_scores_backward", _op_backward, _key)
except RuntimeError:  # already registered in this process (e.g. module reloaded)
    _OPS = None
