"""ctypes binding of the dbs C ABI (include/dbs.h, include/dbs_device.h).

The struct layouts mirror the reference's C ABI (include/dbs.h:29-110 of
maged15/differentiable-beam-search-cuda; the 64-byte DBSOptionsC offsets are
the ones its python/torch_dbs.py:20-76 pins). The binding works over any
library exporting that ABI: this package's lib/libdbs.so, which runs every
decode and backward as sm_100a kernels, or another build of the same ABI.
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import Dict, Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
DEFAULT_LIBRARY = os.path.normpath(os.path.join(_HERE, "..", "lib", "libdbs.so"))

DBS_DTYPE_F32 = 0
DBS_DTYPE_F16 = 1
DBS_DTYPE_BF16 = 2


class DBSOptionsC(ctypes.Structure):
    _fields_ = [
        ("beam_size", ctypes.c_int),
        ("eos_token", ctypes.c_int),
        ("selected_temperature", ctypes.c_float),
        ("soft_topk_temperature", ctypes.c_float),
        ("relaxed_pool_multiplier", ctypes.c_int),
        ("vocab_block", ctypes.c_int),
        ("length_penalty_alpha", ctypes.c_float),
        ("soft_topk_tolerance", ctypes.c_float),
        ("soft_topk_max_iters", ctypes.c_int),
        ("min_length", ctypes.c_int),
        ("validate_inputs", ctypes.c_int),
        ("max_dense_gradient_elements", ctypes.c_int64),
        ("reserved0", ctypes.c_int),
        ("reserved1", ctypes.c_int),
    ]


TOKEN_FILTER_FN = ctypes.CFUNCTYPE(
    ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
    ctypes.POINTER(ctypes.c_int32), ctypes.c_int, ctypes.c_int,
)
MODEL_STEP_FN = ctypes.CFUNCTYPE(
    ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int32),
    ctypes.POINTER(ctypes.c_float), ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_float),
)


class DBSAdvancedConstraintsC(ctypes.Structure):
    _fields_ = [
        ("banned_tokens", ctypes.c_void_p),
        ("forced_tokens", ctypes.c_void_p),
        ("min_length", ctypes.c_int),
        ("repetition_penalty", ctypes.c_float),
        ("no_repeat_ngram_size", ctypes.c_int),
        ("token_filter", TOKEN_FILTER_FN),
        ("token_filter_user_data", ctypes.c_void_p),
        ("batch_index", ctypes.c_int),
    ]


class DBSStatsC(ctypes.Structure):
    _fields_ = [
        ("abi_version", ctypes.c_int),
        ("last_kernel", ctypes.c_int),
        ("used_sparse_backward", ctypes.c_int),
        ("used_dense_backward", ctypes.c_int),
        ("used_batch_threads", ctypes.c_int),
        ("used_model_step_callback", ctypes.c_int),
        ("last_error_category", ctypes.c_int),
        ("last_decode_ns", ctypes.c_int64),
        ("last_backward_ns", ctypes.c_int64),
        ("last_allocation_bytes", ctypes.c_int64),
        ("last_selected_count", ctypes.c_int64),
        ("last_pool_count", ctypes.c_int64),
        ("last_logprob_count", ctypes.c_int64),
        ("last_sparse_grad_count", ctypes.c_int64),
        ("total_allocator_calls", ctypes.c_int64),
        ("total_allocator_bytes", ctypes.c_int64),
        ("reserved_stats0", ctypes.c_int64),
        ("reserved_stats1", ctypes.c_int64),
    ]


class DBSDeviceDecodeOutputs(ctypes.Structure):
    _fields_ = [(name, ctypes.c_void_p) for name in (
        "parents", "tokens", "lengths", "from_logprob", "raw_scores", "scores", "weights",
        "pool_parents", "pool_tokens", "pool_lengths", "pool_from_logprob", "pool_raw_scores",
        "pool_scores", "relaxed_weights", "final_raw_scores", "final_scores",
    )]


assert ctypes.sizeof(DBSOptionsC) == 64
assert ctypes.sizeof(DBSAdvancedConstraintsC) == 56
assert ctypes.sizeof(DBSStatsC) == 120

_VP = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F = ctypes.c_float
_PP = ctypes.POINTER(ctypes.c_void_p)

# name -> (restype, argtypes); the 76 functions of the reference ABI.
ABI_FUNCTIONS = {
    "dbs_abi_version": (_I, []),
    "dbs_version_string": (ctypes.c_char_p, []),
    "dbs_last_global_error": (ctypes.c_char_p, []),
    "dbs_workspace_create": (_I, [_PP]),
    "dbs_workspace_destroy": (None, [_VP]),
    "dbs_workspace_reserve": (_I, [_VP, _I64, _I64]),
    "dbs_workspace_allocated_bytes": (_I64, [_VP]),
    "dbs_create_ex": (_I, [DBSOptionsC, _PP]),
    "dbs_create": (_VP, [DBSOptionsC]),
    "dbs_destroy": (None, [_VP]),
    "dbs_last_error": (ctypes.c_char_p, [_VP]),
    "dbs_decode": (_I, [_VP, _VP, _I, _I, _PP]),
    "dbs_decode_typed": (_I, [_VP, _VP, _I, _I, _I, _PP]),
    "dbs_decode_batch_typed": (_I, [_VP, _VP, _I, _I, _I, _I, _I, _PP]),
    "dbs_decode_constrained": (_I, [_VP, _VP, _I, _I, _VP, _VP, _I, _PP]),
    "dbs_decode_constrained_ex": (_I, [_VP, _VP, _I, _I, ctypes.POINTER(DBSAdvancedConstraintsC), _PP]),
    "dbs_decode_model_steps": (_I, [_VP, MODEL_STEP_FN, _VP, _I, _I, _I, _PP]),
    "dbs_decode_model_steps_with_workspace": (_I, [_VP, _VP, MODEL_STEP_FN, _VP, _I, _I, _I, _PP]),
    "dbs_decode_batch": (_I, [_VP, _VP, _I, _I, _I, _I, _PP]),
    "dbs_decode_batch_variable": (_I, [_VP, _VP, _I, _I, _I, _I, _VP, _VP, _VP, _VP, _VP, _VP, _I, _PP]),
    "dbs_backward": (_I, [_VP, _VP, _VP, _VP, _VP, _PP]),
    "dbs_backward_dense": (_I, [_VP, _VP, _VP, _VP, _VP, _PP]),
    "dbs_backward_sparse": (_I, [_VP, _VP, _VP, _VP, _VP, _PP]),
    "dbs_backward_default": (_I, [_VP, _VP, _VP, _VP, _VP, _PP]),
    "dbs_free_result": (None, [_VP]),
    "dbs_free_batch_result": (None, [_VP]),
    "dbs_free_backward": (None, [_VP]),
    "dbs_batch_result_size": (_I, [_VP]),
    "dbs_batch_result_at": (_VP, [_VP, _I]),
    "dbs_result_steps": (_I, [_VP]),
    "dbs_result_beam_size": (_I, [_VP]),
    "dbs_result_vocab_size": (_I, [_VP]),
    "dbs_result_pool_size": (_I, [_VP]),
    "dbs_result_tokens": (_VP, [_VP]),
    "dbs_result_parents": (_VP, [_VP]),
    "dbs_result_lengths": (_VP, [_VP]),
    "dbs_result_scores": (_VP, [_VP]),
    "dbs_result_raw_scores": (_VP, [_VP]),
    "dbs_result_weights": (_VP, [_VP]),
    "dbs_result_final_scores": (_VP, [_VP]),
    "dbs_result_final_raw_scores": (_VP, [_VP]),
    "dbs_result_relaxed_weights": (_VP, [_VP]),
    "dbs_result_pool_tokens": (_VP, [_VP]),
    "dbs_result_pool_parents": (_VP, [_VP]),
    "dbs_result_pool_lengths": (_VP, [_VP]),
    "dbs_result_pool_scores": (_VP, [_VP]),
    "dbs_result_pool_raw_scores": (_VP, [_VP]),
    "dbs_backward_grad_log_probs": (_VP, [_VP]),
    "dbs_backward_grad_initial_scores": (_VP, [_VP]),
    "dbs_backward_sparse_logprob_indices": (_VP, [_VP]),
    "dbs_backward_sparse_logprob_values": (_VP, [_VP]),
    "dbs_backward_sparse_logprob_count": (_I64, [_VP]),
    "dbs_backward_is_sparse": (_I, [_VP]),
    "dbs_result_selected_count": (_I64, [_VP]),
    "dbs_result_pool_count": (_I64, [_VP]),
    "dbs_result_logprob_count": (_I64, [_VP]),
    "dbs_backward_grad_log_probs_count": (_I64, [_VP]),
    "dbs_backward_grad_initial_scores_count": (_I64, [_VP]),
    "dbs_result_eos_count": (_I64, [_VP, _I]),
    "dbs_result_validate_deterministic_order": (_I, [_VP]),
    "dbs_result_summary_json": (_I, [_VP, _I, ctypes.c_char_p, _I64]),
    "dbs_validate_production_gate_manifest": (_I, [ctypes.c_char_p, ctypes.c_char_p, _I64]),
    "dbs_has_avx512": (_I, []),
    "dbs_has_avx2": (_I, []),
    "dbs_has_sse42": (_I, []),
    "dbs_has_neon": (_I, []),
    "dbs_selected_kernel_name": (ctypes.c_char_p, []),
    "dbs_get_stats": (_I, [_VP, ctypes.POINTER(DBSStatsC)]),
    "dbs_get_stats_json": (_I, [_VP, ctypes.c_char_p, _I64]),
    "dbs_is_deterministic": (_I, []),
    "dbs_set_deterministic_seed": (_I, [_VP, ctypes.c_uint64]),
    "dbs_get_deterministic_seed": (ctypes.c_uint64, [_VP]),
    "dbs_allocator_counters_reset": (None, []),
    "dbs_allocator_call_count": (_I64, []),
    "dbs_allocator_byte_count": (_I64, []),
    "dbs_reset_stats": (None, [_VP]),
}

DEVICE_FUNCTIONS = {
    "dbs_device_decode_batch": (_I, [_VP, _VP, _I, _I, _I, ctypes.POINTER(DBSDeviceDecodeOutputs), _VP]),
    "dbs_device_decode_batch_variable_ex": (
        _I, [_VP, _VP, _I, _I, _I, _I, _VP, _VP, _VP, _VP, _VP, _VP, _F, _I,
             ctypes.POINTER(DBSDeviceDecodeOutputs), _VP]),
    "dbs_device_backward_batch": (
        _I, [_VP, _I, _I, _I, ctypes.POINTER(DBSDeviceDecodeOutputs), _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP]),
    "dbs_device_decode_batch_ex": (_I, [_VP, _VP, _I, _I, _I, ctypes.POINTER(DBSDeviceDecodeOutputs), _VP, _I64, _VP]),
    "dbs_device_backward_batch_ex": (
        _I, [_VP, _I, _I, _I, ctypes.POINTER(DBSDeviceDecodeOutputs), _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _I,
             _VP]),
    "dbs_device_last_rescan_counts": (_I, [_VP, ctypes.POINTER(_I64), ctypes.POINTER(_I64)]),
    "dbs_device_profile": (_I, [_I]),
    "dbs_device_profile_read": (_I, [_I, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(_I64)]),
    "dbs_device_profile_kernels": (_I, [ctypes.c_uint]),
    "dbs_device_kernel_launches": (_I, [ctypes.POINTER(_I64)]),
    "dbs_device_row_list_capacity": (_I, [_VP, _I, ctypes.POINTER(_I)]),
    "dbs_device_scan_rows": (_I, [_VP, _VP, _I, _I, _I, _I, _I64, _I64, _VP, _VP, _VP, _VP]),
    "dbs_device_merge_rows": (_I, [_VP, _VP, _I, _I, _I, _VP, _VP, _VP, ctypes.POINTER(DBSDeviceDecodeOutputs), _VP]),
    "dbs_device_backward_sparse_noalloc": (
        _I, [_VP, _I, _I, _I, ctypes.POINTER(DBSDeviceDecodeOutputs), _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP]),
}

PROFILED_KERNELS = ("validate", "row_scan", "step_merge", "weights", "fill_zero", "backward")
DBS_DEVICE_GRAD_PREZEROED = 1


def load_library(path: Optional[str] = None, device_api: bool = True) -> ctypes.CDLL:
    """Load a dbs library and declare the ABI signatures on it."""
    path = path or os.environ.get("DBS_LIBRARY") or DEFAULT_LIBRARY
    if not os.path.exists(path):
        raise RuntimeError(
            f"dbs library not found at {path}; build it with `make -C differentiable-beam-search-cuda_b200`")
    lib = ctypes.CDLL(path)
    table = dict(ABI_FUNCTIONS)
    if device_api:
        table.update(DEVICE_FUNCTIONS)
    for name, (res, args) in table.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


@dataclass
class Options:
    beam_size: int = 8
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

    def to_c(self) -> DBSOptionsC:
        return DBSOptionsC(
            self.beam_size, self.eos_token, self.selected_temperature, self.soft_topk_temperature,
            self.relaxed_pool_multiplier, self.vocab_block, self.length_penalty_alpha,
            self.soft_topk_tolerance, self.soft_topk_max_iters, self.min_length, self.validate_inputs,
            self.max_dense_gradient_elements, 0, 0,
        )


class DBSError(RuntimeError):
    def __init__(self, what: str, rc: int, message: str):
        super().__init__(f"{what} failed ({rc}): {message}")
        self.rc = rc
        self.message = message


def _ptr(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _read(lib, fn, handle, dtype, count):
    p = getattr(lib, fn)(handle)
    if count == 0:
        return np.zeros(0, dtype=dtype)
    if not p:
        raise RuntimeError(f"{fn} returned NULL")
    buf = (ctypes.c_char * (count * np.dtype(dtype).itemsize)).from_address(p)
    return np.frombuffer(buf, dtype=dtype).copy()


def read_result(lib, r) -> Dict[str, np.ndarray]:
    T = lib.dbs_result_steps(r)
    K = lib.dbs_result_beam_size(r)
    P = lib.dbs_result_pool_size(r)
    out = {"T": T, "K": K, "P": P, "V": lib.dbs_result_vocab_size(r)}
    for name, fn, dt, n in (
        ("parents", "dbs_result_parents", np.int32, T * K),
        ("tokens", "dbs_result_tokens", np.int32, T * K),
        ("lengths", "dbs_result_lengths", np.int32, T * K),
        ("raw_scores", "dbs_result_raw_scores", np.float32, T * K),
        ("scores", "dbs_result_scores", np.float32, T * K),
        ("weights", "dbs_result_weights", np.float32, T * K),
        ("pool_parents", "dbs_result_pool_parents", np.int32, T * P),
        ("pool_tokens", "dbs_result_pool_tokens", np.int32, T * P),
        ("pool_lengths", "dbs_result_pool_lengths", np.int32, T * P),
        ("pool_raw_scores", "dbs_result_pool_raw_scores", np.float32, T * P),
        ("pool_scores", "dbs_result_pool_scores", np.float32, T * P),
        ("relaxed_weights", "dbs_result_relaxed_weights", np.float32, T * P),
        ("final_raw_scores", "dbs_result_final_raw_scores", np.float32, K),
        ("final_scores", "dbs_result_final_scores", np.float32, K),
    ):
        out[name] = _read(lib, fn, r, dt, n)
    return out


def read_backward(lib, b, dense_count: int = 0, K: int = 0) -> Dict[str, np.ndarray]:
    n = lib.dbs_backward_sparse_logprob_count(b)
    out = {
        "sparse": bool(lib.dbs_backward_is_sparse(b)),
        "indices": _read(lib, "dbs_backward_sparse_logprob_indices", b, np.int64, n),
        "values": _read(lib, "dbs_backward_sparse_logprob_values", b, np.float32, n),
        "grad_initial": _read(lib, "dbs_backward_grad_initial_scores", b, np.float32, K),
    }
    if not out["sparse"] and dense_count:
        out["grad_log_probs"] = _read(lib, "dbs_backward_grad_log_probs", b, np.float32, dense_count)
    return out


class Decoder:
    """One decoder handle of a dbs library (host arrays in, host arrays out)."""

    def __init__(self, lib, options: Options):
        self.lib = lib
        self.options = options
        h = ctypes.c_void_p()
        rc = lib.dbs_create_ex(options.to_c(), ctypes.byref(h))
        if rc != 0:
            raise DBSError("dbs_create_ex", rc, lib.dbs_last_global_error().decode())
        self.h = h

    def close(self):
        if self.h:
            self.lib.dbs_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _err(self, what, rc):
        raise DBSError(what, rc, self.lib.dbs_last_error(self.h).decode())

    def decode(self, x: np.ndarray, steps: int, vocab: int):
        r = ctypes.c_void_p()
        rc = self.lib.dbs_decode(self.h, _ptr(x), steps, vocab, ctypes.byref(r))
        if rc != 0:
            self._err("dbs_decode", rc)
        return r

    def decode_constrained_ex(self, x, steps, vocab, banned=None, forced=None, min_length=-1,
                              repetition_penalty=1.0, no_repeat_ngram_size=0, token_filter=None, batch_index=0):
        c = DBSAdvancedConstraintsC()
        c.batch_index = batch_index
        c.banned_tokens = _ptr(banned)
        c.forced_tokens = _ptr(forced)
        c.min_length = min_length
        c.repetition_penalty = repetition_penalty
        c.no_repeat_ngram_size = no_repeat_ngram_size
        if token_filter is not None:
            c.token_filter = token_filter
        r = ctypes.c_void_p()
        rc = self.lib.dbs_decode_constrained_ex(self.h, _ptr(x), steps, vocab, ctypes.byref(c), ctypes.byref(r))
        if rc != 0:
            self._err("dbs_decode_constrained_ex", rc)
        return r

    def decode_batch(self, x, batch, steps, vocab, threads=0):
        br = ctypes.c_void_p()
        rc = self.lib.dbs_decode_batch(self.h, _ptr(x), batch, steps, vocab, threads, ctypes.byref(br))
        if rc != 0:
            self._err("dbs_decode_batch", rc)
        return br

    def decode_batch_variable(self, x, batch, max_steps, max_beam, vocab, steps=None, beams=None, eos=None,
                              min_lengths=None, banned=None, forced=None, threads=0):
        br = ctypes.c_void_p()
        rc = self.lib.dbs_decode_batch_variable(
            self.h, _ptr(x), batch, max_steps, max_beam, vocab, _ptr(steps), _ptr(beams), _ptr(eos),
            _ptr(min_lengths), _ptr(banned), _ptr(forced), threads, ctypes.byref(br))
        if rc != 0:
            self._err("dbs_decode_batch_variable", rc)
        return br

    def backward(self, r, grad_selected=None, grad_relaxed=None, grad_final=None, mode="sparse"):
        fn = {"sparse": "dbs_backward_sparse", "dense": "dbs_backward_dense",
              "default": "dbs_backward", "default2": "dbs_backward_default"}[mode]
        b = ctypes.c_void_p()
        rc = getattr(self.lib, fn)(self.h, r, _ptr(grad_selected), _ptr(grad_relaxed), _ptr(grad_final),
                                   ctypes.byref(b))
        if rc != 0:
            self._err(fn, rc)
        return b

    def stats(self) -> DBSStatsC:
        s = DBSStatsC()
        self.lib.dbs_get_stats(self.h, ctypes.byref(s))
        return s


def decode_and_read(lib, options: Options, x: np.ndarray, steps: int, vocab: int,
                    grad_final: Optional[Sequence[float]] = None, **constraints):
    """Decode one [T,K,V] example and (optionally) run the sparse backward."""
    dec = Decoder(lib, options)
    try:
        if constraints:
            r = dec.decode_constrained_ex(x, steps, vocab, **constraints)
        else:
            r = dec.decode(x, steps, vocab)
        try:
            out = read_result(lib, r)
            if grad_final is not None:
                g = np.asarray(grad_final, dtype=np.float32)
                b = dec.backward(r, None, None, g)
                try:
                    out["backward"] = read_backward(lib, b, K=options.beam_size)
                finally:
                    lib.dbs_free_backward(b)
        finally:
            lib.dbs_free_result(r)
    finally:
        dec.close()
    return out
