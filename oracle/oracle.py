"""Python access to the CPU checkers. TEST INFRASTRUCTURE ONLY.

* `OracleLib`  -- ctypes wrapper of oracle/_build/libdbs_oracle.so, the plain-C
  restatement of the reference decoder (dbs_oracle.c).
* `reference_library_path()` -- oracle/_ref/libdbs_ref.so, the reference
  library compiled from its own source by oracle/Makefile; it exports the
  same C ABI as the product and is driven through dbs_ctypes.Decoder.

Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline arm use this
module; the product never imports it.
"""

from __future__ import annotations

import ctypes
import os
from typing import Dict, Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libdbs_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libdbs_ref.so")


def reference_library_path() -> Optional[str]:
    return REF_SO if os.path.exists(REF_SO) else None


class _Opts(ctypes.Structure):
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
    ]


TOKEN_FILTER_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                   ctypes.POINTER(ctypes.c_int32), ctypes.c_int, ctypes.c_int)


class _Cons(ctypes.Structure):
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


_RESULT_FIELDS = [
    ("parents", np.int32, "sel"), ("tokens", np.int32, "sel"), ("lengths", np.int32, "sel"),
    ("raw_scores", np.float32, "sel"), ("scores", np.float32, "sel"), ("weights", np.float32, "sel"),
    ("from_logprob", np.uint8, "sel"),
    ("pool_parents", np.int32, "pool"), ("pool_tokens", np.int32, "pool"), ("pool_lengths", np.int32, "pool"),
    ("pool_raw_scores", np.float32, "pool"), ("pool_scores", np.float32, "pool"),
    ("relaxed_weights", np.float32, "pool"), ("pool_from_logprob", np.uint8, "pool"),
    ("final_raw_scores", np.float32, "fin"), ("final_scores", np.float32, "fin"),
]


class _Result(ctypes.Structure):
    _fields_ = [(name, ctypes.c_void_p) for name, _, _ in _RESULT_FIELDS]


class OracleLib:
    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            raise RuntimeError(f"oracle library missing: {path} (run `make -C oracle`)")
        self.lib = ctypes.CDLL(path)
        L = self.lib
        L.oracle_options_from_c.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_float,
                                            ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_float,
                                            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int64,
                                            ctypes.POINTER(_Opts)]
        L.oracle_pool_size.argtypes = [ctypes.POINTER(_Opts)]
        L.oracle_pool_size.restype = ctypes.c_int
        L.oracle_decode.argtypes = [ctypes.POINTER(_Opts), ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                    ctypes.POINTER(_Cons), ctypes.POINTER(_Result)]
        L.oracle_decode.restype = ctypes.c_int
        for fn in ("oracle_backward_sparse",):
            getattr(L, fn).argtypes = [ctypes.POINTER(_Opts), ctypes.c_int, ctypes.c_int, ctypes.POINTER(_Result),
                                       ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64), ctypes.c_void_p]
            getattr(L, fn).restype = ctypes.c_int
        L.oracle_backward_dense.argtypes = [ctypes.POINTER(_Opts), ctypes.c_int, ctypes.c_int,
                                            ctypes.POINTER(_Result), ctypes.c_void_p, ctypes.c_void_p,
                                            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        L.oracle_backward_dense.restype = ctypes.c_int
        L.oracle_last_error.restype = ctypes.c_char_p

    def options(self, beam_size=8, eos_token=-1, selected_temperature=1.0, soft_topk_temperature=0.25,
                relaxed_pool_multiplier=8, vocab_block=4096, length_penalty_alpha=0.0,
                soft_topk_tolerance=1.0e-4, soft_topk_max_iters=48, min_length=0, validate_inputs=1,
                max_dense_gradient_elements=100_000_000) -> _Opts:
        o = _Opts()
        self.lib.oracle_options_from_c(beam_size, eos_token, selected_temperature, soft_topk_temperature,
                                       relaxed_pool_multiplier, vocab_block, length_penalty_alpha,
                                       soft_topk_tolerance, soft_topk_max_iters, min_length, validate_inputs,
                                       max_dense_gradient_elements, ctypes.byref(o))
        return o

    def decode(self, opts: _Opts, x: np.ndarray, steps: int, vocab: int, banned=None, forced=None,
               min_length: Optional[int] = None, repetition_penalty: float = 1.0,
               no_repeat_ngram_size: int = 0, token_filter=None, batch_index: int = 0) -> Dict[str, np.ndarray]:
        x = np.ascontiguousarray(x, dtype=np.float32)
        K = opts.beam_size
        P = self.lib.oracle_pool_size(ctypes.byref(opts))
        sizes = {"sel": steps * K, "pool": steps * P, "fin": K}
        arrays = {name: np.zeros(sizes[kind], dtype=dt) for name, dt, kind in _RESULT_FIELDS}
        res = _Result(*[arrays[name].ctypes.data_as(ctypes.c_void_p) for name, _, _ in _RESULT_FIELDS])
        cons_ptr = None
        keep = []
        if banned is not None or forced is not None or min_length is not None or \
                repetition_penalty != 1.0 or no_repeat_ngram_size or token_filter is not None:
            b = None if banned is None else np.ascontiguousarray(banned, dtype=np.uint8)
            f = None if forced is None else np.ascontiguousarray(forced, dtype=np.int32)
            keep += [b, f]
            c = _Cons(None if b is None else b.ctypes.data_as(ctypes.c_void_p),
                      None if f is None else f.ctypes.data_as(ctypes.c_void_p),
                      -1 if min_length is None else min_length, repetition_penalty, no_repeat_ngram_size,
                      TOKEN_FILTER_FN() if token_filter is None else token_filter, None, batch_index)
            cons_ptr = ctypes.byref(c)
        rc = self.lib.oracle_decode(ctypes.byref(opts), x.ctypes.data_as(ctypes.c_void_p), steps, vocab, cons_ptr,
                                    ctypes.byref(res))
        if rc != 0:
            raise ValueError(self.lib.oracle_last_error().decode())
        arrays.update({"T": steps, "K": K, "P": P, "V": vocab, "_res": res, "_opts": opts})
        return arrays

    def backward_sparse(self, fwd: Dict, grad_selected=None, grad_relaxed=None, grad_final=None):
        T, K, P, V = fwd["T"], fwd["K"], fwd["P"], fwd["V"]
        idx = np.zeros(T * (K + P) + 1, dtype=np.int64)
        val = np.zeros(T * (K + P) + 1, dtype=np.float32)
        gi = np.zeros(K, dtype=np.float32)
        nnz = ctypes.c_int64()
        gs = None if grad_selected is None else np.ascontiguousarray(grad_selected, dtype=np.float32)
        gr = None if grad_relaxed is None else np.ascontiguousarray(grad_relaxed, dtype=np.float32)
        gf = None if grad_final is None else np.ascontiguousarray(grad_final, dtype=np.float32)
        p = lambda a: None if a is None else a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
        self.lib.oracle_backward_sparse(ctypes.byref(fwd["_opts"]), T, V, ctypes.byref(fwd["_res"]), p(gs), p(gr),
                                        p(gf), p(idx), p(val), ctypes.byref(nnz), p(gi))
        n = nnz.value
        return {"indices": idx[:n].copy(), "values": val[:n].copy(), "grad_initial": gi}

    def backward_dense(self, fwd: Dict, grad_selected=None, grad_relaxed=None, grad_final=None):
        T, K, V = fwd["T"], fwd["K"], fwd["V"]
        g = np.zeros(T * K * V, dtype=np.float32)
        gi = np.zeros(K, dtype=np.float32)
        gs = None if grad_selected is None else np.ascontiguousarray(grad_selected, dtype=np.float32)
        gr = None if grad_relaxed is None else np.ascontiguousarray(grad_relaxed, dtype=np.float32)
        gf = None if grad_final is None else np.ascontiguousarray(grad_final, dtype=np.float32)
        p = lambda a: None if a is None else a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
        rc = self.lib.oracle_backward_dense(ctypes.byref(fwd["_opts"]), T, V, ctypes.byref(fwd["_res"]), p(gs),
                                            p(gr), p(gf), p(g), p(gi))
        if rc != 0:
            raise ValueError(self.lib.oracle_last_error().decode())
        return {"grad_log_probs": g, "grad_initial": gi}
