"""The drop-in library loads on a machine without a GPU, exports every symbol
its headers declare under the reference's version node, and serves the
host-only parts of the ABI (handles, options, errors, stats, utilities)."""
import ctypes
import os
import re
import subprocess

import pytest

import dbs_ctypes as dc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", h) for h in ("dbs.h", "dbs_device.h")]


def declared_symbols():
    names = set()
    for h in HEADERS:
        text = open(h).read()
        names |= set(re.findall(r"DBS_EXPORT[^;(]*?\b(dbs_\w+)\s*\(", text, flags=re.S))
    return names


def test_library_exports_every_declared_symbol(libdbs):
    out = subprocess.run(["nm", "-D", "--defined-only", libdbs._name], capture_output=True, text=True, check=True)
    exported = {m.group(1) for m in re.finditer(r" T (dbs_\w+)", out.stdout)}
    declared = declared_symbols()
    assert len(declared) >= 76 + 4
    assert declared <= exported, sorted(declared - exported)
    for name in declared:
        assert hasattr(libdbs, name)


def test_reference_abi_symbol_set_and_version_node(libdbs):
    out = subprocess.run(["objdump", "-T", libdbs._name], capture_output=True, text=True, check=True)
    versioned = {m.group(1) for m in re.finditer(r"DBS_0\.6\s+(dbs_\w+)", out.stdout)}
    assert set(dc.ABI_FUNCTIONS) <= versioned
    assert len(dc.ABI_FUNCTIONS) == 76


def test_soname_matches_the_reference(libdbs):
    # binaries linked against the reference look for libdbs.so.10
    out = subprocess.run(["readelf", "-d", libdbs._name], capture_output=True, text=True, check=True)
    assert "Library soname: [libdbs.so.10]" in out.stdout
    assert os.path.exists(os.path.join(os.path.dirname(libdbs._name), "libdbs.so.10"))


def test_version_and_stub_entry_points(libdbs):
    assert libdbs.dbs_abi_version() == 10
    assert libdbs.dbs_version_string() == b"1.0.0"
    assert libdbs.dbs_is_deterministic() == 1
    buf = ctypes.create_string_buffer(256)
    assert libdbs.dbs_validate_production_gate_manifest(b"{}", buf, 256) != 0
    assert b"deprecated" in buf.value
    assert libdbs.dbs_selected_kernel_name() == b"cuda"


def test_create_defaults_errors_and_stats(libdbs):
    opt = dc.DBSOptionsC()  # all zero -> reference defaults
    h = ctypes.c_void_p()
    assert libdbs.dbs_create_ex(opt, ctypes.byref(h)) == 0
    st = dc.DBSStatsC()
    assert libdbs.dbs_get_stats(h, ctypes.byref(st)) == 0
    assert st.abi_version == 10 and st.last_kernel == 5
    js = ctypes.create_string_buffer(2048)
    assert libdbs.dbs_get_stats_json(h, js, 2048) == 0
    assert b'"abi_version":10' in js.value and b'"allocator_calls"' in js.value
    assert libdbs.dbs_set_deterministic_seed(h, 123456789) == 0
    assert libdbs.dbs_get_deterministic_seed(h) == 123456789
    libdbs.dbs_reset_stats(h)
    # null output pointers
    assert libdbs.dbs_decode(h, None, 1, 1, None) == -1
    assert libdbs.dbs_create_ex(opt, None) == -1
    assert libdbs.dbs_last_global_error() == b"out_handle cannot be null"
    libdbs.dbs_destroy(h)


@pytest.mark.parametrize("field,value,msg", [
    ("length_penalty_alpha", -0.5, None),         # negative alpha falls back to 0 (from_c_options)
    ("min_length", -3, None),                     # negative min length falls back to 0
])
def test_option_default_substitution(libdbs, field, value, msg):
    opt = dc.Options()
    setattr(opt, field, value)
    h = ctypes.c_void_p()
    assert libdbs.dbs_create_ex(opt.to_c(), ctypes.byref(h)) == 0
    libdbs.dbs_destroy(h)


def test_invalid_arguments_fail_before_touching_the_device(libdbs):
    h = ctypes.c_void_p()
    assert libdbs.dbs_create_ex(dc.Options(beam_size=2).to_c(), ctypes.byref(h)) == 0
    r = ctypes.c_void_p()
    x = (ctypes.c_float * 8)()
    assert libdbs.dbs_decode(h, None, 1, 4, ctypes.byref(r)) == -2
    assert libdbs.dbs_last_error(h) == b"log_probs cannot be null"
    assert libdbs.dbs_decode(h, x, 0, 4, ctypes.byref(r)) == -2
    assert libdbs.dbs_last_error(h) == b"steps must be positive"
    assert libdbs.dbs_decode(h, x, 1, 0, ctypes.byref(r)) == -2
    assert libdbs.dbs_last_error(h) == b"vocab_size must be positive"
    br = ctypes.c_void_p()
    assert libdbs.dbs_decode_batch(h, x, 0, 1, 4, 1, ctypes.byref(br)) == -1
    st = dc.DBSStatsC()
    libdbs.dbs_get_stats(h, ctypes.byref(st))
    assert st.last_error_category == 1
    libdbs.dbs_destroy(h)


def test_eos_outside_vocab_and_forced_outside_vocab(libdbs):
    h = ctypes.c_void_p()
    assert libdbs.dbs_create_ex(dc.Options(beam_size=2, eos_token=9).to_c(), ctypes.byref(h)) == 0
    x = (ctypes.c_float * 16)()
    r = ctypes.c_void_p()
    assert libdbs.dbs_decode(h, x, 2, 4, ctypes.byref(r)) == -2
    assert libdbs.dbs_last_error(h) == b"eos_token is outside vocab"
    libdbs.dbs_destroy(h)
    assert libdbs.dbs_create_ex(dc.Options(beam_size=2).to_c(), ctypes.byref(h)) == 0
    forced = (ctypes.c_int32 * 2)(1, 7)
    assert libdbs.dbs_decode_constrained(h, x, 2, 4, None, forced, 0, ctypes.byref(r)) == -2
    assert libdbs.dbs_last_error(h) == b"forced token is outside vocab"
    libdbs.dbs_destroy(h)


def test_workspace_api(libdbs):
    ws = ctypes.c_void_p()
    assert libdbs.dbs_workspace_create(ctypes.byref(ws)) == 0
    assert libdbs.dbs_workspace_reserve(ws, 4096, 128) == 0
    assert libdbs.dbs_workspace_allocated_bytes(ws) == 4096 * 4 + 128 * 4
    assert libdbs.dbs_workspace_reserve(ws, -1, 0) == -1
    libdbs.dbs_workspace_destroy(ws)


def test_null_handles_are_safe(libdbs):
    assert libdbs.dbs_result_steps(None) == 0
    assert libdbs.dbs_result_tokens(None) is None
    assert libdbs.dbs_batch_result_size(None) == 0
    assert libdbs.dbs_batch_result_at(None, 0) is None
    assert libdbs.dbs_backward_sparse_logprob_count(None) == 0
    assert libdbs.dbs_get_stats(None, None) == -1
    libdbs.dbs_free_result(None)
    libdbs.dbs_free_batch_result(None)
    libdbs.dbs_free_backward(None)
    libdbs.dbs_destroy(None)


def _reference_lib():
    import sys
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle import reference_library_path
    path = reference_library_path()
    if path is None:
        pytest.skip("oracle/_ref not built")
    return dc.load_library(path, device_api=False)


def _null_out():
    return ctypes.byref(ctypes.c_void_p())


_X = (ctypes.c_float * 64)()
_REJECTED_CALLS = [
    ("null log_probs", lambda L, h: L.dbs_decode(h, None, 1, 4, _null_out())),
    ("zero steps", lambda L, h: L.dbs_decode(h, _X, 0, 4, _null_out())),
    ("zero vocab", lambda L, h: L.dbs_decode(h, _X, 1, 0, _null_out())),
    ("eos outside vocab", lambda L, h: L.dbs_decode(h, _X, 2, 4, _null_out())),
    ("null result out", lambda L, h: L.dbs_decode(h, _X, 2, 16, None)),
    ("empty batch", lambda L, h: L.dbs_decode_batch(h, _X, 0, 1, 16, 1, _null_out())),
    ("null batch out", lambda L, h: L.dbs_decode_batch(h, _X, 1, 1, 16, 1, None)),
    ("backward of null result", lambda L, h: L.dbs_backward(h, None, None, None, None, _null_out())),
    ("backward null out", lambda L, h: L.dbs_backward(h, None, None, None, None, None)),
    ("stats to null", lambda L, h: L.dbs_get_stats(h, None)),
    ("stats json too small", lambda L, h: L.dbs_get_stats_json(h, ctypes.create_string_buffer(4), 4)),
    ("stats json to null", lambda L, h: L.dbs_get_stats_json(h, None, 0)),
]


@pytest.mark.parametrize("name,call", _REJECTED_CALLS, ids=[c[0] for c in _REJECTED_CALLS])
def test_rejected_calls_match_the_reference(libdbs, name, call):
    """Calls the library rejects before any device work: the same return
    code, per-handle message and stats error category as the reference
    library on the same call."""
    ref = _reference_lib()
    seen = []
    for lib in (libdbs, ref):
        h = ctypes.c_void_p()
        assert lib.dbs_create_ex(dc.Options(beam_size=2, eos_token=9).to_c(), ctypes.byref(h)) == 0
        rc = call(lib, h)
        st = dc.DBSStatsC()
        lib.dbs_get_stats(h, ctypes.byref(st))
        seen.append((rc, lib.dbs_last_error(h), st.last_error_category))
        lib.dbs_destroy(h)
    assert seen[0] == seen[1], f"{name}: {seen[0]} here, {seen[1]} in the reference"


@pytest.mark.parametrize("opts", [dict(beam_size=0), dict(beam_size=-3), dict(relaxed_pool_multiplier=0),
                                  dict(selected_temperature=0.0), dict(soft_topk_temperature=-1.0),
                                  dict(length_penalty_alpha=float("nan")), dict(soft_topk_max_iters=0),
                                  dict(vocab_block=0), dict(max_dense_gradient_elements=0)])
def test_option_substitution_matches_the_reference(libdbs, opts):
    """Out-of-range options: created or refused as the reference does, with
    its global message."""
    ref = _reference_lib()
    seen = []
    for lib in (libdbs, ref):
        h = ctypes.c_void_p()
        rc = lib.dbs_create_ex(dc.Options(**opts).to_c(), ctypes.byref(h))
        seen.append((rc, lib.dbs_last_global_error()))
        if rc == 0:
            lib.dbs_destroy(h)
    assert seen[0] == seen[1]


def test_stats_json_matches_the_reference_format(libdbs):
    """dbs_get_stats_json of a fresh handle: the reference's keys, order and
    values, the kernel name aside ("cuda" here, the reference's SIMD level
    there)."""
    ref = _reference_lib()
    texts = []
    for lib in (libdbs, ref):
        h = ctypes.c_void_p()
        assert lib.dbs_create_ex(dc.Options(beam_size=3, eos_token=2, length_penalty_alpha=0.4).to_c(),
                                 ctypes.byref(h)) == 0
        js = ctypes.create_string_buffer(4096)
        assert lib.dbs_get_stats_json(h, js, 4096) == 0
        texts.append(re.sub(rb'"kernel":"[a-z0-9_]+"', b'"kernel":"-"', js.value))
        lib.dbs_destroy(h)
    assert b'"kernel":"-"' in texts[0]
    assert texts[0] == texts[1]


def _host_only_calls(L):
    """The host-only entry points, exercised in one fixed sequence."""
    out = [L.dbs_abi_version(), L.dbs_version_string(), L.dbs_is_deterministic(),
           (L.dbs_has_avx512(), L.dbs_has_avx2(), L.dbs_has_sse42(), L.dbs_has_neon())]
    w = ctypes.c_void_p()
    out += [L.dbs_workspace_create(ctypes.byref(w)), L.dbs_workspace_allocated_bytes(w),
            L.dbs_workspace_reserve(w, 1000, 10), L.dbs_workspace_allocated_bytes(w),
            L.dbs_workspace_reserve(w, -1, 10), L.dbs_workspace_reserve(None, 1, 1),
            L.dbs_workspace_allocated_bytes(None), L.dbs_workspace_create(None), L.dbs_last_global_error()]
    L.dbs_workspace_destroy(w)
    L.dbs_workspace_destroy(None)
    h = ctypes.c_void_p()
    L.dbs_create_ex(dc.Options(beam_size=2).to_c(), ctypes.byref(h))
    out += [L.dbs_get_deterministic_seed(h), L.dbs_set_deterministic_seed(h, 42), L.dbs_get_deterministic_seed(h),
            L.dbs_set_deterministic_seed(None, 1), L.dbs_get_deterministic_seed(None), L.dbs_last_error(None)]
    L.dbs_reset_stats(h)
    L.dbs_reset_stats(None)
    L.dbs_destroy(h)
    L.dbs_destroy(None)
    L.dbs_allocator_counters_reset()
    out += [L.dbs_allocator_call_count(), L.dbs_allocator_byte_count()]
    buf = ctypes.create_string_buffer(256)
    out += [L.dbs_validate_production_gate_manifest(b"{}", buf, 256), buf.value,
            L.dbs_validate_production_gate_manifest(None, None, 0)]
    old = L.dbs_create(dc.Options(beam_size=3).to_c())
    out.append(bool(old))
    L.dbs_destroy(old)
    return out


def test_host_only_entry_points_match_the_reference(libdbs):
    """Version, capability queries, workspaces, seeds, allocator counters,
    the deprecated manifest stub and dbs_create: the same results, codes and
    messages as the reference library."""
    ref = _reference_lib()
    assert _host_only_calls(libdbs) == _host_only_calls(ref)


def test_struct_layouts_equal_the_reference_header():
    """Every public struct's size and every field's offset and size, the
    data-type enum, the callback pointers and the version macros, as
    include/dbs.h declares them and as the reference's header does
    (oracle/abi_layout.c compiled against each by oracle/Makefile)."""
    ours = os.path.join(ROOT, "oracle", "_build", "abi_layout")
    ref = os.path.join(ROOT, "oracle", "_ref", "abi_layout")
    if not os.path.exists(ours):
        pytest.skip("oracle/_build/abi_layout not built (make -C oracle)")
    if not os.path.exists(ref):
        pytest.skip("oracle/_ref/abi_layout not built (needs the reference source tree)")
    a = subprocess.run([ours], capture_output=True, text=True, check=True).stdout
    b = subprocess.run([ref], capture_output=True, text=True, check=True).stdout
    assert "DBSOptionsC size 64" in a and a.count("\n") > 40
    assert a == b


def test_versioned_symbols_equal_the_reference_library(libdbs):
    """The names exported under DBS_0.6: every name the reference library
    exports there (oracle/_ref/libdbs_ref.so, built from its source with its
    version script), and besides them only the device extension's
    dbs_device_* names."""
    import sys
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle import reference_library_path
    path = reference_library_path()
    if path is None:
        pytest.skip("oracle/_ref not built")

    def versioned(lib_path):
        out = subprocess.run(["objdump", "-T", lib_path], capture_output=True, text=True, check=True).stdout
        return {m.group(1) for m in re.finditer(r"DBS_0\.6\s+(dbs_\w+)", out)}

    ours, ref = versioned(libdbs._name), versioned(path)
    assert len(ref) == 76
    assert ref <= ours, sorted(ref - ours)
    assert all(n.startswith("dbs_device_") for n in ours - ref), sorted(ours - ref)
