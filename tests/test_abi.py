"""The C ABI: every entry point declared in include/afb.h is exported by libafb.so and bound by the
Python host, bench.py's probe lives in its own library (include/afb_probe.h), and argument errors come
back as AfbError without touching a GPU."""

import ctypes
import os
import re

import pytest

from conftest import ROOT


def declared():
    inc = os.path.join(ROOT, "include")
    text = "".join(open(os.path.join(inc, f)).read() for f in sorted(os.listdir(inc)) if f.endswith(".h"))
    return sorted(set(re.findall(r"AFB_API\s+[\w\s\*]*?\b(afb_\w+)\s*\(", text)))


def test_header_declares_the_entry_points():
    names = declared()
    assert "afb_cone_forward" in names and "afb_cone_create" in names and len(names) >= 16


def test_library_exports_every_declared_symbol():
    from alphafly_b200 import _lib
    lib = _lib.load()
    for name in declared():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no Python binding"
    assert lib.afb_compiled_arch() == 100 and lib.afb_version() >= 1


def test_probe_is_a_separate_library():
    from alphafly_b200 import _lib
    lib = _lib.load()
    assert not hasattr(lib, "afb_probe_gather")
    probe = _lib.load_probe()
    text = open(os.path.join(ROOT, "include", "afb_probe.h")).read()
    names = sorted(set(re.findall(r"AFB_PROBE_API\s+[\w\s\*]*?\b(afb_\w+)\s*\(", text)))
    assert names == sorted(_lib.PROBE_SIGNATURES)
    for name in names:
        assert hasattr(probe, name), name
    # argument checks come before any device call
    assert probe.afb_probe_gather(9, None, 1, None, 1, None, 0, None) == -1


def test_argument_errors_are_reported_without_a_gpu():
    from alphafly_b200 import _lib
    lib = _lib.load()
    h = ctypes.c_void_p()
    rc = lib.afb_cone_create(ctypes.byref(h), 0, 0, None, None, None, 0, None, 1, 6, None)
    assert rc == _lib.EINVAL and b"n must be" in lib.afb_last_error()
    with pytest.raises(_lib.AfbError, match="steps must be"):
        _lib.check(lib.afb_cone_create(ctypes.byref(h), 10, 0, None, None, None, 0, ctypes.c_void_p(8), 1, 0, None))
    assert lib.afb_cone_forward_workspace(None, 0, 64) == 0
    with pytest.raises(_lib.AfbError, match="unknown mode"):
        _lib.check(lib.afb_cone_forward(ctypes.c_void_p(16), 7, None, 0, 0, None, 0, None, 0, None))


def test_input_map_argument_errors_without_a_gpu():
    from alphafly_b200 import _lib
    lib = _lib.load()
    p = ctypes.c_void_p(256)
    assert lib.afb_input_map_f16(0, 64, 838, p, 840, p, 840, p, 5.0, p, 64, None, None) == _lib.OK   # nothing to do
    with pytest.raises(_lib.AfbError, match="negative size"):
        _lib.check(lib.afb_input_map_f16(-1, 64, 838, p, 840, p, 840, p, 5.0, p, 64, None, None))
    with pytest.raises(_lib.AfbError, match="multiple of 8"):
        _lib.check(lib.afb_input_map_f16(10, 64, 838, p, 838, p, 840, p, 5.0, p, 64, None, None))
    with pytest.raises(_lib.AfbError, match="below the row length"):
        _lib.check(lib.afb_input_map_f16(10, 64, 838, p, 840, p, 840, p, 5.0, p, 32, None, None))
    with pytest.raises(_lib.AfbError, match="16-byte aligned"):
        _lib.check(lib.afb_input_map_f16(10, 64, 838, ctypes.c_void_p(258), 840, p, 840, p, 5.0, p, 64, None, None))


def prototypes():
    """{name: number of parameters} of every AFB_API declaration in include/afb.h."""
    text = open(os.path.join(ROOT, "include", "afb.h")).read()
    out = {}
    for m in re.finditer(r"AFB_API\s+[\w\s\*]*?\b(afb_\w+)\s*\(([^)]*)\)", text):
        params = " ".join(m.group(2).split())
        out[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_bindings_take_as_many_arguments_as_the_header_declares():
    from alphafly_b200 import _lib
    protos = prototypes()
    assert len(protos) == len(declared())
    for name, n in protos.items():
        assert len(_lib.SIGNATURES[name][1]) == n, name


def test_gemm_argument_errors_are_reported_without_a_gpu():
    from alphafly_b200 import _lib
    lib = _lib.load()
    args = [1.0, None, 1, 0, None, 1, 0, None, 0, 1.0, None, 1, None, 0, None, None]
    with pytest.raises(_lib.AfbError, match="negative size"):
        _lib.check(lib.afb_gemm_f32(-1, 1, 1, *args))
    bad_bias = list(args)
    bad_bias[8] = 3
    with pytest.raises(_lib.AfbError, match="bias_dim"):
        _lib.check(lib.afb_gemm_f32(1, 1, 1, *bad_bias))
    assert lib.afb_gemm_f32(0, 5, 7, *args) == 0                      # an empty product is a no-op
    assert lib.afb_gemm_workspace(0, 4, 4) == 0 and lib.afb_gemm_workspace(4, 4, 4) > 0
