"""ctypes binding of libafb.so, the package's CUDA library (C ABI declared in include/afb.h).

The library is built in-tree (``python __graft_entry__.py build`` or ``make -C alphafly_b200/csrc``).
There is no fallback: if it is missing or cannot be loaded, importing a module that needs it fails
with the reason.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libafb.so")
PROBE_PATH = os.path.join(_HERE, "libafb_probe.so")      # bench.py's gather-ceiling probe (include/afb_probe.h)

OK, EINVAL, ECUDA, ESTATE = 0, -1, -2, -3
MODE_F32, MODE_DEV16 = 0, 1
FIELDS = {"rows": 0, "carried": 1, "keep_next": 2, "keep_prev": 3, "prev_row": 4, "u_pos": 5, "u_src": 6,
          "edges": 7, "post": 8, "pre": 9, "crow": 10, "t_order": 11, "t_crow": 12, "t_col": 13,
          "out_pos": 14, "out_src": 15}

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f = ctypes.c_float
_sz = ctypes.c_size_t
_pp = ctypes.POINTER(ctypes.c_void_p)

# name -> (restype, argtypes); every entry point of include/afb.h
SIGNATURES = {
    "afb_last_error": (ctypes.c_char_p, []),
    "afb_version": (_int, []),
    "afb_compiled_arch": (_int, []),
    "afb_edge_weights": (_int, [_i64, _p, _p, _p, _p, _p]),
    "afb_cone_create": (_int, [_pp, _i64, _i64, _p, _p, _p, _i64, _p, _i64, _int, _p]),
    "afb_cone_destroy": (None, [_p]),
    "afb_cone_sizes": (_int, [_p, _p, _p, _p, _p, _p, _p]),
    "afb_cone_export": (_int, [_p, _int, _int, _p, _p]),
    "afb_cone_set_weights": (_int, [_p, _int, _p, _p, _p, _f, _p]),
    "afb_cone_resting": (_int, [_p, _int, _p, _p]),
    "afb_cone_forward_workspace": (_sz, [_p, _int, _i64]),
    "afb_cone_forward": (_int, [_p, _int, _p, _i64, _i64, _p, _i64, _p, _sz, _p]),
    "afb_cone_forward_timed": (_int, [_p, _int, _p, _i64, _i64, _p, _i64, _p, _sz, _p, _p]),
    "afb_cone_forward_noalloc": (_int, [_p, _int, _p, _i64, _i64, _p, _i64, _p]),
    "afb_cone_status": (_int, [_p, _p, _int, _p]),
    "afb_cone_train_workspace": (_sz, [_p, _i64]),
    "afb_cone_forward_train": (_int, [_p, _p, _i64, _i64, _p, _i64, _p, _sz, _p]),
    "afb_cone_backward_workspace": (_sz, [_p, _i64]),
    "afb_cone_backward": (_int, [_p, _p, _i64, _i64, _p, _sz, _p, _i64, _p, _p, _p, _p, _sz, _p]),
    "afb_graph_status": (_int, [_p, _p, _int, _p]),
    "afb_graph_create": (_int, [_pp, _i64, _i64, _p, _p, _p]),
    "afb_graph_destroy": (None, [_p]),
    "afb_graph_forward_workspace": (_sz, [_p, _i64]),
    "afb_graph_forward": (_int, [_p, _p, _p, _p, _f, _p, _i64, _i64, _int, _p, _i64, _p, _sz, _p]),
    "afb_input_map_f16": (_int, [_i64, _i64, _i64, _p, _i64, _p, _i64, _p, _f, _p, _i64, _p, _p]),
    "afb_heads_split": (_int, [_i64, _i64, _p, _i64, _p, _p, _i64, _p]),
    "afb_readout_workspace": (_sz, [_i64, _i64]),
    "afb_readout_heads": (_int, [_i64, _i64, _p, _i64, _p, _p, _f, _f, _i64, _i64, _p, _p, _i64, _p, _p, _i64, _int, _p,
                                 _i64, _p, _sz, _p, _p]),
    "afb_gemm_workspace": (_sz, [_i64, _i64, _i64]),
    "afb_gemm_f32": (_int, [_i64, _i64, _i64, _f, _p, _i64, _int, _p, _i64, _int, _p, _int, _f, _p, _i64, _p, _sz, _p, _p]),
}

# the entry points of include/afb_probe.h (libafb_probe.so)
PROBE_SIGNATURES = {
    "afb_probe_gather_sink_words": (_i64, []),
    "afb_probe_gather": (_int, [_int, _p, _i64, _p, _i64, _p, _i64, _p]),
}

_lib = None
_probe = None


def load() -> ctypes.CDLL:
    """The loaded library; raises ImportError with the reason when it is absent or unloadable."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python __graft_entry__.py` (build) or "
                              f"`make -C {os.path.join(_HERE, 'csrc')}`; alphafly_b200 has no CPU path")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def load_probe() -> ctypes.CDLL:
    """bench.py's gather-ceiling probe library (built beside libafb.so by the same Makefile)."""
    global _probe
    if _probe is None:
        if not os.path.exists(PROBE_PATH):
            raise ImportError(f"{PROBE_PATH} is missing: build it with `make -C {os.path.join(_HERE, 'csrc')}`")
        lib = ctypes.CDLL(PROBE_PATH)
        for name, (res, args) in PROBE_SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _probe = lib
    return _probe


class AfbError(RuntimeError):
    """A failed call into libafb (argument check or CUDA error); the message is the library's."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


def check(code: int) -> None:
    if code != OK:
        raise AfbError(code, load().afb_last_error().decode())


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))
