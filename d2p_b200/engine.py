"""Which engine computed the problems: counters kept by libd2p_b200.

The fast kernels flag problems they cannot finish within their numeric range
(very low temperatures, extreme scores); the normalised log-domain kernel
recomputes those, and the plane engine takes whatever it flags in turn, as well
as shapes no fast kernel covers.  ``engine_counts`` reads the device-side
counters so that such fall-backs are visible (no reference counterpart: the
reference has one engine per family).
"""
from __future__ import annotations

import ctypes
import os

_LIB = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libd2p_b200.so")
_KEYS = ("logdomain_fixups", "plane_linear", "plane_affine")


def engine_counts() -> dict:
    """Counters of the current CUDA device, cumulative since the library was
    loaded: ``logdomain_fixups`` (linear problems the log-domain kernel
    recomputed after a linear-domain kernel flagged them), ``plane_linear`` and
    ``plane_affine`` (problems the plane engine computed).  Synchronises with
    the device."""
    lib = ctypes.CDLL(_LIB)
    fn = lib.d2p_engine_counts
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(ctypes.c_ulonglong), ctypes.c_int]
    out = (ctypes.c_ulonglong * len(_KEYS))()
    rc = fn(out, len(_KEYS))
    if rc != 0:
        lib.d2p_error_string.restype = ctypes.c_char_p
        lib.d2p_error_string.argtypes = [ctypes.c_int]
        raise RuntimeError(f"d2p_engine_counts failed: {lib.d2p_error_string(rc).decode()} (code {rc})")
    return dict(zip(_KEYS, (int(v) for v in out)))


_ENGINES = {"auto": 0, "plane": 1, "pipeline": 2}


def set_engine(name: str) -> str:
    """Select the engine for the whole process: ``"auto"`` (per shape, the
    default), ``"plane"`` (the general plane engine for every operator) or
    ``"pipeline"`` (the anti-diagonal row-block pipeline for linear value +
    marginals at every size).  The engines compute the same results; this
    exists to cross-check and time them.  Returns the previous setting."""
    if name not in _ENGINES:
        raise ValueError(f"engine must be one of {sorted(_ENGINES)}, got {name!r}")
    lib = ctypes.CDLL(_LIB)
    fn = lib.d2p_set_engine
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
    prev = ctypes.c_int(0)
    rc = fn(_ENGINES[name], ctypes.byref(prev))
    if rc != 0:
        raise RuntimeError(f"d2p_set_engine failed (code {rc})")
    return {v: k for k, v in _ENGINES.items()}[prev.value]


class use_engine:
    """``with use_engine("plane"): ...`` -- set_engine for a block."""

    def __init__(self, name: str):
        self.name = name
        self.prev = None

    def __enter__(self):
        self.prev = set_engine(self.name)
        return self

    def __exit__(self, *exc):
        set_engine(self.prev)
        return False
