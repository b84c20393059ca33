"""Parity checker for d2p_b200 -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg (``cpu_baseline`` and ``--impl reference``) import this package.  The
d2p_b200 product never imports, links or calls it.

Two CPU implementations sit behind one numpy interface:

* ``impl="f32"`` / ``impl="f64"`` -- ``sw_oracle.c``, a restatement of the
  reference CPU algorithms (src/sw/kernels_cpu.cpp, src/sw_affine/kernels_cpu.cpp)
  in float and in double precision (the double build is the noise-floor
  reference).
* ``impl="ref"`` -- the reference's own CPU kernels compiled from its sources
  into ``_ref/libref_sw_cpu.so`` by ``oracle/Makefile``.

The op-level orchestration mirrors the reference's CPU bindings
(src/sw/torch_cpu.cpp:140-520, src/sw_affine/torch_cpu.cpp): e.g. the
parameter Jacobian runs forward + backward to obtain dS/dtheta and then the
param-grad sweep; ``backward_full`` is HVP + one Jacobian per parameter,
reduced against the incoming gradient.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Dict, Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_D = ctypes.c_double

_libs: Dict[str, ctypes.CDLL] = {}


def build(quiet: bool = True) -> None:
    """Compile liboracle_sw.so (and _ref/ when the reference sources exist)."""
    out = subprocess.run(["make", "-C", _HERE], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout)


def _lib(name: str) -> ctypes.CDLL:
    if name in _libs:
        return _libs[name]
    if name == "oracle":
        path = os.path.join(_HERE, "liboracle_sw.so")
        if not os.path.exists(path):
            build()
    else:
        path = os.path.join(_HERE, "_ref", "libref_sw_cpu.so")
        if not os.path.exists(path):
            build()
        if not os.path.exists(path):
            raise FileNotFoundError("reference CPU build missing: " + path)
        import torch  # noqa: F401  (loads libc10 / libtorch_cpu the build links to)
    lib = ctypes.CDLL(path)
    _libs[name] = lib
    return lib


def ref_available() -> bool:
    try:
        _lib("ref")
        return True
    except (OSError, FileNotFoundError, RuntimeError):
        return False


def set_threads(n: int) -> None:
    """Thread count for both CPU paths (OpenMP for the restatement, ATen for ref)."""
    os.environ["OMP_NUM_THREADS"] = str(n)
    try:
        ctypes.CDLL("libgomp.so.1").omp_set_num_threads(int(n))
    except OSError:
        pass
    try:
        import torch

        torch.set_num_threads(int(n))
    except Exception:
        pass


# ----------------------------------------------------------------------------
# helpers
# ----------------------------------------------------------------------------

def _dt(impl: str):
    return np.float64 if impl == "f64" else np.float32


def _arr(x, dtype):
    return np.ascontiguousarray(np.asarray(x, dtype=dtype))


def _lens(lengths, B, L1, L2):
    if lengths is None:
        return np.ascontiguousarray(np.tile(np.array([[L1, L2]], np.int32), (B, 1)))
    return np.ascontiguousarray(np.asarray(lengths, dtype=np.int32).reshape(B, 2))


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_P)


def _fn(lib, name, argtypes):
    f = getattr(lib, name)
    f.argtypes = argtypes
    f.restype = None
    return f


# ----------------------------------------------------------------------------
# linear gap
# ----------------------------------------------------------------------------

def sw_linear(scores, lengths=None, gap=-1.0, T=1.0, impl="f32") -> dict:
    """value, marginals, grad_gap, grad_T (+ alpha) for soft_sw_with_grads."""
    dt = _dt(impl)
    s = _arr(scores, dt)
    B, L1, L2 = s.shape
    ln = _lens(lengths, B, L1, L2)
    A = (L1 + 1) * (L2 + 1)
    alpha = np.zeros((B, A), dt)
    value = np.zeros(B, dt)
    beta = np.zeros((B, A), dt)
    marg = np.zeros((B, L1, L2), dt)
    gg = np.zeros(B, dt)
    gT = np.zeros(B, dt)
    if impl == "ref":
        lib = _lib("ref")
        f = _fn(lib, "sw_regular_forward_cpu", [_P] * 4 + [_I] * 3 + [_F] * 2)
        f(_ptr(s), _ptr(alpha), _ptr(value), _ptr(ln), B, L1, L2, gap, T)
        g = _fn(lib, "sw_regular_backward_cpu", [_P] * 8 + [_I] * 3 + [_F] * 2)
        g(_ptr(alpha), _ptr(s), _ptr(value), _ptr(beta), _ptr(marg), _ptr(gg), _ptr(gT), _ptr(ln), B, L1, L2, gap, T)
    else:
        lib = _lib("oracle")
        R = _D if impl == "f64" else _F
        sfx = "_f64" if impl == "f64" else "_f32"
        f = _fn(lib, "oracle_sw_forward" + sfx, [_P, _P, _I, _I, _I, R, R, _P, _P])
        f(_ptr(s), _ptr(ln), B, L1, L2, gap, T, _ptr(alpha), _ptr(value))
        g = _fn(lib, "oracle_sw_backward" + sfx, [_P, _P, _I, _I, _I, R, R] + [_P] * 6)
        g(_ptr(s), _ptr(ln), B, L1, L2, gap, T, _ptr(alpha), _ptr(value), _ptr(beta), _ptr(marg), _ptr(gg), _ptr(gT))
    return {"value": value, "marginals": marg, "grad_gap": gg, "grad_T": gT, "alpha": alpha}


def sw_linear_hvp(scores, V, lengths=None, gap=-1.0, T=1.0, impl="f32") -> np.ndarray:
    dt = _dt(impl)
    s = _arr(scores, dt)
    v = _arr(V, dt)
    B, L1, L2 = s.shape
    ln = _lens(lengths, B, L1, L2)
    A = (L1 + 1) * (L2 + 1)
    alpha = np.zeros((B, A), dt)
    value = np.zeros(B, dt)
    w1, w2, w3 = (np.zeros((B, A), dt) for _ in range(3))
    H = np.zeros((B, L1, L2), dt)
    if impl == "ref":
        lib = _lib("ref")
        f = _fn(lib, "sw_regular_forward_cpu", [_P] * 4 + [_I] * 3 + [_F] * 2)
        f(_ptr(s), _ptr(alpha), _ptr(value), _ptr(ln), B, L1, L2, gap, T)
        dpart = np.zeros(B, dt)
        h = _fn(lib, "sw_regular_hvp_cpu", [_P] * 10 + [_I] * 3 + [_F] * 2)
        h(_ptr(alpha), _ptr(s), _ptr(value), _ptr(v), _ptr(w1), _ptr(dpart), _ptr(w2), _ptr(w3), _ptr(H), _ptr(ln),
          B, L1, L2, gap, T)
    else:
        lib = _lib("oracle")
        R = _D if impl == "f64" else _F
        sfx = "_f64" if impl == "f64" else "_f32"
        f = _fn(lib, "oracle_sw_forward" + sfx, [_P, _P, _I, _I, _I, R, R, _P, _P])
        f(_ptr(s), _ptr(ln), B, L1, L2, gap, T, _ptr(alpha), _ptr(value))
        h = _fn(lib, "oracle_sw_hvp" + sfx, [_P, _P, _P, _I, _I, _I, R, R] + [_P] * 6)
        h(_ptr(s), _ptr(v), _ptr(ln), B, L1, L2, gap, T, _ptr(alpha), _ptr(value), _ptr(w1), _ptr(w2), _ptr(w3),
          _ptr(H))
    return H


def sw_linear_param_jacobian(scores, param_type, lengths=None, gap=-1.0, T=1.0, impl="f32") -> np.ndarray:
    if param_type not in (0, 1):
        raise ValueError("param_type must be 0 or 1")
    dt = _dt(impl)
    s = _arr(scores, dt)
    B, L1, L2 = s.shape
    ln = _lens(lengths, B, L1, L2)
    base = sw_linear(s, ln, gap, T, impl)
    dS = base["grad_gap"] if param_type == 0 else base["grad_T"]
    A = (L1 + 1) * (L2 + 1)
    w1, w2, w3 = (np.zeros((B, A), dt) for _ in range(3))
    dP = np.zeros((B, L1, L2), dt)
    alpha, value = base["alpha"], base["value"]
    if impl == "ref":
        lib = _lib("ref")
        p = _fn(lib, "sw_regular_param_grad_cpu", [_P] * 9 + [_I] * 3 + [_F] * 2 + [_I])
        p(_ptr(alpha), _ptr(s), _ptr(value), _ptr(dS), _ptr(w1), _ptr(w2), _ptr(w3), _ptr(dP), _ptr(ln), B, L1, L2,
          gap, T, param_type)
    else:
        lib = _lib("oracle")
        R = _D if impl == "f64" else _F
        sfx = "_f64" if impl == "f64" else "_f32"
        p = _fn(lib, "oracle_sw_param_grad" + sfx, [_P, _P, _I, _I, _I, R, R] + [_P] * 7 + [_I])
        p(_ptr(s), _ptr(ln), B, L1, L2, gap, T, _ptr(alpha), _ptr(value), _ptr(dS), _ptr(w1), _ptr(w2), _ptr(w3),
          _ptr(dP), param_type)
    return dP


def sw_linear_backward_full(scores, grad_alignment, lengths=None, gap=-1.0, T=1.0, impl="f32"):
    """(grad_scores, grad_gap[1], grad_T[1]) as soft_sw_backward_full (torch_cpu.cpp:440-520)."""
    dt = _dt(impl)
    G = _arr(grad_alignment, dt)
    gs = sw_linear_hvp(scores, G, lengths, gap, T, impl)
    jg = sw_linear_param_jacobian(scores, 0, lengths, gap, T, impl)
    jt = sw_linear_param_jacobian(scores, 1, lengths, gap, T, impl)
    return gs, np.array([(G * jg).sum()], dt), np.array([(G * jt).sum()], dt)


# ----------------------------------------------------------------------------
# affine gap
# ----------------------------------------------------------------------------

def sw_affine(scores, lengths=None, gap_open=-2.0, gap_ext=-0.5, T=1.0, impl="f32") -> dict:
    dt = _dt(impl)
    s = _arr(scores, dt)
    B, L1, L2 = s.shape
    ln = _lens(lengths, B, L1, L2)
    A = 3 * (L1 + 1) * (L2 + 1)
    alpha = np.zeros((B, A), dt)
    value = np.zeros(B, dt)
    beta = np.zeros((B, A), dt)
    marg = np.zeros((B, L1, L2), dt)
    go_, ge_, gT = (np.zeros(B, dt) for _ in range(3))
    if impl == "ref":
        lib = _lib("ref")
        f = _fn(lib, "sw_affine_forward_cpu", [_P] * 4 + [_I] * 3 + [_F] * 3)
        f(_ptr(s), _ptr(alpha), _ptr(value), _ptr(ln), B, L1, L2, gap_open, gap_ext, T)
        g = _fn(lib, "sw_affine_backward_cpu", [_P] * 9 + [_I] * 3 + [_F] * 3)
        g(_ptr(alpha), _ptr(s), _ptr(value), _ptr(beta), _ptr(marg), _ptr(go_), _ptr(ge_), _ptr(gT), _ptr(ln),
          B, L1, L2, gap_open, gap_ext, T)
    else:
        lib = _lib("oracle")
        R = _D if impl == "f64" else _F
        sfx = "_f64" if impl == "f64" else "_f32"
        f = _fn(lib, "oracle_sw_affine_forward" + sfx, [_P, _P, _I, _I, _I, R, R, R, _P, _P])
        f(_ptr(s), _ptr(ln), B, L1, L2, gap_open, gap_ext, T, _ptr(alpha), _ptr(value))
        g = _fn(lib, "oracle_sw_affine_backward" + sfx, [_P, _P, _I, _I, _I, R, R, R] + [_P] * 7)
        g(_ptr(s), _ptr(ln), B, L1, L2, gap_open, gap_ext, T, _ptr(alpha), _ptr(value), _ptr(beta), _ptr(marg),
          _ptr(go_), _ptr(ge_), _ptr(gT))
    return {"value": value, "marginals": marg, "grad_open": go_, "grad_ext": ge_, "grad_T": gT, "alpha": alpha}


def sw_affine_hvp(scores, V, lengths=None, gap_open=-2.0, gap_ext=-0.5, T=1.0, impl="f32") -> np.ndarray:
    dt = _dt(impl)
    s = _arr(scores, dt)
    v = _arr(V, dt)
    B, L1, L2 = s.shape
    ln = _lens(lengths, B, L1, L2)
    A = 3 * (L1 + 1) * (L2 + 1)
    alpha = np.zeros((B, A), dt)
    value = np.zeros(B, dt)
    w1, w2, w3 = (np.zeros((B, A), dt) for _ in range(3))
    H = np.zeros((B, L1, L2), dt)
    if impl == "ref":
        lib = _lib("ref")
        f = _fn(lib, "sw_affine_forward_cpu", [_P] * 4 + [_I] * 3 + [_F] * 3)
        f(_ptr(s), _ptr(alpha), _ptr(value), _ptr(ln), B, L1, L2, gap_open, gap_ext, T)
        dpart = np.zeros(B, dt)
        h = _fn(lib, "sw_affine_hvp_cpu", [_P] * 9 + [_I] * 3 + [_F] * 3)
        h(_ptr(alpha), _ptr(s), _ptr(value), _ptr(v), _ptr(w1), _ptr(dpart), _ptr(w3), _ptr(H), _ptr(ln),
          B, L1, L2, gap_open, gap_ext, T)
    else:
        lib = _lib("oracle")
        R = _D if impl == "f64" else _F
        sfx = "_f64" if impl == "f64" else "_f32"
        f = _fn(lib, "oracle_sw_affine_forward" + sfx, [_P, _P, _I, _I, _I, R, R, R, _P, _P])
        f(_ptr(s), _ptr(ln), B, L1, L2, gap_open, gap_ext, T, _ptr(alpha), _ptr(value))
        h = _fn(lib, "oracle_sw_affine_hvp" + sfx, [_P, _P, _P, _I, _I, _I, R, R, R] + [_P] * 6)
        h(_ptr(s), _ptr(v), _ptr(ln), B, L1, L2, gap_open, gap_ext, T, _ptr(alpha), _ptr(value), _ptr(w1),
          _ptr(w2), _ptr(w3), _ptr(H))
    return H


def sw_affine_param_jacobian(scores, param_type, lengths=None, gap_open=-2.0, gap_ext=-0.5, T=1.0,
                             impl="f32") -> np.ndarray:
    if param_type not in (0, 1, 2):
        raise ValueError("param_type must be 0, 1, or 2")
    dt = _dt(impl)
    s = _arr(scores, dt)
    B, L1, L2 = s.shape
    ln = _lens(lengths, B, L1, L2)
    base = sw_affine(s, ln, gap_open, gap_ext, T, impl)
    dS = [base["grad_open"], base["grad_ext"], base["grad_T"]][param_type]
    A = 3 * (L1 + 1) * (L2 + 1)
    w1, w2, w3 = (np.zeros((B, A), dt) for _ in range(3))
    dP = np.zeros((B, L1, L2), dt)
    alpha, value = base["alpha"], base["value"]
    if impl == "ref":
        lib = _lib("ref")
        p = _fn(lib, "sw_affine_param_grad_cpu", [_P] * 9 + [_I] * 3 + [_F] * 3 + [_I])
        p(_ptr(alpha), _ptr(s), _ptr(value), _ptr(dS), _ptr(w1), _ptr(w2), _ptr(w3), _ptr(dP), _ptr(ln), B, L1, L2,
          gap_open, gap_ext, T, param_type)
    else:
        lib = _lib("oracle")
        R = _D if impl == "f64" else _F
        sfx = "_f64" if impl == "f64" else "_f32"
        p = _fn(lib, "oracle_sw_affine_param_grad" + sfx, [_P, _P, _I, _I, _I, R, R, R] + [_P] * 7 + [_I])
        p(_ptr(s), _ptr(ln), B, L1, L2, gap_open, gap_ext, T, _ptr(alpha), _ptr(value), _ptr(dS), _ptr(w1),
          _ptr(w2), _ptr(w3), _ptr(dP), param_type)
    return dP


def sw_affine_backward_full(scores, grad_alignment, lengths=None, gap_open=-2.0, gap_ext=-0.5, T=1.0,
                            impl="f32"):
    dt = _dt(impl)
    G = _arr(grad_alignment, dt)
    gs = sw_affine_hvp(scores, G, lengths, gap_open, gap_ext, T, impl)
    outs = [gs]
    for p in range(3):
        jac = sw_affine_param_jacobian(scores, p, lengths, gap_open, gap_ext, T, impl)
        outs.append(np.array([(G * jac).sum()], dt))
    return tuple(outs)


# ----------------------------------------------------------------------------
# Needleman-Wunsch (global alignment, linear gap): nw_oracle.c, or the
# reference's src/nw/kernels_cpu.cpp; op-level orchestration as
# src/nw/torch_cpu.cpp:294-520
# ----------------------------------------------------------------------------

def _nw_call(impl, name_ref, name_oracle):
    if impl == "ref":
        return _lib("ref"), name_ref, _F
    return _lib("oracle"), name_oracle + ("_f64" if impl == "f64" else "_f32"), (_D if impl == "f64" else _F)


def nw_linear(scores, lengths=None, gap=-1.0, T=1.0, impl="f32") -> dict:
    """value, marginals, grad_gap, grad_T (+ alpha) as soft_nw_with_grads."""
    dt = _dt(impl)
    s = _arr(scores, dt)
    B, L1, L2 = s.shape
    ln = _lens(lengths, B, L1, L2)
    A = (L1 + 1) * (L2 + 1)
    alpha = np.zeros((B, A), dt)
    value = np.zeros(B, dt)
    beta = np.zeros((B, A), dt)
    marg = np.zeros((B, L1, L2), dt)
    gg = np.zeros(B, dt)
    gT = np.zeros(B, dt)
    lib, name, R = _nw_call(impl, "nw_forward_cpu", "oracle_nw_forward")
    if impl == "ref":
        _fn(lib, name, [_P] * 4 + [_I] * 3 + [_F] * 2)(_ptr(s), _ptr(alpha), _ptr(value), _ptr(ln), B, L1, L2, gap,
                                                        T)
        _fn(lib, "nw_backward_cpu", [_P] * 8 + [_I] * 3 + [_F] * 2)(
            _ptr(alpha), _ptr(s), _ptr(value), _ptr(beta), _ptr(marg), _ptr(gg), _ptr(gT), _ptr(ln), B, L1, L2, gap,
            T)
    else:
        _fn(lib, name, [_P, _P, _I, _I, _I, R, R, _P, _P])(_ptr(s), _ptr(ln), B, L1, L2, gap, T, _ptr(alpha),
                                                          _ptr(value))
        g = _fn(lib, name.replace("forward", "backward"), [_P, _P, _I, _I, _I, R, R] + [_P] * 6)
        g(_ptr(s), _ptr(ln), B, L1, L2, gap, T, _ptr(alpha), _ptr(value), _ptr(beta), _ptr(marg), _ptr(gg), _ptr(gT))
    return {"value": value, "marginals": marg, "grad_gap": gg, "grad_T": gT, "alpha": alpha}


def nw_linear_hvp(scores, V, lengths=None, gap=-1.0, T=1.0, impl="f32") -> np.ndarray:
    dt = _dt(impl)
    s = _arr(scores, dt)
    v = _arr(V, dt)
    B, L1, L2 = s.shape
    ln = _lens(lengths, B, L1, L2)
    A = (L1 + 1) * (L2 + 1)
    base = nw_linear(s, ln, gap, T, impl)
    alpha, value = base["alpha"], base["value"]
    w1, w2, w3 = (np.zeros((B, A), dt) for _ in range(3))
    H = np.zeros((B, L1, L2), dt)
    lib, name, R = _nw_call(impl, "nw_hvp_cpu", "oracle_nw_hvp")
    if impl == "ref":
        dsc = np.zeros(B, dt)
        _fn(lib, name, [_P] * 10 + [_I] * 3 + [_F] * 2)(
            _ptr(alpha), _ptr(s), _ptr(value), _ptr(v), _ptr(w1), _ptr(dsc), _ptr(w2), _ptr(w3), _ptr(H), _ptr(ln),
            B, L1, L2, gap, T)
    else:
        _fn(lib, name, [_P, _P, _P, _I, _I, _I, R, R] + [_P] * 5)(
            _ptr(s), _ptr(v), _ptr(ln), B, L1, L2, gap, T, _ptr(alpha), _ptr(w1), _ptr(w2), _ptr(w3), _ptr(H))
    return H


def nw_linear_param_jacobian(scores, param_type, lengths=None, gap=-1.0, T=1.0, impl="f32") -> np.ndarray:
    """dP/dgap (param_type 0) or dP/dT (1), as soft_nw_param_jacobian_cpu."""
    if param_type not in (0, 1):
        raise ValueError("param_type must be 0 or 1")
    dt = _dt(impl)
    s = _arr(scores, dt)
    B, L1, L2 = s.shape
    ln = _lens(lengths, B, L1, L2)
    base = nw_linear(s, ln, gap, T, impl)
    dS = base["grad_gap"] if param_type == 0 else base["grad_T"]
    alpha, value = base["alpha"], base["value"]
    A = (L1 + 1) * (L2 + 1)
    w1, w2, w3 = (np.zeros((B, A), dt) for _ in range(3))
    dP = np.zeros((B, L1, L2), dt)
    lib, name, R = _nw_call(impl, "nw_param_grad_cpu", "oracle_nw_param_grad")
    if impl == "ref":
        _fn(lib, name, [_P] * 9 + [_I] * 3 + [_F] * 2 + [_I])(
            _ptr(alpha), _ptr(s), _ptr(value), _ptr(dS), _ptr(w1), _ptr(w2), _ptr(w3), _ptr(dP), _ptr(ln), B, L1, L2,
            gap, T, param_type)
    else:
        _fn(lib, name, [_P, _P, _I, _I, _I, R, R] + [_P] * 5 + [_I])(
            _ptr(s), _ptr(ln), B, L1, L2, gap, T, _ptr(alpha), _ptr(w1), _ptr(w2), _ptr(w3), _ptr(dP), param_type)
    return dP


def nw_linear_backward_full(scores, grad_alignment, lengths=None, gap=-1.0, T=1.0, impl="f32"):
    """(grad_scores, grad_gap[1], grad_T[1]) as soft_nw_backward_full_cpu (torch_cpu.cpp:430-520)."""
    dt = _dt(impl)
    G = _arr(grad_alignment, dt)
    gs = nw_linear_hvp(scores, G, lengths, gap, T, impl)
    jg = nw_linear_param_jacobian(scores, 0, lengths, gap, T, impl)
    jt = nw_linear_param_jacobian(scores, 1, lengths, gap, T, impl)
    return gs, np.array([(G * jg).sum()], dt), np.array([(G * jt).sum()], dt)


# ----------------------------------------------------------------------------
# Needleman-Wunsch, affine gaps: nw_affine_oracle.c, or the reference's
# src/nw_affine/kernels_cpu.cpp; op-level orchestration as
# src/nw_affine/torch_cpu.cpp:180-580
# ----------------------------------------------------------------------------

def _nwa_call(impl, name_ref, name_oracle):
    if impl == "ref":
        return _lib("ref"), name_ref, _F
    return _lib("oracle"), name_oracle + ("_f64" if impl == "f64" else "_f32"), (_D if impl == "f64" else _F)


def nw_affine(scores, lengths=None, gap_open=-2.0, gap_ext=-0.5, T=1.0, impl="f32") -> dict:
    """value, marginals, grad_open, grad_ext, grad_T (+ alpha) as soft_nw_affine_with_grads."""
    dt = _dt(impl)
    s = _arr(scores, dt)
    B, L1, L2 = s.shape
    ln = _lens(lengths, B, L1, L2)
    A3 = 3 * (L1 + 1) * (L2 + 1)
    alpha = np.zeros((B, A3), dt)
    beta = np.zeros((B, A3), dt)
    value = np.zeros(B, dt)
    marg = np.zeros((B, L1, L2), dt)
    go_, ge_, gT = (np.zeros(B, dt) for _ in range(3))
    lib, name, R = _nwa_call(impl, "nw_affine_forward_cpu", "oracle_nwa_forward")
    if impl == "ref":
        _fn(lib, name, [_P] * 4 + [_I] * 3 + [_F] * 3)(_ptr(s), _ptr(alpha), _ptr(value), _ptr(ln), B, L1, L2,
                                                        gap_open, gap_ext, T)
        _fn(lib, "nw_affine_backward_cpu", [_P] * 9 + [_I] * 3 + [_F] * 3)(
            _ptr(alpha), _ptr(s), _ptr(value), _ptr(beta), _ptr(marg), _ptr(go_), _ptr(ge_), _ptr(gT), _ptr(ln),
            B, L1, L2, gap_open, gap_ext, T)
    else:
        _fn(lib, name, [_P, _P, _I, _I, _I, R, R, R, _P, _P])(_ptr(s), _ptr(ln), B, L1, L2, gap_open, gap_ext, T,
                                                             _ptr(alpha), _ptr(value))
        _fn(lib, name.replace("forward", "backward"), [_P, _P, _I, _I, _I, R, R, R] + [_P] * 7)(
            _ptr(s), _ptr(ln), B, L1, L2, gap_open, gap_ext, T, _ptr(alpha), _ptr(value), _ptr(beta), _ptr(marg),
            _ptr(go_), _ptr(ge_), _ptr(gT))
    return {"value": value, "marginals": marg, "grad_open": go_, "grad_ext": ge_, "grad_T": gT, "alpha": alpha}


def nw_affine_hvp(scores, V, lengths=None, gap_open=-2.0, gap_ext=-0.5, T=1.0, impl="f32") -> np.ndarray:
    dt = _dt(impl)
    s = _arr(scores, dt)
    v = _arr(V, dt)
    B, L1, L2 = s.shape
    ln = _lens(lengths, B, L1, L2)
    A3 = 3 * (L1 + 1) * (L2 + 1)
    base = nw_affine(s, ln, gap_open, gap_ext, T, impl)
    alpha, value = base["alpha"], base["value"]
    w1, w2, w3 = (np.zeros((B, A3), dt) for _ in range(3))
    H = np.zeros((B, L1, L2), dt)
    lib, name, R = _nwa_call(impl, "nw_affine_hvp_cpu", "oracle_nwa_hvp")
    if impl == "ref":
        dsc = np.zeros(B, dt)
        _fn(lib, name, [_P] * 10 + [_I] * 3 + [_F] * 3)(
            _ptr(alpha), _ptr(s), _ptr(value), _ptr(v), _ptr(w1), _ptr(dsc), _ptr(w2), _ptr(w3), _ptr(H), _ptr(ln),
            B, L1, L2, gap_open, gap_ext, T)
    else:
        _fn(lib, name, [_P, _P, _P, _I, _I, _I, R, R, R] + [_P] * 5)(
            _ptr(s), _ptr(v), _ptr(ln), B, L1, L2, gap_open, gap_ext, T, _ptr(alpha), _ptr(w1), _ptr(w2), _ptr(w3),
            _ptr(H))
    return H


def nw_affine_param_jacobian(scores, param_type, lengths=None, gap_open=-2.0, gap_ext=-0.5, T=1.0,
                             impl="f32") -> np.ndarray:
    """dP/dgap_open (param_type 0), dP/dgap_ext (1) or dP/dT (2)."""
    if param_type not in (0, 1, 2):
        raise ValueError("param_type must be 0, 1, or 2")
    dt = _dt(impl)
    s = _arr(scores, dt)
    B, L1, L2 = s.shape
    ln = _lens(lengths, B, L1, L2)
    base = nw_affine(s, ln, gap_open, gap_ext, T, impl)
    dS = base[("grad_open", "grad_ext", "grad_T")[param_type]]
    alpha, value = base["alpha"], base["value"]
    A3 = 3 * (L1 + 1) * (L2 + 1)
    w1, w2, w3 = (np.zeros((B, A3), dt) for _ in range(3))
    dP = np.zeros((B, L1, L2), dt)
    lib, name, R = _nwa_call(impl, "nw_affine_param_grad_cpu", "oracle_nwa_param_grad")
    if impl == "ref":
        _fn(lib, name, [_P] * 9 + [_I] * 3 + [_F] * 3 + [_I])(
            _ptr(alpha), _ptr(s), _ptr(value), _ptr(dS), _ptr(w1), _ptr(w2), _ptr(w3), _ptr(dP), _ptr(ln), B, L1, L2,
            gap_open, gap_ext, T, param_type)
    else:
        _fn(lib, name, [_P, _P, _I, _I, _I, R, R, R] + [_P] * 5 + [_I])(
            _ptr(s), _ptr(ln), B, L1, L2, gap_open, gap_ext, T, _ptr(alpha), _ptr(w1), _ptr(w2), _ptr(w3), _ptr(dP),
            param_type)
    return dP


def nw_affine_backward_full(scores, grad_alignment, lengths=None, gap_open=-2.0, gap_ext=-0.5, T=1.0,
                            impl="f32"):
    """(grad_scores, grad_open[1], grad_ext[1], grad_T[1]) as soft_nw_affine_backward_full_cpu
    (src/nw_affine/torch_cpu.cpp:474-570)."""
    dt = _dt(impl)
    G = _arr(grad_alignment, dt)
    gs = nw_affine_hvp(scores, G, lengths, gap_open, gap_ext, T, impl)
    js = [nw_affine_param_jacobian(scores, p, lengths, gap_open, gap_ext, T, impl) for p in (0, 1, 2)]
    return (gs,) + tuple(np.array([(G * j).sum()], dt) for j in js)


# ----------------------------------------------------------------------------
# soft DTW: dtw_oracle.c, or the reference's src/dtw/kernels_cpu.cpp;
# op-level orchestration as src/dtw/torch_cpu.cpp (bandwidth < 0: no band)
# ----------------------------------------------------------------------------
_L = ctypes.c_int64


def _dtw_call(impl, name_ref, name_oracle):
    if impl == "ref":
        return _lib("ref"), name_ref, _F
    return _lib("oracle"), name_oracle + ("_f64" if impl == "f64" else "_f32"), (_D if impl == "f64" else _F)


def dtw(costs, lengths=None, T=1.0, bandwidth=-1, impl="f32") -> dict:
    """value, marginals (visit probabilities), grad_T (+ alpha) as soft_dtw_with_grads."""
    dt = _dt(impl)
    c = _arr(costs, dt)
    B, L1, L2 = c.shape
    ln = _lens(lengths, B, L1, L2)
    A = (L1 + 1) * (L2 + 1)
    alpha = np.zeros((B, A), dt)
    beta = np.zeros((B, A), dt)
    value = np.zeros(B, dt)
    marg = np.zeros((B, L1, L2), dt)
    gT = np.zeros(B, dt)
    lib, name, R = _dtw_call(impl, "dtw_forward_cpu", "oracle_dtw_forward")
    if impl == "ref":
        _fn(lib, name, [_P] * 4 + [_I] * 3 + [_F, _L])(_ptr(c), _ptr(alpha), _ptr(value), _ptr(ln), B, L1, L2, T,
                                                        bandwidth)
        _fn(lib, "dtw_backward_cpu", [_P] * 7 + [_I] * 3 + [_F, _L])(
            _ptr(alpha), _ptr(c), _ptr(value), _ptr(beta), _ptr(marg), _ptr(gT), _ptr(ln), B, L1, L2, T, bandwidth)
    else:
        _fn(lib, name, [_P, _P, _I, _I, _I, R, _L, _P, _P])(_ptr(c), _ptr(ln), B, L1, L2, T, bandwidth, _ptr(alpha),
                                                           _ptr(value))
        _fn(lib, name.replace("forward", "backward"), [_P, _P, _I, _I, _I, R, _L] + [_P] * 4)(
            _ptr(c), _ptr(ln), B, L1, L2, T, bandwidth, _ptr(alpha), _ptr(beta), _ptr(marg), _ptr(gT))
    return {"value": value, "marginals": marg, "grad_T": gT, "alpha": alpha}


def dtw_hvp(costs, V, lengths=None, T=1.0, bandwidth=-1, impl="f32") -> np.ndarray:
    dt = _dt(impl)
    c = _arr(costs, dt)
    v = _arr(V, dt)
    B, L1, L2 = c.shape
    ln = _lens(lengths, B, L1, L2)
    base = dtw(c, ln, T, bandwidth, impl)
    alpha, value = base["alpha"], base["value"]
    A = (L1 + 1) * (L2 + 1)
    w1, w2, w3 = (np.zeros((B, A), dt) for _ in range(3))
    H = np.zeros((B, L1, L2), dt)
    lib, name, R = _dtw_call(impl, "dtw_hvp_cpu", "oracle_dtw_hvp")
    if impl == "ref":
        dsc = np.zeros(B, dt)
        _fn(lib, name, [_P] * 10 + [_I] * 3 + [_F, _L])(
            _ptr(alpha), _ptr(c), _ptr(value), _ptr(v), _ptr(w1), _ptr(dsc), _ptr(w2), _ptr(w3), _ptr(H), _ptr(ln),
            B, L1, L2, T, bandwidth)
    else:
        _fn(lib, name, [_P, _P, _P, _I, _I, _I, R, _L] + [_P] * 5)(
            _ptr(c), _ptr(v), _ptr(ln), B, L1, L2, T, bandwidth, _ptr(alpha), _ptr(w1), _ptr(w2), _ptr(w3), _ptr(H))
    return H


def dtw_param_jacobian(costs, lengths=None, T=1.0, bandwidth=-1, impl="f32") -> np.ndarray:
    """dP/dT, as soft_dtw_param_jacobian."""
    dt = _dt(impl)
    c = _arr(costs, dt)
    B, L1, L2 = c.shape
    ln = _lens(lengths, B, L1, L2)
    base = dtw(c, ln, T, bandwidth, impl)
    alpha, value = base["alpha"], base["value"]
    A = (L1 + 1) * (L2 + 1)
    w1, w2, w3 = (np.zeros((B, A), dt) for _ in range(3))
    dP = np.zeros((B, L1, L2), dt)
    lib, name, R = _dtw_call(impl, "dtw_param_grad_cpu", "oracle_dtw_param_grad")
    if impl == "ref":
        _fn(lib, name, [_P] * 8 + [_I] * 3 + [_F, _L])(
            _ptr(alpha), _ptr(c), _ptr(value), _ptr(w1), _ptr(w2), _ptr(w3), _ptr(dP), _ptr(ln), B, L1, L2, T,
            bandwidth)
    else:
        _fn(lib, name, [_P, _P, _I, _I, _I, R, _L] + [_P] * 5)(
            _ptr(c), _ptr(ln), B, L1, L2, T, bandwidth, _ptr(alpha), _ptr(w1), _ptr(w2), _ptr(w3), _ptr(dP))
    return dP


def dtw_backward_full(costs, grad_alignment, lengths=None, T=1.0, bandwidth=-1, impl="f32"):
    """(grad_costs, grad_T[1]) as soft_dtw_backward_full (src/dtw/torch_cpu.cpp)."""
    dt = _dt(impl)
    G = _arr(grad_alignment, dt)
    gs = dtw_hvp(costs, G, lengths, T, bandwidth, impl)
    j = dtw_param_jacobian(costs, lengths, T, bandwidth, impl)
    return gs, np.array([(G * j).sum()], dt)
