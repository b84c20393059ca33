"""Shared helpers for the GPU parity tests (test infrastructure)."""
from __future__ import annotations

import json
import os

import numpy as np
import torch

# BASELINE.json tolerances for fp32: value, marginals, gradients and HVPs
# within 1e-5 relative / 1e-6 absolute; bf16 inputs compared after upcast
# within 1e-2 relative.
RTOL = 1e-5
ATOL = 1e-6
BF16_RTOL = 1e-2


def scores(B, L1, L2, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(B, L1, L2, generator=g) * scale


def plane_engine(op, s, *params):
    """Outputs of `op(scores, *params, None)` computed by the plane engine
    (d2p_b200.use_engine("plane")): bitwise what the plane engine gives for a
    problem a fast kernel flags."""
    from d2p_b200.engine import use_engine

    with use_engine("plane"):
        outs = op(s, *params, None)
        torch.cuda.synchronize()
    return list(outs)


def lengths_for(B, L1, L2, seed=1, lo=1):
    g = torch.Generator().manual_seed(seed)
    l1 = torch.randint(lo, L1 + 1, (B,), generator=g)
    l2 = torch.randint(lo, L2 + 1, (B,), generator=g)
    return torch.stack([l1, l2], 1).to(torch.int32)


def err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b))) if a.size else 0.0


# Where the reference's own fp32 result misses the tolerance against fp64 (the
# fp32 noise floor of a long logsumexp chain: 2.5e-5 absolute on 512x512
# marginals already), no fp32 kernel can meet it.  Such a result is judged
# against that floor instead: its error against fp64 may be at most
# NOISE_FACTOR x the reference's own fp32 error, i.e. no worse than the
# reference.
NOISE_FACTOR = 1.0


def _log(rec):
    """Append one parity record (JSON line) to $D2P_PARITY_LOG when it is set."""
    path = os.environ.get("D2P_PARITY_LOG")
    if not path:
        return
    rec["test"] = os.environ.get("PYTEST_CURRENT_TEST", "").split(" ")[0]
    with open(path, "a") as f:
        f.write(json.dumps(rec) + "\n")


def check(name, ours, ref64, ref32=None, rtol=RTOL, atol=ATOL, noise=NOISE_FACTOR):
    """ours within (rtol, atol) of the fp64 oracle -- or, where the reference's
    own fp32 result is further than that from fp64, with an fp64 error no
    larger than `noise` x the reference's."""
    ours = np.asarray(ours.detach().cpu().numpy() if isinstance(ours, torch.Tensor) else ours, np.float64)
    r64 = np.asarray(ref64, np.float64)
    assert ours.shape == r64.shape, (name, ours.shape, r64.shape)
    assert np.all(np.isfinite(ours)), f"{name}: non-finite output"
    ok = np.allclose(ours, r64, rtol=rtol, atol=atol)
    e_ours = err(ours, r64)
    e_ref = err(ref32, r64) if ref32 is not None else None
    _log({"name": name, "ours": e_ours, "ref32": e_ref, "tol_ok": bool(ok), "rtol": rtol, "atol": atol,
          "scale": float(np.max(np.abs(r64))) if r64.size else 0.0})
    if ok:
        return e_ours
    msg = f"{name}: max|ours - f64| = {e_ours:.3e} exceeds rtol={rtol}, atol={atol}"
    if e_ref is not None:
        msg += f"; reference fp32 vs f64 = {e_ref:.3e}"
        ref_ok = np.allclose(np.asarray(ref32, np.float64), r64, rtol=rtol, atol=atol)
        assert not ref_ok, msg + " (the reference itself meets the tolerance)"
        assert e_ours <= noise * e_ref, msg
        return e_ours
    raise AssertionError(msg)
