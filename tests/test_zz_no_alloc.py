"""d2p_sw_forward_backward_static: the allocation-free linear forward/backward.

Called through the C ABI with ctypes and compared against
d2p_sw_forward_backward (caller workspace) on the same inputs, for two calls in
a row with different inputs, so a stale scratch state would show.  This file is
collected last on purpose: the entry point's per-device set-up must also work
after the other tests have used the device.
"""
import ctypes
import os

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "d2p_b200", "libd2p_b200.so")
STATIC_BYTES = 64 * 1024 * 1024
RTOL, ATOL = 1e-5, 1e-6

P = ctypes.c_void_p
F = ctypes.c_float
I = ctypes.c_int


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(LIB):
        from d2p_b200 import _build

        _build.build_cuda_lib()
    L = ctypes.CDLL(LIB)
    L.d2p_sw_forward_backward_static.restype = I
    L.d2p_sw_forward_backward_static.argtypes = [P, P, I, I, I, F, F, P, P, P, P, P, P, P]
    L.d2p_sw_forward_backward.restype = I
    L.d2p_sw_forward_backward.argtypes = [P, P, I, I, I, F, F, P, P, P, P, P, P, P, ctypes.c_size_t, P]
    L.d2p_sw_workspace_bytes.restype = ctypes.c_size_t
    L.d2p_sw_workspace_bytes.argtypes = [I] * 5
    return L


def test_rejects_sizes_beyond_static_scratch(lib):
    """Too-large problems are refused on the host, before any device call."""
    B, L1, L2 = 256, 512, 512
    assert lib.d2p_sw_workspace_bytes(0, 0, B, L1, L2) > STATIC_BYTES
    rc = lib.d2p_sw_forward_backward_static(P(16), None, B, L1, L2, -1.0, 1.0, None, None, None, None,
                                           None, None, None)
    assert rc == 1002  # D2P_ERR_WORKSPACE_TOO_SMALL


def _run(lib, fn_static, s, ln, gap, T, grads=True):
    """One call; without `grads` no dS/dgap, dS/dT pointers are passed, which
    sends the call through the value + marginals kernel instead of the
    gradient sweep."""
    import torch

    B, L1, L2 = s.shape
    dev = s.device
    v = torch.empty(B, device=dev)
    m = torch.empty(B, L1, L2, device=dev)
    gg = torch.zeros(B, device=dev)
    gt = torch.zeros(B, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    lp = P(ln.data_ptr()) if ln is not None else None
    args = [P(s.data_ptr()), lp, B, L1, L2, gap, T, None, None, P(v.data_ptr()), P(m.data_ptr()),
            P(gg.data_ptr()) if grads else None, P(gt.data_ptr()) if grads else None]
    if fn_static:
        rc = lib.d2p_sw_forward_backward_static(*args, P(st))
    else:
        nb = lib.d2p_sw_workspace_bytes(0, 0, B, L1, L2)
        ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=dev)
        rc = lib.d2p_sw_forward_backward(*args, P(ws.data_ptr()), nb, P(st))
    assert rc == 0, rc
    torch.cuda.synchronize()
    return v.cpu(), m.cpu(), gg.cpu(), gt.cpu()


def _case(B, L1, L2, seed, ragged, device):
    import torch

    g = torch.Generator().manual_seed(seed)
    s = torch.randn(B, L1, L2, generator=g, dtype=torch.float32).to(device)
    ln = None
    if ragged:
        l1 = torch.randint(1, L1 + 1, (B,), generator=g)
        l2 = torch.randint(1, L2 + 1, (B,), generator=g)
        ln = torch.stack([l1, l2], 1).to(torch.int32).to(device)
    return s, ln


@pytest.mark.gpu
@pytest.mark.parametrize("B,L1,L2,ragged,grads", [
    (8, 96, 128, False, True), (5, 70, 66, True, True), (3, 40, 37, True, True),
    # value + marginals only: the linear-domain kernel runs in the scratch
    (8, 96, 128, False, False), (5, 70, 64, True, False),
    # few large problems: each is spread over several CTAs, whose progress
    # words and partition partials also live in the scratch (cleared per call)
    (2, 1024, 1024, False, False),
])
def test_static_matches_workspace_entry_point(lib, cuda_device, B, L1, L2, ragged, grads):
    import torch

    assert lib.d2p_sw_workspace_bytes(0, 0, B, L1, L2) <= STATIC_BYTES
    for call in range(2):  # two calls in a row, different inputs
        s, ln = _case(B, L1, L2, seed=1000 * call + L1 + L2, ragged=ragged, device=cuda_device)
        gap, T = -0.5 - 0.25 * call, 1.0 - 0.3 * call
        got = _run(lib, True, s, ln, gap, T, grads)
        ref = _run(lib, False, s, ln, gap, T, grads)
        for name, a, b in zip(("value", "marginals", "grad_gap", "grad_T"), got, ref):
            assert torch.isfinite(a).all(), name
            np.testing.assert_allclose(a.numpy(), b.numpy(), rtol=RTOL, atol=ATOL, err_msg=f"call {call}: {name}")
