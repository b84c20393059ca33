"""Bounded device waits: a wait on a progress word that nothing sets gives up,
reports it, and leaves the context usable (no GPU fault, no hang).

The kernels' waits (sw_ring.cuh: wait_flag between the warps of a CTA,
wait_flag_gpu between the CTAs of a problem spread over several CTAs) are run
through d2p_wait_selftest on a word nothing ever sets.
"""
import ctypes
import os
import time

import pytest
import torch

import oracle
from tests._parity import check, scores

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "d2p_b200", "libd2p_b200.so")


@pytest.fixture(scope="module")
def lib():
    import d2p_b200  # noqa: F401  (builds / loads the extension and the C library)

    L = ctypes.CDLL(LIB)
    L.d2p_wait_selftest.restype = ctypes.c_int
    L.d2p_wait_selftest.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    return L


@pytest.mark.parametrize("scope", [0, 1])
def test_wait_on_unset_word_gives_up(lib, cuda_device, scope):
    word = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    status = torch.full((1,), -1, dtype=torch.int32, device=cuda_device)
    st = torch.cuda.current_stream().cuda_stream
    torch.cuda.synchronize()
    t0 = time.time()
    rc = lib.d2p_wait_selftest(scope, ctypes.c_void_p(word.data_ptr()), ctypes.c_void_p(status.data_ptr()),
                               ctypes.c_void_p(st))
    assert rc == 0
    torch.cuda.synchronize()
    dt = time.time() - t0
    assert int(status.item()) == 1, "the wait must report that it gave up"
    assert int(word.item()) == 0
    assert dt < 30.0, f"the bounded wait took {dt:.1f} s"
    # the context is still usable: an ordinary op runs and matches the oracle
    s = scores(2, 40, 48, seed=9)
    v, m = torch.ops.d2p.soft_sw_float(s.to(cuda_device), -1.0, 1.0, None)
    r64 = oracle.sw_linear(s.numpy(), None, -1.0, 1.0, "f64")
    r32 = oracle.sw_linear(s.numpy(), None, -1.0, 1.0, "f32")
    check("value", v, r64["value"], r32["value"])
    check("marginals", m, r64["marginals"], r32["marginals"])


def test_wait_selftest_rejects_bad_arguments(lib):
    assert lib.d2p_wait_selftest(2, None, ctypes.c_void_p(16), None) != 0
    assert lib.d2p_wait_selftest(1, None, ctypes.c_void_p(16), None) != 0
    assert lib.d2p_wait_selftest(0, None, None, None) != 0
