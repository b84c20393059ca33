"""Soft DTW on the GPU against the CPU oracle.

The oracle (oracle/dtw_oracle.c) restates src/dtw/kernels_cpu.cpp and is
pinned bit for bit to the reference's own CPU build by
tests/test_oracle_golden.py.  Every output -- value, alignment marginals,
dS/dT, the HVP, dP/dT and backward_full -- is checked within 1e-5 relative /
1e-6 absolute of the oracle's fp64 evaluation, or, where the reference's own
fp32 result misses that, no further from fp64 than the reference is
(tests/_parity.py).  Cases: no band and Sakoe-Chiba bands, ragged lengths,
empty sequences (whose value is the reference's +inf sentinel 1e30), one-row
problems, low temperature.
"""
import numpy as np
import pytest
import torch

import oracle
from _parity import check, lengths_for

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def d2p(cuda_device):
    import d2p_b200

    return d2p_b200


def costs(B, L1, L2, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.rand(B, L1, L2, generator=g)


CASES = [
    # (B, L1, L2, T, bandwidth, ragged, seed)
    (2, 100, 120, 1.0, -1, False, 0),
    (3, 64, 80, 0.5, 10, True, 1),
    (2, 1, 37, 1.0, -1, False, 2),
    (2, 48, 48, 0.1, 5, False, 4),
    (2, 256, 200, 1.0, 20, True, 5),
    (2, 30, 45, 1.0, 0, False, 6),
]
IDS = [f"{c[0]}x{c[1]}x{c[2]}-T{c[3]}-bw{c[4]}{'-ragged' if c[5] else ''}" for c in CASES]


def _lengths(B, L1, L2, ragged, seed):
    if not ragged:
        return np.tile(np.array([[L1, L2]], np.int32), (B, 1))
    ln = lengths_for(B, L1, L2, seed=seed + 10, lo=1).numpy()
    ln[0, 0] = 0   # an empty sequence: the +inf sentinel
    return ln


def _finite(ref, ours):
    """Values of unreached ends are the 1e30 sentinel on both sides."""
    r = np.asarray(ref, np.float64)
    o = ours.detach().cpu().numpy().astype(np.float64)
    inf = r >= 1e29
    assert np.all(o[inf] >= 1e29), "an unreached end must keep the sentinel"
    return ~inf


@pytest.mark.parametrize("B,L1,L2,T,bw,ragged,seed", CASES, ids=IDS)
def test_value_marginals_grad_T(d2p, cuda_device, B, L1, L2, T, bw, ragged, seed):
    c0 = costs(B, L1, L2, seed)
    ln = _lengths(B, L1, L2, ragged, seed)
    lnd = torch.from_numpy(ln).to(cuda_device)
    v, m, gt = d2p.soft_dtw_with_grads(c0.to(cuda_device), T, lnd, bw)
    r64 = oracle.dtw(c0.numpy(), ln, T, bw, "f64")
    r32 = oracle.dtw(c0.numpy(), ln, T, bw, "f32")
    fin = _finite(r64["value"], v)
    check("dtw value", v[torch.from_numpy(fin).to(cuda_device)], r64["value"][fin], r32["value"][fin])
    check("dtw marginals", m, r64["marginals"], r32["marginals"])
    check("dtw grad_T", gt, r64["grad_T"], r32["grad_T"])
    v2, m2 = d2p.soft_dtw_float(c0.to(cuda_device), T, lnd, bw)
    assert torch.equal(v, v2) and torch.equal(m, m2)


@pytest.mark.parametrize("B,L1,L2,T,bw,ragged,seed", CASES, ids=IDS)
def test_hvp(d2p, cuda_device, B, L1, L2, T, bw, ragged, seed):
    c0 = costs(B, L1, L2, seed)
    g = torch.Generator().manual_seed(seed + 100)
    V = torch.randn(B, L1, L2, generator=g)
    ln = _lengths(B, L1, L2, ragged, seed)
    H = d2p.soft_dtw_hvp(c0.to(cuda_device), V.to(cuda_device), T, torch.from_numpy(ln).to(cuda_device), bw)
    check("dtw hvp", H, oracle.dtw_hvp(c0.numpy(), V.numpy(), ln, T, bw, "f64"),
          oracle.dtw_hvp(c0.numpy(), V.numpy(), ln, T, bw, "f32"))


@pytest.mark.parametrize("B,L1,L2,T,bw,ragged,seed", CASES, ids=IDS)
def test_param_jacobian(d2p, cuda_device, B, L1, L2, T, bw, ragged, seed):
    c0 = costs(B, L1, L2, seed)
    ln = _lengths(B, L1, L2, ragged, seed)
    J = d2p.soft_dtw_param_jacobian(c0.to(cuda_device), T, torch.from_numpy(ln).to(cuda_device), bw)
    check("dtw jacobian", J, oracle.dtw_param_jacobian(c0.numpy(), ln, T, bw, "f64"),
          oracle.dtw_param_jacobian(c0.numpy(), ln, T, bw, "f32"))


@pytest.mark.parametrize("B,L1,L2,T,bw,ragged,seed", CASES, ids=IDS)
def test_backward_full(d2p, cuda_device, B, L1, L2, T, bw, ragged, seed):
    c0 = costs(B, L1, L2, seed)
    g = torch.Generator().manual_seed(seed + 200)
    G = torch.randn(B, L1, L2, generator=g)
    ln = _lengths(B, L1, L2, ragged, seed)
    gc, gt = d2p.soft_dtw_backward_full(c0.to(cuda_device), G.to(cuda_device), T,
                                        torch.from_numpy(ln).to(cuda_device), bw)
    r64 = oracle.dtw_backward_full(c0.numpy(), G.numpy(), ln, T, bw, "f64")
    r32 = oracle.dtw_backward_full(c0.numpy(), G.numpy(), ln, T, bw, "f32")
    check("dtw backward_full costs", gc, r64[0], r32[0])
    check("dtw backward_full T", gt, r64[1], r32[1])


def test_public_api_autograd_and_module(d2p, cuda_device):
    """soft_dtw through autograd (reference SoftDTWCUDAFunction,
    src/dtw/torch_cuda.cpp:140-325): the value branch gives g[b] x marginals
    and sum g dS/dT, the marginal branch adds backward_full's terms; the
    Python API maps bandwidth 0 to no band (d2p/dtw.py:90-96)."""
    B, L1, L2, T = 3, 40, 50, 0.7
    c0 = costs(B, L1, L2, 7)
    g = torch.Generator().manual_seed(8)
    G = torch.randn(B, L1, L2, generator=g)
    c = c0.to(cuda_device).requires_grad_(True)
    t = torch.tensor([T], device=cuda_device, requires_grad=True)
    res = d2p.soft_dtw(c, temperature=t, bandwidth=0)
    w = torch.arange(1, B + 1, dtype=torch.float32, device=cuda_device)
    ((res.cost * w).sum() + (res.alignment * G.to(cuda_device)).sum()).backward()
    r64 = oracle.dtw(c0.numpy(), None, T, -1, "f64")
    bf = oracle.dtw_backward_full(c0.numpy(), G.numpy(), None, T, -1, "f64")
    wn = w.cpu().numpy()
    check("dtw autograd costs", c.grad, wn[:, None, None] * r64["marginals"] + bf[0], None, rtol=1e-4, atol=1e-5)
    check("dtw autograd T", t.grad, [(wn * r64["grad_T"]).sum() + bf[1][0]], None, rtol=1e-4)
    # value-only backward is the marginals; the module takes a learnable temperature
    c2 = c0.to(cuda_device).requires_grad_(True)
    r2 = d2p.soft_dtw(c2, temperature=1.0, bandwidth=5)
    r2.cost.sum().backward()
    assert torch.equal(c2.grad, r2.alignment)
    mod = d2p.SoftDTW(temperature=1.0, bandwidth=5, learnable=True).to(cuda_device)
    out = mod(c0.to(cuda_device))
    out.cost.sum().backward()
    assert mod.temperature.grad is not None
    assert torch.allclose(out.cost, r2.cost) and torch.allclose(out.alignment, r2.alignment)


def test_compile_fullgraph(d2p, cuda_device):
    """torch.compile(fullgraph=True) traces soft_dtw through the d2p_py custom
    ops and their autograd formulas; results equal the eager ones."""
    torch._dynamo.reset()
    c0 = costs(2, 12, 16, 9).to(cuda_device)
    W = costs(2, 12, 16, 10).to(cuda_device)

    def run(fn, tensor_t):
        c = c0.clone().requires_grad_(True)
        t = torch.tensor([0.9], device=cuda_device, requires_grad=True) if tensor_t else 0.9
        loss, v, m = fn(c, t)
        loss.backward()
        return v.detach(), m.detach(), [c.grad] + ([t.grad] if tensor_t else [])

    def f(c, t):
        r = d2p.soft_dtw(c, temperature=t, bandwidth=4)
        return r.cost.sum() + (r.alignment * W).sum(), r.cost, r.alignment

    for tensor_t in (False, True):
        torch._dynamo.reset()
        ve, me, ge = run(f, tensor_t)
        vc, mc, gc = run(torch.compile(f, fullgraph=True, backend="aot_eager"), tensor_t)
        torch.testing.assert_close(vc, ve, rtol=0, atol=0)
        torch.testing.assert_close(mc, me, rtol=0, atol=0)
        for a, b in zip(gc, ge):
            torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)


def _kernel_names(fn):
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        torch.ones(1, device="cuda").add_(1)   # a torch launch first (a session's first launches can go unrecorded)
        torch.cuda.synchronize()
        fn()
        torch.cuda.synchronize()
    return [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]


WAVE_CASES = [
    # (B, L1, L2, T, bandwidth, ragged, seed): more row-blocks than the CTA has
    # warps, widths that are not multiples of 4 or 16, one column, a band
    (3, 512, 512, 1.0, -1, False, 11),
    (3, 300, 701, 0.5, 60, True, 12),
    (2, 33, 1, 1.0, -1, False, 13),
    (2, 1000, 64, 0.25, -1, True, 14),
]
WAVE_IDS = [f"{c[0]}x{c[1]}x{c[2]}-T{c[3]}-bw{c[4]}{'-ragged' if c[5] else ''}" for c in WAVE_CASES]


@pytest.mark.parametrize("B,L1,L2,T,bw,ragged,seed", WAVE_CASES, ids=WAVE_IDS)
def test_wavefront_value_pass(d2p, cuda_device, B, L1, L2, T, bw, ragged, seed):
    """The value pass in row-block wavefront form (dtw_wave_kernel) against the
    oracle, and repeatable bit for bit.  An empty sequence in the ragged cases
    is flagged by it and recomputed by the diagonal engine."""
    c0 = costs(B, L1, L2, seed)
    ln = _lengths(B, L1, L2, ragged, seed)
    lnd = torch.from_numpy(ln).to(cuda_device)
    cd = c0.to(cuda_device)
    names = _kernel_names(lambda: d2p.soft_dtw_with_grads(cd, T, lnd, bw))
    assert any("dtw_wave_kernel" in n for n in names), names
    v, m, gt = d2p.soft_dtw_with_grads(cd, T, lnd, bw)
    r64 = oracle.dtw(c0.numpy(), ln, T, bw, "f64")
    r32 = oracle.dtw(c0.numpy(), ln, T, bw, "f32")
    fin = _finite(r64["value"], v)
    check("dtw value", v[torch.from_numpy(fin).to(cuda_device)], r64["value"][fin], r32["value"][fin])
    check("dtw marginals", m, r64["marginals"], r32["marginals"])
    check("dtw grad_T", gt, r64["grad_T"], r32["grad_T"])
    v2, m2, gt2 = d2p.soft_dtw_with_grads(cd, T, lnd, bw)
    assert torch.equal(v, v2) and torch.equal(m, m2) and torch.equal(gt, gt2)


@pytest.mark.parametrize("B,L1,L2,T,bw,ragged,seed", WAVE_CASES, ids=WAVE_IDS)
def test_wavefront_hvp_backward_full(d2p, cuda_device, B, L1, L2, T, bw, ragged, seed):
    """The Hessian-vector product and dP/dT in wavefront form
    (dtw_wave_tan_kernel<HVP / PT>), and backward_full through both, against the
    oracle; repeatable bit for bit."""
    c0 = costs(B, L1, L2, seed)
    g = torch.Generator().manual_seed(seed + 300)
    V = torch.randn(B, L1, L2, generator=g)
    ln = _lengths(B, L1, L2, ragged, seed)
    lnd = torch.from_numpy(ln).to(cuda_device)
    cd, Vd = c0.to(cuda_device), V.to(cuda_device)
    names = _kernel_names(lambda: d2p.soft_dtw_hvp(cd, Vd, T, lnd, bw))
    assert any("dtw_wave_tan_kernel" in n for n in names), names
    H = d2p.soft_dtw_hvp(cd, Vd, T, lnd, bw)
    check("dtw wave hvp", H, oracle.dtw_hvp(c0.numpy(), V.numpy(), ln, T, bw, "f64"),
          oracle.dtw_hvp(c0.numpy(), V.numpy(), ln, T, bw, "f32"))
    assert torch.equal(H, d2p.soft_dtw_hvp(cd, Vd, T, lnd, bw))
    gc, gt = d2p.soft_dtw_backward_full(cd, Vd, T, lnd, bw)
    r64 = oracle.dtw_backward_full(c0.numpy(), V.numpy(), ln, T, bw, "f64")
    r32 = oracle.dtw_backward_full(c0.numpy(), V.numpy(), ln, T, bw, "f32")
    check("dtw wave backward_full costs", gc, r64[0], r32[0])
    check("dtw wave backward_full T", gt, r64[1], r32[1])
    J = d2p.soft_dtw_param_jacobian(cd, T, lnd, bw)
    check("dtw wave jacobian", J, oracle.dtw_param_jacobian(c0.numpy(), ln, T, bw, "f64"),
          oracle.dtw_param_jacobian(c0.numpy(), ln, T, bw, "f32"))
    assert torch.equal(J, d2p.soft_dtw_param_jacobian(cd, T, lnd, bw))
