"""Soft Needleman-Wunsch (linear gap) on the GPU against the CPU oracle.

The oracle (oracle/nw_oracle.c) restates src/nw/kernels_cpu.cpp:79-642 and is
pinned bit for bit to the reference's own CPU build by
tests/test_oracle_golden.py.  Every output of the operator set -- value,
alignment marginals, dS/dgap, dS/dT, the HVP, both parameter Jacobians and
backward_full -- is checked within 1e-5 relative / 1e-6 absolute of the
oracle's fp64 evaluation, or, where the reference's own fp32 result misses that,
no further from fp64 than the reference is (tests/_parity.py).  Cases follow
the reference's NW tests: full and ragged lengths, empty problems, one-row and
one-column problems, and low temperature.
"""
import numpy as np
import pytest
import torch

import oracle
from _parity import check, lengths_for, scores

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def d2p(cuda_device):
    import d2p_b200

    return d2p_b200


CASES = [
    # (B, L1, L2, gap, T, ragged, seed)
    (2, 100, 120, -1.0, 1.0, False, 0),
    (3, 64, 80, -0.5, 0.5, True, 1),
    (2, 1, 37, -1.0, 1.0, False, 2),
    (2, 41, 1, -1.0, 1.0, False, 3),
    (2, 48, 48, -1.0, 0.1, False, 4),
    (2, 256, 200, -1.0, 1.0, True, 5),
]


def _lengths(B, L1, L2, ragged, seed, dev):
    if not ragged:
        return None, None
    ln = lengths_for(B, L1, L2, seed=seed + 10, lo=0)
    ln[0, 0] = 0   # an empty problem: the value is L2 gaps, no marginals
    return ln, ln.to(dev)


@pytest.mark.parametrize("B,L1,L2,gap,T,ragged,seed", CASES)
def test_value_marginals_param_grads(d2p, cuda_device, B, L1, L2, gap, T, ragged, seed):
    s0 = scores(B, L1, L2, seed=seed)
    ln, lnd = _lengths(B, L1, L2, ragged, seed, cuda_device)
    v, m, gg, gt = d2p.soft_nw_with_grads(s0.to(cuda_device), gap, T, lnd)
    r64 = oracle.nw_linear(s0.numpy(), ln, gap, T, "f64")
    r32 = oracle.nw_linear(s0.numpy(), ln, gap, T, "f32")
    check("nw value", v, r64["value"], r32["value"])
    check("nw marginals", m, r64["marginals"], r32["marginals"])
    check("nw grad_gap", gg, r64["grad_gap"], r32["grad_gap"])
    check("nw grad_T", gt, r64["grad_T"], r32["grad_T"])
    # the float op (value + marginals only: the strip kernel) against the oracle too
    v2, m2 = d2p.soft_nw_float(s0.to(cuda_device), gap, T, lnd)
    check("nw value (strip)", v2, r64["value"], r32["value"])
    check("nw marginals (strip)", m2, r64["marginals"], r32["marginals"])


@pytest.mark.parametrize("B,L1,L2,gap,T,ragged,seed", CASES)
def test_hvp(d2p, cuda_device, B, L1, L2, gap, T, ragged, seed):
    s0 = scores(B, L1, L2, seed=seed)
    V = scores(B, L1, L2, seed=seed + 100)
    ln, lnd = _lengths(B, L1, L2, ragged, seed, cuda_device)
    H = d2p.soft_nw_hvp(s0.to(cuda_device), V.to(cuda_device), gap, T, lnd)
    check("nw hvp", H, oracle.nw_linear_hvp(s0.numpy(), V.numpy(), ln, gap, T, "f64"),
          oracle.nw_linear_hvp(s0.numpy(), V.numpy(), ln, gap, T, "f32"))


@pytest.mark.parametrize("param_type", [0, 1])
@pytest.mark.parametrize("B,L1,L2,gap,T,ragged,seed", CASES)
def test_param_jacobian(d2p, cuda_device, param_type, B, L1, L2, gap, T, ragged, seed):
    s0 = scores(B, L1, L2, seed=seed)
    ln, lnd = _lengths(B, L1, L2, ragged, seed, cuda_device)
    J = d2p.soft_nw_param_jacobian(s0.to(cuda_device), param_type, gap, T, lnd)
    check(f"nw jacobian {param_type}", J, oracle.nw_linear_param_jacobian(s0.numpy(), param_type, ln, gap, T, "f64"),
          oracle.nw_linear_param_jacobian(s0.numpy(), param_type, ln, gap, T, "f32"))


@pytest.mark.parametrize("B,L1,L2,gap,T,ragged,seed", CASES)
def test_backward_full(d2p, cuda_device, B, L1, L2, gap, T, ragged, seed):
    s0 = scores(B, L1, L2, seed=seed)
    G = scores(B, L1, L2, seed=seed + 200)
    ln, lnd = _lengths(B, L1, L2, ragged, seed, cuda_device)
    gs, gg, gt = d2p.soft_nw_backward_full(s0.to(cuda_device), G.to(cuda_device), gap, T, lnd)
    r64 = oracle.nw_linear_backward_full(s0.numpy(), G.numpy(), ln, gap, T, "f64")
    r32 = oracle.nw_linear_backward_full(s0.numpy(), G.numpy(), ln, gap, T, "f32")
    check("nw backward_full scores", gs, r64[0], r32[0])
    check("nw backward_full gap", gg, r64[1], r32[1])
    check("nw backward_full T", gt, r64[2], r32[2])


def test_autograd_value_and_marginal_branches(d2p, cuda_device):
    """soft_nw through autograd: the value branch gives grad = g[b] x marginals,
    dS/dgap and dS/dT summed over the batch; the marginal branch adds
    backward_full's terms (reference SoftNWCUDAFunction, src/nw/torch_cuda.cpp:115-330)."""
    B, L1, L2 = 3, 50, 70
    s0 = scores(B, L1, L2, seed=7)
    G = scores(B, L1, L2, seed=8)
    s = s0.to(cuda_device).requires_grad_(True)
    gap = torch.tensor([-0.7], device=cuda_device, requires_grad=True)
    T = torch.tensor([0.8], device=cuda_device, requires_grad=True)
    res = d2p.soft_nw(s, gap, T)
    w = torch.arange(1, B + 1, dtype=torch.float32, device=cuda_device)
    ((res.score * w).sum() + (res.alignment * G.to(cuda_device)).sum()).backward()
    r64 = oracle.nw_linear(s0.numpy(), None, -0.7, 0.8, "f64")
    bf = oracle.nw_linear_backward_full(s0.numpy(), G.numpy(), None, -0.7, 0.8, "f64")
    wn = w.cpu().numpy()[:, None, None]
    check("nw autograd scores", s.grad, wn * r64["marginals"] + bf[0], None, rtol=1e-4, atol=1e-5)
    check("nw autograd gap", gap.grad, [(w.cpu().numpy() * r64["grad_gap"]).sum() + bf[1][0]], None, rtol=1e-4)
    check("nw autograd T", T.grad, [(w.cpu().numpy() * r64["grad_T"]).sum() + bf[2][0]], None, rtol=1e-4)


def test_value_backward_is_the_marginals(d2p, cuda_device):
    B, L1, L2 = 4, 33, 65
    s = scores(B, L1, L2, seed=9).to(cuda_device).requires_grad_(True)
    res = d2p.soft_nw(s, gap=-1.0, temperature=1.0)
    res.score.sum().backward()
    assert torch.equal(s.grad, res.alignment)


def test_module_and_aliases(d2p, cuda_device):
    B, L1, L2 = 2, 30, 40
    s = scores(B, L1, L2, seed=11).to(cuda_device)
    mod = d2p.SoftNW(gap=-1.0, temperature=1.0, learnable=True).to(cuda_device)
    out = mod(s)
    out.score.sum().backward()
    assert mod.gap.grad is not None and mod.temperature.grad is not None
    ref = d2p.soft_nw(s, gap=-1.0, temperature=1.0)
    assert torch.allclose(out.score, ref.score) and torch.allclose(out.alignment, ref.alignment)
    v, m = d2p.ops.nw_forward(s, -1.0, 1.0, None)
    assert torch.equal(v, ref.score) and torch.equal(m, ref.alignment)
    gg, gt = d2p.ops.nw_value_grad_params(s, -1.0, 1.0, None)
    _, _, gg2, gt2 = d2p.soft_nw_with_grads(s, -1.0, 1.0, None)
    assert torch.equal(gg, gg2) and torch.equal(gt, gt2)
    assert torch.allclose(mod.gap.grad, gg.sum().reshape(1), rtol=1e-5, atol=1e-4)
    J = d2p.ops.nw_marginals_grad_gap(s, -1.0, 1.0, None)
    assert torch.equal(J, d2p.soft_nw_param_jacobian(s, 0, -1.0, 1.0, None))


def test_nw_value_is_global(d2p, cuda_device):
    """Closed forms: with one row, every global path has that row's one
    diagonal cell or none; an empty problem is all gaps."""
    L2 = 9
    s0 = scores(1, 1, L2, seed=12)
    gap, T = -1.0, 1.0
    v, m = d2p.soft_nw_float(s0.to(cuda_device), gap, T, None)
    # paths: all gaps (L2 + 1 of them) in C(L2+1, 1) = L2 + 1 orders, or one match at column j
    # with L2 - 1 gaps: Z = (L2 + 1) e^{(L2+1) gap} + sum_j e^{s_j + (L2-1) gap}
    z = (L2 + 1) * np.exp((L2 + 1) * gap) + np.exp(s0.numpy()[0, 0] + (L2 - 1) * gap).sum()
    assert abs(float(v[0]) - np.log(z)) < 1e-5
    ln = torch.tensor([[0, L2]], dtype=torch.int32)
    v0, m0 = d2p.soft_nw_float(s0.to(cuda_device), gap, T, ln.to(cuda_device))
    assert abs(float(v0[0]) - L2 * gap) < 1e-6 and float(m0.abs().max()) == 0.0


# value + marginals on the column-sweep strip kernel (problems of at most 512
# rows): full, ragged (packed several per CTA), odd widths (padded copies),
# one row, and a cut that a single column block does not reach
STRIP = [  # (B, L1, L2, gap, T, ragged, seed)
    (4, 512, 512, -1.0, 1.0, False, 20),
    (6, 512, 300, -0.5, 0.5, True, 21),
    (3, 100, 57, -1.0, 1.0, False, 22),
    (3, 1, 64, -1.0, 1.0, False, 23),
    (5, 200, 8, -1.0, 0.7, True, 24),
    (2, 128, 1000, -1.0, 1.0, False, 25),
]


@pytest.mark.parametrize("B,L1,L2,gap,T,ragged,seed", STRIP)
def test_strip_kernel_nw(d2p, cuda_device, B, L1, L2, gap, T, ragged, seed):
    """soft_nw_float on the strip kernel against the oracle, padding exactly
    zero, and its own result: the general engine (use_engine("plane")) rounds
    differently."""
    s0 = scores(B, L1, L2, seed=seed)
    ln, lnd = _lengths(B, L1, L2, ragged, seed, cuda_device)
    v, m = d2p.soft_nw_float(s0.to(cuda_device), gap, T, lnd)
    r64 = oracle.nw_linear(s0.numpy(), ln, gap, T, "f64")
    r32 = oracle.nw_linear(s0.numpy(), ln, gap, T, "f32")
    check("nw strip value", v, r64["value"], r32["value"])
    check("nw strip marginals", m, r64["marginals"], r32["marginals"])
    if ln is not None:
        mc = m.cpu()
        for b, (l1, l2) in enumerate(ln.tolist()):
            assert torch.count_nonzero(mc[b, l1:, :]) == 0 and torch.count_nonzero(mc[b, :, l2:]) == 0
    with d2p.use_engine("plane"):
        ve, me = d2p.soft_nw_float(s0.to(cuda_device), gap, T, lnd)
    full = [b for b in range(B) if ln is None or (ln[b, 0] > 1 and ln[b, 1] > 1)]
    assert any(not torch.equal(m[b], me[b]) for b in full), "the strip kernel did not run"
    v2, m2 = d2p.soft_nw_float(s0.to(cuda_device), gap, T, lnd)
    assert torch.equal(v, v2) and torch.equal(m, m2)


def _tan_kernel_names(fn):
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        torch.ones(1, device="cuda").add_(1)   # a torch launch first (a session's first launches can go unrecorded)
        torch.cuda.synchronize()
        fn()
        torch.cuda.synchronize()
    return [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]


WAVE_TAN_CASES = [
    # (B, L1, L2, gap, T, ragged, seed): more row-blocks than the CTA has warps,
    # widths that are not multiples of 4 or 16, one column, ragged with an empty problem
    (3, 512, 512, -1.0, 1.0, False, 31),
    (3, 300, 701, -0.5, 0.5, True, 32),
    (2, 33, 1, -1.0, 1.0, False, 33),
    (2, 1000, 64, -1.0, 0.25, True, 34),
]


@pytest.mark.parametrize("B,L1,L2,gap,T,ragged,seed", WAVE_TAN_CASES,
                         ids=[f"{c[0]}x{c[1]}x{c[2]}-T{c[4]}{'-ragged' if c[5] else ''}" for c in WAVE_TAN_CASES])
def test_wavefront_tangents(d2p, cuda_device, B, L1, L2, gap, T, ragged, seed):
    """The tangent operators in wavefront form (nw_wave_tan_kernel<HVP / PGAP /
    PT>): HVP, both Jacobians and backward_full against the oracle, each
    repeatable bit for bit."""
    s0 = scores(B, L1, L2, seed=seed)
    V = scores(B, L1, L2, seed=seed + 100)
    ln, lnd = _lengths(B, L1, L2, ragged, seed, cuda_device)
    sd, Vd = s0.to(cuda_device), V.to(cuda_device)
    names = _tan_kernel_names(lambda: d2p.soft_nw_hvp(sd, Vd, gap, T, lnd))
    assert any("nw_wave_tan_kernel" in n for n in names), names
    H = d2p.soft_nw_hvp(sd, Vd, gap, T, lnd)
    check("nw wave hvp", H, oracle.nw_linear_hvp(s0.numpy(), V.numpy(), ln, gap, T, "f64"),
          oracle.nw_linear_hvp(s0.numpy(), V.numpy(), ln, gap, T, "f32"))
    assert torch.equal(H, d2p.soft_nw_hvp(sd, Vd, gap, T, lnd))
    for pt in (0, 1):
        J = d2p.soft_nw_param_jacobian(sd, pt, gap, T, lnd)
        check(f"nw wave jacobian {pt}", J, oracle.nw_linear_param_jacobian(s0.numpy(), pt, ln, gap, T, "f64"),
              oracle.nw_linear_param_jacobian(s0.numpy(), pt, ln, gap, T, "f32"))
        assert torch.equal(J, d2p.soft_nw_param_jacobian(sd, pt, gap, T, lnd))
    gs, gg, gt = d2p.soft_nw_backward_full(sd, Vd, gap, T, lnd)
    r64 = oracle.nw_linear_backward_full(s0.numpy(), V.numpy(), ln, gap, T, "f64")
    r32 = oracle.nw_linear_backward_full(s0.numpy(), V.numpy(), ln, gap, T, "f32")
    check("nw wave backward_full scores", gs, r64[0], r32[0])
    check("nw wave backward_full gap", gg, r64[1], r32[1])
    check("nw wave backward_full T", gt, r64[2], r32[2])
