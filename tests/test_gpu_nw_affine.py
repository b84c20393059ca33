"""Soft Needleman-Wunsch with affine gaps on the GPU against the CPU oracle.

The oracle (oracle/nw_affine_oracle.c) restates src/nw_affine/kernels_cpu.cpp
and is pinned bit for bit to the reference's own CPU build by
tests/test_oracle_golden.py.  Every output of the operator set -- value,
alignment marginals, the three parameter gradients, the HVP, the three
parameter Jacobians and backward_full -- is checked within 1e-5 relative /
1e-6 absolute of the oracle's fp64 evaluation, or, where the reference's own
fp32 result misses that, no further from fp64 than the reference is
(tests/_parity.py).  Cases: full and ragged lengths, empty problems, one-row
and one-column problems, low temperature.
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
    # (B, L1, L2, gap_open, gap_ext, T, ragged, seed)
    (2, 100, 120, -2.0, -0.5, 1.0, False, 0),
    (3, 64, 80, -1.5, -0.3, 0.5, True, 1),
    (2, 1, 37, -2.0, -0.5, 1.0, False, 2),
    (2, 41, 1, -2.0, -0.5, 1.0, False, 3),
    (2, 48, 48, -2.0, -0.5, 0.1, False, 4),
    (2, 256, 200, -2.0, -0.5, 1.0, True, 5),
]
IDS = [f"{c[0]}x{c[1]}x{c[2]}-T{c[5]}{'-ragged' if c[6] else ''}" for c in CASES]


def _lengths(B, L1, L2, ragged, seed, dev):
    if not ragged:
        return None, None
    ln = lengths_for(B, L1, L2, seed=seed + 10, lo=0)
    ln[0, 0] = 0   # an empty problem: one all-gap path
    return ln, ln.to(dev)


@pytest.mark.parametrize("B,L1,L2,go,ge,T,ragged,seed", CASES, ids=IDS)
def test_value_marginals_param_grads(d2p, cuda_device, B, L1, L2, go, ge, T, ragged, seed):
    s0 = scores(B, L1, L2, seed=seed)
    ln, lnd = _lengths(B, L1, L2, ragged, seed, cuda_device)
    v, m, g_o, g_e, g_t = d2p.soft_nw_affine_with_grads(s0.to(cuda_device), go, ge, T, lnd)
    r64 = oracle.nw_affine(s0.numpy(), ln, go, ge, T, "f64")
    r32 = oracle.nw_affine(s0.numpy(), ln, go, ge, T, "f32")
    check("nwa value", v, r64["value"], r32["value"])
    check("nwa marginals", m, r64["marginals"], r32["marginals"])
    check("nwa grad_open", g_o, r64["grad_open"], r32["grad_open"])
    check("nwa grad_ext", g_e, r64["grad_ext"], r32["grad_ext"])
    check("nwa grad_T", g_t, r64["grad_T"], r32["grad_T"])
    v2, m2 = d2p.soft_nw_affine_float(s0.to(cuda_device), go, ge, T, lnd)
    assert torch.equal(v, v2) and torch.equal(m, m2)


@pytest.mark.parametrize("B,L1,L2,go,ge,T,ragged,seed", CASES, ids=IDS)
def test_hvp(d2p, cuda_device, B, L1, L2, go, ge, T, ragged, seed):
    s0 = scores(B, L1, L2, seed=seed)
    V = scores(B, L1, L2, seed=seed + 100)
    ln, lnd = _lengths(B, L1, L2, ragged, seed, cuda_device)
    H = d2p.soft_nw_affine_hvp(s0.to(cuda_device), V.to(cuda_device), go, ge, T, lnd)
    check("nwa hvp", H, oracle.nw_affine_hvp(s0.numpy(), V.numpy(), ln, go, ge, T, "f64"),
          oracle.nw_affine_hvp(s0.numpy(), V.numpy(), ln, go, ge, T, "f32"))


@pytest.mark.parametrize("param_type", [0, 1, 2])
@pytest.mark.parametrize("B,L1,L2,go,ge,T,ragged,seed", CASES, ids=IDS)
def test_param_jacobian(d2p, cuda_device, param_type, B, L1, L2, go, ge, T, ragged, seed):
    s0 = scores(B, L1, L2, seed=seed)
    ln, lnd = _lengths(B, L1, L2, ragged, seed, cuda_device)
    J = d2p.soft_nw_affine_param_jacobian(s0.to(cuda_device), param_type, go, ge, T, lnd)
    check(f"nwa jacobian {param_type}", J,
          oracle.nw_affine_param_jacobian(s0.numpy(), param_type, ln, go, ge, T, "f64"),
          oracle.nw_affine_param_jacobian(s0.numpy(), param_type, ln, go, ge, T, "f32"))


@pytest.mark.parametrize("B,L1,L2,go,ge,T,ragged,seed", CASES, ids=IDS)
def test_backward_full(d2p, cuda_device, B, L1, L2, go, ge, T, ragged, seed):
    s0 = scores(B, L1, L2, seed=seed)
    G = scores(B, L1, L2, seed=seed + 200)
    ln, lnd = _lengths(B, L1, L2, ragged, seed, cuda_device)
    out = d2p.soft_nw_affine_backward_full(s0.to(cuda_device), G.to(cuda_device), go, ge, T, lnd)
    r64 = oracle.nw_affine_backward_full(s0.numpy(), G.numpy(), ln, go, ge, T, "f64")
    r32 = oracle.nw_affine_backward_full(s0.numpy(), G.numpy(), ln, go, ge, T, "f32")
    for q, name in enumerate(("scores", "open", "ext", "T")):
        check(f"nwa backward_full {name}", out[q], r64[q], r32[q])


def test_autograd_value_and_marginal_branches(d2p, cuda_device):
    """soft_nw_affine through autograd (reference SoftNWAffineCUDAFunction,
    src/nw_affine/torch_cuda.cpp:170-420): the value branch gives g[b] x
    marginals and batch-summed parameter gradients, the marginal branch adds
    backward_full's terms."""
    B, L1, L2 = 3, 50, 70
    go, ge, T = -1.7, -0.4, 0.8
    s0 = scores(B, L1, L2, seed=7)
    G = scores(B, L1, L2, seed=8)
    s = s0.to(cuda_device).requires_grad_(True)
    params = [torch.tensor([x], device=cuda_device, requires_grad=True) for x in (go, ge, T)]
    res = d2p.soft_nw_affine(s, *params)
    w = torch.arange(1, B + 1, dtype=torch.float32, device=cuda_device)
    ((res.score * w).sum() + (res.alignment * G.to(cuda_device)).sum()).backward()
    r64 = oracle.nw_affine(s0.numpy(), None, go, ge, T, "f64")
    bf = oracle.nw_affine_backward_full(s0.numpy(), G.numpy(), None, go, ge, T, "f64")
    wn = w.cpu().numpy()
    check("nwa autograd scores", s.grad, wn[:, None, None] * r64["marginals"] + bf[0], None, rtol=1e-4, atol=1e-5)
    for q, key in enumerate(("grad_open", "grad_ext", "grad_T")):
        check(f"nwa autograd {key}", params[q].grad, [(wn * r64[key]).sum() + bf[1 + q][0]], None, rtol=1e-4)


def test_value_backward_is_the_marginals(d2p, cuda_device):
    s = scores(4, 33, 65, seed=9).to(cuda_device).requires_grad_(True)
    res = d2p.soft_nw_affine(s, gap_open=-2.0, gap_ext=-0.5, temperature=1.0)
    res.score.sum().backward()
    assert torch.equal(s.grad, res.alignment)


def test_module_and_aliases(d2p, cuda_device):
    B, L1, L2 = 2, 30, 40
    s = scores(B, L1, L2, seed=11).to(cuda_device)
    mod = d2p.SoftNWAffine(gap_open=-2.0, gap_ext=-0.5, temperature=1.0, learnable=True).to(cuda_device)
    out = mod(s)
    out.score.sum().backward()
    assert all(p.grad is not None for p in (mod.gap_open, mod.gap_ext, mod.temperature))
    ref = d2p.soft_nw_affine(s, gap_open=-2.0, gap_ext=-0.5, temperature=1.0)
    assert torch.allclose(out.score, ref.score) and torch.allclose(out.alignment, ref.alignment)
    ops = torch.ops.d2p
    p = (-2.0, -0.5, 1.0)
    v, m = ops.nw_affine_forward(s, *p, None)
    assert torch.equal(v, ref.score) and torch.equal(m, ref.alignment)
    wg = ops.soft_nw_affine_with_grads(s, *p, None)
    vg = ops.nw_affine_value_grad_params(s, *p, None)
    assert all(torch.equal(a, b) for a, b in zip(vg, wg[2:]))
    G = scores(B, L1, L2, seed=12).to(cuda_device)
    mb = ops.nw_affine_marginals_backward(s, G, *p, None)
    bf = ops.soft_nw_affine_backward_full(s, G, *p, None)
    assert all(torch.equal(a, b) for a, b in zip(mb, bf))
    assert torch.equal(ops.nw_affine_marginals_hvp(s, G, *p, None), ops.soft_nw_affine_hvp(s, G, *p, None))
    for q, name in enumerate(("gap_open", "gap_ext", "temp")):
        assert torch.equal(getattr(ops, f"nw_affine_marginals_grad_{name}")(s, *p, None),
                           ops.soft_nw_affine_param_jacobian(s, q, *p, None))
    gt = [mod.gap_open.grad, mod.gap_ext.grad, mod.temperature.grad]
    for q in range(3):
        assert torch.allclose(gt[q], wg[2 + q].sum().reshape(1), rtol=1e-5, atol=1e-4)


def test_empty_problems_are_all_gap_paths(d2p, cuda_device):
    """An empty side leaves one path, all gaps: open + (n - 1) ext for n > 0
    gaps, 0 for none; no marginals; dS/dopen = 1, dS/dext = n - 1, dS/dT = 0."""
    go, ge = -2.0, -0.5
    s = scores(4, 6, 9, seed=13).to(cuda_device)
    ln = torch.tensor([[0, 9], [6, 0], [0, 0], [0, 1]], dtype=torch.int32, device=cuda_device)
    v, m, g_o, g_e, g_t = d2p.soft_nw_affine_with_grads(s, go, ge, 1.0, ln)
    n = (ln.sum(1)).cpu().numpy()
    want = np.where(n > 0, go + (n - 1) * ge, 0.0)
    assert np.allclose(v.cpu().numpy(), want, atol=1e-6)
    assert float(m.abs().max()) == 0.0
    assert np.allclose(g_o.cpu().numpy(), (n > 0).astype(float), atol=1e-6)
    assert np.allclose(g_e.cpu().numpy(), np.maximum(n - 1, 0), atol=1e-6)
    assert np.allclose(g_t.cpu().numpy(), 0.0, atol=1e-6)


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
    # (B, L1, L2, gap_open, gap_ext, T, ragged, seed): more row-blocks than the
    # CTA has warps, widths that are not multiples of 4 or 16, one column, a
    # ragged batch with an empty problem, low temperature
    (3, 512, 512, -2.0, -0.5, 1.0, False, 21),
    (3, 300, 701, -1.5, -0.3, 0.5, True, 22),
    (2, 33, 1, -2.0, -0.5, 1.0, False, 23),
    (2, 1000, 64, -2.0, -0.5, 0.25, True, 24),
]
WAVE_IDS = [f"{c[0]}x{c[1]}x{c[2]}-T{c[5]}{'-ragged' if c[6] else ''}" for c in WAVE_CASES]


@pytest.mark.parametrize("B,L1,L2,go,ge,T,ragged,seed", WAVE_CASES, ids=WAVE_IDS)
def test_wavefront_value_pass(d2p, cuda_device, B, L1, L2, go, ge, T, ragged, seed):
    """The value pass in row-block wavefront form (nwa_wave_kernel) against the
    oracle -- value, marginals and the three parameter gradients (leading gaps
    of row 0 and column 0 included) -- and repeatable bit for bit.  An empty
    problem is flagged by it and recomputed by the diagonal engine."""
    s0 = scores(B, L1, L2, seed=seed)
    ln, lnd = _lengths(B, L1, L2, ragged, seed, cuda_device)
    sd = s0.to(cuda_device)
    names = _kernel_names(lambda: d2p.soft_nw_affine_with_grads(sd, go, ge, T, lnd))
    assert any("nwa_wave_kernel" in n for n in names), names
    out = d2p.soft_nw_affine_with_grads(sd, go, ge, T, lnd)
    r64 = oracle.nw_affine(s0.numpy(), ln, go, ge, T, "f64")
    r32 = oracle.nw_affine(s0.numpy(), ln, go, ge, T, "f32")
    for name, x, key in zip(("value", "marginals", "grad_open", "grad_ext", "grad_T"), out,
                            ("value", "marginals", "grad_open", "grad_ext", "grad_T")):
        check("nwa " + name, x, r64[key], r32[key])
    again = d2p.soft_nw_affine_with_grads(sd, go, ge, T, lnd)
    assert all(torch.equal(a, b) for a, b in zip(out, again))
