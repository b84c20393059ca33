"""GPU parity of the affine-gap soft Smith-Waterman ops against the CPU oracle."""
import numpy as np
import pytest
import torch

import oracle
from tests._parity import check, lengths_for, plane_engine, scores

pytestmark = pytest.mark.gpu

CASES = [  # (B, L1, L2, T, gap_open, gap_ext)
    (1, 8, 10, 1.0, -2.0, -0.5),
    (4, 16, 16, 0.1, -2.0, -0.5),
    (2, 5, 20, 2.0, -1.7, -0.4),
    (3, 33, 47, 0.5, -2.0, -0.5),
    (2, 64, 80, 1.0, -2.0, -0.5),
    (2, 1, 7, 1.0, -2.0, -0.5),
]


@pytest.fixture(scope="module")
def d2p():
    import d2p_b200

    return d2p_b200


@pytest.mark.parametrize("B,L1,L2,T,go,ge", CASES)
def test_forward_backward(d2p, cuda_device, B, L1, L2, T, go, ge):
    s = scores(B, L1, L2, seed=B * 100 + L2)
    v, m, a, b, c = torch.ops.d2p.soft_sw_affine_with_grads(s.to(cuda_device), go, ge, T, None)
    r64 = oracle.sw_affine(s.numpy(), None, go, ge, T, "f64")
    r32 = oracle.sw_affine(s.numpy(), None, go, ge, T, "f32")
    check("value", v, r64["value"], r32["value"])
    check("marginals", m, r64["marginals"], r32["marginals"])
    check("grad_open", a, r64["grad_open"], r32["grad_open"])
    check("grad_ext", b, r64["grad_ext"], r32["grad_ext"])
    check("grad_T", c, r64["grad_T"], r32["grad_T"])


@pytest.mark.parametrize("B,L1,L2,T,go,ge", CASES[:5])
def test_variable_lengths_and_padding(d2p, cuda_device, B, L1, L2, T, go, ge):
    s = scores(B, L1, L2, seed=17)
    ln = lengths_for(B, L1, L2, seed=20260707)
    v, m, a, b, c = torch.ops.d2p.soft_sw_affine_with_grads(s.to(cuda_device), go, ge, T, ln.to(cuda_device))
    r64 = oracle.sw_affine(s.numpy(), ln.numpy(), go, ge, T, "f64")
    r32 = oracle.sw_affine(s.numpy(), ln.numpy(), go, ge, T, "f32")
    check("value", v, r64["value"], r32["value"])
    check("marginals", m, r64["marginals"], r32["marginals"])
    check("grad_open", a, r64["grad_open"], r32["grad_open"])
    check("grad_ext", b, r64["grad_ext"], r32["grad_ext"])
    mc = m.cpu()
    for bb, (l1, l2) in enumerate(ln.tolist()):
        assert torch.count_nonzero(mc[bb, l1:, :]) == 0
        assert torch.count_nonzero(mc[bb, :, l2:]) == 0


@pytest.mark.parametrize("B,L1,L2,T,go,ge", CASES[:4])
def test_hvp(d2p, cuda_device, B, L1, L2, T, go, ge):
    s = scores(B, L1, L2, seed=3)
    V = scores(B, L1, L2, seed=4)
    H = torch.ops.d2p.soft_sw_affine_hvp(s.to(cuda_device), V.to(cuda_device), go, ge, T, None)
    h64 = oracle.sw_affine_hvp(s.numpy(), V.numpy(), None, go, ge, T, "f64")
    h32 = oracle.sw_affine_hvp(s.numpy(), V.numpy(), None, go, ge, T, "f32")
    check("hvp", H, h64, h32)


@pytest.mark.parametrize("param_type", [0, 1, 2])
@pytest.mark.parametrize("B,L1,L2,T,go,ge", CASES[:4])
def test_param_jacobian(d2p, cuda_device, B, L1, L2, T, go, ge, param_type):
    s = scores(B, L1, L2, seed=5)
    J = torch.ops.d2p.soft_sw_affine_param_jacobian(s.to(cuda_device), param_type, go, ge, T, None)
    j64 = oracle.sw_affine_param_jacobian(s.numpy(), param_type, None, go, ge, T, "f64")
    j32 = oracle.sw_affine_param_jacobian(s.numpy(), param_type, None, go, ge, T, "f32")
    check(f"jac{param_type}", J, j64, j32)


@pytest.mark.parametrize("B,L1,L2,T,go,ge", CASES[:3])
def test_backward_full(d2p, cuda_device, B, L1, L2, T, go, ge):
    s = scores(B, L1, L2, seed=8)
    G = scores(B, L1, L2, seed=9)
    out = torch.ops.d2p.soft_sw_affine_backward_full(s.to(cuda_device), G.to(cuda_device), go, ge, T, None)
    r64 = oracle.sw_affine_backward_full(s.numpy(), G.numpy(), None, go, ge, T, "f64")
    r32 = oracle.sw_affine_backward_full(s.numpy(), G.numpy(), None, go, ge, T, "f32")
    check("grad_scores", out[0], r64[0], r32[0])
    for k in range(1, 4):
        check(f"grad_param{k}", out[k], r64[k], r32[k])


# Shapes routed to the affine linear-domain tangent kernel (L2 % 4 == 0).
ATAN = [  # (B, L1, L2, T, gap_open, gap_ext, ragged)
    (2, 33, 64, 1.0, -2.0, -0.5, False), (3, 100, 36, 0.5, -2.0, -0.5, False),
    (2, 130, 260, 1.0, -1.7, -0.4, False), (1, 200, 8, 1.0, -2.0, -0.5, False),
    (4, 70, 96, 1.0, -2.0, -0.5, True), (1, 1024, 256, 1.0, -2.0, -0.5, False),
]


def _atan_inputs(B, L1, L2, ragged, seed):
    s = scores(B, L1, L2, seed=seed)
    ln = lengths_for(B, L1, L2, seed=seed + 1) if ragged else None
    if ln is not None:
        ln[0] = torch.tensor([L1, L2], dtype=torch.int32)
    return s, ln


@pytest.mark.parametrize("B,L1,L2,T,go,ge,ragged", ATAN)
def test_tangent_hvp(d2p, cuda_device, B, L1, L2, T, go, ge, ragged):
    s, ln = _atan_inputs(B, L1, L2, ragged, 81)
    V = scores(B, L1, L2, seed=82)
    lnd = None if ln is None else ln.to(cuda_device)
    H = torch.ops.d2p.soft_sw_affine_hvp(s.to(cuda_device), V.to(cuda_device), go, ge, T, lnd)
    lnp = None if ln is None else ln.numpy()
    h64 = oracle.sw_affine_hvp(s.numpy(), V.numpy(), lnp, go, ge, T, "f64")
    h32 = oracle.sw_affine_hvp(s.numpy(), V.numpy(), lnp, go, ge, T, "f32")
    check("hvp", H, h64, h32)


@pytest.mark.parametrize("param_type", [0, 1, 2])
@pytest.mark.parametrize("B,L1,L2,T,go,ge,ragged", ATAN)
def test_tangent_param_jacobian(d2p, cuda_device, B, L1, L2, T, go, ge, ragged, param_type):
    s, ln = _atan_inputs(B, L1, L2, ragged, 83)
    lnd = None if ln is None else ln.to(cuda_device)
    J = torch.ops.d2p.soft_sw_affine_param_jacobian(s.to(cuda_device), param_type, go, ge, T, lnd)
    lnp = None if ln is None else ln.numpy()
    j64 = oracle.sw_affine_param_jacobian(s.numpy(), param_type, lnp, go, ge, T, "f64")
    j32 = oracle.sw_affine_param_jacobian(s.numpy(), param_type, lnp, go, ge, T, "f32")
    check(f"jac{param_type}", J, j64, j32)


@pytest.mark.parametrize("B,L1,L2,T,go,ge,ragged", ATAN)
def test_tangent_backward_full(d2p, cuda_device, B, L1, L2, T, go, ge, ragged):
    s, ln = _atan_inputs(B, L1, L2, ragged, 85)
    Gm = scores(B, L1, L2, seed=86)
    lnd = None if ln is None else ln.to(cuda_device)
    out = torch.ops.d2p.soft_sw_affine_backward_full(s.to(cuda_device), Gm.to(cuda_device), go, ge, T, lnd)
    lnp = None if ln is None else ln.numpy()
    r64 = oracle.sw_affine_backward_full(s.numpy(), Gm.numpy(), lnp, go, ge, T, "f64")
    r32 = oracle.sw_affine_backward_full(s.numpy(), Gm.numpy(), lnp, go, ge, T, "f32")
    check("grad_scores", out[0], r64[0], r32[0])
    for k in range(1, 4):
        check(f"grad_param{k}", out[k], r64[k], r32[k])


def test_bf16_scores(d2p, cuda_device):
    s = scores(3, 40, 50, seed=12).to(torch.bfloat16)
    res = d2p.soft_sw_affine(s.to(cuda_device), gap_open=-2.0, gap_ext=-0.5, temperature=1.0)
    r64 = oracle.sw_affine(s.float().numpy(), None, -2.0, -0.5, 1.0, "f64")
    r32 = oracle.sw_affine(s.float().numpy(), None, -2.0, -0.5, 1.0, "f32")
    check("value", res.value, r64["value"], r32["value"])
    check("marginals", res.marginals, r64["marginals"], r32["marginals"])


def test_autograd_value_sum(d2p, cuda_device):
    s = scores(4, 30, 41, seed=21).to(cuda_device).requires_grad_(True)
    res = d2p.soft_sw_affine(s, gap_open=-2.0, gap_ext=-0.5, temperature=1.0)
    res.value.sum().backward()
    assert torch.equal(s.grad, res.marginals.detach())


def test_autograd_tensor_params(d2p, cuda_device):
    s0 = scores(3, 12, 17, seed=22)
    s = s0.to(cuda_device).requires_grad_(True)
    go = torch.tensor([-2.0], device=cuda_device, requires_grad=True)
    ge = torch.tensor([-0.5], device=cuda_device, requires_grad=True)
    T = torch.tensor([0.9], device=cuda_device, requires_grad=True)
    res = d2p.soft_sw_affine(s, gap_open=go, gap_ext=ge, temperature=T)
    res.value.sum().backward()
    r64 = oracle.sw_affine(s0.numpy(), None, -2.0, -0.5, 0.9, "f64")
    r32 = oracle.sw_affine(s0.numpy(), None, -2.0, -0.5, 0.9, "f32")
    for name, key, g in (("dopen", "grad_open", go), ("dext", "grad_ext", ge), ("dT", "grad_T", T)):
        check(name, g.grad, np.array([r64[key].sum()]), np.array([r32[key].astype(np.float64).sum()]))


# Shapes for the linear-domain fast path (value + marginals, L2 % 4 == 0):
# single and multiple row-blocks, a partial last row-block, rows shorter than a
# stage, ragged lengths.
FASTAFF = [  # (B, L1, L2, T, gap_open, gap_ext, ragged)
    (2, 1, 4, 1.0, -2.0, -0.5, False), (3, 31, 16, 1.0, -2.0, -0.5, False), (2, 32, 20, 0.5, -2.0, -0.5, False),
    (2, 33, 64, 1.0, -2.0, -0.5, False), (4, 64, 100, 2.0, -1.7, -0.4, False), (2, 130, 260, 1.0, -2.0, -0.5, False),
    (1, 200, 8, 1.0, -2.0, -0.5, False), (2, 100, 120, 1.0, -2.0, -0.5, False), (1, 520, 48, 1.0, -2.0, -0.5, False),
    (6, 70, 96, 1.0, -2.0, -0.5, True), (5, 130, 200, 0.5, -2.0, -0.5, True),
]


@pytest.mark.parametrize("B,L1,L2,T,go,ge,ragged", FASTAFF)
def test_fast_value_marginals(d2p, cuda_device, B, L1, L2, T, go, ge, ragged):
    """soft_sw_affine_float with parameters that need no gradient runs the
    linear-domain kernel (the plane engine recomputes whatever it flags)."""
    s = scores(B, L1, L2, seed=L1 * 11 + L2 + B)
    ln = lengths_for(B, L1, L2, seed=L2) if ragged else None
    if ln is not None:
        ln[0] = torch.tensor([L1, L2], dtype=torch.int32)
    v, m = torch.ops.d2p.soft_sw_affine_float(s.to(cuda_device), go, ge, T, None if ln is None else ln.to(cuda_device))
    lnp = None if ln is None else ln.numpy()
    r64 = oracle.sw_affine(s.numpy(), lnp, go, ge, T, "f64")
    r32 = oracle.sw_affine(s.numpy(), lnp, go, ge, T, "f32")
    check("value", v, r64["value"], r32["value"])
    check("marginals", m, r64["marginals"], r32["marginals"])
    if ln is not None:
        mc = m.cpu()
        for b, (l1, l2) in enumerate(ln.tolist()):
            assert torch.count_nonzero(mc[b, l1:, :]) == 0
            assert torch.count_nonzero(mc[b, :, l2:]) == 0


@pytest.mark.parametrize("B,L1,L2", [(4, 256, 1024), (2, 1024, 1024), (3, 768, 700), (2, 70, 2000)])
def test_fast_long_rows(d2p, cuda_device, B, L1, L2):
    """Long rows, more row-blocks than warps and partitions beyond the double
    range of a single accumulator (S > 1023 log2 units at 1024 x 1024): every
    problem must come out of the linear-domain kernels themselves (one they
    flag is recomputed by the plane engine, whose result would be bitwise the
    plane engine's own) and match the oracle -- value + marginals, and with
    parameter gradients (the tangent kernel's gap sweep pair)."""
    s = scores(B, L1, L2, seed=L1 + 5 * L2)
    v, m = torch.ops.d2p.soft_sw_affine_float(s.to(cuda_device), -2.0, -0.5, 1.0, None)
    v2, m2, g1, g2, g3 = torch.ops.d2p.soft_sw_affine_with_grads(s.to(cuda_device), -2.0, -0.5, 1.0, None)
    _, mp = plane_engine(torch.ops.d2p.soft_sw_affine_float, s.to(cuda_device), -2.0, -0.5, 1.0)
    for b in range(B):
        assert not torch.equal(m[b], mp[b]), f"problem {b} was recomputed by the plane engine"
        assert not torch.equal(m2[b], mp[b]), f"problem {b} (with gradients) was recomputed by the plane engine"
    v4, m4 = torch.ops.d2p.soft_sw_affine_float(s.to(cuda_device), -2.0, -0.5, 1.0, None)
    assert torch.equal(v4, v) and torch.equal(m4, m), "problems spread over several CTAs must repeat bitwise"
    idx = [0, B - 1]
    r64 = oracle.sw_affine(s[idx].numpy(), None, -2.0, -0.5, 1.0, "f64")
    r32 = oracle.sw_affine(s[idx].numpy(), None, -2.0, -0.5, 1.0, "f32")
    check("value", v[idx], r64["value"], r32["value"])
    check("marginals", m[idx], r64["marginals"], r32["marginals"])
    check("value (with grads)", v2[idx], r64["value"], r32["value"])
    check("marginals (with grads)", m2[idx], r64["marginals"], r32["marginals"])
    check("grad_open", g1[idx], r64["grad_open"], r32["grad_open"])
    check("grad_ext", g2[idx], r64["grad_ext"], r32["grad_ext"])
    check("grad_T", g3[idx], r64["grad_T"], r32["grad_T"])


def test_fast_bf16_matches_widened_fp32(d2p, cuda_device):
    """bf16 scores on the fast path give exactly the fp32 result of the
    widened scores (the widening is exact)."""
    s = scores(3, 96, 128, seed=77).to(torch.bfloat16)
    v1, m1 = torch.ops.d2p.soft_sw_affine_float(s.to(cuda_device), -2.0, -0.5, 1.0, None)
    v2, m2 = torch.ops.d2p.soft_sw_affine_float(s.float().to(cuda_device), -2.0, -0.5, 1.0, None)
    assert torch.equal(v1, v2) and torch.equal(m1, m2)
    r64 = oracle.sw_affine(s.float().numpy(), None, -2.0, -0.5, 1.0, "f64")
    r32 = oracle.sw_affine(s.float().numpy(), None, -2.0, -0.5, 1.0, "f32")
    check("marginals", m1, r64["marginals"], r32["marginals"])


def test_fast_and_plane_agree_and_repeat(d2p, cuda_device):
    """The fast paths (value + marginals; with parameter gradients, over more
    than one wave of CTAs) and the plane engine agree, and the fast path is
    bitwise repeatable with many row-blocks and more problems than two per SM
    (ragged, so the CTA order is by cost)."""
    B, L1, L2 = 320, 200, 64
    s = scores(B, L1, L2, seed=5).to(cuda_device)
    ln = lengths_for(B, L1, L2, seed=6).to(cuda_device)
    v1, m1 = torch.ops.d2p.soft_sw_affine_float(s, -2.0, -0.5, 1.0, ln)
    v2, m2, a2, b2, c2 = torch.ops.d2p.soft_sw_affine_with_grads(s, -2.0, -0.5, 1.0, ln)
    torch.testing.assert_close(v1, v2, rtol=1e-5, atol=1e-4)
    torch.testing.assert_close(m1, m2, rtol=0, atol=5e-5)
    sp = torch.nn.functional.pad(s, (0, 1)).contiguous()  # row length 65: the plane engine
    v3, m3, a3, b3, c3 = torch.ops.d2p.soft_sw_affine_with_grads(sp, -2.0, -0.5, 1.0, ln)
    torch.testing.assert_close(v2, v3, rtol=1e-5, atol=1e-4)
    torch.testing.assert_close(m2, m3[..., :L2], rtol=0, atol=5e-5)
    for x, y in ((a2, a3), (b2, b3), (c2, c3)):  # two engines: rounding-level agreement
        torch.testing.assert_close(x, y, rtol=1e-5, atol=1e-4)
    for _ in range(3):
        v3, m3 = torch.ops.d2p.soft_sw_affine_float(s, -2.0, -0.5, 1.0, ln)
        assert torch.equal(v3, v1) and torch.equal(m3, m1)
        out = torch.ops.d2p.soft_sw_affine_with_grads(s, -2.0, -0.5, 1.0, ln)
        for x, y in zip(out, (v2, m2, a2, b2, c2)):
            assert torch.equal(x, y)


@pytest.mark.parametrize("B,L1,L2,T,go,ge,ragged", [
    (3, 100, 120, 1.0, -2.0, -0.5, False),
    (5, 64, 256, 0.5, -1.5, -0.3, True),
    (1, 1024, 256, 1.0, -2.0, -0.5, False),  # one large problem: spread over several CTAs
    (2, 300, 512, 1.0, -2.0, -0.5, True),
    (160, 40, 64, 1.0, -2.0, -0.5, True),  # more problems than SMs
])
def test_fast_param_grads(d2p, cuda_device, B, L1, L2, T, go, ge, ragged):
    """Value, marginals and dS/dgap_open, dS/dgap_ext, dS/dT from the tangent
    kernel's gap sweep pair (dS/dgap_ext from the I and D visits, Euler's
    identity for dS/dT) against the oracle;
    no problem may have been handed to the plane engine."""
    s = scores(B, L1, L2, seed=B + L1 + 7 * L2)
    ln = lengths_for(B, L1, L2, seed=L2, lo=L1 // 2) if ragged else None
    lnd = None if ln is None else ln.to(cuda_device)
    v, m, a, b, c = torch.ops.d2p.soft_sw_affine_with_grads(s.to(cuda_device), go, ge, T, lnd)
    lnp = None if ln is None else ln.numpy()
    r64 = oracle.sw_affine(s.numpy(), lnp, go, ge, T, "f64")
    r32 = oracle.sw_affine(s.numpy(), lnp, go, ge, T, "f32")
    check("value", v, r64["value"], r32["value"])
    check("marginals", m, r64["marginals"], r32["marginals"])
    check("grad_open", a, r64["grad_open"], r32["grad_open"])
    check("grad_ext", b, r64["grad_ext"], r32["grad_ext"])
    check("grad_T", c, r64["grad_T"], r32["grad_T"])
    sp = torch.nn.functional.pad(s, (0, 1)).contiguous().to(cuda_device)
    lp = lnd if lnd is not None else torch.tensor([[L1, L2]] * B, dtype=torch.int32, device=cuda_device)
    _, mp, _, _, _ = torch.ops.d2p.soft_sw_affine_with_grads(sp, go, ge, T, lp)
    for bb in range(B):
        assert not torch.equal(m[bb], mp[bb, :, :L2]), f"problem {bb} was recomputed by the plane engine"
    if ln is not None:
        mc = m.cpu()
        for bb, (l1, l2) in enumerate(ln.tolist()):
            assert torch.count_nonzero(mc[bb, l1:, :]) == 0
            assert torch.count_nonzero(mc[bb, :, l2:]) == 0


def test_low_temperature_fix_up_precision(d2p, cuda_device):
    """T = 0.1 on N(0,1) scores: the linear-domain kernels flag these problems
    and the plane engine recomputes them, its reverse normalising each state's
    incoming weights; value, marginals and the three gradients must stay at
    the reference's own fp32 level."""
    B, L, T, go, ge = 3, 96, 0.1, -2.0, -0.5
    s = scores(B, L, L, seed=L + B)
    r64 = oracle.sw_affine(s.numpy(), None, go, ge, T, "f64")
    r32 = oracle.sw_affine(s.numpy(), None, go, ge, T, "f32")
    v, m = torch.ops.d2p.soft_sw_affine_float(s.to(cuda_device), go, ge, T, None)
    check("value", v, r64["value"], r32["value"])
    check("marginals", m, r64["marginals"], r32["marginals"])
    v2, m2, a, b, c = torch.ops.d2p.soft_sw_affine_with_grads(s.to(cuda_device), go, ge, T, None)
    check("value (with grads)", v2, r64["value"], r32["value"])
    check("marginals (with grads)", m2, r64["marginals"], r32["marginals"])
    check("grad_open", a, r64["grad_open"], r32["grad_open"])
    check("grad_ext", b, r64["grad_ext"], r32["grad_ext"])
    check("grad_T", c, r64["grad_T"], r32["grad_T"])


def test_empty_problems_every_path(d2p, cuda_device):
    """Problems with a zero length (S = 0: only the empty alignment) beside
    full ones, on every value path of both families: value + marginals, with
    parameter gradients in one wave, and (linear) over more than one wave.
    Values, marginals and gradients against the oracle; the empty problems'
    outputs are exactly zero."""
    L1, L2 = 40, 48
    s = scores(4, L1, L2, seed=44)
    ln = torch.tensor([[0, L2], [L1, 0], [0, 0], [L1, L2]], dtype=torch.int32)
    sd, lnd = s.to(cuda_device), ln.to(cuda_device)
    a64 = oracle.sw_affine(s.numpy(), ln.numpy(), -2.0, -0.5, 1.0, "f64")
    a32 = oracle.sw_affine(s.numpy(), ln.numpy(), -2.0, -0.5, 1.0, "f32")
    v, m = torch.ops.d2p.soft_sw_affine_float(sd, -2.0, -0.5, 1.0, lnd)
    check("affine value", v, a64["value"], a32["value"])
    check("affine marginals", m, a64["marginals"], a32["marginals"])
    v, m, go, ge, gT = torch.ops.d2p.soft_sw_affine_with_grads(sd, -2.0, -0.5, 1.0, lnd)
    check("affine value (with grads)", v, a64["value"], a32["value"])
    check("affine marginals (with grads)", m, a64["marginals"], a32["marginals"])
    for name, g, key in (("grad_open", go, "grad_open"), ("grad_ext", ge, "grad_ext"), ("grad_T", gT, "grad_T")):
        check(f"affine {name}", g, a64[key], a32[key])
        assert torch.all(g[:3] == 0)
    assert torch.all(v[:3] == 0) and torch.count_nonzero(m[:3]) == 0
    r64 = oracle.sw_linear(s.numpy(), ln.numpy(), -1.0, 1.0, "f64")
    r32 = oracle.sw_linear(s.numpy(), ln.numpy(), -1.0, 1.0, "f32")
    sms = torch.cuda.get_device_properties(cuda_device).multi_processor_count
    big_s = torch.cat([sd, sd[3:].expand(sms, -1, -1)]).contiguous()
    big_l = torch.cat([lnd, lnd[3:].expand(sms, -1)]).contiguous()
    v1, m1 = torch.ops.d2p.soft_sw_float(sd, -1.0, 1.0, lnd)
    runs = [("one wave", torch.ops.d2p.soft_sw_with_grads(sd, -1.0, 1.0, lnd)),
            ("log-domain kernel", [t[:4] for t in torch.ops.d2p.soft_sw_with_grads(big_s, -1.0, 1.0, big_l)])]
    check("linear value", v1, r64["value"], r32["value"])
    check("linear marginals", m1, r64["marginals"], r32["marginals"])
    for name, (v, m, gg, gt) in runs:
        check(f"linear value ({name})", v, r64["value"], r32["value"])
        check(f"linear marginals ({name})", m, r64["marginals"], r32["marginals"])
        check(f"linear grad_gap ({name})", gg, r64["grad_gap"], r32["grad_gap"])
        check(f"linear grad_T ({name})", gt, r64["grad_T"], r32["grad_T"])
        assert torch.all(v[:3] == 0) and torch.all(gg[:3] == 0) and torch.all(gt[:3] == 0)
        assert torch.count_nonzero(m[:3]) == 0


def test_bf16_param_grads_on_the_tangent_kernel(d2p, cuda_device):
    """bf16 scores with parameter gradients: the scores are widened (exactly)
    for the tangent kernel's gap sweep pair, so every output equals the fp32
    result of the widened scores bitwise, and no problem falls back to the
    plane engine."""
    B, L1, L2 = 4, 96, 128
    s = scores(B, L1, L2, seed=88).to(torch.bfloat16)
    w = s.float()
    out_b = torch.ops.d2p.soft_sw_affine_with_grads(s.to(cuda_device), -2.0, -0.5, 1.0, None)
    out_f = torch.ops.d2p.soft_sw_affine_with_grads(w.to(cuda_device), -2.0, -0.5, 1.0, None)
    for x, y in zip(out_b, out_f):
        assert torch.equal(x, y)
    wp = torch.nn.functional.pad(w, (0, 1)).contiguous().to(cuda_device)  # row length 129: the plane engine
    lp = torch.tensor([[L1, L2]] * B, dtype=torch.int32, device=cuda_device)
    mp = torch.ops.d2p.soft_sw_affine_with_grads(wp, -2.0, -0.5, 1.0, lp)[1][..., :L2]
    for b in range(B):
        assert not torch.equal(out_b[1][b], mp[b]), f"problem {b} was recomputed by the plane engine"
    r64 = oracle.sw_affine(w.numpy(), None, -2.0, -0.5, 1.0, "f64")
    r32 = oracle.sw_affine(w.numpy(), None, -2.0, -0.5, 1.0, "f32")
    check("marginals", out_b[1], r64["marginals"], r32["marginals"])
    check("grad_open", out_b[2], r64["grad_open"], r32["grad_open"])
    check("grad_ext", out_b[3], r64["grad_ext"], r32["grad_ext"])
    check("grad_T", out_b[4], r64["grad_T"], r32["grad_T"])


def test_backward_full_is_two_sweep_pairs(d2p, cuda_device):
    """backward_full runs two tangent-kernel launches: the dot sweep along
    gap_ext, then the BF sweep (H g, the gap_open part and, by Euler's
    identity, the temperature part), where it ran four; the plane engine's
    fix-up launches find nothing to do.  A problem spread over several CTAs
    (B = 1) takes the same two launches."""
    from torch.profiler import ProfilerActivity, profile

    for B, L1, L2 in [(3, 130, 260), (1, 1024, 256)]:
        s = scores(B, L1, L2, seed=91).to(cuda_device)
        G = scores(B, L1, L2, seed=92).to(cuda_device)
        torch.ops.d2p.soft_sw_affine_backward_full(s, G, -2.0, -0.5, 1.0, None)
        c0 = d2p.engine_counts()
        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            torch.ops.d2p.soft_sw_affine_backward_full(s, G, -2.0, -0.5, 1.0, None)
            torch.cuda.synchronize()
        names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
        assert sum("aff_tan_kernel" in n for n in names) == 2, names
        assert d2p.engine_counts() == c0, "a problem reached the plane engine"
