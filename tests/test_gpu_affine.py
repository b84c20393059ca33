"""GPU parity of the affine-gap soft Smith-Waterman ops against the CPU oracle."""
import numpy as np
import pytest
import torch

import oracle
from tests._parity import check, lengths_for, scores

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
    check("grad_open", a, r64["grad_open"], r32["grad_open"], rtol=1e-4, atol=1e-5)
    check("grad_ext", b, r64["grad_ext"], r32["grad_ext"], rtol=1e-4, atol=1e-5)
    check("grad_T", c, r64["grad_T"], r32["grad_T"], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("B,L1,L2,T,go,ge", CASES[:5])
def test_variable_lengths_and_padding(d2p, cuda_device, B, L1, L2, T, go, ge):
    s = scores(B, L1, L2, seed=17)
    ln = lengths_for(B, L1, L2, seed=20260707)
    v, m, a, b, c = torch.ops.d2p.soft_sw_affine_with_grads(s.to(cuda_device), go, ge, T, ln.to(cuda_device))
    r64 = oracle.sw_affine(s.numpy(), ln.numpy(), go, ge, T, "f64")
    r32 = oracle.sw_affine(s.numpy(), ln.numpy(), go, ge, T, "f32")
    check("value", v, r64["value"], r32["value"])
    check("marginals", m, r64["marginals"], r32["marginals"])
    check("grad_open", a, r64["grad_open"], r32["grad_open"], rtol=1e-4, atol=1e-5)
    check("grad_ext", b, r64["grad_ext"], r32["grad_ext"], rtol=1e-4, atol=1e-5)
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
    check("hvp", H, h64, h32, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("param_type", [0, 1, 2])
@pytest.mark.parametrize("B,L1,L2,T,go,ge", CASES[:4])
def test_param_jacobian(d2p, cuda_device, B, L1, L2, T, go, ge, param_type):
    s = scores(B, L1, L2, seed=5)
    J = torch.ops.d2p.soft_sw_affine_param_jacobian(s.to(cuda_device), param_type, go, ge, T, None)
    j64 = oracle.sw_affine_param_jacobian(s.numpy(), param_type, None, go, ge, T, "f64")
    j32 = oracle.sw_affine_param_jacobian(s.numpy(), param_type, None, go, ge, T, "f32")
    check(f"jac{param_type}", J, j64, j32, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("B,L1,L2,T,go,ge", CASES[:3])
def test_backward_full(d2p, cuda_device, B, L1, L2, T, go, ge):
    s = scores(B, L1, L2, seed=8)
    G = scores(B, L1, L2, seed=9)
    out = torch.ops.d2p.soft_sw_affine_backward_full(s.to(cuda_device), G.to(cuda_device), go, ge, T, None)
    r64 = oracle.sw_affine_backward_full(s.numpy(), G.numpy(), None, go, ge, T, "f64")
    r32 = oracle.sw_affine_backward_full(s.numpy(), G.numpy(), None, go, ge, T, "f32")
    check("grad_scores", out[0], r64[0], r32[0], rtol=1e-4, atol=1e-5)
    for k in range(1, 4):
        check(f"grad_param{k}", out[k], r64[k], r32[k], rtol=1e-4, atol=1e-4)


def test_bf16_scores(d2p, cuda_device):
    s = scores(3, 40, 50, seed=12).to(torch.bfloat16)
    res = d2p.soft_sw_affine(s.to(cuda_device), gap_open=-2.0, gap_ext=-0.5, temperature=1.0)
    r64 = oracle.sw_affine(s.float().numpy(), None, -2.0, -0.5, 1.0, "f64")
    check("value", res.value, r64["value"])
    check("marginals", res.marginals, r64["marginals"])


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
    check("dopen", go.grad, np.array([r64["grad_open"].sum()]), rtol=1e-4, atol=1e-5)
    check("dext", ge.grad, np.array([r64["grad_ext"].sum()]), rtol=1e-4, atol=1e-5)
    check("dT", T.grad, np.array([r64["grad_T"].sum()]), rtol=1e-4, atol=1e-5)
