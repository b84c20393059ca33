"""Parity at the BASELINE configurations, at their own shapes, seeds and parameters.

Each test runs the product on the configuration's full batch (the same seeded
inputs bench.py uses: scores ``randn`` from a CPU generator seeded 0, C3
lengths from seed 1, the C5 HVP direction from seed 2) and compares a sample
of its problems -- the first, the last and, for the ragged batch, the
smallest and the largest -- with the CPU oracle in fp64 and fp32.  The
tolerance is BASELINE's: 1e-5 relative / 1e-6 absolute for fp32 results, and
for bf16 inputs after upcast 1e-2 relative; where the reference's own fp32
result misses that against fp64 (long logsumexp chains), ours must be no
further from fp64 than the reference is (tests/_parity.py).

  C1  soft_sw [2,100,120] fp32, gap -1, T 1; forward + value.sum().backward()
  C2  soft_sw [256,512,512] fp32, gap -1, T 1; forward + backward; HVP
  C3  soft_sw [1024,512,512] fp32, lengths U[64,512], gap -0.5, T 0.5
  C4  soft_sw_affine [64,1024,1024] bf16, open -2, ext -0.5, T 1
  C5  soft_sw [32,4096,4096] 0.5 N(0,1), gap -1, T 1; forward, backward, HVP
      (one problem of the batch: the first 4096 x 4096 problem of the seeded
      batch equals a seeded draw of that one problem, since torch.randn fills
      a CPU tensor in order)
"""
import numpy as np
import pytest
import torch

import oracle
from tests._parity import BF16_RTOL, check

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def d2p():
    import d2p_b200

    return d2p_b200


def _randn(shape, seed, scale=1.0):
    return torch.randn(*shape, generator=torch.Generator().manual_seed(seed)) * scale


def _fwd_bwd(d2p, s_dev, fn):
    """forward (value + marginals) and value.sum().backward(), as bench.py's step"""
    x = s_dev.detach().requires_grad_(True)
    res = fn(x)
    res.value.sum().backward()
    return res.value.detach(), res.marginals.detach(), x.grad


def _linear_checks(tag, v, m, g, s_np, ln_np, gap, T, idx):
    r64 = oracle.sw_linear(s_np, ln_np, gap, T, "f64")
    r32 = oracle.sw_linear(s_np, ln_np, gap, T, "f32")
    check(f"{tag} value", v[idx], r64["value"], r32["value"])
    check(f"{tag} marginals", m[idx], r64["marginals"], r32["marginals"])
    # value.sum().backward() gives grad = 1 * marginals
    check(f"{tag} grad", g[idx], r64["marginals"], r32["marginals"])
    return r64, r32


def test_c1(d2p, cuda_device):
    s = _randn((2, 100, 120), 0)
    v, m, g = _fwd_bwd(d2p, s.to(cuda_device), lambda x: d2p.soft_sw(x, gap=-1.0, temperature=1.0))
    r64, r32 = _linear_checks("c1", v, m, g, s.numpy(), None, -1.0, 1.0, [0, 1])
    _, _, gg, gt = torch.ops.d2p.soft_sw_with_grads(s.to(cuda_device), -1.0, 1.0, None)
    check("c1 grad_gap", gg, r64["grad_gap"], r32["grad_gap"])
    check("c1 grad_T", gt, r64["grad_T"], r32["grad_T"])


@pytest.fixture(scope="module")
def c2_inputs():
    return _randn((256, 512, 512), 0)


def test_c2_forward_backward(d2p, cuda_device, c2_inputs):
    s = c2_inputs
    v, m, g = _fwd_bwd(d2p, s.to(cuda_device), lambda x: d2p.soft_sw(x, gap=-1.0, temperature=1.0))
    assert torch.equal(g, m)
    idx = [0, 1, 147, 255]
    _linear_checks("c2", v, m, g, s[idx].numpy(), None, -1.0, 1.0, idx)


def test_c2_param_grads(d2p, cuda_device, c2_inputs):
    """Learnable gap and temperature at C2: dS/dgap, dS/dT per problem."""
    s = c2_inputs
    v, m, gg, gt = torch.ops.d2p.soft_sw_with_grads(s.to(cuda_device), -1.0, 1.0, None)
    idx = [0, 255]
    r64 = oracle.sw_linear(s[idx].numpy(), None, -1.0, 1.0, "f64")
    r32 = oracle.sw_linear(s[idx].numpy(), None, -1.0, 1.0, "f32")
    check("c2 value (with grads)", v[idx], r64["value"], r32["value"])
    check("c2 marginals (with grads)", m[idx], r64["marginals"], r32["marginals"])
    check("c2 grad_gap", gg[idx], r64["grad_gap"], r32["grad_gap"])
    check("c2 grad_T", gt[idx], r64["grad_T"], r32["grad_T"])


def test_c2_hvp(d2p, cuda_device, c2_inputs):
    """HVP along a seeded N(0,1) direction over the whole C2 batch."""
    s = c2_inputs
    V = _randn((256, 512, 512), 2)
    H = torch.ops.d2p.soft_sw_hvp(s.to(cuda_device), V.to(cuda_device), -1.0, 1.0, None)
    idx = [0, 255]
    h64 = oracle.sw_linear_hvp(s[idx].numpy(), V[idx].numpy(), None, -1.0, 1.0, "f64")
    h32 = oracle.sw_linear_hvp(s[idx].numpy(), V[idx].numpy(), None, -1.0, 1.0, "f32")
    check("c2 hvp", H[idx], h64, h32)


def test_c2_backward_full(d2p, cuda_device, c2_inputs):
    """A loss on the marginals at C2 (grad_scores, grad_gap, grad_T)."""
    s = c2_inputs[:8]
    G = _randn((8, 512, 512), 3)
    gs, gg, gt = torch.ops.d2p.soft_sw_backward_full(s.to(cuda_device), G.to(cuda_device), -1.0, 1.0, None)
    idx = [0, 7]
    r64 = oracle.sw_linear_backward_full(s[idx].numpy(), G[idx].numpy(), None, -1.0, 1.0, "f64")
    r32 = oracle.sw_linear_backward_full(s[idx].numpy(), G[idx].numpy(), None, -1.0, 1.0, "f32")
    check("c2 backward_full grad_scores", gs[idx], r64[0], r32[0])
    # the parameter gradients are batch sums: compare the two problems' sum
    gs2, gg2, gt2 = torch.ops.d2p.soft_sw_backward_full(s[idx].to(cuda_device), G[idx].to(cuda_device), -1.0, 1.0,
                                                        None)
    check("c2 backward_full grad_gap", gg2, r64[1], r32[1])
    check("c2 backward_full grad_T", gt2, r64[2], r32[2])
    assert torch.equal(gs2, gs[idx])


def test_c3_ragged(d2p, cuda_device):
    s = _randn((1024, 512, 512), 0)
    ln = torch.randint(64, 513, (1024, 2), generator=torch.Generator().manual_seed(1), dtype=torch.int32)
    lnd = ln.to(cuda_device)
    v, m, g = _fwd_bwd(d2p, s.to(cuda_device),
                       lambda x: d2p.soft_sw(x, gap=-0.5, temperature=0.5, lengths=lnd))
    assert torch.equal(g, m)
    area = (ln[:, 0].long() * ln[:, 1].long())
    idx = sorted({0, 1023, int(area.argmin()), int(area.argmax()), 517})
    _linear_checks("c3", v, m, g, s[idx].numpy(), ln[idx].numpy(), -0.5, 0.5, idx)
    mc = m[idx].cpu()
    for k, b in enumerate(idx):
        l1, l2 = ln[b].tolist()
        assert torch.count_nonzero(mc[k, l1:, :]) == 0 and torch.count_nonzero(mc[k, :, l2:]) == 0


def test_c4_affine_bf16(d2p, cuda_device):
    s = _randn((64, 1024, 1024), 0).to(torch.bfloat16)
    v, m, g = _fwd_bwd(d2p, s.to(cuda_device),
                       lambda x: d2p.soft_sw_affine(x, gap_open=-2.0, gap_ext=-0.5, temperature=1.0))
    assert g.dtype == torch.bfloat16
    idx = [0, 63]
    sw = s[idx].float().numpy()  # the reference runs on the upcast scores
    r64 = oracle.sw_affine(sw, None, -2.0, -0.5, 1.0, "f64")
    r32 = oracle.sw_affine(sw, None, -2.0, -0.5, 1.0, "f32")
    # computed in fp32 on the exactly widened scores: BASELINE's fp32 bar
    check("c4 value", v[idx], r64["value"], r32["value"])
    check("c4 marginals", m[idx], r64["marginals"], r32["marginals"])
    # and BASELINE's bf16 bar: after upcast, within 1e-2 relative of the reference
    np.testing.assert_allclose(v[idx].cpu().numpy(), r32["value"], rtol=BF16_RTOL, atol=0)
    np.testing.assert_allclose(m[idx].cpu().numpy(), r32["marginals"], rtol=BF16_RTOL, atol=1e-6)
    # the backward's gradient is in the scores' dtype: bf16(marginals)
    np.testing.assert_allclose(g[idx].float().cpu().numpy(), r32["marginals"], rtol=BF16_RTOL, atol=1e-6)
    assert torch.equal(g, m.to(torch.bfloat16))


def test_c4_affine_bf16_param_grads(d2p, cuda_device):
    """C4 with learnable gap penalties and temperature: dS/d(open, ext, T)."""
    s = _randn((64, 1024, 1024), 0).to(torch.bfloat16)
    out = torch.ops.d2p.soft_sw_affine_with_grads(s.to(cuda_device), -2.0, -0.5, 1.0, None)
    idx = [0, 63]
    sw = s[idx].float().numpy()
    r64 = oracle.sw_affine(sw, None, -2.0, -0.5, 1.0, "f64")
    r32 = oracle.sw_affine(sw, None, -2.0, -0.5, 1.0, "f32")
    for k, key in ((0, "value"), (1, "marginals"), (2, "grad_open"), (3, "grad_ext"), (4, "grad_T")):
        check(f"c4 {key} (with grads)", out[k][idx], r64[key], r32[key])


@pytest.fixture(scope="module")
def c5_inputs():
    s = _randn((1, 4096, 4096), 0, scale=0.5)  # problem 0 of 0.5 * randn(32, 4096, 4096), seed 0
    V = _randn((1, 4096, 4096), 2)             # problem 0 of randn(32, 4096, 4096), seed 2
    return s, V


def test_c5_forward_backward(d2p, cuda_device, c5_inputs):
    s, _ = c5_inputs
    # four problems per GPU at 8 GPUs: problem 0 beside three others
    batch = torch.cat([s, _randn((3, 4096, 4096), 5, scale=0.5)])
    v, m, g = _fwd_bwd(d2p, batch.to(cuda_device), lambda x: d2p.soft_sw(x, gap=-1.0, temperature=1.0))
    assert torch.equal(g, m)
    _linear_checks("c5", v, m, g, s.numpy(), None, -1.0, 1.0, [0])


def test_c5_hvp(d2p, cuda_device, c5_inputs):
    s, V = c5_inputs
    H = torch.ops.d2p.soft_sw_hvp(s.to(cuda_device), V.to(cuda_device), -1.0, 1.0, None)
    h64 = oracle.sw_linear_hvp(s.numpy(), V.numpy(), None, -1.0, 1.0, "f64")
    h32 = oracle.sw_linear_hvp(s.numpy(), V.numpy(), None, -1.0, 1.0, "f32")
    check("c5 hvp", H, h64, h32)
