"""The reference's own contract tests, run against the drop-in on CUDA.

Ported from the reference's test files (their CUDA parametrisations):
validation messages (tests/test_soft_sw_regular.py:376-452, :632-719;
tests/test_soft_sw_affine.py:397-580), autocast (tests/test_autocast.py:17-140),
masks and the modules (d2p/sw.py:153-239, :429-604), the alias ops
(src/sw/torch_cuda.cpp:778-848), torch.compile over the ``d2p_py::`` custom
ops (d2p/_pt2_ops.py) and the device guard (current device != the scores'
device).
"""
import numpy as np
import pytest
import torch

import oracle
from tests._parity import check, scores

pytestmark = pytest.mark.gpu

TWO_GPUS = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                              reason="requires two CUDA devices")


@pytest.fixture(scope="module")
def d2p():
    import d2p_b200

    return d2p_b200


# ------------------------------------------------------------------ validation
@pytest.mark.parametrize("op", ["soft_sw_float", "soft_sw_affine_float"])
@pytest.mark.parametrize("lengths,match", [([[-1, 5]], r"lengths\[0,0\] must be between 0 and 4"),
                                           ([[4, 6]], r"lengths\[0,1\] must be between 0 and 5")])
def test_invalid_lengths_raise(d2p, cuda_device, op, lengths, match):
    s = torch.randn(1, 4, 5, device=cuda_device)
    ln = torch.tensor(lengths, dtype=torch.int32, device=cuda_device)
    params = (-2.0, -0.5, 1.0) if "affine" in op else (-1.0, 1.0)
    with pytest.raises(RuntimeError, match=match):
        getattr(d2p, op)(s, *params, ln)


def test_hvp_and_backward_full_shape_mismatch(d2p, cuda_device):
    s = torch.randn(1, 4, 5, device=cuda_device)
    bad = torch.randn(1, 4, 4, device=cuda_device)
    with pytest.raises(RuntimeError, match="scores and tangent must have same shape"):
        d2p.soft_sw_hvp(s, bad, -1.0, 1.0, None)
    with pytest.raises(RuntimeError, match="scores and tangent must have same shape"):
        d2p.soft_sw_affine_hvp(s, bad, -2.0, -0.5, 1.0, None)
    with pytest.raises(RuntimeError, match="grad_alignment must have same shape as scores"):
        d2p.soft_sw_backward_full(s, bad, -1.0, 1.0, None)
    with pytest.raises(RuntimeError, match="grad_alignment must have same shape as scores"):
        d2p.soft_sw_affine_backward_full(s, bad, -2.0, -0.5, 1.0, None)
    with pytest.raises(RuntimeError, match="grad_alignment must be a CUDA tensor"):
        d2p.soft_sw_affine_backward_full(s, torch.randn(1, 4, 5), -2.0, -0.5, 1.0, None)
    with pytest.raises(RuntimeError, match="scores must be 3D"):
        d2p.soft_sw_affine_hvp(torch.randn(4, 5, device=cuda_device), torch.randn(4, 5, device=cuda_device),
                               -2.0, -0.5, 1.0, None)
    with pytest.raises(RuntimeError, match="param_type must be 0 or 1"):
        d2p.soft_sw_param_jacobian(s, 2, -1.0, 1.0, None)
    with pytest.raises(RuntimeError, match="param_type must be 0, 1, or 2"):
        d2p.soft_sw_affine_param_jacobian(s, 3, -2.0, -0.5, 1.0, None)


def test_oversized_dp_table_rejected_before_allocation(d2p, cuda_device):
    s = torch.empty((0, 46341, 46341), device=cuda_device)
    t = torch.empty_like(s)
    ln = torch.empty((0, 2), dtype=torch.int32, device=cuda_device)
    gap = torch.tensor([-1.0], device=cuda_device)
    T = torch.tensor([1.0], device=cuda_device)
    calls = (lambda: d2p.ops.sw.forward_t(s, gap, T, ln),
             lambda: torch.ops.d2p.soft_sw(s, gap, T, ln),
             lambda: d2p.soft_sw_float(s, -1.0, 1.0, None),
             lambda: d2p.soft_sw_with_grads(s, -1.0, 1.0, None),
             lambda: d2p.soft_sw_hvp(s, t, -1.0, 1.0, None),
             lambda: d2p.soft_sw_param_jacobian(s, 0, -1.0, 1.0, None),
             lambda: d2p.soft_sw_backward_full(s, t, -1.0, 1.0, None))
    for call in calls:
        with pytest.raises(RuntimeError, match="SW CUDA DP table is too large"):
            call()
    wide = torch.empty((1, 0, torch.iinfo(torch.int32).max // 3), device=cuda_device)
    with pytest.raises(RuntimeError, match="sw_affine DP table too large"):
        d2p.soft_sw_affine_with_grads(wide, -2.0, -0.5, 1.0, None)


def test_half_precision_inputs_need_autocast(d2p, cuda_device):
    """fp16 scores outside autocast are refused (src/common/torch_utils.h:619-621);
    the affine kernels take bf16 scores directly."""
    s16 = torch.randn(2, 4, 5, device=cuda_device, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="must be float32"):
        d2p.soft_sw_float(s16, -1.0, 1.0, None)
    v, m = d2p.soft_sw_affine_float(s16.to(torch.bfloat16), -2.0, -0.5, 1.0, None)
    assert v.dtype == torch.float32 and m.dtype == torch.float32


# ------------------------------------------------------------------ autocast
class TestAutocast:
    def test_soft_sw_promotes_fp16(self, d2p, cuda_device):
        s = torch.randn(2, 8, 10, device=cuda_device, dtype=torch.float16)
        with torch.autocast("cuda", dtype=torch.float16):
            r = d2p.soft_sw(s, gap=-1.0)
        assert r.value.dtype == torch.float32 and r.marginals.dtype == torch.float32

    def test_soft_sw_bf16(self, d2p, cuda_device):
        s = torch.randn(2, 8, 10, device=cuda_device, dtype=torch.bfloat16)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            r = d2p.soft_sw(s, gap=-1.0)
        assert r.value.dtype == torch.float32 and r.marginals.dtype == torch.float32

    def test_soft_sw_affine(self, d2p, cuda_device):
        s = torch.randn(2, 8, 10, device=cuda_device, dtype=torch.float16)
        with torch.autocast("cuda", dtype=torch.float16):
            r = d2p.soft_sw_affine(s, gap_open=-2.0, gap_ext=-0.5)
        assert r.value.dtype == torch.float32 and r.marginals.dtype == torch.float32

    def test_gradient_flow(self, d2p, cuda_device):
        s = torch.randn(2, 8, 10, device=cuda_device, dtype=torch.float16, requires_grad=True)
        with torch.autocast("cuda", dtype=torch.float16):
            loss = d2p.soft_sw(s, gap=-1.0).value.sum()
        loss.backward()
        assert s.grad is not None and s.grad.dtype == torch.float16

    def test_matches_explicit_fp32(self, d2p, cuda_device):
        torch.manual_seed(42)
        s16 = torch.randn(4, 16, 20, device=cuda_device, dtype=torch.float16)
        with torch.autocast("cuda", dtype=torch.float16):
            ra = d2p.soft_sw(s16, gap=-1.0)
        rf = d2p.soft_sw(s16.float(), gap=-1.0)
        assert torch.equal(ra.value, rf.value) and torch.equal(ra.marginals, rf.marginals)

    def test_fp32_unchanged(self, d2p, cuda_device):
        s = torch.randn(2, 8, 10, device=cuda_device)
        with torch.autocast("cuda", dtype=torch.float16):
            r = d2p.soft_sw(s, gap=-1.0)
        assert r.value.dtype == torch.float32 and torch.equal(r.value, d2p.soft_sw(s, gap=-1.0).value)

    def test_low_level_forward(self, d2p, cuda_device):
        from d2p_b200 import sw as swmod

        s = torch.randn(2, 8, 10, device=cuda_device, dtype=torch.float16)
        with torch.autocast("cuda", dtype=torch.float16):
            v, m = swmod.soft_sw_forward(s, -1.0, 1.0, None)
            va, ma = swmod.soft_sw_affine_forward(s, -2.0, -0.5, 1.0, None)
        assert {v.dtype, m.dtype, va.dtype, ma.dtype} == {torch.float32}


# ------------------------------------------------------------------ masks, modules
def test_masks_equal_lengths(d2p, cuda_device):
    B, L1, L2 = 4, 20, 24
    s = scores(B, L1, L2, seed=5).to(cuda_device)
    l1 = torch.tensor([20, 7, 1, 13])
    l2 = torch.tensor([24, 9, 24, 2])
    m1 = torch.arange(L1)[None, :] < l1[:, None]
    m2 = torch.arange(L2)[None, :] < l2[:, None]
    ln = torch.stack([l1, l2], 1).to(torch.int32).to(cuda_device)
    for fn, kw in ((d2p.soft_sw, {}), (d2p.soft_sw_affine, {}), (d2p.soft_sw, {"gap": torch.tensor(-1.0)})):
        a = fn(s, lengths=ln, **kw)
        b = fn(s, mask1=m1.to(cuda_device), mask2=m2.to(cuda_device), **kw)
        assert torch.equal(a.value, b.value) and torch.equal(a.marginals, b.marginals)
    bad = m1.clone()
    bad[1, 12] = True  # a hole
    with pytest.raises(ValueError, match="mask1 is not prefix-only"):
        d2p.soft_sw(s, mask1=bad.to(cuda_device))


def test_soft_sw_module_gradients(d2p, cuda_device):
    """SoftSW with learnable gap and temperature: the parameters receive the
    batch sums of dS/dgap, dS/dT (d2p/sw.py:429-510)."""
    s0 = scores(3, 24, 28, seed=31)
    mod = d2p.SoftSW(gap=-1.0, temperature=0.8, learn_gap=True, learn_temperature=True).to(cuda_device)
    s = s0.to(cuda_device).requires_grad_(True)
    res = mod(s)
    res.value.sum().backward()
    r64 = oracle.sw_linear(s0.numpy(), None, -1.0, 0.8, "f64")
    r32 = oracle.sw_linear(s0.numpy(), None, -1.0, 0.8, "f32")
    check("module value", res.value, r64["value"], r32["value"])
    check("module dgap", mod.gap.grad, np.array([r64["grad_gap"].sum()]),
          np.array([r32["grad_gap"].astype(np.float64).sum()]))
    check("module dT", mod.temperature.grad, np.array([r64["grad_T"].sum()]),
          np.array([r32["grad_T"].astype(np.float64).sum()]))
    check("module dscores", s.grad, r64["marginals"], r32["marginals"])


def test_soft_sw_affine_module_gradients(d2p, cuda_device):
    s0 = scores(2, 20, 24, seed=32)
    mod = d2p.SoftSWAffine(learn_gap_open=True, learn_gap_ext=True, learn_temperature=True).to(cuda_device)
    res = mod(s0.to(cuda_device))
    res.value.sum().backward()
    r64 = oracle.sw_affine(s0.numpy(), None, -2.0, -0.5, 1.0, "f64")
    r32 = oracle.sw_affine(s0.numpy(), None, -2.0, -0.5, 1.0, "f32")
    for p, key in ((mod.gap_open, "grad_open"), (mod.gap_ext, "grad_ext"), (mod.temperature, "grad_T")):
        check(f"module {key}", p.grad, np.array([r64[key].sum()]), np.array([r32[key].astype(np.float64).sum()]))


# ------------------------------------------------------------------ alias ops
def test_alias_ops_match_primary_ops(d2p, cuda_device):
    """The sw_* / sw_affine_* schemas are the same computations under the
    reference's structured names (src/sw/torch_cuda.cpp:778-848)."""
    s = scores(3, 17, 20, seed=33).to(cuda_device)
    G = scores(3, 17, 20, seed=34).to(cuda_device)
    ln = torch.tensor([[17, 20], [9, 11], [17, 4]], dtype=torch.int32, device=cuda_device)
    ops = torch.ops.d2p
    gap, T = torch.tensor([-1.0], device=cuda_device), torch.tensor([1.0], device=cuda_device)

    def same(a, b):
        a = list(a) if isinstance(a, (list, tuple)) else [a]
        b = list(b) if isinstance(b, (list, tuple)) else [b]
        assert len(a) == len(b) and all(torch.equal(x, y) for x, y in zip(a, b))

    same(ops.sw_forward(s, -1.0, 1.0, ln), ops.soft_sw_float(s, -1.0, 1.0, ln))
    same(ops.sw_forward_t(s, gap, T, ln), ops.soft_sw(s, gap, T, ln))
    wg = ops.soft_sw_with_grads(s, -1.0, 1.0, ln)
    same(ops.sw_value_grad_params(s, -1.0, 1.0, ln), (wg[2], wg[3]))
    same(ops.sw_marginals_backward(s, G, -1.0, 1.0, ln), ops.soft_sw_backward_full(s, G, -1.0, 1.0, ln))
    same(ops.sw_marginals_hvp(s, G, -1.0, 1.0, ln), ops.soft_sw_hvp(s, G, -1.0, 1.0, ln))
    same(ops.sw_marginals_grad_gap(s, -1.0, 1.0, ln), ops.soft_sw_param_jacobian(s, 0, -1.0, 1.0, ln))
    same(ops.sw_marginals_grad_temp(s, -1.0, 1.0, ln), ops.soft_sw_param_jacobian(s, 1, -1.0, 1.0, ln))
    go, ge = torch.tensor([-2.0], device=cuda_device), torch.tensor([-0.5], device=cuda_device)
    p = (-2.0, -0.5, 1.0)
    same(ops.sw_affine_forward(s, *p, ln), ops.soft_sw_affine_float(s, *p, ln))
    same(ops.sw_affine_forward_t(s, go, ge, T, ln), ops.soft_sw_affine(s, go, ge, T, ln))
    wa = ops.soft_sw_affine_with_grads(s, *p, ln)
    same(ops.sw_affine_value_grad_params(s, *p, ln), (wa[2], wa[3], wa[4]))
    same(ops.sw_affine_marginals_backward(s, G, *p, ln), ops.soft_sw_affine_backward_full(s, G, *p, ln))
    same(ops.sw_affine_marginals_hvp(s, G, *p, ln), ops.soft_sw_affine_hvp(s, G, *p, ln))
    same(ops.sw_affine_marginals_grad_gap_open(s, *p, ln), ops.soft_sw_affine_param_jacobian(s, 0, *p, ln))
    same(ops.sw_affine_marginals_grad_gap_ext(s, *p, ln), ops.soft_sw_affine_param_jacobian(s, 1, *p, ln))
    same(ops.sw_affine_marginals_grad_temp(s, *p, ln), ops.soft_sw_affine_param_jacobian(s, 2, *p, ln))
    # the nw_* names of the linear soft Needleman-Wunsch ops (src/nw/torch_cuda.cpp:700-785)
    same(ops.nw_forward(s, -1.0, 1.0, ln), ops.soft_nw_float(s, -1.0, 1.0, ln))
    same(ops.nw_forward_t(s, gap, T, ln), ops.soft_nw(s, gap, T, ln))
    wn = ops.soft_nw_with_grads(s, -1.0, 1.0, ln)
    same(ops.nw_value_grad_params(s, -1.0, 1.0, ln), (wn[2], wn[3]))
    same(ops.nw_marginals_backward(s, G, -1.0, 1.0, ln), ops.soft_nw_backward_full(s, G, -1.0, 1.0, ln))
    same(ops.nw_marginals_hvp(s, G, -1.0, 1.0, ln), ops.soft_nw_hvp(s, G, -1.0, 1.0, ln))
    same(ops.nw_marginals_grad_gap(s, -1.0, 1.0, ln), ops.soft_nw_param_jacobian(s, 0, -1.0, 1.0, ln))
    same(ops.nw_marginals_grad_temp(s, -1.0, 1.0, ln), ops.soft_nw_param_jacobian(s, 1, -1.0, 1.0, ln))


def test_outputs_are_independent_tensors(d2p, cuda_device):
    """Schemas without alias annotations return fresh tensors: no output shares
    storage with another (custom ops and functionalization rely on it)."""
    s = scores(3, 9, 12, seed=38).to(cuda_device)
    for out in (torch.ops.d2p.soft_sw_with_grads(s, -1.0, 1.0, None),
                torch.ops.d2p.soft_sw_affine_with_grads(s, -2.0, -0.5, 1.0, None),
                torch.ops.d2p.sw_value_grad_params(s, -1.0, 1.0, None),
                torch.ops.d2p.sw_affine_value_grad_params(s, -2.0, -0.5, 1.0, None)):
        ptrs = [t.untyped_storage().data_ptr() for t in out]
        assert len(set(ptrs)) == len(ptrs)


# ------------------------------------------------------------------ torch.compile
def test_fake_shapes_match_real_outputs(d2p, cuda_device):
    """Every op's fake kernel (d2p/_compile.py:24-250) describes the real
    outputs: shape, dtype and device."""
    from torch._subclasses.fake_tensor import FakeTensorMode

    from tests.test_api_host import SCHEMAS, _call_args

    real = scores(2, 6, 8, seed=35).to(cuda_device)
    for name in sorted(SCHEMAS):
        out_r = getattr(torch.ops.d2p, name)(*_call_args(name, real, 2))
        with FakeTensorMode() as mode:
            fake = mode.from_tensor(real)
            out_f = getattr(torch.ops.d2p, name)(*_call_args(name, fake, 2))
        rs = list(out_r) if isinstance(out_r, (list, tuple)) else [out_r]
        fs = list(out_f) if isinstance(out_f, (list, tuple)) else [out_f]
        assert [(t.shape, t.dtype, t.device) for t in rs] == [(t.shape, t.dtype, t.device) for t in fs], name


@pytest.mark.parametrize("tensor_params", [False, True])
@pytest.mark.parametrize("family", ["linear", "affine", "nw", "nw_affine"])
def test_compile_fullgraph_forward_backward(d2p, cuda_device, family, tensor_params):
    """torch.compile(fullgraph=True) traces the public API through the
    d2p_py:: custom ops and their autograd formulas: value, marginals and every
    gradient equal the eager ones, including a loss on the marginals."""
    torch._dynamo.reset()
    s0 = scores(2, 12, 16, seed=36).to(cuda_device)
    W = scores(2, 12, 16, seed=37).to(cuda_device)

    def run(fn):
        s = s0.clone().requires_grad_(True)
        if family in ("linear", "nw"):
            params = [torch.tensor([-1.0], device=cuda_device, requires_grad=True),
                      torch.tensor([0.9], device=cuda_device, requires_grad=True)] if tensor_params else [-1.0, 0.9]
        else:
            params = [torch.tensor([v], device=cuda_device, requires_grad=True) for v in (-2.0, -0.5, 0.9)] \
                if tensor_params else [-2.0, -0.5, 0.9]
        loss, v, m = fn(s, *params)
        loss.backward()
        grads = [s.grad] + ([p.grad for p in params] if tensor_params else [])
        return v.detach(), m.detach(), grads

    def f(s, *params):
        if family == "linear":
            r = d2p.soft_sw(s, gap=params[0], temperature=params[1])
        elif family == "nw":
            r = d2p.soft_nw(s, gap=params[0], temperature=params[1])
            return r.score.sum() + (r.alignment * W).sum(), r.score, r.alignment
        elif family == "nw_affine":
            r = d2p.soft_nw_affine(s, gap_open=params[0], gap_ext=params[1], temperature=params[2])
            return r.score.sum() + (r.alignment * W).sum(), r.score, r.alignment
        else:
            r = d2p.soft_sw_affine(s, gap_open=params[0], gap_ext=params[1], temperature=params[2])
        return r.value.sum() + (r.marginals * W).sum(), r.value, r.marginals

    ve, me, ge = run(f)
    vc, mc, gc = run(torch.compile(f, fullgraph=True, backend="aot_eager"))
    torch.testing.assert_close(vc, ve, rtol=0, atol=0)
    torch.testing.assert_close(mc, me, rtol=0, atol=0)
    for a, b in zip(gc, ge):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)


# ------------------------------------------------------------------ device guard
@TWO_GPUS
def test_entrypoints_honor_scores_device(d2p):
    """Current device cuda:0, scores on cuda:1: every op runs on the scores'
    device and returns its outputs there (tests/test_soft_sw_regular.py:693-719)."""
    s = torch.randn(4, 4, 5, device="cuda:1")
    t = torch.randn_like(s)
    ln = torch.tensor([[4, 5], [3, 5], [4, 4], [2, 3]], dtype=torch.int32, device="cuda:1")
    prev = torch.cuda.current_device()
    try:
        torch.cuda.set_device(0)
        v, m = d2p.soft_sw_float(s, -1.0, 1.0, ln)
        assert v.device == s.device and m.device == s.device
        outs = [d2p.soft_sw_with_grads(s, -1.0, 1.0, ln), d2p.soft_sw_hvp(s, t, -1.0, 1.0, ln),
                d2p.soft_sw_param_jacobian(s, 0, -1.0, 1.0, ln), d2p.soft_sw_param_jacobian(s, 1, -1.0, 1.0, ln),
                d2p.soft_sw_backward_full(s, t, -1.0, 1.0, ln),
                d2p.soft_sw_affine_float(s, -2.0, -0.5, 1.0, ln), d2p.soft_sw_affine_hvp(s, t, -2.0, -0.5, 1.0, ln),
                d2p.soft_sw_affine_backward_full(s, t, -2.0, -0.5, 1.0, ln)]
        for o in outs:
            for x in (o if isinstance(o, (list, tuple)) else [o]):
                assert x.device == s.device
        sr = s.detach().clone().requires_grad_(True)
        vr, _ = d2p.soft_sw_float(sr, -1.0, 1.0, ln)
        vr.sum().backward()
        assert sr.grad is not None and sr.grad.device == sr.device
        torch.cuda.synchronize(s.device)
        # the same results as on the current device
        v0, m0 = d2p.soft_sw_float(s.to("cuda:0"), -1.0, 1.0, ln.to("cuda:0"))
        assert torch.equal(v0.cpu(), v.cpu()) and torch.equal(m0.cpu(), m.cpu())
    finally:
        torch.cuda.set_device(prev)


@TWO_GPUS
def test_lengths_and_gradients_must_share_the_scores_device(d2p):
    s = torch.randn(1, 4, 5, device="cuda:0")
    ln = torch.tensor([[4, 5]], dtype=torch.int32, device="cuda:1")
    with pytest.raises(RuntimeError, match="lengths must be on same device as scores"):
        d2p.soft_sw_float(s, -1.0, 1.0, ln)
    with pytest.raises(RuntimeError, match="lengths must be on same device as scores"):
        d2p.soft_sw_affine_float(s, -2.0, -0.5, 1.0, ln)
    with pytest.raises(RuntimeError, match="grad_alignment must be on same device as scores"):
        d2p.soft_sw_affine_backward_full(s, torch.randn(1, 4, 5, device="cuda:1"), -2.0, -0.5, 1.0, None)
