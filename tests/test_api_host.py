"""Host-side contract of the drop-in, checked without a GPU.

The dispatcher schemas, the fake (meta) kernels that torch.compile traces
through, the rejection of CPU tensors, and the Python layer's validation
(temperature, gap sign, masks vs lengths), result aliases and modules.  Each
item follows the reference (d2p/sw.py, d2p/_compile.py, src/sw/registry.cpp,
src/sw_affine/registry.cpp); the CUDA behaviour of the same surface is in
tests/test_gpu_contract.py.
"""
import warnings

import pytest
import torch

import d2p_b200 as d2p
from d2p_b200 import _ops
from d2p_b200.sw import SWResult, _masks_to_lengths, _resolve_lengths, _validate_temperature

# src/sw/registry.cpp:30-44 and src/sw_affine/registry.cpp:27-42, verbatim
SCHEMAS = {
    "soft_sw": "soft_sw(Tensor scores, Tensor gap, Tensor temperature, Tensor lengths) -> Tensor[]",
    "soft_sw_float": "soft_sw_float(Tensor scores, float gap, float temperature, Tensor? lengths) -> Tensor[]",
    "soft_sw_with_grads": "soft_sw_with_grads(Tensor scores, float gap, float temperature, Tensor? lengths) -> "
                          "(Tensor, Tensor, Tensor, Tensor)",
    "soft_sw_hvp": "soft_sw_hvp(Tensor scores, Tensor tangent, float gap, float temperature, Tensor? lengths) -> "
                   "Tensor",
    "soft_sw_param_jacobian": "soft_sw_param_jacobian(Tensor scores, int param_type, float gap, float temperature, "
                              "Tensor? lengths) -> Tensor",
    "soft_sw_backward_full": "soft_sw_backward_full(Tensor scores, Tensor grad_alignment, float gap, "
                             "float temperature, Tensor? lengths) -> (Tensor, Tensor, Tensor)",
    "sw_forward": "sw_forward(Tensor scores, float gap, float temp, Tensor? lengths) -> Tensor[]",
    "sw_forward_t": "sw_forward_t(Tensor scores, Tensor gap, Tensor temp, Tensor lengths) -> Tensor[]",
    "sw_value_grad_params": "sw_value_grad_params(Tensor scores, float gap, float temp, Tensor? lengths) -> "
                            "(Tensor, Tensor)",
    "sw_marginals_backward": "sw_marginals_backward(Tensor scores, Tensor grad_marginals, float gap, float temp, "
                             "Tensor? lengths) -> (Tensor, Tensor, Tensor)",
    "sw_marginals_hvp": "sw_marginals_hvp(Tensor scores, Tensor v, float gap, float temp, Tensor? lengths) -> "
                        "Tensor",
    "sw_marginals_grad_gap": "sw_marginals_grad_gap(Tensor scores, float gap, float temp, Tensor? lengths) -> "
                             "Tensor",
    "sw_marginals_grad_temp": "sw_marginals_grad_temp(Tensor scores, float gap, float temp, Tensor? lengths) -> "
                              "Tensor",
    "soft_sw_affine": "soft_sw_affine(Tensor scores, Tensor gap_open, Tensor gap_ext, Tensor temperature, "
                      "Tensor lengths) -> Tensor[]",
    "soft_sw_affine_float": "soft_sw_affine_float(Tensor scores, float gap_open, float gap_ext, "
                            "float temperature, Tensor? lengths) -> Tensor[]",
    "soft_sw_affine_with_grads": "soft_sw_affine_with_grads(Tensor scores, float gap_open, float gap_ext, "
                                 "float temperature, Tensor? lengths) -> (Tensor, Tensor, Tensor, Tensor, Tensor)",
    "soft_sw_affine_hvp": "soft_sw_affine_hvp(Tensor scores, Tensor tangent, float gap_open, float gap_ext, "
                          "float temperature, Tensor? lengths) -> Tensor",
    "soft_sw_affine_param_jacobian": "soft_sw_affine_param_jacobian(Tensor scores, int param_type, float gap_open, "
                                     "float gap_ext, float temperature, Tensor? lengths) -> Tensor",
    "soft_sw_affine_backward_full": "soft_sw_affine_backward_full(Tensor scores, Tensor grad_alignment, "
                                    "float gap_open, float gap_ext, float temperature, Tensor? lengths) -> "
                                    "(Tensor, Tensor, Tensor, Tensor)",
    "sw_affine_forward": "sw_affine_forward(Tensor scores, float gap_open, float gap_ext, float temp, "
                         "Tensor? lengths) -> Tensor[]",
    "sw_affine_forward_t": "sw_affine_forward_t(Tensor scores, Tensor gap_open, Tensor gap_ext, Tensor temp, "
                           "Tensor lengths) -> Tensor[]",
    "sw_affine_value_grad_params": "sw_affine_value_grad_params(Tensor scores, float gap_open, float gap_ext, "
                                   "float temp, Tensor? lengths) -> (Tensor, Tensor, Tensor)",
    "sw_affine_marginals_backward": "sw_affine_marginals_backward(Tensor scores, Tensor grad_marginals, "
                                    "float gap_open, float gap_ext, float temp, Tensor? lengths) -> "
                                    "(Tensor, Tensor, Tensor, Tensor)",
    "sw_affine_marginals_hvp": "sw_affine_marginals_hvp(Tensor scores, Tensor v, float gap_open, float gap_ext, "
                               "float temp, Tensor? lengths) -> Tensor",
    "sw_affine_marginals_grad_gap_open": "sw_affine_marginals_grad_gap_open(Tensor scores, float gap_open, "
                                         "float gap_ext, float temp, Tensor? lengths) -> Tensor",
    "sw_affine_marginals_grad_gap_ext": "sw_affine_marginals_grad_gap_ext(Tensor scores, float gap_open, "
                                        "float gap_ext, float temp, Tensor? lengths) -> Tensor",
    "sw_affine_marginals_grad_temp": "sw_affine_marginals_grad_temp(Tensor scores, float gap_open, float gap_ext, "
                                     "float temp, Tensor? lengths) -> Tensor",
}
# src/nw/registry.cpp:35-49, verbatim: the linear soft Needleman-Wunsch ops have
# the linear soft Smith-Waterman schemas under their own names
SCHEMAS.update({
    name.replace("soft_sw", "soft_nw").replace("sw_", "nw_"):
        SCHEMAS[name].replace("soft_sw", "soft_nw").replace("sw_", "nw_")
    for name in list(SCHEMAS) if "affine" not in name
})
# src/nw_affine/registry.cpp:35-50, verbatim: the affine soft Smith-Waterman
# schemas under the Needleman-Wunsch names
SCHEMAS.update({
    name.replace("soft_sw", "soft_nw").replace("sw_", "nw_"):
        SCHEMAS[name].replace("soft_sw", "soft_nw").replace("sw_", "nw_")
    for name in list(SCHEMAS) if "affine" in name and "sw" in name
})
# src/dtw/registry.cpp:35-40, verbatim
SCHEMAS.update({
    "soft_dtw": "soft_dtw(Tensor costs, Tensor temperature, Tensor lengths, int bandwidth) -> Tensor[]",
    "soft_dtw_float": "soft_dtw_float(Tensor costs, float temperature, Tensor? lengths, int? bandwidth) -> Tensor[]",
    "soft_dtw_with_grads": "soft_dtw_with_grads(Tensor costs, float temperature, Tensor? lengths, int? bandwidth) -> "
                           "(Tensor, Tensor, Tensor)",
    "soft_dtw_hvp": "soft_dtw_hvp(Tensor costs, Tensor tangent, float temperature, Tensor? lengths, int? bandwidth) "
                    "-> Tensor",
    "soft_dtw_param_jacobian": "soft_dtw_param_jacobian(Tensor costs, float temperature, Tensor? lengths, "
                               "int? bandwidth) -> Tensor",
    "soft_dtw_backward_full": "soft_dtw_backward_full(Tensor costs, Tensor grad_alignment, float temperature, "
                              "Tensor? lengths, int? bandwidth) -> (Tensor, Tensor)",
})


def _schema(name):
    s = str(getattr(torch.ops.d2p, name).default._schema)
    return s.split("::", 1)[1] if "::" in s else s


def test_every_reference_schema_is_registered_verbatim():
    assert set(SCHEMAS) == set(_ops.OP_NAMES)
    for name, want in SCHEMAS.items():
        assert _schema(name) == want, name


def _call_args(name, s, B):
    """Arguments of op `name` for scores `s` (float parameters, full lengths)."""
    if "dtw" in name:
        ln = torch.full((B, 2), 1, dtype=torch.int32, device=s.device)
        if name == "soft_dtw":
            return (s, s.new_tensor([1.0]), ln, -1)
        if "hvp" in name or "backward" in name:
            return (s, torch.zeros_like(s), 1.0, None, None)
        return (s, 1.0, None, None)
    aff = "affine" in name
    fl = (-2.0, -0.5, 1.0) if aff else (-1.0, 1.0)
    t = [s.new_tensor([v]) for v in fl]
    ln = torch.full((B, 2), 1, dtype=torch.int32, device=s.device)
    if name in ("soft_sw", "sw_forward_t", "soft_sw_affine", "sw_affine_forward_t", "soft_nw", "nw_forward_t",
                "soft_nw_affine", "nw_affine_forward_t"):
        return (s, *t, ln)
    if "hvp" in name or "backward" in name:
        return (s, torch.zeros_like(s), *fl, None)
    if "param_jacobian" in name:
        return (s, 0, *fl, None)
    return (s, *fl, None)


# output layout per op: "B" = [B], "P" = [B, L1, L2], "1" = [1]
LAYOUT = {
    "soft_sw": "BP", "soft_sw_float": "BP", "soft_sw_with_grads": "BPBB", "soft_sw_hvp": "P",
    "soft_sw_param_jacobian": "P", "soft_sw_backward_full": "P11", "sw_forward": "BP", "sw_forward_t": "BP",
    "sw_value_grad_params": "BB", "sw_marginals_backward": "P11", "sw_marginals_hvp": "P",
    "sw_marginals_grad_gap": "P", "sw_marginals_grad_temp": "P", "soft_sw_affine": "BP",
    "soft_sw_affine_float": "BP", "soft_sw_affine_with_grads": "BPBBB", "soft_sw_affine_hvp": "P",
    "soft_sw_affine_param_jacobian": "P", "soft_sw_affine_backward_full": "P111", "sw_affine_forward": "BP",
    "sw_affine_forward_t": "BP", "sw_affine_value_grad_params": "BBB", "sw_affine_marginals_backward": "P111",
    "sw_affine_marginals_hvp": "P", "sw_affine_marginals_grad_gap_open": "P",
    "sw_affine_marginals_grad_gap_ext": "P", "sw_affine_marginals_grad_temp": "P",
}
LAYOUT.update({k.replace("soft_sw", "soft_nw").replace("sw_", "nw_"): v for k, v in list(LAYOUT.items())
               if "sw" in k})
LAYOUT.update({"soft_dtw": "BP", "soft_dtw_float": "BP", "soft_dtw_with_grads": "BPB", "soft_dtw_hvp": "P",
               "soft_dtw_param_jacobian": "P", "soft_dtw_backward_full": "P1"})


@pytest.mark.parametrize("name", sorted(SCHEMAS))
def test_fake_kernels_give_the_reference_shapes(name):
    """Under FakeTensorMode every op runs its registered fake (d2p/_compile.py:24-250):
    values [B], planes [B, L1, L2], batch-summed parameter gradients [1]."""
    from torch._subclasses.fake_tensor import FakeTensorMode

    B, L1, L2 = 3, 7, 9
    with FakeTensorMode() as mode:
        s = mode.from_tensor(torch.empty(B, L1, L2))
        out = getattr(torch.ops.d2p, name)(*_call_args(name, s, B))
    outs = list(out) if isinstance(out, (list, tuple)) else [out]
    shapes = {"B": (B,), "P": (B, L1, L2), "1": (1,)}
    assert [tuple(o.shape) for o in outs] == [shapes[k] for k in LAYOUT[name]]
    assert all(o.dtype == torch.float32 for o in outs)


@pytest.mark.parametrize("name", ["soft_sw_float", "soft_sw_hvp", "soft_sw_affine_float", "sw_affine_marginals_hvp",
                                  "soft_nw_float", "nw_marginals_backward", "soft_nw_affine_float",
                                  "nw_affine_marginals_hvp", "soft_dtw_float", "soft_dtw_backward_full"])
def test_cpu_tensors_are_rejected(name):
    """No CPU kernel and no silent fallback: a CPU input raises, naming CUDA."""
    s = torch.randn(2, 4, 5)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        getattr(torch.ops.d2p, name)(*_call_args(name, s, 2))


# ---------------------------------------------------------------- Python layer
def test_temperature_validation():
    """d2p/sw.py:90-99: a non-positive temperature (float or fixed scalar tensor)."""
    for T in (0.0, -1.0, torch.tensor(0.0), torch.tensor([-0.5])):
        with pytest.raises(ValueError, match="temperature must be positive"):
            _validate_temperature(T)
    _validate_temperature(0.5)
    _validate_temperature(torch.tensor([1.0]))
    _validate_temperature(torch.tensor([-1.0], requires_grad=True))  # learnable: not checked
    s = torch.randn(1, 3, 4)
    with pytest.raises(ValueError, match="temperature must be positive"):
        d2p.soft_sw(s, temperature=0.0)
    with pytest.raises(ValueError, match="temperature must be positive"):
        d2p.soft_sw_affine(s, temperature=-2.0)


def test_positive_gap_warns():
    """d2p/sw.py:102-113: a positive float gap is almost always a sign error."""
    s = torch.randn(1, 3, 4)
    with pytest.warns(UserWarning, match="gap=0.5 is positive"):
        with pytest.raises(RuntimeError, match="CUDA"):
            d2p.soft_sw(s, gap=0.5)
    with pytest.warns(UserWarning, match="gap_open=1.0 is positive"):
        with pytest.raises(RuntimeError, match="CUDA"):
            d2p.soft_sw_affine(s, gap_open=1.0)
    with warnings.catch_warnings():
        warnings.simplefilter("error")
        with pytest.raises(RuntimeError, match="CUDA"):
            d2p.soft_sw(s, gap=torch.tensor([0.5]))  # a tensor gap is taken as intended


def test_masks_to_lengths():
    m1 = torch.tensor([[1, 1, 1, 0], [1, 0, 0, 0], [0, 0, 0, 0]], dtype=torch.bool)
    m2 = torch.tensor([[1, 1, 1, 1, 1], [1, 1, 0, 0, 0], [1, 0, 0, 0, 0]], dtype=torch.bool)
    ln = _masks_to_lengths(m1, m2, 3, 4, 5, torch.device("cpu"))
    assert ln.dtype == torch.int32 and ln.tolist() == [[3, 5], [1, 2], [0, 1]]
    ln = _masks_to_lengths(m1, None, 3, 4, 5, torch.device("cpu"))
    assert ln.tolist() == [[3, 5], [1, 5], [0, 5]]


def test_non_prefix_mask_rejected():
    m1 = torch.tensor([[1, 0, 1, 0], [1, 1, 0, 0]], dtype=torch.bool)
    with pytest.raises(ValueError, match=r"mask1 is not prefix-only \(has holes\) at batch indices: \[0\]"):
        _masks_to_lengths(m1, None, 2, 4, 5, torch.device("cpu"))


def test_lengths_and_masks_are_exclusive():
    s = torch.randn(2, 4, 5)
    m1 = torch.ones(2, 4, dtype=torch.bool)
    ln = torch.tensor([[4, 5], [4, 5]], dtype=torch.int32)
    with pytest.raises(ValueError, match="Cannot specify both 'lengths' and 'mask1'/'mask2'"):
        _resolve_lengths(s, ln, m1, None, need_tensor=False)
    with pytest.raises(ValueError, match="Cannot specify both"):
        d2p.soft_sw(s, lengths=ln, mask1=m1)
    # float parameters with no lengths: no [B, 2] tensor is built (no host->device copy)
    assert _resolve_lengths(s, None, None, None, need_tensor=False) is None
    assert _resolve_lengths(s, None, None, None, need_tensor=True).tolist() == [[4, 5], [4, 5]]


def test_result_aliases():
    v, m = torch.zeros(2), torch.ones(2, 3, 4)
    r = SWResult(v, m)
    assert r.score is v and r.alignment is m and r.posteriors is m
    vv, mm = r
    assert vv is v and mm is m


def test_modules_parameters_and_buffers():
    sw = d2p.SoftSW(gap=-1.5, temperature=0.7)
    assert not list(sw.parameters())
    assert sw.gap.tolist() == [-1.5] and sw.temperature.tolist() == [pytest.approx(0.7)]
    sw = d2p.SoftSW(learn_gap=True)
    assert [n for n, _ in sw.named_parameters()] == ["gap"]
    with pytest.warns(DeprecationWarning, match="'learnable' parameter is deprecated"):
        sw = d2p.SoftSW(learnable=True)
    assert sorted(n for n, _ in sw.named_parameters()) == ["gap", "temperature"]
    with pytest.raises(ValueError, match="temperature must be positive"):
        d2p.SoftSW(temperature=0.0)
    aff = d2p.SoftSWAffine(learn_gap_ext=True)
    assert [n for n, _ in aff.named_parameters()] == ["gap_ext"]
    assert sorted(n for n, _ in aff.named_buffers()) == ["gap_open", "temperature"]
    with pytest.warns(DeprecationWarning):
        aff = d2p.SoftSWAffine(learnable=True)
    assert sorted(n for n, _ in aff.named_parameters()) == ["gap_ext", "gap_open", "temperature"]


def test_flat_and_module_aliases():
    """d2p/__init__.py:119-131 and d2p/sw.py:612-620 re-export the ops."""
    from d2p_b200 import sw as swmod

    for name in ("soft_sw_float", "soft_sw_with_grads", "soft_sw_hvp", "soft_sw_param_jacobian",
                 "soft_sw_backward_full", "soft_sw_affine_float", "soft_sw_affine_with_grads",
                 "soft_sw_affine_hvp", "soft_sw_affine_param_jacobian", "soft_sw_affine_backward_full"):
        assert getattr(d2p, name) is getattr(_ops, name)
    assert swmod.soft_sw_forward is _ops.soft_sw_float
    assert swmod.soft_sw_affine_forward is _ops.soft_sw_affine_float
    for name in ("forward", "forward_t", "value_grad_params", "marginals_backward", "marginals_hvp",
                 "marginals_grad_gap", "marginals_grad_temp"):
        assert callable(getattr(d2p.ops.sw, name))
    for name in ("forward", "forward_t", "value_grad_params", "marginals_backward", "marginals_hvp",
                 "marginals_grad_gap_open", "marginals_grad_gap_ext", "marginals_grad_temp"):
        assert callable(getattr(d2p.ops.sw_affine, name))


def test_public_api_on_fake_tensors_uses_the_custom_ops():
    """Fake tensors through the public API take the d2p_py:: custom ops
    (d2p/_pt2_ops.py), whose fakes and autograd formulas torch.compile uses."""
    from torch._subclasses.fake_tensor import FakeTensorMode

    from d2p_b200 import _pt2_ops

    assert _ops._get_pt2_ops() is _pt2_ops
    with FakeTensorMode() as mode:
        s = mode.from_tensor(torch.empty(2, 5, 6))
        r = d2p.soft_sw(s, gap=-1.0, temperature=0.5)
        assert r.value.shape == (2,) and r.marginals.shape == (2, 5, 6)
        ra = d2p.soft_sw_affine(s, gap_open=mode.from_tensor(torch.tensor([-2.0])))
        assert ra.marginals.shape == (2, 5, 6)
        gs, gg, gt = d2p.soft_sw_backward_full(s, s, -1.0, 1.0, None)
        assert gs.shape == (2, 5, 6) and gg.shape == (1,) and gt.shape == (1,)


# ---------------------------------------------------------------- score producer
def test_embed_scores_validation():
    """embed_scores / soft_sw_embed check dtype, shapes and D before any launch."""
    x = torch.zeros(2, 5, 16, dtype=torch.bfloat16)
    with pytest.raises(TypeError, match="bfloat16"):
        d2p.embed_scores(x.float(), x)
    with pytest.raises(ValueError, match="same B and D"):
        d2p.embed_scores(x, torch.zeros(3, 5, 16, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="same B and D"):
        d2p.embed_scores(x, torch.zeros(2, 5, 8, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="exceeds 256"):
        big = torch.zeros(1, 2, 320, dtype=torch.bfloat16)
        d2p.embed_scores(big, big)
    with pytest.raises(ValueError):
        d2p.soft_sw_embed(x, x, temperature=0.0)
    assert "embed_scores" in d2p.__all__ and "soft_sw_embed" in d2p.__all__


def test_embed_scores_fake_shape():
    """Under FakeTensorMode the producer op gives [B, L1, L2] fp32 (its register_fake)."""
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode() as mode:
        x = mode.from_tensor(torch.empty(2, 5, 64, dtype=torch.bfloat16))
        y = mode.from_tensor(torch.empty(2, 7, 64, dtype=torch.bfloat16))
        s = torch.ops.d2p_b200.embed_scores(x, y, 1.0)
    assert tuple(s.shape) == (2, 5, 7) and s.dtype == torch.float32


def test_embed_scores_cpu_rejected():
    """No CPU producer and no silent fallback."""
    x = torch.zeros(1, 4, 64, dtype=torch.bfloat16)
    with pytest.raises((RuntimeError, NotImplementedError)):
        torch.ops.d2p_b200.embed_scores(x, x, 1.0)
