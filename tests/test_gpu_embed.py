"""The score producer (d2p_b200/csrc/sw_embed.cu) and soft_sw_embed on the GPU.

scores = scale * x y^T from bf16 embeddings on the tcgen05 tensor cores,
against an fp64 product of the same bf16 values (every bf16 product is exact
in fp32, so the only error is the fp32 accumulation: bounded here by 1e-5 of
sum |x| |y| per entry).  Through the C ABI the status word must stay 0: every
tile came from the tensor cores, none from the kernel's CUDA-core recovery
path.  soft_sw_embed: value and marginals at the default parity criterion
against the oracle on the fp64 scores, and the embeddings' gradients against
fp64 products of the oracle's marginals (bf16 outputs: 1e-2 relative, the bf16
tolerance).
"""
import ctypes
import os

import numpy as np
import pytest
import torch

import oracle
from _parity import check

pytestmark = pytest.mark.gpu

LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "d2p_b200", "libd2p_b200.so")


@pytest.fixture(scope="module")
def d2p(cuda_device):
    import d2p_b200

    return d2p_b200


@pytest.fixture(scope="module")
def lib():
    lib = ctypes.CDLL(LIB)
    f = lib.d2p_embed_scores
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int] * 4 + [ctypes.c_float, ctypes.c_void_p,
                                                                               ctypes.c_void_p, ctypes.c_void_p]
    return lib


def embeddings(B, L, D, seed):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(B, L, D, generator=g) / D ** 0.25).to(torch.bfloat16)


def reference(x, y, scale):
    x64, y64 = x.double(), y.double()
    s = torch.bmm(x64, y64.transpose(1, 2)) * scale
    mag = torch.bmm(x64.abs(), y64.abs().transpose(1, 2)) * abs(scale)
    return s, mag


SHAPES = [
    # (B, L1, L2, D): whole tiles, ragged tiles, one row, the largest D, odd widths
    (2, 256, 256, 128),
    (3, 100, 120, 64),
    (2, 300, 77, 256),
    (1, 5, 3, 64),
    (4, 129, 513, 192),
]


@pytest.mark.parametrize("B,L1,L2,D", SHAPES, ids=[f"{s[0]}x{s[1]}x{s[2]}xD{s[3]}" for s in SHAPES])
def test_embed_scores_c_abi(lib, cuda_device, B, L1, L2, D):
    x = embeddings(B, L1, D, 1).to(cuda_device)
    y = embeddings(B, L2, D, 2).to(cuda_device)
    out = torch.full((B, L1, L2), float("nan"), device=cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):   # twice: the second call reuses the device set-up
        rc = lib.d2p_embed_scores(x.data_ptr(), y.data_ptr(), B, L1, L2, D, ctypes.c_float(0.5), out.data_ptr(),
                                  status.data_ptr(), stream)
        assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0, "a tile fell back to the CUDA cores"
    ref, mag = reference(x.cpu(), y.cpu(), 0.5)
    err = (out.double().cpu() - ref).abs()
    assert torch.all(err <= 1e-5 * mag + 1e-7), float((err / (mag + 1e-30)).max())


def test_embed_scores_rejects(lib, cuda_device):
    x = embeddings(1, 8, 40, 1).to(cuda_device)
    out = torch.empty(1, 8, 8, device=cuda_device)
    stream = torch.cuda.current_stream().cuda_stream
    # D not a multiple of 64 (the Python layer pads), D above 256
    assert lib.d2p_embed_scores(x.data_ptr(), x.data_ptr(), 1, 8, 8, 40, ctypes.c_float(1.0), out.data_ptr(),
                                None, stream) == 1001
    assert lib.d2p_embed_scores(x.data_ptr(), x.data_ptr(), 1, 8, 8, 320, ctypes.c_float(1.0), out.data_ptr(),
                                None, stream) == 1003


def test_embed_scores_op_pads_d(d2p, cuda_device):
    x = embeddings(2, 70, 40, 3).to(cuda_device)
    y = embeddings(2, 90, 40, 4).to(cuda_device)
    s = d2p.embed_scores(x, y, 2.0)
    ref, mag = reference(x.cpu(), y.cpu(), 2.0)
    assert torch.all((s.double().cpu() - ref).abs() <= 1e-5 * mag + 1e-7)


@pytest.mark.parametrize("ragged", [False, True])
def test_soft_sw_embed_value_marginals_grads(d2p, cuda_device, ragged):
    B, L1, L2, D, gap, T = 3, 160, 200, 96, -1.0, 1.0
    x = embeddings(B, L1, D, 5).to(cuda_device).requires_grad_(True)
    y = embeddings(B, L2, D, 6).to(cuda_device).requires_grad_(True)
    ln = None
    if ragged:
        ln = torch.tensor([[160, 200], [90, 150], [31, 7]], dtype=torch.int32)
    res = d2p.soft_sw_embed(x, y, gap=gap, temperature=T, lengths=None if ln is None else ln.to(cuda_device))
    res.value.sum().backward()
    s64 = torch.bmm(x.detach().cpu().double(), y.detach().cpu().double().transpose(1, 2)).numpy()
    lnp = None if ln is None else ln.numpy()
    r64 = oracle.sw_linear(s64, lnp, gap, T, "f64")
    r32 = oracle.sw_linear(s64.astype(np.float32), lnp, gap, T, "f32")
    check("embed value", res.value, r64["value"], r32["value"])
    check("embed marginals", res.marginals, r64["marginals"], r32["marginals"])
    P = torch.from_numpy(r64["marginals"])
    gx_ref = torch.bmm(P, y.detach().cpu().double())
    gy_ref = torch.bmm(P.transpose(1, 2), x.detach().cpu().double())
    for name, got, want in (("grad_x", x.grad, gx_ref), ("grad_y", y.grad, gy_ref)):
        err = (got.double().cpu() - want).abs()
        assert torch.all(err <= 1e-2 * want.abs() + 1e-2 * want.abs().max()), (name, float(err.max()))


def test_embed_kernel_runs(d2p, cuda_device):
    from torch.profiler import ProfilerActivity, profile

    x = embeddings(2, 128, 64, 7).to(cuda_device)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        torch.ones(1, device="cuda").add_(1)
        torch.cuda.synchronize()
        d2p.embed_scores(x, x)
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    assert any("embed_scores_kernel" in n for n in names), names


def test_soft_sw_embed_marginal_loss(d2p, cuda_device):
    """A loss of the values and of the marginals: dL/dscores = g P + H W (the
    Hessian-vector product along the marginals' weights W, from backward_full),
    then the embeddings' GEMMs; against fp64 (oracle HVP) at the bf16 tolerance."""
    B, L1, L2, D, gap, T = 2, 64, 80, 64, -1.0, 1.0
    x = embeddings(B, L1, D, 8).to(cuda_device).requires_grad_(True)
    y = embeddings(B, L2, D, 9).to(cuda_device).requires_grad_(True)
    g = torch.Generator().manual_seed(10)
    W = torch.randn(B, L1, L2, generator=g)
    res = d2p.soft_sw_embed(x, y, gap=gap, temperature=T)
    (res.value.sum() + (res.marginals * W.to(cuda_device)).sum()).backward()
    s64 = torch.bmm(x.detach().cpu().double(), y.detach().cpu().double().transpose(1, 2)).numpy()
    P = oracle.sw_linear(s64, None, gap, T, "f64")["marginals"]
    HW = oracle.sw_linear_hvp(s64, W.double().numpy(), None, gap, T, "f64")
    G = torch.from_numpy(P + HW)
    gx_ref = torch.bmm(G, y.detach().cpu().double())
    gy_ref = torch.bmm(G.transpose(1, 2), x.detach().cpu().double())
    for name, got, want in (("grad_x", x.grad, gx_ref), ("grad_y", y.grad, gy_ref)):
        err = (got.double().cpu() - want).abs()
        assert torch.all(err <= 1e-2 * want.abs() + 1e-2 * want.abs().max()), (name, float(err.max()))


@pytest.mark.parametrize("L1,L2", [(40, 56), (37, 51)], ids=["whole-8", "odd"])
def test_embed_grad_scores_op(d2p, cuda_device, L1, L2):
    g = torch.Generator().manual_seed(11)
    P = torch.rand(3, L1, L2, generator=g)
    gv = torch.randn(3, generator=g)
    G = torch.ops.d2p_b200.embed_grad_scores(P.to(cuda_device), gv.to(cuda_device), 0.5)
    assert G.dtype == torch.bfloat16
    want = (0.5 * gv[:, None, None] * P).to(torch.bfloat16)
    assert torch.equal(G.cpu(), want)


def test_soft_sw_embed_odd_shape_backward(d2p, cuda_device):
    """Planes that are not whole 8-element units, D that is padded (40 -> 64)."""
    B, L1, L2, D = 2, 37, 51, 40
    x = embeddings(B, L1, D, 12).to(cuda_device).requires_grad_(True)
    y = embeddings(B, L2, D, 13).to(cuda_device).requires_grad_(True)
    res = d2p.soft_sw_embed(x, y, gap=-1.0, temperature=1.0)
    res.value.sum().backward()
    s64 = torch.bmm(x.detach().cpu().double(), y.detach().cpu().double().transpose(1, 2)).numpy()
    P = torch.from_numpy(oracle.sw_linear(s64, None, -1.0, 1.0, "f64")["marginals"])
    for name, got, want in (("grad_x", x.grad, torch.bmm(P, y.detach().cpu().double())),
                            ("grad_y", y.grad, torch.bmm(P.transpose(1, 2), x.detach().cpu().double()))):
        err = (got.double().cpu() - want).abs()
        assert torch.all(err <= 1e-2 * want.abs() + 1e-2 * want.abs().max()), (name, float(err.max()))
