"""Generate the golden fixtures in tests/golden/ from the REFERENCE's own CPU
kernels (src/sw/kernels_cpu.cpp, src/sw_affine/kernels_cpu.cpp,
src/nw/kernels_cpu.cpp, src/nw_affine/kernels_cpu.cpp, src/dtw/kernels_cpu.cpp compiled from the reference sources into
oracle/_ref/libref_sw_cpu.so by oracle/Makefile).

Run in a container where the reference sources are present:
    make -C oracle && python tests/golden/make_golden.py
Inputs are seeded (torch.Generator) so the fixtures are reproducible; each .npz
holds the inputs and the reference outputs of every operator mode.
"""
import os
import sys

import zlib

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
import oracle  # noqa: E402

CASES = [
    # name, B, L1, L2, T, linear gap, (affine open, ext), with_lengths
    ("small_t1", 2, 7, 9, 1.0, -1.0, (-2.0, -0.5), False),
    ("ragged_t05", 3, 12, 10, 0.5, -0.5, (-1.7, -0.4), True),
    ("sharp_t01", 2, 6, 11, 0.1, -1.0, (-2.0, -0.5), False),
    ("row1", 2, 1, 8, 1.0, -1.0, (-2.0, -0.5), False),
]

# Needleman-Wunsch only (files named nw_*): name, B, L1, L2, T, gap, lengths
NW_CASES = [
    ("nw_edges", 6, 9, 7, 0.8, -0.7, [[9, 7], [0, 7], [9, 0], [0, 0], [1, 7], [9, 1]]),
]
# the affine gap penalties of the Needleman-Wunsch edge cases
NW_AFFINE = (-1.5, -0.4)

# soft DTW (files named dtw_*): name, B, L1, L2, T, bandwidth (-1: none), lengths
DTW_CASES = [
    ("dtw_full", 3, 9, 12, 1.0, -1, None),
    ("dtw_band", 5, 11, 8, 0.5, 2, [[11, 8], [0, 8], [11, 0], [7, 8], [11, 5]]),
    ("dtw_sharp", 2, 10, 10, 0.1, 3, None),
]


def main():
    assert oracle.ref_available(), "reference CPU build missing: run `make -C oracle` with the reference present"
    oracle.set_threads(1)
    for name, B, L1, L2, T, gap, (go, ge), with_len in CASES:
        g = torch.Generator().manual_seed(zlib.crc32(name.encode()))
        s = torch.randn(B, L1, L2, generator=g).numpy()
        V = torch.randn(B, L1, L2, generator=g).numpy()
        G = torch.randn(B, L1, L2, generator=g).numpy()
        ln = None
        if with_len:
            l1 = torch.randint(1, L1 + 1, (B,), generator=g)
            l2 = torch.randint(1, L2 + 1, (B,), generator=g)
            ln = torch.stack([l1, l2], 1).to(torch.int32).numpy()
        out = dict(scores=s, tangent=V, grad_marginals=G, T=np.float32(T), gap=np.float32(gap),
                   gap_open=np.float32(go), gap_ext=np.float32(ge),
                   lengths=ln if ln is not None else np.zeros((0, 2), np.int32))
        r = oracle.sw_linear(s, ln, gap, T, "ref")
        for k in ("value", "marginals", "grad_gap", "grad_T"):
            out["lin_" + k] = r[k]
        out["lin_hvp"] = oracle.sw_linear_hvp(s, V, ln, gap, T, "ref")
        out["lin_jac0"] = oracle.sw_linear_param_jacobian(s, 0, ln, gap, T, "ref")
        out["lin_jac1"] = oracle.sw_linear_param_jacobian(s, 1, ln, gap, T, "ref")
        bf = oracle.sw_linear_backward_full(s, G, ln, gap, T, "ref")
        out["lin_bf_scores"], out["lin_bf_gap"], out["lin_bf_T"] = bf
        r = oracle.sw_affine(s, ln, go, ge, T, "ref")
        for k in ("value", "marginals", "grad_open", "grad_ext", "grad_T"):
            out["aff_" + k] = r[k]
        out["aff_hvp"] = oracle.sw_affine_hvp(s, V, ln, go, ge, T, "ref")
        for p in range(3):
            out[f"aff_jac{p}"] = oracle.sw_affine_param_jacobian(s, p, ln, go, ge, T, "ref")
        bf = oracle.sw_affine_backward_full(s, G, ln, go, ge, T, "ref")
        out["aff_bf_scores"], out["aff_bf_open"], out["aff_bf_ext"], out["aff_bf_T"] = bf
        out.update(_nw_outputs(s, V, G, ln, gap, T))
        out.update(_nwa_outputs(s, V, G, ln, go, ge, T))
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **out)
        print("wrote", name)
    # Needleman-Wunsch edge cases: empty sequences (lengths 0 on either side)
    # and a single row / column
    for name, B, L1, L2, T, gap, lens in NW_CASES:
        g = torch.Generator().manual_seed(zlib.crc32(name.encode()))
        s = torch.randn(B, L1, L2, generator=g).numpy()
        V = torch.randn(B, L1, L2, generator=g).numpy()
        G = torch.randn(B, L1, L2, generator=g).numpy()
        ln = np.array(lens, np.int32)
        go, ge = NW_AFFINE
        out = dict(scores=s, tangent=V, grad_marginals=G, T=np.float32(T), gap=np.float32(gap),
                   gap_open=np.float32(go), gap_ext=np.float32(ge), lengths=ln)
        out.update(_nw_outputs(s, V, G, ln, gap, T))
        out.update(_nwa_outputs(s, V, G, ln, go, ge, T))
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **out)
        print("wrote", name)
    # soft DTW: non-negative costs, with and without a band, empty sequences
    for name, B, L1, L2, T, bw, lens in DTW_CASES:
        g = torch.Generator().manual_seed(zlib.crc32(name.encode()))
        c = torch.rand(B, L1, L2, generator=g).numpy()
        V = torch.randn(B, L1, L2, generator=g).numpy()
        G = torch.randn(B, L1, L2, generator=g).numpy()
        ln = np.array(lens, np.int32) if lens is not None else np.tile(np.array([[L1, L2]], np.int32), (B, 1))
        out = dict(costs=c, tangent=V, grad_marginals=G, T=np.float32(T), bandwidth=np.int64(bw), lengths=ln)
        r = oracle.dtw(c, ln, T, bw, "ref")
        for k in ("value", "marginals", "grad_T"):
            out["dtw_" + k] = r[k]
        out["dtw_hvp"] = oracle.dtw_hvp(c, V, ln, T, bw, "ref")
        out["dtw_jac"] = oracle.dtw_param_jacobian(c, ln, T, bw, "ref")
        out["dtw_bf_costs"], out["dtw_bf_T"] = oracle.dtw_backward_full(c, G, ln, T, bw, "ref")
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **out)
        print("wrote", name)


def _nw_outputs(s, V, G, ln, gap, T):
    out = {}
    r = oracle.nw_linear(s, ln, gap, T, "ref")
    for k in ("value", "marginals", "grad_gap", "grad_T"):
        out["nw_" + k] = r[k]
    out["nw_hvp"] = oracle.nw_linear_hvp(s, V, ln, gap, T, "ref")
    out["nw_jac0"] = oracle.nw_linear_param_jacobian(s, 0, ln, gap, T, "ref")
    out["nw_jac1"] = oracle.nw_linear_param_jacobian(s, 1, ln, gap, T, "ref")
    out["nw_bf_scores"], out["nw_bf_gap"], out["nw_bf_T"] = oracle.nw_linear_backward_full(s, G, ln, gap, T, "ref")
    return out


def _nwa_outputs(s, V, G, ln, go, ge, T):
    out = {}
    r = oracle.nw_affine(s, ln, go, ge, T, "ref")
    for k in ("value", "marginals", "grad_open", "grad_ext", "grad_T"):
        out["nwa_" + k] = r[k]
    out["nwa_hvp"] = oracle.nw_affine_hvp(s, V, ln, go, ge, T, "ref")
    for p in range(3):
        out[f"nwa_jac{p}"] = oracle.nw_affine_param_jacobian(s, p, ln, go, ge, T, "ref")
    bf = oracle.nw_affine_backward_full(s, G, ln, go, ge, T, "ref")
    out["nwa_bf_scores"], out["nwa_bf_open"], out["nwa_bf_ext"], out["nwa_bf_T"] = bf
    return out


if __name__ == "__main__":
    main()
