"""The oracle is pinned to the reference: its fp32 restatement must reproduce the
golden vectors that tests/golden/make_golden.py generated from the reference's
own CPU kernels (and, when oracle/_ref is present, the live reference build).
CPU only."""
import glob
import os

import numpy as np
import pytest

import oracle

ALL = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz")))
# Smith-Waterman fixtures; files named nw_* hold Needleman-Wunsch cases only
GOLDEN = [p for p in ALL if not os.path.basename(p).startswith(("nw_", "dtw_"))]
NW_GOLDEN = [p for p in ALL if "nw_value" in np.load(p).files]
DTW_GOLDEN = [p for p in ALL if "dtw_value" in np.load(p).files]


def _load(path):
    z = np.load(path)
    d = {k: z[k] for k in z.files}
    if d["lengths"].shape[0] == 0:
        d["lengths"] = None
    return d


def _close(a, b, rtol, atol, what):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    assert a.shape == b.shape, what
    assert np.allclose(a, b, rtol=rtol, atol=atol), f"{what}: max abs diff {np.abs(a - b).max():.3e}"


def test_fixtures_present():
    assert len(GOLDEN) >= 4
    assert len(NW_GOLDEN) >= 5


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p) for p in GOLDEN])
def test_linear_restatement_matches_reference_golden(path):
    d = _load(path)
    s, ln, gap, T = d["scores"], d["lengths"], float(d["gap"]), float(d["T"])
    r = oracle.sw_linear(s, ln, gap, T, "f32")
    # the fp32 restatement follows the reference's operation order: bit-exact
    for k in ("value", "marginals", "grad_gap", "grad_T"):
        _close(r[k], d["lin_" + k], 0, 0, k)
    _close(oracle.sw_linear_hvp(s, d["tangent"], ln, gap, T, "f32"), d["lin_hvp"], 0, 0, "hvp")
    for p in (0, 1):
        _close(oracle.sw_linear_param_jacobian(s, p, ln, gap, T, "f32"), d[f"lin_jac{p}"], 0, 0, f"jac{p}")
    bf = oracle.sw_linear_backward_full(s, d["grad_marginals"], ln, gap, T, "f32")
    _close(bf[0], d["lin_bf_scores"], 0, 0, "bf scores")
    _close(bf[1], d["lin_bf_gap"], 1e-6, 1e-7, "bf gap")
    _close(bf[2], d["lin_bf_T"], 1e-6, 1e-7, "bf T")


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p) for p in GOLDEN])
def test_affine_restatement_matches_reference_golden(path):
    d = _load(path)
    s, ln, go, ge, T = d["scores"], d["lengths"], float(d["gap_open"]), float(d["gap_ext"]), float(d["T"])
    r = oracle.sw_affine(s, ln, go, ge, T, "f32")
    # affine: same algorithm; float rounding may differ in the last bits
    for k in ("value", "marginals", "grad_open", "grad_ext", "grad_T"):
        _close(r[k], d["aff_" + k], 1e-6, 1e-6, k)
    _close(oracle.sw_affine_hvp(s, d["tangent"], ln, go, ge, T, "f32"), d["aff_hvp"], 1e-6, 1e-6, "hvp")
    for p in range(3):
        _close(oracle.sw_affine_param_jacobian(s, p, ln, go, ge, T, "f32"), d[f"aff_jac{p}"], 1e-5, 1e-6, f"jac{p}")
    bf = oracle.sw_affine_backward_full(s, d["grad_marginals"], ln, go, ge, T, "f32")
    _close(bf[0], d["aff_bf_scores"], 1e-5, 1e-6, "bf scores")
    for k, name in ((1, "open"), (2, "ext"), (3, "T")):
        _close(bf[k], d["aff_bf_" + name], 1e-5, 1e-5, "bf " + name)


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p) for p in GOLDEN])
def test_fp64_restatement_near_reference(path):
    """The double-precision build (the noise-floor reference) agrees with the
    reference's fp32 to fp32 accuracy on these small problems."""
    d = _load(path)
    s, ln, gap, T = d["scores"], d["lengths"], float(d["gap"]), float(d["T"])
    r = oracle.sw_linear(s, ln, gap, T, "f64")
    _close(r["value"], d["lin_value"], 1e-5, 1e-6, "value")
    _close(r["marginals"], d["lin_marginals"], 1e-4, 1e-5, "marginals")
    ra = oracle.sw_affine(s, ln, float(d["gap_open"]), float(d["gap_ext"]), T, "f64")
    _close(ra["value"], d["aff_value"], 1e-5, 1e-6, "aff value")
    _close(ra["marginals"], d["aff_marginals"], 1e-4, 1e-5, "aff marginals")


@pytest.mark.skipif(not oracle.ref_available(), reason="reference CPU build (oracle/_ref) not present")
def test_restatement_matches_live_reference_build():
    rng = np.random.default_rng(5)
    s = rng.standard_normal((3, 21, 17)).astype(np.float32)
    ln = np.array([[21, 17], [10, 17], [21, 3]], np.int32)
    a = oracle.sw_linear(s, ln, -0.7, 0.6, "f32")
    b = oracle.sw_linear(s, ln, -0.7, 0.6, "ref")
    for k in ("value", "marginals", "grad_gap", "grad_T"):
        _close(a[k], b[k], 0, 0, k)
    a = oracle.sw_affine(s, ln, -1.5, -0.3, 0.6, "f32")
    b = oracle.sw_affine(s, ln, -1.5, -0.3, 0.6, "ref")
    for k in ("value", "marginals", "grad_open", "grad_ext", "grad_T"):
        _close(a[k], b[k], 1e-6, 1e-6, k)


def test_oracle_semantics_value_includes_origin():
    """S includes alpha[0,0] = 0 (reference kernels_cpu.cpp:125-147): an empty
    problem has value 0 and a 1x1 problem has value log(1 + exp(s))."""
    s = np.zeros((1, 1, 1), np.float32) + 0.3
    r = oracle.sw_linear(s, None, -1.0, 1.0, "f64")
    x = float(np.float32(0.3))
    assert abs(r["value"][0] - np.log(1 + np.exp(x))) < 1e-12
    r0 = oracle.sw_linear(s, np.array([[0, 1]], np.int32), -1.0, 1.0, "f64")
    assert r0["value"][0] == 0.0 and np.all(r0["marginals"] == 0)


@pytest.mark.parametrize("path", NW_GOLDEN, ids=[os.path.basename(p) for p in NW_GOLDEN])
def test_nw_restatement_matches_reference_golden(path):
    """nw_oracle.c reproduces the reference's src/nw/kernels_cpu.cpp bit for bit
    (same operation order), including empty sequences on either side."""
    d = _load(path)
    s, ln, gap, T = d["scores"], d["lengths"], float(d["gap"]), float(d["T"])
    r = oracle.nw_linear(s, ln, gap, T, "f32")
    for k in ("value", "marginals", "grad_gap", "grad_T"):
        _close(r[k], d["nw_" + k], 0, 0, k)
    _close(oracle.nw_linear_hvp(s, d["tangent"], ln, gap, T, "f32"), d["nw_hvp"], 0, 0, "hvp")
    for p in (0, 1):
        _close(oracle.nw_linear_param_jacobian(s, p, ln, gap, T, "f32"), d[f"nw_jac{p}"], 0, 0, f"jac{p}")
    bf = oracle.nw_linear_backward_full(s, d["grad_marginals"], ln, gap, T, "f32")
    _close(bf[0], d["nw_bf_scores"], 0, 0, "bf scores")
    _close(bf[1], d["nw_bf_gap"], 1e-6, 1e-7, "bf gap")
    _close(bf[2], d["nw_bf_T"], 1e-6, 1e-7, "bf T")
    # the double build agrees to fp32 accuracy, and the closed forms hold:
    # dS/dgap = L1 + L2 - 2 sum(marginals) (every global path with m diagonal
    # cells has L1 + L2 - 2m gaps), dS/dT = (S - sum s mu - gap dS/dgap) / T
    r64 = oracle.nw_linear(s, ln, gap, T, "f64")
    _close(r64["value"], d["nw_value"], 1e-5, 1e-5, "f64 value")
    _close(r64["marginals"], d["nw_marginals"], 1e-4, 1e-5, "f64 marginals")
    B, L1, L2 = s.shape
    lens = np.tile([L1, L2], (B, 1)) if ln is None else ln
    mu = r64["marginals"]
    _close(r64["grad_gap"], lens.sum(1) - 2 * mu.sum((1, 2)), 1e-9, 1e-9, "dS/dgap closed form")
    _close(r64["grad_T"], (r64["value"] - (s * mu).sum((1, 2)) - gap * r64["grad_gap"]) / T, 1e-9, 1e-9,
           "dS/dT closed form")


NWA_GOLDEN = [p for p in ALL if "nwa_value" in np.load(p).files]


@pytest.mark.parametrize("path", NWA_GOLDEN, ids=[os.path.basename(p) for p in NWA_GOLDEN])
def test_nw_affine_restatement_matches_reference_golden(path):
    """nw_affine_oracle.c reproduces the reference's src/nw_affine/kernels_cpu.cpp
    bit for bit (same operation order, Kahan sums and skip thresholds),
    including empty sequences on either side; the double build agrees to fp32
    accuracy."""
    d = _load(path)
    s, ln, go, ge, T = d["scores"], d["lengths"], float(d["gap_open"]), float(d["gap_ext"]), float(d["T"])
    r = oracle.nw_affine(s, ln, go, ge, T, "f32")
    for k in ("value", "marginals", "grad_open", "grad_ext", "grad_T"):
        _close(r[k], d["nwa_" + k], 0, 0, k)
    _close(oracle.nw_affine_hvp(s, d["tangent"], ln, go, ge, T, "f32"), d["nwa_hvp"], 0, 0, "hvp")
    for p in (0, 1, 2):
        _close(oracle.nw_affine_param_jacobian(s, p, ln, go, ge, T, "f32"), d[f"nwa_jac{p}"], 0, 0, f"jac{p}")
    bf = oracle.nw_affine_backward_full(s, d["grad_marginals"], ln, go, ge, T, "f32")
    _close(bf[0], d["nwa_bf_scores"], 0, 0, "bf scores")
    for q, k in ((1, "open"), (2, "ext"), (3, "T")):
        _close(bf[q], d["nwa_bf_" + k], 1e-6, 1e-7, "bf " + k)
    r64 = oracle.nw_affine(s, ln, go, ge, T, "f64")
    _close(r64["value"], d["nwa_value"], 1e-5, 1e-5, "f64 value")
    _close(r64["marginals"], d["nwa_marginals"], 1e-4, 1e-5, "f64 marginals")
    # the marginals of an empty problem are zero, and its value is the single
    # all-gap path's: open + (L - 1) ext for L > 0 gaps, 0 for none
    B, L1, L2 = s.shape
    lens = np.tile([L1, L2], (B, 1)) if ln is None or ln.size == 0 else ln
    for b, (l1, l2) in enumerate(lens):
        if l1 == 0 or l2 == 0:
            n = int(l1 + l2)
            want = 0.0 if n == 0 else go + (n - 1) * ge
            assert abs(float(r64["value"][b]) - want) < 1e-9, (b, r64["value"][b], want)
            assert np.all(r64["marginals"][b] == 0)


@pytest.mark.parametrize("path", DTW_GOLDEN, ids=[os.path.basename(p) for p in DTW_GOLDEN])
def test_dtw_restatement_matches_reference_golden(path):
    """dtw_oracle.c reproduces the reference's src/dtw/kernels_cpu.cpp bit for
    bit, with and without a Sakoe-Chiba band and with empty sequences (whose
    value stays at the +inf sentinel 1e30, as in the reference)."""
    z = np.load(path)
    c, ln, T, bw = z["costs"], z["lengths"], float(z["T"]), int(z["bandwidth"])
    r = oracle.dtw(c, ln, T, bw, "f32")
    for k in ("value", "marginals", "grad_T"):
        _close(r[k], z["dtw_" + k], 0, 0, k)
    _close(oracle.dtw_hvp(c, z["tangent"], ln, T, bw, "f32"), z["dtw_hvp"], 0, 0, "hvp")
    _close(oracle.dtw_param_jacobian(c, ln, T, bw, "f32"), z["dtw_jac"], 0, 0, "jac")
    bf = oracle.dtw_backward_full(c, z["grad_marginals"], ln, T, bw, "f32")
    _close(bf[0], z["dtw_bf_costs"], 0, 0, "bf costs")
    _close(bf[1], z["dtw_bf_T"], 1e-6, 1e-7, "bf T")
    r64 = oracle.dtw(c, ln, T, bw, "f64")
    fin = np.abs(z["dtw_value"]) < 1e29
    _close(r64["value"][fin], z["dtw_value"][fin], 1e-5, 1e-5, "f64 value")
    _close(r64["marginals"], z["dtw_marginals"], 1e-4, 1e-5, "f64 marginals")
    # every warping path ends at (L1, L2): the marginals of the last cell are 1
    for b, (l1, l2) in enumerate(ln):
        if l1 > 0 and l2 > 0:
            assert abs(r64["marginals"][b, l1 - 1, l2 - 1] - 1.0) < 1e-12
