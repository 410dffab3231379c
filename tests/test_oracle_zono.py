"""The zonotope (zono.cf, zono2.cf), interval (ibp.cf) and polyzono.cf oracles against the
reference's own outputs (tests/golden/zono_*.npz, zono2_*.npz, ibp_*.npz, pz_*.npz), planted
mistakes, and soundness: concrete points of the input box stay inside every affine layer's
bounds.
Tolerances: tests/parity.py.
"""
import numpy as np
import pytest

import parity
from golden_cases import Case, names
from oracle import deeppoly_oracle as O
from oracle import zono_oracle as Z
from cfgpu import nets

ZONO_CASES = names("zono", max_wid=9) + names("zono2", max_wid=9)
IBP_CASES = names("ibp", max_wid=9)
PZ_CASES = names("polyzono", max_wid=9)
ZID_CASES = names("zid", max_wid=9)


def _run(c, program=None, relu=None):
    program = program or c.program
    if program == "ibp":
        bounds, lb, ub = Z.ibp(c.wl.layers, c.l0, c.u0, c.spec_W)
        br = None
    elif program == "polyzono":
        bounds, lb, ub = Z.polyzono(c.wl.layers, c.l0, c.u0, c.spec_W)
        br = None
    elif program == "zid":
        bounds, lb, ub = Z.zid(c.wl.layers, c.l0, c.u0, c.spec_W)
        br = None
    else:
        saved = Z.zono_relu
        if relu is not None:
            Z.zono_relu = relu
        try:
            bounds, lb, ub, br = Z.zono(c.wl.layers, c.l0, c.u0, c.spec_W, program)
        finally:
            Z.zono_relu = saved
    xl, xu = O.flatten_bounds(c.wl.input_size, bounds, c.B)
    return xl, xu, lb, ub, br


def test_cases_present():
    assert len(names("zono", max_wid=9)) >= 7 and len(names("zono2", max_wid=9)) >= 2 and len(IBP_CASES) >= 4
    assert {Case(n).wid for n in ZONO_CASES + IBP_CASES} >= {0, 1, 2, 3, 5}
    assert len(PZ_CASES) >= 4 and {Case(n).wid for n in PZ_CASES} >= {0, 1, 2}


@pytest.mark.parametrize("name", ZONO_CASES + IBP_CASES + PZ_CASES + ZID_CASES)
def test_oracle_matches_reference(name):
    c = Case(name)
    xl, xu, lb, ub, br = _run(c)
    worst, where = parity.continuous_errors(xl, xu, c.l_all, c.u_all, c.sizes, label=(c.name, "oracle vs reference"))
    assert worst <= 1.0, f"{name}: oracle vs reference {worst:.3g}x tolerance at {where}"
    assert parity.verdicts_match(lb, c.lb, np.abs(c.lb).max(axis=1))[0]
    if c.program == "zono2":
        assert br == ([Z.BRANCH_ZERO] + [Z.BRANCH_PASS] * (len(br) - 1) if c.eps >= 0.05 else [Z.BRANCH_PASS] * len(br))


def test_planted_missing_symbol_fails():
    """A mistake planted in the oracle (the fresh noise symbol of a crossing ReLU neuron
    dropped) breaks the zonotope cases."""
    original = Z.zono_relu

    def no_symbol(l, u, M, c):
        Mn, cn = original(l, u, M, c)
        Mn[:, :, M.shape[2]:] = 0.0
        return Mn, cn
    c = Case("zono_w2_b4_e2e-3")
    xl, xu, _, _, _ = _run(c, relu=no_symbol)
    worst, _ = parity.continuous_errors(xl, xu, c.l_all, c.u_all, c.sizes)
    assert worst > 10.0


def test_polyzono_meets_both_certifiers():
    """polyzono's bounds are the tightest of its two halves: at the first affine layer (the
    same input box for both) they are exactly max / min of DeepPoly's and the zonotope's,
    and the property bounds are at least as tight as either program's alone."""
    from oracle import crown_oracle as C
    c = Case("pz_w2_b4_e2e-3")
    bp, lbp, ubp = Z.polyzono(c.wl.layers, c.l0, c.u0, c.spec_W)
    bz, lbz, _, _ = Z.zono(c.wl.layers, c.l0, c.u0, c.spec_W, "zono")
    bd, lbd, _, _ = C.certify(c.wl.layers, c.l0, c.u0, c.spec_W, "deeppoly")
    np.testing.assert_array_equal(bp[0][0], np.maximum(bz[0][0], bd[0][0]))
    np.testing.assert_array_equal(bp[0][1], np.minimum(bz[0][1], bd[0][1]))
    assert (lbp >= np.maximum(lbz, lbd) - 1e-5 * np.abs(lbp).max()).all()


def test_planted_unmet_bounds_fail():
    """A mistake planted in the oracle (the zonotope ReLU relaxed with a lower bound 5% of
    the interval below the met one) breaks a polyzono case where the zonotope is the
    tighter half (the larger box)."""
    c = Case("pz_w0_b4_e1e-2")
    saved = Z.zono_relu

    def looser(l, u, M, c_):
        return saved(l - np.float32(0.05) * (u - l), u, M, c_)
    Z.zono_relu = looser
    try:
        bounds, _, _ = Z.polyzono(c.wl.layers, c.l0, c.u0, c.spec_W)
    finally:
        Z.zono_relu = saved
    xl, xu = O.flatten_bounds(c.wl.input_size, bounds, c.B)
    worst, _ = parity.continuous_errors(xl, xu, c.l_all, c.u_all, c.sizes)
    assert worst > 10.0


def _activations(layers, x, spec_W):
    """float64 values of every layer (and the property rows) at flat inputs x [P, n0]."""
    vals = []
    for i, L in enumerate(layers):
        ps = nets.parents_of(layers, i)
        h = [x if p < 0 else vals[p] for p in ps]
        if L.kind == "relu":
            vals.append(np.maximum(h[0], 0.0))
        elif L.kind == "add":
            vals.append(h[0] + h[1])
        elif L.kind == "concat":
            vals.append(np.concatenate(h, axis=1))
        else:
            W = Z.weight_matrix(L).astype(np.float64)
            vals.append(h[0] @ W.T + O.layer_bias(L).astype(np.float64))
    vals.append(np.einsum("ij,pj->pi", spec_W.astype(np.float64), vals[-1]))
    return vals


@pytest.mark.parametrize("program,wid,eps", [("zono", 0, 0.01), ("zono", 1, 0.005), ("zono", 2, 0.002),
                                             ("ibp", 3, 0.002), ("ibp", 5, 0.002)])
def test_soundness_by_sampling(program, wid, eps):
    """Chain networks.  (On a residual network zono.cf is not sound by construction: a
    ReLU layer's l, u are 0, the Add layer sums its parents' l, u, and the ReLU after the
    Add relaxes with those bounds; the reference computes the same, tests/golden/zono_w5_*.
    zono2.cf's whole-layer branches are not sound either: the pass-through branch keeps a
    whole layer linear as soon as one neuron of one region has l >= 0.)"""
    wl = nets.workload(wid)
    X = nets.centres(wl, 2)
    y = nets.labels(wl, X)
    l0, u0 = (t.numpy() for t in nets.input_box(X, eps, wl.dataset))
    W = nets.spec_weight(y).numpy()
    if program == "ibp":
        bounds, _, _ = Z.ibp(wl.layers, l0, u0, W)
    else:
        bounds, _, _, _ = Z.zono(wl.layers, l0, u0, W, program)
    rng = np.random.default_rng(0)
    kinds = [L.kind for L in wl.layers] + ["spec"]
    for b in range(2):
        t = rng.random((256, l0.shape[1]))
        t[:2] = np.array([0.0, 1.0])[:, None]                 # the box corners
        x = l0[b].astype(np.float64) + t * (u0[b] - l0[b]).astype(np.float64)
        acts = _activations(wl.layers, x, W[b])
        for k, (kind, (lo, hi)) in enumerate(zip(kinds, bounds)):
            if program == "zono" and kind == "relu":
                continue                                      # zono.cf sets a ReLU layer's l, u to 0
            scale = max(1.0, float(np.abs(acts[k]).max()))
            assert (acts[k] >= lo[b].astype(np.float64) - 1e-4 * scale).all(), (program, k, kind)
            assert (acts[k] <= hi[b].astype(np.float64) + 1e-4 * scale).all(), (program, k, kind)


def test_zid_layer_threshold_is_pinned():
    """zid.cf switches from zonotope to interval bounds above layer 4; a threshold planted
    one layer pair lower or higher in the oracle breaks every zid case."""
    assert len(ZID_CASES) >= 4 and {Case(n).wid for n in ZID_CASES} >= {0, 1, 2, 3}
    for name in ZID_CASES:
        c = Case(name)
        for upto in (2, 6):
            bounds, _, _ = Z.zid(c.wl.layers, c.l0, c.u0, c.spec_W, upto)
            xl, xu = O.flatten_bounds(c.wl.input_size, bounds, c.B)
            assert parity.continuous_errors(xl, xu, c.l_all, c.u_all, c.sizes)[0] > 10.0, (name, upto)
