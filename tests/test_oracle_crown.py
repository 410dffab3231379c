"""The CROWN oracle (oracle/crown_oracle.py) against the reference's own CROWN outputs,
deeppoly_efficient.cf's reference outputs against the DeepPoly oracle, and the crownibp.cf
oracle (interval bounds below the property) against the reference's crownibp outputs.

The reference cases (tests/golden/crown_*.npz, dpe_*.npz, made by gen_golden.py) cover
CROWN's pass-through branch (eps 1e-3 .. 1e-2) and its all-crossing branch (eps >= 0.1,
polyexps that mix layers, where the lowest-layer-first traversal order matters).  The
reference crashes in CROWN's zero branch (abs_elem.py:929 on a PolyExpSparse built with a
float matrix), so that branch is checked against its stated semantics instead.
Tolerances: tests/parity.py.
"""
import numpy as np
import pytest
import torch

import parity
from golden_cases import Case, chain_names, names
from oracle import crown_oracle as C
from oracle import deeppoly_oracle as O
from cfgpu import nets

CROWN_CASES = names("crown")
DPE_CASES = names("deeppoly_efficient")
CIBP_CASES = chain_names("crownibp")


def _crown(c, **kw):
    bounds, lb, ub, br = C.crown(c.wl.layers, c.l0, c.u0, c.spec_W, **kw)
    xl, xu = O.flatten_bounds(c.wl.input_size, bounds, c.B)
    return xl, xu, lb, ub, br


@pytest.mark.parametrize("name", CROWN_CASES)
def test_crown_oracle_matches_reference(name):
    c = Case(name)
    xl, xu, lb, ub, br = _crown(c)
    worst, where = parity.continuous_errors(xl, xu, c.l_all, c.u_all, c.sizes, label=(c.name, "oracle vs reference"))
    assert worst <= 1.0, f"{name}: oracle vs reference {worst:.3g}x tolerance at {where}"
    assert parity.verdicts_match(lb, c.lb, np.abs(c.lb).max(axis=1))[0]
    # the branch taken is visible in the reference's ReLU bounds
    expect = C.BRANCH_CROSS if c.eps >= 0.1 else C.BRANCH_PASS
    assert br == [expect] * len(br)


def test_traversal_order_is_pinned():
    """A mistake planted in the oracle (highest live layer first) breaks the crossing cases."""
    c = Case("crown_w0_b2_e1e-1")
    xl, xu, _, _, _ = _crown(c, order=max)
    worst, _ = parity.continuous_errors(xl, xu, c.l_all, c.u_all, c.sizes)
    assert worst > 10.0


def test_zero_branch_semantics():
    """Workload 1 at eps 0.05: the first ReLU takes the zero branch; every later bound is
    the plain forward pass of the biases (the remaining ReLUs pass through)."""
    wl = nets.workload(1)
    X = nets.centres(wl, 2)
    y = nets.labels(wl, X)
    l0, u0 = nets.input_box(X, 0.05, wl.dataset)
    W = nets.spec_weight(y).numpy()
    bounds, lb, ub, br = C.crown(wl.layers, l0.numpy(), u0.numpy(), W)
    assert br[0] == C.BRANCH_ZERO and all(b == C.BRANCH_PASS for b in br[1:])
    h = np.zeros((2, bounds[1][0].shape[1]), np.float32)   # the zeroed ReLU output
    affine = [L for L in wl.layers if L.kind != "relu"]
    k = 2
    for L in affine[1:]:
        h = (h @ L.W.T.astype(np.float32) + L.b.astype(np.float32)).astype(np.float32)
        np.testing.assert_allclose(bounds[k][0], h, rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(bounds[k][1], h, rtol=1e-5, atol=1e-6)
        k += 2   # skip the pass-through ReLU (identical bounds)
    spec = np.einsum('bij,bj->bi', W, h)
    np.testing.assert_allclose(lb, spec, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(ub, spec, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("name", DPE_CASES)
def test_deeppoly_efficient_is_deeppoly(name):
    """deeppoly_efficient.cf's reference bounds agree with the DeepPoly oracle."""
    c = Case(name)
    bounds, lb, _ = O.deeppoly(c.wl.layers, c.l0, c.u0, c.spec_W)
    xl, xu = O.flatten_bounds(c.wl.input_size, bounds, c.B)
    worst, where = parity.continuous_errors(xl, xu, c.l_all, c.u_all, c.sizes, label=(c.name, "oracle vs reference"))
    assert worst <= 1.0, f"{name}: DeepPoly oracle vs reference {worst:.3g}x tolerance at {where}"
    assert parity.verdicts_match(lb, c.lb, np.abs(c.lb).max(axis=1))[0]


@pytest.mark.parametrize("name", CIBP_CASES)
def test_crownibp_oracle_matches_reference(name):
    c = Case(name)
    bounds, lb, ub, _ = C.crownibp(c.wl.layers, c.l0, c.u0, c.spec_W)
    xl, xu = O.flatten_bounds(c.wl.input_size, bounds, c.B)
    worst, where = parity.continuous_errors(xl, xu, c.l_all, c.u_all, c.sizes, label=(c.name, "oracle vs reference"))
    assert worst <= 1.0, f"{name}: oracle vs reference {worst:.3g}x tolerance at {where}"
    assert parity.verdicts_match(lb, c.lb, np.abs(c.lb).max(axis=1))[0]


def test_crownibp_cases_present():
    assert len(CIBP_CASES) >= 5 and {Case(n).wid for n in CIBP_CASES} >= {0, 1, 2, 3}


def test_crownibp_planted_backsubstitution_fails():
    """A mistake planted in the oracle (every layer backsubstituted, i.e. DeepPoly) breaks
    the crownibp cases: the reference's intermediate bounds are the interval ones."""
    c = Case("cibp_w2_b4_e2e-4")
    bounds, _, _, _ = C.certify(c.wl.layers, c.l0, c.u0, c.spec_W, "deeppoly")
    xl, xu = O.flatten_bounds(c.wl.input_size, bounds, c.B)
    worst, _ = parity.continuous_errors(xl, xu, c.l_all, c.u_all, c.sizes)
    assert worst > 10.0


CS_CASES = sorted(n for p in ("deeppoly_custom_stop",) + tuple(f"custom_stops/deeppoly_custom_stop{d:02d}"
                                                                for d in range(19)) for n in chain_names(p))


def _cs_depth(name):
    return int(name[2:name.index("_")])


@pytest.mark.parametrize("name", CS_CASES)
def test_custom_stop_oracle_matches_reference(name):
    c = Case(name)
    bounds, lb, ub, _ = C.custom_stop(c.wl.layers, c.l0, c.u0, c.spec_W, _cs_depth(name))
    xl, xu = O.flatten_bounds(c.wl.input_size, bounds, c.B)
    worst, where = parity.continuous_errors(xl, xu, c.l_all, c.u_all, c.sizes, label=(c.name, "oracle vs reference"))
    assert worst <= 1.0, f"{name}: oracle vs reference {worst:.3g}x tolerance at {where}"
    assert parity.verdicts_match(lb, c.lb, np.abs(c.lb).max(axis=1))[0]


def test_custom_stop_depth_is_pinned():
    """The depth is pinned by the reference's outputs: one layer more (a mistake planted in
    the oracle) breaks every custom-stop case."""
    assert len(CS_CASES) >= 7 and {_cs_depth(n) for n in CS_CASES} >= {0, 1, 2, 3, 5, 8}
    for name in CS_CASES:
        c = Case(name)
        bounds, _, _, _ = C.custom_stop(c.wl.layers, c.l0, c.u0, c.spec_W, _cs_depth(name) + 1)
        xl, xu = O.flatten_bounds(c.wl.input_size, bounds, c.B)
        assert parity.continuous_errors(xl, xu, c.l_all, c.u_all, c.sizes)[0] > 10.0, name


def test_relu_tie_rule_is_pinned():
    """The tied network (workload 7) has 32 first-layer neurons with l + u == 0 exactly in
    every region.  The reference's bounds there follow each program's own relu_n: strict
    (l + u > 0) for zid.cf and the custom-stop programs, non-strict (l + u >= 0) for
    deeppoly.cf and crownibp.cf.  The oracle with the other rule planted misses every one of
    these cases by far more than the tolerance."""
    from oracle import zono_oracle as Z

    def run(name, strict):
        c = Case(name)
        if name.startswith("zid"):
            bounds = Z.zid(c.wl.layers, c.l0, c.u0, c.spec_W, strict=strict)[0]
        elif name.startswith("cs3"):
            bounds = C.certify(c.wl.layers, c.l0, c.u0, c.spec_W, "deeppoly", min, stop_depth=3, strict=strict)[0]
        elif name.startswith("cibp"):
            bounds = C.certify(c.wl.layers, c.l0, c.u0, c.spec_W, "deeppoly", max, interval=True, strict=strict)[0]
        else:
            bounds = C.certify(c.wl.layers, c.l0, c.u0, c.spec_W, "deeppoly", min, strict=strict)[0]
        xl, xu = O.flatten_bounds(c.wl.input_size, bounds, c.B)
        return c, parity.continuous_errors(xl, xu, c.l_all, c.u_all, c.sizes)[0]

    for name, strict in (("zid_w7_b4_e1e-2", True), ("cs3_w7_b4_e1e-2", True), ("dp_w7_b4_e1e-2", False),
                         ("cibp_w7_b4_e1e-2", False)):
        c, worst = run(name, strict)
        n_tied = int((c.l_all[:, :32] + c.u_all[:, :32] == 0).sum())
        assert n_tied == 32 * c.B and (c.l_all[:, :32] < 0).all(), name
        assert worst <= 1.0, (name, worst)
        assert run(name, not strict)[1] > 100.0, name
