"""The general oracle (oracle/crown_oracle.certify) on networks with residual Add and
Concat layers, against the reference's own DeepPoly and CROWN outputs
(tests/golden/dp_w5_*, dp_w6_*, crown_w5_*, crown_w6_*: workload 5 = residual MLP,
workload 6 = two branches joined by Concat), and on chains against the chain DeepPoly
oracle.  Tolerances: tests/parity.py.
"""
import numpy as np
import pytest

import parity
from golden_cases import Case, names
from oracle import crown_oracle as C
from oracle import deeppoly_oracle as O
from cfgpu import nets

DAG_CASES = [n for p in ("deeppoly", "crown") for n in names(p, max_wid=9)
             if not nets.is_chain(Case(n).wl.layers)]


def _certify(c, layers=None, **kw):
    rel = "crown" if c.program == "crown" else "deeppoly"
    bounds, lb, ub, br = C.certify(layers or c.wl.layers, c.l0, c.u0, c.spec_W, rel, **kw)
    xl, xu = O.flatten_bounds(c.wl.input_size, bounds, c.B)
    return xl, xu, lb, ub, br


def test_dag_cases_present():
    assert {Case(n).wid for n in DAG_CASES} == {5, 6, 8}
    assert {Case(n).program for n in DAG_CASES} == {"deeppoly", "crown"}


@pytest.mark.parametrize("name", DAG_CASES)
def test_dag_oracle_matches_reference(name):
    c = Case(name)
    xl, xu, lb, ub, _ = _certify(c)
    worst, where = parity.continuous_errors(xl, xu, c.l_all, c.u_all, c.sizes, label=(c.name, "oracle vs reference"))
    assert worst <= 1.0, f"{name}: oracle vs reference {worst:.3g}x tolerance at {where}"
    assert parity.verdicts_match(lb, c.lb, np.abs(c.lb).max(axis=1))[0]


def test_dag_layouts_follow_the_reference_reader():
    """Workload 6 lists its layers breadth first from the input, as the reference's ONNX
    reader orders them: both branch Linears before both branch ReLUs."""
    kinds = [L.kind for L in nets.workload(6).layers]
    assert kinds == ["linear", "relu", "linear", "linear", "relu", "relu", "concat", "linear"]
    assert [nets.parents_of(nets.workload(6).layers, i) for i in range(8)] == [
        (-1,), (0,), (1,), (1,), (2,), (3,), (4, 5), (6,)]
    assert not nets.is_chain(nets.workload(5).layers) and nets.is_chain(nets.workload(0).layers)


def test_planted_missing_skip_fails():
    """A mistake planted in the oracle's input (the residual Add reading one parent twice)
    breaks the residual cases."""
    c = Case("dp_w5_b4_e2e-3")
    layers = list(c.wl.layers)
    i = next(k for k, L in enumerate(layers) if L.kind == "add")
    p = layers[i].parents
    layers[i] = nets.Layer(**{**layers[i].__dict__, "parents": (p[0], p[0])})
    xl, xu, _, _, _ = _certify(c, layers)
    worst, _ = parity.continuous_errors(xl, xu, c.l_all, c.u_all, c.sizes)
    assert worst > 10.0


@pytest.mark.parametrize("name", ["dp_w0_b4_e1e-3", "dp_w2_b8_e2e-4"])
def test_general_oracle_is_chain_oracle(name):
    """On a chain network the general traversal computes the chain DeepPoly oracle's
    bounds (same operations in a different grouping: within float32 rounding)."""
    c = Case(name)
    xl, xu, lb, _, _ = _certify(c)
    bounds, lb2, _ = O.deeppoly(c.wl.layers, c.l0, c.u0, c.spec_W)
    yl, yu = O.flatten_bounds(c.wl.input_size, bounds, c.B)
    worst, where = parity.continuous_errors(xl, xu, yl, yu, c.sizes)
    assert worst <= 1.0, f"{name}: general vs chain oracle {worst:.3g}x tolerance at {where}"
