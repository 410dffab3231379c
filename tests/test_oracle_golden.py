"""The CPU oracle against the reference's own outputs (golden vectors).

Pins oracle/deeppoly_oracle.py: on every golden case the oracle, replaying the
reference's ReLU decisions, matches every neuron bound of the reference within the
parity tolerance; its own decisions differ from the reference's only on ties; and
its input box equals the reference's input columns bit for bit.
"""
import numpy as np
import pytest

import parity
from golden_cases import Case, chain_names, names
from oracle import deeppoly_oracle as O

FAST = [n for n in chain_names() if Case(n).wid != 4 and Case(n).B <= 16]
SLOW = [n for n in chain_names() if Case(n).wid == 4 or Case(n).B > 16]
CONV_FAST = [n for n in FAST if Case(n).wid == 3]


def _check(name, run=O.deeppoly):
    c = Case(name)
    # input layer: bit-identical to the reference's clip + normalisation
    r = c.l0_ref.shape[0]
    assert np.array_equal(c.l0[:r], c.l0_ref) and np.array_equal(c.u0[:r], c.u0_ref)
    # replay the reference's decisions: continuous agreement on every neuron
    bounds, lb, ub = run(c.wl.layers, c.l0, c.u0, c.spec_W, force=(c.l_all, c.u_all))
    xl, xu = O.flatten_bounds(c.wl.input_size, bounds, c.B)
    worst, where = parity.continuous_errors(xl, xu, c.l_all, c.u_all, c.sizes)
    parity.record(name, f"oracle[{run.__name__}] vs reference", worst)
    assert worst <= 1.0, f"{name}: oracle vs reference {worst:.3g}x tolerance at {where}"
    loose, where = parity.looser_errors(xl, xu, c.l_all, c.u_all, c.sizes)
    assert loose <= 1.0, f"{name}: oracle looser than the reference by {loose:.3g}x tolerance at {where}"
    # with the same upstream decisions, the oracle would decide differently only on ties
    ok, flips, ratio = parity.decision_flips_are_ties(xl, xu, c.l_all, c.u_all, c.sizes, c.relu_layers)
    assert ok, f"{name}: {flips} decision flips, worst at {ratio:.3g} of layer scale"
    # verdicts of the oracle's own (unforced) run
    bounds2, lb2, ub2 = run(c.wl.layers, c.l0, c.u0, c.spec_W)
    scale = np.abs(c.lb).max(axis=1)
    same, nd = parity.verdicts_match(lb2, c.lb, scale)
    assert same, f"{name}: {nd} verdicts differ"
    assert lb.dtype == np.float64 and lb.shape == c.lb.shape


@pytest.mark.parametrize("name", FAST)
def test_oracle_matches_reference(name):
    _check(name)


@pytest.mark.slow
@pytest.mark.parametrize("name", [n for n in SLOW if Case(n).wid <= 3])
def test_oracle_matches_reference_large_batch(name):
    _check(name)


@pytest.mark.parametrize("name", CONV_FAST)
def test_window_oracle_matches_reference(name):
    """The receptive-field-window restatement (deeppoly_windows) on the 1x28x28 conv net."""
    _check(name, O.deeppoly_windows)


def test_window_oracle_matches_dense_oracle():
    """Windows and dense rows give the same bounds on an MLP (whole-image windows) and on the
    1x28x28 conv net (receptive-field windows), decisions replayed."""
    for name in (FAST[0], CONV_FAST[0]):
        c = Case(name)
        b1, _, _ = O.deeppoly(c.wl.layers, c.l0, c.u0, c.spec_W, force=(c.l_all, c.u_all))
        b2, _, _ = O.deeppoly_windows(c.wl.layers, c.l0, c.u0, c.spec_W, force=(c.l_all, c.u_all))
        x1 = O.flatten_bounds(c.wl.input_size, b1, c.B)
        x2 = O.flatten_bounds(c.wl.input_size, b2, c.B)
        worst, where = parity.continuous_errors(x2[0], x2[1], x1[0], x1[1], c.sizes)
        assert worst <= 1.0, f"{name}: windows vs dense {worst:.3g}x tolerance at {where}"


@pytest.mark.slow
@pytest.mark.parametrize("name", [n for n in SLOW if Case(n).wid == 4])
def test_window_oracle_matches_reference_cifar_conv(name):
    """The 3x32x32 CIFAR-shaped conv net (dense rows would take minutes per region)."""
    _check(name, O.deeppoly_windows)


def test_relu_relax_formulae():
    """Hand-checked relaxation values (deeppoly.cf:20-24)."""
    l = np.array([[-2.0, 1.0, -3.0, -1.0, 0.0]], np.float32)
    u = np.array([[2.0, 3.0, -1.0, 3.0, 0.0]], np.float32)
    ln, un, a, lam, mu = O.relu_relax(l, u)
    np.testing.assert_array_equal(ln, [[0, 1, 0, 0, 0]])
    np.testing.assert_array_equal(un, [[2, 3, 0, 3, 0]])
    np.testing.assert_array_equal(a, [[1, 1, 0, 1, 1]])
    np.testing.assert_allclose(lam, [[0.5, 1, 0, 0.75, 1]])
    np.testing.assert_allclose(mu, [[1.0, 0, 0, 0.75, 0]])


def test_oracle_detects_planted_error():
    """A mistake planted in the oracle (wrong lower slope) is caught by the criterion."""
    c = Case(FAST[0])
    saved = O.relu_relax

    def bad(l, u, force=None):
        ln, un, a, lam, mu = saved(l, u, force)
        return ln, un, np.ones_like(a), lam, mu
    O.relu_relax = bad
    try:
        bounds, lb, ub = O.deeppoly(c.wl.layers, c.l0, c.u0, c.spec_W, force=(c.l_all, c.u_all))
    finally:
        O.relu_relax = saved
    xl, xu = O.flatten_bounds(c.wl.input_size, bounds, c.B)
    worst, _ = parity.continuous_errors(xl, xu, c.l_all, c.u_all, c.sizes)
    assert worst > 1.0
