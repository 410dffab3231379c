"""Parity criteria shared by the CPU and GPU test suites.

Floating-point parity (float32 everywhere, as in the reference):

* Continuous agreement.  Two float32 implementations that sum in different orders
  differ by rounding; through deep backsubstitution that difference is a fraction
  of the layer's bound magnitude, not of each bound.  A neuron bound passes when
      |x - ref| <= RTOL * |ref| + ATOL * S
  with S = max |bound| over that layer for that region (l and u together),
  RTOL = 1e-5 and ATOL = 8e-5.  The absolute floor is the measured disagreement of two
  float32 implementations with identical decisions: on the 9x200 MLP (256 regions) the
  oracle and the reference differ by up to 4.4e-5*S and the GPU and the reference by up to
  4.2e-5*S; the largest is the custom-stop program at depth 5, whose property rows are
  concretised against a hidden layer's bounds (much larger than S): oracle vs reference
  7.3e-5*S, GPU vs oracle 5.1e-5*S.  Every test records its worst ratio (tests/conftest.py
  prints them; CF_PARITY_LOG keeps them).
* Discrete decisions.  The ReLU transformer branches on l>=0, u<=0 and l+u>=0
  (deeppoly.cf:20-24).  A bound a few ulps from 0 can take either branch and every
  later layer then differs by far more than rounding.  The continuous comparison is
  therefore made against the oracle replaying the SAME decisions as the
  implementation under test (oracle ``force=``), and every decision that differs
  from the reference's own run must sit on a tie: the deciding quantity within
  TIE * S of zero.
* Verdicts (all 9 property lower bounds >= 0) must be identical, except for a
  region whose smallest margin is itself within tolerance of 0.
* Never looser: lb >= lb_ref - tol and ub <= ub_ref + tol on every neuron whose
  upstream decisions agree.
"""
import json
import os

import numpy as np

RTOL = 1e-5
ATOL = 8e-5
TIE = 1e-4

# Worst observed ratio (error / tolerance) per (case, check), printed at the end of the
# session (tests/conftest.py) and written to $CF_PARITY_LOG as JSON when that is set.
OBSERVED = {}


def record(case, check, ratio):
    """Keep the worst ratio seen for (case, check); returns the ratio."""
    key = f"{case}::{check}"
    r = float(ratio)
    if key not in OBSERVED or r > OBSERVED[key]:
        OBSERVED[key] = r
    return r


def dump_observed():
    path = os.environ.get("CF_PARITY_LOG")
    if path and OBSERVED:
        old = {}
        if os.path.exists(path):
            try:
                old = json.load(open(path))
            except Exception:
                old = {}
        old.update(OBSERVED)
        with open(path, "w") as fh:
            json.dump(old, fh, indent=1, sort_keys=True)


def layer_slices(layout_sizes):
    out, pos = [], 0
    for n in layout_sizes:
        out.append(slice(pos, pos + n))
        pos += n
    return out


def continuous_errors(x_l, x_u, r_l, r_u, sizes, label=None):
    """Max of |x-ref| / (RTOL|ref| + ATOL*S) over all neurons (<= 1 passes); recorded under
    label = (case, check) when given."""
    worst = 0.0
    where = None
    for li, sl in enumerate(layer_slices(sizes)):
        rl, ru = r_l[:, sl].astype(np.float64), r_u[:, sl].astype(np.float64)
        S = np.maximum(np.abs(rl).max(axis=1, keepdims=True), np.abs(ru).max(axis=1, keepdims=True))
        S = np.maximum(S, 1e-30)
        for x, r in ((x_l[:, sl], rl), (x_u[:, sl], ru)):
            tol = RTOL * np.abs(r) + ATOL * S
            q = np.abs(x.astype(np.float64) - r) / tol
            m = float(q.max()) if q.size else 0.0
            if m > worst:
                worst = m
                where = (li, np.unravel_index(int(np.argmax(q)), q.shape))
    if label is not None:
        record(label[0], label[1], worst)
    return worst, where


def looser_errors(x_l, x_u, r_l, r_u, sizes, label=None):
    """Never looser: how far x's lower bounds lie below, and its upper bounds above, the
    reference's, in units of the tolerance RTOL|ref| + ATOL*S.  Returns the worst ratio
    (<= 1 passes; 0 when x is nowhere looser) and where it occurs."""
    worst = 0.0
    where = None
    for li, sl in enumerate(layer_slices(sizes)):
        rl, ru = r_l[:, sl].astype(np.float64), r_u[:, sl].astype(np.float64)
        S = np.maximum(np.abs(rl).max(axis=1, keepdims=True), np.abs(ru).max(axis=1, keepdims=True))
        S = np.maximum(S, 1e-30)
        for over, r in ((rl - x_l[:, sl].astype(np.float64), rl), (x_u[:, sl].astype(np.float64) - ru, ru)):
            q = np.maximum(over, 0.0) / (RTOL * np.abs(r) + ATOL * S)
            m = float(q.max()) if q.size else 0.0
            if m > worst:
                worst = m
                where = (li, np.unravel_index(int(np.argmax(q)), q.shape))
    if label is not None:
        record(label[0], label[1], worst)
    return worst, where


def decision_masks(l, u):
    return (l >= 0), (u <= 0), ((l + u) >= 0)


def decision_flips_are_ties(x_l, x_u, r_l, r_u, sizes, relu_layers):
    """All ReLU decisions of x that differ from ref's lie within TIE*S of the threshold.

    x must come from a run that replayed ref's decisions (same upstream branches), so
    that a difference here is the decision x would take on its own bounds.

    relu_layers: indices (into sizes) of the pre-activation layers that feed a ReLU.
    Returns (ok, n_flips, worst_ratio).
    """
    sls = layer_slices(sizes)
    n_flips, worst, ok = 0, 0.0, True
    for li in relu_layers:
        sl = sls[li]
        xl, xu, rl, ru = x_l[:, sl], x_u[:, sl], r_l[:, sl], r_u[:, sl]
        S = np.maximum(np.abs(rl).max(axis=1, keepdims=True), np.abs(ru).max(axis=1, keepdims=True))
        for a, b, q in zip(decision_masks(xl, xu), decision_masks(rl, ru), (rl, ru, rl + ru)):
            d = a != b
            if d.any():
                n_flips += int(d.sum())
                ratio = float((np.abs(q)[d] / np.broadcast_to(S, q.shape)[d]).max())
                worst = max(worst, ratio)
                if ratio > TIE:
                    ok = False
    return ok, n_flips, worst


def verdicts_match(lb, lb_ref, scale):
    """Certified verdicts identical except where the reference margin is a tie."""
    v, vr = (lb >= 0).all(axis=1), (lb_ref >= 0).all(axis=1)
    margin = np.abs(lb_ref).min(axis=1)
    tie = margin <= (RTOL * np.abs(lb_ref).min(axis=1) + ATOL * scale)
    return bool(np.all((v == vr) | tie)), int((v != vr).sum())
