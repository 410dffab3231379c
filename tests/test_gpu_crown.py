"""GPU parity of the network driver running the reference's CROWN program
(DeepPolyEngine(certifier='crown') -> cf_deeppoly_run with CF_RELAX_CROWN), and its
crownibp.cf program (certifier='crownibp', CF_RELAX_CROWNIBP: interval bounds below the
property, one backsubstitution of the property rows).

CROWN's ReLU takes one branch per layer for the whole batch (crown.cf:25 as the
reference compiles it): pass-through and zero run in the fused driver; the all-crossing
branch (mixed-layer polyexps) runs the general traversal of cfgpu.general.  Every case is
compared with the reference's golden bounds where the reference has them and with the
CROWN oracle.  Tolerances: tests/parity.py.
"""
import ctypes

import numpy as np
import pytest
import torch

import parity
from golden_cases import Case, chain_names, names
from oracle import crown_oracle as C
from oracle import deeppoly_oracle as O
from cfgpu import nets

pytestmark = pytest.mark.gpu

PASS_CASES = [n for n in names("crown") if Case(n).eps < 0.1]
CROSS_CASES = [n for n in names("crown") if Case(n).eps >= 0.1]


def _engine(wl):
    from cfgpu.engine import DeepPolyEngine
    return DeepPolyEngine(wl.layers, wl.input_size, "cuda:0", certifier="crown")


def _run(eng, l0, u0, W):
    dev = torch.device("cuda:0")
    lb, ub, sl, su = eng.run(torch.from_numpy(l0).to(dev), torch.from_numpy(u0).to(dev),
                             torch.from_numpy(W).to(dev), want_state=True)
    torch.cuda.synchronize()
    return lb.cpu().numpy(), ub.cpu().numpy(), sl.cpu().numpy(), su.cpu().numpy()


def _against_oracle(wl, l0, u0, W, lb, sl, su):
    n0 = wl.input_size
    bounds, olb, _, br = C.crown(wl.layers, l0, u0, W)
    ol, ou = O.flatten_bounds(n0, bounds, l0.shape[0])
    sizes = [L.n_out for L in wl.layers] + [9]
    worst, where = parity.continuous_errors(sl[:, n0:], su[:, n0:], ol, ou, sizes)
    assert worst <= 1.0, f"GPU vs CROWN oracle {worst:.3g}x tolerance at {where}"
    np.testing.assert_array_equal(lb, sl[:, -9:].astype(np.float64))
    return br


@pytest.mark.parametrize("name", PASS_CASES)
def test_gpu_crown_matches_reference(name):
    c = Case(name)
    lb, ub, sl, su = _run(_engine(c.wl), c.l0, c.u0, c.spec_W)
    n0 = c.wl.input_size
    assert np.array_equal(sl[:, :n0], c.l0) and np.array_equal(su[:, :n0], c.u0)
    worst, where = parity.continuous_errors(sl[:, n0:], su[:, n0:], c.l_all, c.u_all, c.sizes, label=(c.name, "gpu vs reference"))
    assert worst <= 1.0, f"{name}: GPU vs reference {worst:.3g}x tolerance at {where}"
    assert parity.verdicts_match(lb, c.lb, np.abs(c.lb).max(axis=1))[0]
    assert _against_oracle(c.wl, c.l0, c.u0, c.spec_W, lb, sl, su) == [C.BRANCH_PASS] * len(c.relu_layers)


def test_gpu_crown_zero_branch():
    wl = nets.workload(1)
    X = nets.centres(wl, 2)
    y = nets.labels(wl, X)
    l0, u0 = (t.numpy() for t in nets.input_box(X, 0.05, wl.dataset))
    W = nets.spec_weight(y).numpy()
    lb, ub, sl, su = _run(_engine(wl), l0, u0, W)
    br = _against_oracle(wl, l0, u0, W, lb, sl, su)
    assert br[0] == C.BRANCH_ZERO


@pytest.mark.parametrize("name", CROSS_CASES)
def test_gpu_crown_crossing_branch_matches_reference(name):
    c = Case(name)
    lb, ub, sl, su = _run(_engine(c.wl), c.l0, c.u0, c.spec_W)
    n0 = c.wl.input_size
    worst, where = parity.continuous_errors(sl[:, n0:], su[:, n0:], c.l_all, c.u_all, c.sizes, label=(c.name, "gpu vs reference"))
    assert worst <= 1.0, f"{name}: GPU vs reference {worst:.3g}x tolerance at {where}"
    assert parity.verdicts_match(lb, c.lb, np.abs(c.lb).max(axis=1))[0]
    assert _against_oracle(c.wl, c.l0, c.u0, c.spec_W, lb, sl, su) == [C.BRANCH_CROSS] * len(c.relu_layers)


def test_gpu_crown_branch_is_batch_wide():
    """A region whose box alone makes every neuron cross zero (all-crossing branch) is
    bounded with the pass-through branch when another region of the same batch has an
    active neuron."""
    wl = nets.workload(0)
    X = nets.centres(wl, 2)
    y = nets.labels(wl, X)
    l_small, u_small = (t.numpy() for t in nets.input_box(X[:1], 0.001, wl.dataset))
    l_big, u_big = (t.numpy() for t in nets.input_box(X[1:], 0.3, wl.dataset))
    W = nets.spec_weight(y).numpy()
    eng = _engine(wl)
    lb1, _, sl1, su1 = _run(eng, l_big, u_big, W[1:])
    assert _against_oracle(wl, l_big, u_big, W[1:], lb1, sl1, su1) == [C.BRANCH_CROSS] * 3
    l0 = np.concatenate([l_small, l_big])
    u0 = np.concatenate([u_small, u_big])
    lb, ub, sl, su = _run(eng, l0, u0, W)
    assert _against_oracle(wl, l0, u0, W, lb, sl, su) == [C.BRANCH_PASS] * 3


def test_gpu_crown_needs_one_chunk():
    """The C driver refuses a CROWN batch that does not fit one workspace chunk."""
    from cfgpu import _lib
    c = Case(PASS_CASES[0])
    eng = _engine(c.wl)
    dev = torch.device("cuda:0")
    l0, u0 = torch.from_numpy(c.l0).to(dev), torch.from_numpy(c.u0).to(dev)
    W = torch.from_numpy(c.spec_W).to(dev)
    lb = torch.empty(c.B, 9, dtype=torch.float64, device=dev)
    ub = torch.empty_like(lb)
    one = eng.workspace_bytes(1)
    ws = torch.empty(one, dtype=torch.uint8, device=dev)
    st = _lib.lib.cf_deeppoly_run(ctypes.byref(eng.net), c.B, l0.data_ptr(), u0.data_ptr(), W.data_ptr(), None,
                                  None, lb.data_ptr(), ub.data_ptr(), ws.data_ptr(), one,
                                  torch.cuda.current_stream().cuda_stream)
    assert st == _lib.CF_ERR_WORKSPACE
    assert b"whole batch" in _lib.lib.cf_last_error()


CIBP_CASES = chain_names("crownibp")


def _cibp_run(wl, l0, u0, W, budget=None):
    from cfgpu.engine import DeepPolyEngine
    eng = DeepPolyEngine(wl.layers, wl.input_size, "cuda:0", certifier="crownibp")
    dev = torch.device("cuda:0")
    kw = {} if budget is None else {"workspace_budget": eng.workspace_bytes(budget)}
    lb, ub, sl, su = eng.run(torch.from_numpy(l0).to(dev), torch.from_numpy(u0).to(dev),
                             torch.from_numpy(W).to(dev), want_state=True, check_device=True, **kw)
    torch.cuda.synchronize()
    return lb.cpu().numpy(), ub.cpu().numpy(), sl.cpu().numpy(), su.cpu().numpy()


@pytest.mark.parametrize("name", CIBP_CASES)
def test_gpu_crownibp_matches_reference(name):
    c = Case(name)
    lb, ub, sl, su = _cibp_run(c.wl, c.l0, c.u0, c.spec_W)
    n0 = c.wl.input_size
    assert np.array_equal(sl[:, :n0], c.l0) and np.array_equal(su[:, :n0], c.u0)
    worst, where = parity.continuous_errors(sl[:, n0:], su[:, n0:], c.l_all, c.u_all, c.sizes, label=(c.name, "gpu vs reference"))
    assert worst <= 1.0, f"{name}: GPU vs reference {worst:.3g}x tolerance at {where}"
    assert parity.verdicts_match(lb, c.lb, np.abs(c.lb).max(axis=1))[0]
    np.testing.assert_array_equal(lb, sl[:, -9:].astype(np.float64))
    bounds, _, _, _ = C.crownibp(c.wl.layers, c.l0, c.u0, c.spec_W)
    ol, ou = O.flatten_bounds(n0, bounds, c.B)
    worst, where = parity.continuous_errors(sl[:, n0:], su[:, n0:], ol, ou, c.sizes, label=(c.name, "gpu vs oracle"))
    assert worst <= 1.0, f"{name}: GPU vs oracle {worst:.3g}x tolerance at {where}"


def test_gpu_crownibp_full_batch_and_chunks():
    """The default workload's full batch: the first regions agree with the oracle, a
    workspace of one region at a time gives the same bounds, and the property bounds are
    no tighter than DeepPoly's (interval bounds below the property are looser)."""
    from cfgpu.engine import DeepPolyEngine
    wl = nets.workload(2)
    B = 256
    X = nets.centres(wl, B)
    y = nets.labels(wl, X)
    l0, u0 = (t.numpy() for t in nets.input_box(X, 0.002, wl.dataset))
    W = nets.spec_weight(y).numpy()
    lb, ub, sl, su = _cibp_run(wl, l0, u0, W)
    lb1, ub1, _, _ = _cibp_run(wl, l0, u0, W, budget=1)
    assert np.array_equal(lb, lb1) and np.array_equal(ub, ub1)
    nb = 2
    bounds, _, _, _ = C.crownibp(wl.layers, l0[:nb], u0[:nb], W[:nb])
    n0 = wl.input_size
    ol, ou = O.flatten_bounds(n0, bounds, nb)
    worst, where = parity.continuous_errors(sl[:nb, n0:], su[:nb, n0:], ol, ou, [L.n_out for L in wl.layers] + [9])
    assert worst <= 1.0, f"GPU vs oracle {worst:.3g}x tolerance at {where}"
    dev = torch.device("cuda:0")
    eng = DeepPolyEngine(wl.layers, wl.input_size, dev)
    lbd, _ = eng.run(torch.from_numpy(l0).to(dev), torch.from_numpy(u0).to(dev), torch.from_numpy(W).to(dev))
    lbd = lbd.cpu().numpy()
    assert (lb <= lbd + 1e-4 * np.abs(lbd).max()).all()


def test_gpu_crownibp_refuses_dag():
    from cfgpu.engine import DeepPolyEngine
    with pytest.raises(NotImplementedError):
        DeepPolyEngine(nets.workload(5).layers, nets.workload(5).input_size, "cuda:0", certifier="crownibp")
