"""GPU parity of the custom-stop DeepPoly programs (deeppoly_custom_stop.cf and
custom_stops/deeppoly_custom_stopNN.cf): DeepPolyEngine(stop_depth=get_start,
relu_strict=True) -> cf_deeppoly_run with cf_network.stop_depth, against the reference's
own outputs (tests/golden/cs*_*.npz) and the oracle (crown_oracle.custom_stop), on the
tensor-core chain and on the CUDA-core steps.  Tolerances: tests/parity.py."""
import numpy as np
import pytest
import torch

import parity
from golden_cases import Case, chain_names, names
from oracle import crown_oracle as C
from oracle import deeppoly_oracle as O
from cfgpu import nets

pytestmark = pytest.mark.gpu

CS_CASES = sorted(n for p in ("deeppoly_custom_stop",) + tuple(f"custom_stops/deeppoly_custom_stop{d:02d}"
                                                                for d in range(19)) for n in chain_names(p))


def _depth(name):
    return int(name[2:name.index("_")])


def _run(wl, l0, u0, W, depth, budget=None):
    from cfgpu.engine import DeepPolyEngine
    eng = DeepPolyEngine(wl.layers, wl.input_size, "cuda:0", stop_depth=depth, relu_strict=True)
    dev = torch.device("cuda:0")
    kw = {} if budget is None else {"workspace_budget": eng.workspace_bytes(budget)}
    lb, ub, sl, su = eng.run(torch.from_numpy(l0).to(dev), torch.from_numpy(u0).to(dev),
                             torch.from_numpy(W).to(dev), want_state=True, check_device=True, **kw)
    torch.cuda.synchronize()
    return lb.cpu().numpy(), ub.cpu().numpy(), sl.cpu().numpy(), su.cpu().numpy()


def _check(c, sl, su, lb, depth):
    n0 = c.wl.input_size
    worst, where = parity.continuous_errors(sl[:, n0:], su[:, n0:], c.l_all, c.u_all, c.sizes, label=(c.name, "gpu vs reference"))
    assert worst <= 1.0, f"{c.name}: GPU vs reference {worst:.3g}x tolerance at {where}"
    assert parity.verdicts_match(lb, c.lb, np.abs(c.lb).max(axis=1))[0]
    np.testing.assert_array_equal(lb, sl[:, -9:].astype(np.float64))
    bounds, _, _, _ = C.custom_stop(c.wl.layers, c.l0, c.u0, c.spec_W, depth)
    ol, ou = O.flatten_bounds(n0, bounds, c.B)
    worst, where = parity.continuous_errors(sl[:, n0:], su[:, n0:], ol, ou, c.sizes, label=(c.name, "gpu vs oracle"))
    assert worst <= 1.0, f"{c.name}: GPU vs oracle {worst:.3g}x tolerance at {where}"


@pytest.mark.parametrize("name", CS_CASES)
def test_gpu_custom_stop_matches_reference(name):
    c = Case(name)
    lb, ub, sl, su = _run(c.wl, c.l0, c.u0, c.spec_W, _depth(name))
    _check(c, sl, su, lb, _depth(name))


@pytest.mark.parametrize("name", ["cs3_w2_b4_e2e-4", "cs1_w0_b4_e1e-3", "cs0_w0_b4_e1e-3"])
def test_gpu_custom_stop_cuda_core_steps(name, monkeypatch):
    """The CUDA-core steps (CF_STEP_IMPL=simt) take the same stops."""
    monkeypatch.setenv("CF_STEP_IMPL", "simt")
    c = Case(name)
    lb, ub, sl, su = _run(c.wl, c.l0, c.u0, c.spec_W, _depth(name))
    _check(c, sl, su, lb, _depth(name))


@pytest.mark.parametrize("depth", [2, 3, 7])
def test_gpu_custom_stop_full_batch(depth):
    """The default workload's full batch: one region at a time gives the same bounds, the
    first regions agree with the oracle, and the deepest stop equals DeepPoly."""
    wl = nets.workload(2)
    B = 256
    X = nets.centres(wl, B)
    y = nets.labels(wl, X)
    l0, u0 = (t.numpy() for t in nets.input_box(X, 0.002, wl.dataset))
    W = nets.spec_weight(y).numpy()
    lb, ub, sl, su = _run(wl, l0, u0, W, depth)
    lb1, ub1, _, _ = _run(wl, l0, u0, W, depth, budget=1)
    assert np.array_equal(lb, lb1) and np.array_equal(ub, ub1)
    nb = 2
    bounds, _, _, _ = C.custom_stop(wl.layers, l0[:nb], u0[:nb], W[:nb], depth)
    n0 = wl.input_size
    ol, ou = O.flatten_bounds(n0, bounds, nb)
    sizes = [L.n_out for L in wl.layers] + [9]
    worst, where = parity.continuous_errors(sl[:nb, n0:], su[:nb, n0:], ol, ou, sizes)
    assert worst <= 1.0, f"GPU vs oracle {worst:.3g}x tolerance at {where}"


def test_gpu_custom_stop_deep_enough_is_deeppoly():
    """A stop below the input layer traverses to the input: DeepPoly's bounds."""
    from cfgpu.engine import DeepPolyEngine
    c = Case("dp_w2_b8_e2e-4")
    dev = torch.device("cuda:0")
    args = [torch.from_numpy(a).to(dev) for a in (c.l0, c.u0, c.spec_W)]
    lb1, ub1 = DeepPolyEngine(c.wl.layers, c.wl.input_size, dev).run(*args)
    lb2, ub2 = DeepPolyEngine(c.wl.layers, c.wl.input_size, dev, stop_depth=40).run(*args)
    torch.cuda.synchronize()
    assert torch.equal(lb1, lb2) and torch.equal(ub1, ub2)


def test_gpu_custom_stop_refusals():
    from cfgpu.engine import DeepPolyEngine
    with pytest.raises(NotImplementedError):
        DeepPolyEngine(nets.workload(3).layers, nets.workload(3).input_size, "cuda:0", stop_depth=3)
    with pytest.raises(NotImplementedError):
        DeepPolyEngine(nets.workload(0).layers, nets.workload(0).input_size, "cuda:0", certifier="crown",
                       stop_depth=3)
