"""GPU parity on networks with residual Add and Concat layers (DeepPolyEngine on a
non-chain layer list -> the general traversal of cfgpu.general over libcfgpu kernels),
against the reference's own DeepPoly and CROWN outputs (tests/golden/dp_w5_*, dp_w6_*,
dp_w8_* (conv layers inside a residual block), crown_w5_*, crown_w6_*) and the general
oracle; and the general traversal on chain
networks against the fused driver.  Tolerances: tests/parity.py.
"""
import numpy as np
import pytest
import torch

import parity
from golden_cases import Case, names
from oracle import crown_oracle as C
from oracle import deeppoly_oracle as O
from cfgpu import nets

pytestmark = pytest.mark.gpu

DAG_CASES = [n for p in ("deeppoly", "crown") for n in names(p, max_wid=9)
             if not nets.is_chain(Case(n).wl.layers)]


def _run(wl, certifier, l0, u0, W):
    from cfgpu.engine import DeepPolyEngine
    eng = DeepPolyEngine(wl.layers, wl.input_size, "cuda:0", certifier=certifier)
    dev = torch.device("cuda:0")
    lb, ub, sl, su = eng.run(torch.from_numpy(l0).to(dev), torch.from_numpy(u0).to(dev),
                             torch.from_numpy(W).to(dev), want_state=True)
    torch.cuda.synchronize()
    return eng, lb.cpu().numpy(), ub.cpu().numpy(), sl.cpu().numpy(), su.cpu().numpy()


@pytest.mark.parametrize("name", DAG_CASES)
def test_gpu_dag_matches_reference(name):
    c = Case(name)
    rel = "crown" if c.program == "crown" else "deeppoly"
    eng, lb, ub, sl, su = _run(c.wl, rel, c.l0, c.u0, c.spec_W)
    assert not eng.chain and eng.net is None
    n0 = c.wl.input_size
    assert sl.shape[1] == n0 + sum(c.sizes)
    assert np.array_equal(sl[:, :n0], c.l0) and np.array_equal(su[:, :n0], c.u0)
    worst, where = parity.continuous_errors(sl[:, n0:], su[:, n0:], c.l_all, c.u_all, c.sizes, label=(c.name, "gpu vs reference"))
    assert worst <= 1.0, f"{name}: GPU vs reference {worst:.3g}x tolerance at {where}"
    assert parity.verdicts_match(lb, c.lb, np.abs(c.lb).max(axis=1))[0]
    np.testing.assert_array_equal(lb, sl[:, -9:].astype(np.float64))
    np.testing.assert_array_equal(ub, su[:, -9:].astype(np.float64))
    bounds, _, _, _ = C.certify(c.wl.layers, c.l0, c.u0, c.spec_W, rel)
    ol, ou = O.flatten_bounds(n0, bounds, c.B)
    worst, where = parity.continuous_errors(sl[:, n0:], su[:, n0:], ol, ou, c.sizes, label=(c.name, "gpu vs oracle"))
    assert worst <= 1.0, f"{name}: GPU vs oracle {worst:.3g}x tolerance at {where}"


@pytest.mark.parametrize("wid,eps", [(5, 0.1), (6, 0.3), (8, 1.0), (3, 1.0), (8, 0.3), (3, 0.2)])
def test_gpu_dag_crown_crossing(wid, eps):
    """Wide boxes: CROWN ReLU layers of the residual / concat / residual-conv network and of
    the conv chain take the all-crossing branch (every layer at the first four settings; the
    last ReLU, or the two conv ReLUs, at the other two).  The reference itself raises there
    on the residual network (abs_elem.py:459) and on any conv network (sparse_block.py:1726);
    its concat-network output at eps 0.1 is a golden case.  The GPU traversal (conv layers
    substituted by transposed convolutions) matches the general oracle."""
    wl = nets.workload(wid)
    X = nets.centres(wl, 2)
    y = nets.labels(wl, X)
    l0, u0 = (t.numpy() for t in nets.input_box(X, eps, wl.dataset))
    W = nets.spec_weight(y).numpy()
    _, lb, ub, sl, su = _run(wl, "crown", l0, u0, W)
    bounds, olb, _, br = C.certify(wl.layers, l0, u0, W, "crown")
    assert br == [C.BRANCH_CROSS] * len(br) if eps >= 0.1 and wid in (5, 6) or eps == 1.0 else C.BRANCH_CROSS in br
    ol, ou = O.flatten_bounds(wl.input_size, bounds, 2)
    sizes = [L.n_out for L in wl.layers] + [9]
    n0 = wl.input_size
    worst, where = parity.continuous_errors(sl[:, n0:], su[:, n0:], ol, ou, sizes)
    assert worst <= 1.0, f"GPU vs oracle {worst:.3g}x tolerance at {where}"


@pytest.mark.parametrize("name", ["dp_w0_b4_e1e-3", "dp_w2_b8_e2e-4"])
def test_gpu_general_on_chain_matches_fused_driver(name):
    """The general traversal over a chain network gives the fused driver's bounds."""
    from cfgpu import general
    from cfgpu.engine import DeepPolyEngine
    c = Case(name)
    eng, lb, ub, sl, su = _run(c.wl, "deeppoly", c.l0, c.u0, c.spec_W)
    assert eng.chain
    dev = torch.device("cuda:0")
    l0, u0 = torch.from_numpy(c.l0).to(dev), torch.from_numpy(c.u0).to(dev)
    bounds, _ = general.run(eng._general, l0, u0, torch.from_numpy(c.spec_W).to(dev), "deeppoly")
    gl, gu = (t.cpu().numpy() for t in general.state(l0, u0, bounds))
    n0 = c.wl.input_size
    worst, where = parity.continuous_errors(gl[:, n0:], gu[:, n0:], sl[:, n0:], su[:, n0:], c.sizes)
    assert worst <= 1.0, f"{name}: general vs fused {worst:.3g}x tolerance at {where}"
    del DeepPolyEngine


def test_gpu_dag_rejects_bad_layers():
    from cfgpu.engine import DeepPolyEngine
    wl = nets.workload(5)
    layers = list(wl.layers)
    i = next(k for k, L in enumerate(layers) if L.kind == "add")
    bad = nets.Layer(**{**layers[i].__dict__, "parents": (i + 1, 0)})
    with pytest.raises(ValueError):
        DeepPolyEngine(layers[:i] + [bad] + layers[i + 1:], wl.input_size, "cuda:0")


@pytest.mark.parametrize("wid", [5, 6, 8])
def test_gpu_dag_graph_replay_equals_eager(wid):
    """DeepPoly's general traversal is captured in a CUDA graph per batch size and
    replayed with new inputs: bitwise the eager traversal, for two different batches."""
    from cfgpu.engine import DeepPolyEngine
    wl = nets.workload(wid)
    dev = torch.device("cuda:0")
    eng = DeepPolyEngine(wl.layers, wl.input_size, dev)
    ref = DeepPolyEngine(wl.layers, wl.input_size, dev)
    ref.graphs = False
    for eps, seed_off in ((0.002, 0), (0.004, 8)):
        X = nets.centres(wl, 16)[seed_off // 8:seed_off // 8 + 8]
        y = nets.labels(wl, X)
        l0, u0 = (t.to(dev) for t in nets.input_box(X, eps, wl.dataset))
        W = nets.spec_weight(y).to(dev)
        lb, ub, sl, su = eng.run(l0, u0, W, want_state=True)
        lb2, ub2, sl2, su2 = ref.run(l0, u0, W, want_state=True)
        torch.cuda.synchronize()
        assert torch.equal(lb, lb2) and torch.equal(sl, sl2) and torch.equal(su, su2)
    assert eng.graphs and len(eng._graph_cache) == 1
