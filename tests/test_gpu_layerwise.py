"""The per-layer entry point (cf_deeppoly_layer through cfgpu.layerwise.LayerRun) gives the
whole-network driver's bounds for every program it runs, layer by layer; and it refuses
calls out of order or with a workspace smaller than the whole batch needs."""
import ctypes

import pytest
import torch

from cfgpu import _lib, nets
from cfgpu.engine import DeepPolyEngine
from cfgpu.layerwise import LayerRun

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("certifier,wid,B,eps", [("deeppoly", 2, 32, 0.002), ("deeppoly", 3, 4, 0.02),
                                                 ("crown", 0, 8, 0.005), ("zono", 1, 16, 0.005),
                                                 ("ibp", 3, 8, 0.02), ("deeppoly", 0, 1, 0.01),
                                                 ("zono", 3, 4, 0.02), ("crownibp", 2, 16, 0.002),
                                                 ("crownibp", 3, 4, 0.02), ("deeppoly", 4, 2, 2 / 255)])
def test_layerwise_equals_whole_pass(certifier, wid, B, eps):
    wl = nets.workload(wid)
    dev = torch.device("cuda:0")
    X = nets.centres(wl, B)
    y = nets.labels(wl, X)
    l0, u0 = (t.to(dev) for t in nets.input_box(X, eps, wl.dataset))
    W = nets.spec_weight(y).to(dev)
    eng = DeepPolyEngine(wl.layers, wl.input_size, dev, certifier=certifier)
    lb, ub, sl, su = eng.run(l0, u0, W, want_state=True, workspace_budget=eng.workspace_bytes(B))
    run = LayerRun(eng, l0, u0, W)
    for i in range(run.n_layers + 1):
        run.layer(i)
    lb2, ub2 = run.finish()
    torch.cuda.synchronize()
    assert torch.equal(lb, lb2) and torch.equal(ub, ub2)
    assert torch.equal(sl, run.state_l) and torch.equal(su, run.state_u)


def test_layerwise_refusals():
    wl = nets.workload(0)
    dev = torch.device("cuda:0")
    X = nets.centres(wl, 2)
    l0, u0 = (t.to(dev) for t in nets.input_box(X, 0.01, wl.dataset))
    W = nets.spec_weight(nets.labels(wl, X)).to(dev)
    eng = DeepPolyEngine(wl.layers, wl.input_size, dev)
    run = LayerRun(eng, l0, u0, W)
    with pytest.raises(ValueError):
        run.layer(1)
    small = eng.workspace_bytes(1)
    st = _lib.lib.cf_deeppoly_layer(ctypes.byref(eng.net), 0, 2, l0.data_ptr(), u0.data_ptr(), W.data_ptr(),
                                    run.state_l.data_ptr(), run.state_u.data_ptr(), run.lb.data_ptr(),
                                    run.ub.data_ptr(), run.ws.data_ptr(), small, None)
    assert st == _lib.CF_ERR_WORKSPACE and b"whole batch" in _lib.lib.cf_last_error()
    st = _lib.lib.cf_deeppoly_layer(ctypes.byref(eng.net), 99, 2, l0.data_ptr(), u0.data_ptr(), W.data_ptr(),
                                    run.state_l.data_ptr(), run.state_u.data_ptr(), run.lb.data_ptr(),
                                    run.ub.data_ptr(), run.ws.data_ptr(), run.ws.numel(), None)
    assert st == _lib.CF_ERR_SHAPE
    with pytest.raises(NotImplementedError):
        LayerRun(DeepPolyEngine(nets.workload(5).layers, 784, dev), l0, u0, W)
