"""Region lanes of a chained DeepPoly pass (cf_deeppoly_run): when a hidden layer's chain
launch spans at least two waves, the regions of a chunk run as 2 (CF_CHAIN_LANES: 1-4)
lanes on separate streams.  A region's arithmetic does not depend on which lane or tile
holds it, so every bound -- every neuron of the state and the float64 property bounds --
is bit-identical to the single-stream run, and the error word stays clear.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(wl, B, dev):
    from cfgpu import nets
    X = nets.centres(wl, B)
    y = nets.labels(wl, X)
    l0, u0 = nets.input_box(X, wl.eps, wl.dataset)
    return l0.to(dev), u0.to(dev), nets.spec_weight(y).to(dev)


@pytest.mark.parametrize("wid,B", [(2, 256), (2, 203)])
def test_lanes_are_bit_identical_to_one_stream(monkeypatch, wid, B):
    from cfgpu import nets
    from cfgpu.engine import DeepPolyEngine
    dev = torch.device("cuda:0")
    wl = nets.workload(wid)
    eng = DeepPolyEngine(wl.layers, wl.input_size, dev)
    l0, u0, W = _inputs(wl, B, dev)
    runs = {}
    for lanes in ("1", "2", "3", "4"):
        monkeypatch.setenv("CF_CHAIN_LANES", lanes)
        lb, ub, sl, su = eng.run(l0, u0, W, want_state=True, check_device=True)
        torch.cuda.synchronize()
        runs[lanes] = [t.cpu().numpy() for t in (lb, ub, sl, su)]
    ref = runs["1"]
    assert all(np.isfinite(a).all() for a in ref)
    for lanes, got in runs.items():
        for name, a, b in zip(("lb", "ub", "state_l", "state_u"), got, ref):
            assert np.array_equal(a, b), (lanes, name, float(np.abs(a - b).max()))
