"""GPU parity of the forward programs: zono.cf (DeepZ) and ibp.cf through
DeepPolyEngine(certifier='zono' | 'ibp') -> cf_deeppoly_run with CF_RELAX_ZONO /
CF_RELAX_IBP, and polyzono.cf through cfgpu.polyzono (DeepPoly and zonotope layer runs met
by cf_bounds_meet), against the reference's own outputs (tests/golden/zono_*, ibp_*,
pz_*) and the oracle; full-size soundness by sampling; the driver's refusals.
Tolerances: tests/parity.py.
"""
import numpy as np
import pytest
import torch

import parity
from golden_cases import Case, names
from oracle import deeppoly_oracle as O
from oracle import zono_oracle as Z
from cfgpu import nets

pytestmark = pytest.mark.gpu

CHAIN_ZONO = [n for n in names("zono", max_wid=9) if nets.is_chain(Case(n).wl.layers)]
CHAIN_IBP = [n for n in names("ibp", max_wid=9) if nets.is_chain(Case(n).wl.layers)]
PZ = names("polyzono", max_wid=9)
ZID = names("zid", max_wid=9)


def _engine(wl, certifier):
    from cfgpu.engine import DeepPolyEngine
    if certifier == "polyzono":
        from cfgpu.polyzono import PolyZonoEngine
        return PolyZonoEngine(wl.layers, wl.input_size, "cuda:0")
    if certifier == "zid":
        from cfgpu.zid import ZidEngine
        return ZidEngine(wl.layers, wl.input_size, "cuda:0")
    return DeepPolyEngine(wl.layers, wl.input_size, "cuda:0", certifier=certifier)


def _run(eng, l0, u0, W):
    dev = torch.device("cuda:0")
    lb, ub, sl, su = eng.run(torch.from_numpy(l0).to(dev), torch.from_numpy(u0).to(dev),
                             torch.from_numpy(W).to(dev), want_state=True, check_device=True)
    torch.cuda.synchronize()
    return lb.cpu().numpy(), ub.cpu().numpy(), sl.cpu().numpy(), su.cpu().numpy()


def _oracle(program, layers, l0, u0, W):
    if program == "ibp":
        return Z.ibp(layers, l0, u0, W)[0]
    if program == "polyzono":
        return Z.polyzono(layers, l0, u0, W)[0]
    if program == "zid":
        return Z.zid(layers, l0, u0, W)[0]
    return Z.zono(layers, l0, u0, W)[0]


@pytest.mark.parametrize("name", CHAIN_ZONO + CHAIN_IBP + PZ + ZID)
def test_gpu_forward_matches_reference(name):
    c = Case(name)
    lb, ub, sl, su = _run(_engine(c.wl, c.program), c.l0, c.u0, c.spec_W)
    n0 = c.wl.input_size
    assert np.array_equal(sl[:, :n0], c.l0) and np.array_equal(su[:, :n0], c.u0)
    worst, where = parity.continuous_errors(sl[:, n0:], su[:, n0:], c.l_all, c.u_all, c.sizes, label=(c.name, "gpu vs reference"))
    assert worst <= 1.0, f"{name}: GPU vs reference {worst:.3g}x tolerance at {where}"
    assert parity.verdicts_match(lb, c.lb, np.abs(c.lb).max(axis=1))[0]
    np.testing.assert_array_equal(lb, sl[:, -9:].astype(np.float64))
    np.testing.assert_array_equal(ub, su[:, -9:].astype(np.float64))
    bounds = _oracle(c.program, c.wl.layers, c.l0, c.u0, c.spec_W)
    ol, ou = O.flatten_bounds(n0, bounds, c.B)
    worst, where = parity.continuous_errors(sl[:, n0:], su[:, n0:], ol, ou, c.sizes, label=(c.name, "gpu vs oracle"))
    assert worst <= 1.0, f"{name}: GPU vs oracle {worst:.3g}x tolerance at {where}"


@pytest.mark.parametrize("certifier,wid,B,eps", [("zono", 2, 256, 0.002), ("zono", 1, 64, 0.005),
                                                 ("ibp", 4, 8, 2.0 / 255.0), ("zono", 3, 128, 0.02),
                                                 ("polyzono", 1, 64, 0.005), ("polyzono", 3, 32, 0.02),
                                                 ("zid", 2, 256, 0.002), ("zid", 3, 32, 0.02)])
def test_gpu_forward_full_size_sound(certifier, wid, B, eps):
    """The workload's full batch: concrete points of every box (its corners included) stay
    inside the bounds of every affine layer and of the property rows; the first regions
    also agree with the oracle."""
    wl = nets.workload(wid)
    X = nets.centres(wl, B)
    y = nets.labels(wl, X)
    l0, u0 = (t.numpy() for t in nets.input_box(X, eps, wl.dataset))
    W = nets.spec_weight(y).numpy()
    lb, ub, sl, su = _run(_engine(wl, certifier), l0, u0, W)
    assert np.isfinite(sl).all() and np.isfinite(su).all() and (sl <= su).all()
    n0 = wl.input_size
    kinds = [L.kind for L in wl.layers] + ["spec"]
    cols = np.cumsum([n0] + [L.n_out for L in wl.layers] + [9])
    rng = np.random.default_rng(1)
    dev = torch.device("cuda:0")
    for b in rng.choice(B, size=min(B, 4), replace=False):
        t = rng.random((64, n0)).astype(np.float32)
        t[:2] = np.array([0.0, 1.0])[:, None]
        x = torch.from_numpy(l0[b] + t * (u0[b] - l0[b])).to(dev, torch.float64)
        acts = _activations(wl, x, torch.from_numpy(W[b]).to(dev, torch.float64))
        for k, kind in enumerate(kinds):
            if kind == "relu" and certifier == "zono":
                continue
            lo = torch.from_numpy(sl[b, cols[k]:cols[k + 1]]).to(dev, torch.float64)
            hi = torch.from_numpy(su[b, cols[k]:cols[k + 1]]).to(dev, torch.float64)
            scale = max(1.0, float(acts[k].abs().max()))
            assert bool((acts[k] >= lo - 1e-4 * scale).all()) and bool((acts[k] <= hi + 1e-4 * scale).all()), \
                (certifier, int(b), k, kind)
    if wid != 4:
        nb = 2
        bounds = _oracle(certifier, wl.layers, l0[:nb], u0[:nb], W[:nb])
        ol, ou = O.flatten_bounds(n0, bounds, nb)
        sizes = [L.n_out for L in wl.layers] + [9]
        worst, where = parity.continuous_errors(sl[:nb, n0:], su[:nb, n0:], ol, ou, sizes)
        assert worst <= 1.0, f"GPU vs oracle {worst:.3g}x tolerance at {where}"


def _activations(wl, x, spec_W):
    """float64 torch forward of the layer list on flat inputs x [P, n0]: every layer's values."""
    vals = []
    h = x
    for L in wl.layers:
        if L.kind == "relu":
            h = torch.relu(h)
        elif L.kind == "linear":
            h = h @ torch.from_numpy(L.W).to(x).T + torch.from_numpy(L.b).to(x)
        else:
            img = h.reshape(h.shape[0], *L.in_shape)
            h = torch.nn.functional.conv2d(img, torch.from_numpy(L.W).to(x), torch.from_numpy(L.b).to(x),
                                           stride=L.stride, padding=L.pad).reshape(h.shape[0], -1)
        vals.append(h)
    vals.append(h @ spec_W.T)
    return vals


def test_gpu_ibp_conv_matches_reference():
    c = Case("ibp_w3_b2_e2e-3")
    lb, ub, sl, su = _run(_engine(c.wl, "ibp"), c.l0, c.u0, c.spec_W)
    n0 = c.wl.input_size
    worst, where = parity.continuous_errors(sl[:, n0:], su[:, n0:], c.l_all, c.u_all, c.sizes, label=(c.name, "gpu vs reference"))
    assert worst <= 1.0, f"GPU vs reference {worst:.3g}x tolerance at {where}"


def test_gpu_zono_refusals():
    """Networks with Add / Concat layers are refused by the zonotope driver with the
    reference's exception type."""
    with pytest.raises(NotImplementedError):
        _engine(nets.workload(5), "zono")
    with pytest.raises(NotImplementedError):
        _engine(nets.workload(5), "polyzono")


def test_gpu_polyzono_tighter_than_either_half():
    """The met property bounds are at least as tight as DeepPoly's and the zonotope's alone
    on the same regions."""
    c = Case("pz_w0_b4_e1e-2")
    lbp, ubp, _, _ = _run(_engine(c.wl, "polyzono"), c.l0, c.u0, c.spec_W)
    lbz, ubz, _, _ = _run(_engine(c.wl, "zono"), c.l0, c.u0, c.spec_W)
    lbd, ubd, _, _ = _run(_engine(c.wl, "deeppoly"), c.l0, c.u0, c.spec_W)
    tol = 1e-5 * np.abs(lbp).max()
    assert (lbp >= np.maximum(lbz, lbd) - tol).all() and (ubp <= np.minimum(ubz, ubd) + tol).all()
    assert (lbp > np.maximum(lbz, lbd) + tol).any()     # the meet inside the network tightens further


def test_gpu_forward_chunks_match_one_pass():
    """A workspace that holds one region at a time gives the same bounds as one pass."""
    c = Case("zono_w1_b8_e5e-4")
    eng = _engine(c.wl, "zono")
    dev = torch.device("cuda:0")
    l0, u0 = torch.from_numpy(c.l0).to(dev), torch.from_numpy(c.u0).to(dev)
    W = torch.from_numpy(c.spec_W).to(dev)
    lb1, ub1 = eng.run(l0, u0, W)
    lb2, ub2 = eng.run(l0, u0, W, workspace_budget=eng.workspace_bytes(1))
    torch.cuda.synchronize()
    assert torch.equal(lb1, lb2) and torch.equal(ub1, ub2)
