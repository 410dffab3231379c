"""GPU parity of the DeepPoly network driver (libcfgpu through its C ABI).

Every case runs on cuda:0 through cfgpu.engine -> cf_deeppoly_run and is compared with
(1) the oracle replaying the GPU's own ReLU decisions (continuous agreement on every
neuron), and (2) the reference's golden outputs: identical decisions up to the first
tie, continuous agreement before it, identical verdicts.  Tolerances: tests/parity.py.
"""
import numpy as np
import pytest
import torch

import parity
from golden_cases import Case, chain_names, has_conv, names
from oracle import deeppoly_oracle as O

pytestmark = pytest.mark.gpu

MLP_CASES = [n for n in chain_names() if not has_conv(n)]
CONV_CASES = [n for n in chain_names() if has_conv(n)]
# the 3x32x32 net at 8 regions: compared with the reference (own and replayed decisions); the
# oracle's window restatement needs tens of seconds per region of it


def _engine(wl):
    from cfgpu.engine import DeepPolyEngine
    return DeepPolyEngine(wl.layers, wl.input_size, "cuda:0")


def _gpu_run(c, eng=None):
    eng = eng or _engine(c.wl)
    dev = torch.device("cuda:0")
    l0 = torch.from_numpy(c.l0).to(dev)
    u0 = torch.from_numpy(c.u0).to(dev)
    W = torch.from_numpy(c.spec_W).to(dev)
    lb, ub, sl, su = eng.run(l0, u0, W, want_state=True)
    torch.cuda.synchronize()
    return lb.cpu().numpy(), ub.cpu().numpy(), sl.cpu().numpy(), su.cpu().numpy()


def _first_flip_layer(xl, xu, rl, ru, sizes, relu_layers):
    sls = parity.layer_slices(sizes)
    for li in relu_layers:
        sl = sls[li]
        for a, b in zip(parity.decision_masks(xl[:, sl], xu[:, sl]), parity.decision_masks(rl[:, sl], ru[:, sl])):
            if (a != b).any():
                return li
    return None


def _check_case(c, lb, ub, sl, su, with_oracle=True):
    n0 = c.wl.input_size
    # input columns: the box itself, bit for bit
    assert np.array_equal(sl[:, :n0], c.l0) and np.array_equal(su[:, :n0], c.u0)
    xl, xu = sl[:, n0:], su[:, n0:]
    assert lb.dtype == np.float64 and lb.shape == (c.B, 9)
    np.testing.assert_array_equal(lb, xl[:, -9:].astype(np.float64))
    if with_oracle:
        # (1) against the oracle replaying the GPU's decisions
        run = O.deeppoly_windows if c.wid >= 3 else O.deeppoly
        bounds, _, _ = run(c.wl.layers, c.l0, c.u0, c.spec_W, force=(xl, xu))
        ol, ou = O.flatten_bounds(n0, bounds, c.B)
        worst, where = parity.continuous_errors(xl, xu, ol, ou, c.sizes, label=(c.name, "gpu vs oracle"))
        assert worst <= 1.0, f"{c.name}: GPU vs oracle {worst:.3g}x tolerance at {where}"
        ok, flips, ratio = parity.decision_flips_are_ties(ol, ou, xl, xu, c.sizes, c.relu_layers)
        assert ok, f"{c.name}: oracle would branch differently off-tie ({flips}, {ratio:.3g})"
    # (2) against the reference itself, up to its first tie-induced branch difference
    ff = _first_flip_layer(xl, xu, c.l_all, c.u_all, c.sizes, c.relu_layers)
    upto = len(c.sizes) if ff is None else ff + 1
    cut = sum(c.sizes[:upto])
    worst, where = parity.continuous_errors(xl[:, :cut], xu[:, :cut], c.l_all[:, :cut], c.u_all[:, :cut],
                                            c.sizes[:upto], label=(c.name, "gpu vs reference (own decisions)"))
    assert worst <= 1.0, f"{c.name}: GPU vs reference {worst:.3g}x tolerance at {where}"
    loose, where = parity.looser_errors(xl[:, :cut], xu[:, :cut], c.l_all[:, :cut], c.u_all[:, :cut],
                                        c.sizes[:upto], label=(c.name, "gpu looser than reference (own decisions)"))
    assert loose <= 1.0, f"{c.name}: GPU looser than the reference by {loose:.3g}x tolerance at {where}"
    if ff is not None:
        # the first differing branch must be a tie of the reference's own bounds
        sizes_cut = c.sizes[:ff + 1]
        ok, flips, ratio = parity.decision_flips_are_ties(xl[:, :cut], xu[:, :cut], c.l_all[:, :cut],
                                                          c.u_all[:, :cut], sizes_cut, [ff])
        assert ok, f"{c.name}: first branch difference is not a tie ({ratio:.3g})"
    same, nd = parity.verdicts_match(lb, c.lb, np.abs(c.lb).max(axis=1))
    assert same, f"{c.name}: {nd} verdicts differ from the reference"
    parity.record(c.name, "verdicts differing from the reference", nd)


@pytest.mark.parametrize("name", MLP_CASES)
def test_deeppoly_mlp_matches_reference(name):
    c = Case(name)
    _check_case(c, *_gpu_run(c))


@pytest.mark.parametrize("name", CONV_CASES)
def test_deeppoly_conv_matches_reference(name):
    """Conv networks (receptive-field windows).  The 3x32x32 net is compared with the
    reference's golden bounds directly (its CPU oracle takes tens of seconds per region) and,
    with the reference's decisions replayed, on every layer (test_replay_matches_reference)."""
    c = Case(name)
    _check_case(c, *_gpu_run(c), with_oracle=c.wid <= 3)


@pytest.mark.parametrize("name", MLP_CASES + CONV_CASES)
def test_replay_matches_reference(name):
    """The GPU replaying the reference's own ReLU decisions (cf_deeppoly_run_replay): every
    neuron of every layer, including the layers below a tie-induced branch difference of the
    GPU's own run, agrees with the reference within the tolerance and is never looser than
    it; the verdicts are identical."""
    c = Case(name)
    eng = _engine(c.wl)
    dev = torch.device("cuda:0")
    n0 = c.wl.input_size
    dl = torch.from_numpy(np.concatenate([c.l0, c.l_all], axis=1)).to(dev).contiguous()
    du = torch.from_numpy(np.concatenate([c.u0, c.u_all], axis=1)).to(dev).contiguous()
    lb, ub, sl, su = eng.run(torch.from_numpy(c.l0).to(dev), torch.from_numpy(c.u0).to(dev),
                             torch.from_numpy(c.spec_W).to(dev), want_state=True, replay=(dl, du))
    xl, xu = sl.cpu().numpy()[:, n0:], su.cpu().numpy()[:, n0:]
    lb = lb.cpu().numpy()
    worst, where = parity.continuous_errors(xl, xu, c.l_all, c.u_all, c.sizes,
                                            label=(c.name, "gpu vs reference (reference decisions)"))
    assert worst <= 1.0, f"{c.name}: replayed GPU vs reference {worst:.3g}x tolerance at {where}"
    loose, where = parity.looser_errors(xl, xu, c.l_all, c.u_all, c.sizes,
                                        label=(c.name, "gpu looser than reference (reference decisions)"))
    assert loose <= 1.0, f"{c.name}: replayed GPU looser than the reference by {loose:.3g}x tolerance at {where}"
    # with the same decisions every branch of the GPU's own bounds agrees except on ties
    ok, flips, ratio = parity.decision_flips_are_ties(xl, xu, c.l_all, c.u_all, c.sizes, c.relu_layers)
    assert ok, f"{c.name}: replayed GPU would branch differently off-tie ({flips}, {ratio:.3g})"
    same, nd = parity.verdicts_match(lb, c.lb, np.abs(c.lb).max(axis=1))
    assert same, f"{c.name}: {nd} verdicts differ from the reference"


def test_replay_of_own_decisions_is_identity():
    """Replaying the GPU's own decisions reproduces its bounds bit for bit."""
    c = Case([n for n in MLP_CASES if n.startswith("dp_w1")][0])
    eng = _engine(c.wl)
    lb, ub, sl, su = _gpu_run(c, eng)
    dev = torch.device("cuda:0")
    lb2, ub2, sl2, su2 = eng.run(torch.from_numpy(c.l0).to(dev), torch.from_numpy(c.u0).to(dev),
                                 torch.from_numpy(c.spec_W).to(dev), want_state=True,
                                 replay=(torch.from_numpy(sl).to(dev), torch.from_numpy(su).to(dev)))
    assert np.array_equal(sl2.cpu().numpy(), sl) and np.array_equal(su2.cpu().numpy(), su)


def test_batch_independence_and_determinism():
    """A region's bounds do not depend on the batch around it; reruns are bit-identical."""
    c = Case([n for n in MLP_CASES if n.startswith("dp_w2")][0])
    eng = _engine(c.wl)
    lb, ub, sl, su = _gpu_run(c, eng)
    lb2, ub2, sl2, su2 = _gpu_run(c, eng)
    assert np.array_equal(sl, sl2) and np.array_equal(su, su2)
    dev = torch.device("cuda:0")
    for b in (0, c.B - 1):
        l0 = torch.from_numpy(c.l0[b:b + 1]).to(dev)
        u0 = torch.from_numpy(c.u0[b:b + 1]).to(dev)
        W = torch.from_numpy(c.spec_W[b:b + 1]).to(dev)
        lb1, ub1, s1, u1 = eng.run(l0, u0, W, want_state=True)
        assert np.array_equal(s1.cpu().numpy()[0], sl[b]) and np.array_equal(u1.cpu().numpy()[0], su[b])


def test_chunked_workspace_matches_single_chunk():
    """A workspace that holds only a few regions (several chunks per call) gives the same bits."""
    c = Case([n for n in MLP_CASES if n.startswith("dp_w1")][0])
    eng = _engine(c.wl)
    lb, ub, sl, su = _gpu_run(c, eng)
    dev = torch.device("cuda:0")
    eng2 = _engine(c.wl)
    small = eng2.workspace_bytes(3)
    l0 = torch.from_numpy(c.l0).to(dev)
    u0 = torch.from_numpy(c.u0).to(dev)
    W = torch.from_numpy(c.spec_W).to(dev)
    lbc, ubc, slc, suc = eng2.run(l0, u0, W, want_state=True, workspace_budget=small)
    assert eng2._ws.numel() == small
    assert np.array_equal(slc.cpu().numpy(), sl) and np.array_equal(lbc.cpu().numpy(), lb)


@pytest.mark.parametrize("wid,B,sample", [(1, 64, 16), (2, 256, 12)])
def test_full_size_batch_against_oracle(wid, B, sample):
    """The full benchmark batch on the GPU; a seeded sample of its regions checked by the oracle."""
    from cfgpu import nets
    wl = nets.workload(wid)
    X = nets.centres(wl, B)
    y = nets.labels(wl, X)
    l0, u0 = nets.input_box(X, wl.eps, wl.dataset)
    W = nets.spec_weight(y)
    eng = _engine(wl)
    dev = torch.device("cuda:0")
    lb, ub, sl, su = eng.run(l0.to(dev), u0.to(dev), W.to(dev), want_state=True)
    sl, su = sl.cpu().numpy()[:, wl.input_size:], su.cpu().numpy()[:, wl.input_size:]
    idx = np.sort(np.random.default_rng(wid).choice(B, sample, replace=False))
    bounds, _, _ = O.deeppoly(wl.layers, l0.numpy()[idx], u0.numpy()[idx], W.numpy()[idx],
                              force=(sl[idx], su[idx]))
    ol, ou = O.flatten_bounds(wl.input_size, bounds, sample)
    sizes = [L.n_out for L in wl.layers] + [9]
    worst, where = parity.continuous_errors(sl[idx], su[idx], ol, ou, sizes)
    assert worst <= 1.0, f"workload {wid}: {worst:.3g}x tolerance at {where}"
    assert np.isfinite(sl).all() and np.isfinite(su).all()
    assert (sl <= su + 1e-4 * np.abs(su).max()).all(), "lower bound above upper bound"


@pytest.mark.parametrize("wid,B", [(3, 16), (4, 2)])
def test_conv_tensor_core_matches_cuda_core(wid, B, monkeypatch):
    """The tcgen05 transposed convolution of the conv windows (3xTF32) against the CUDA-core
    float32 implicit GEMM (CF_CONV_IMPL=simt) on the same regions: every neuron within the
    parity tolerance, decisions replayed so that a tie cannot make the two runs diverge."""
    from cfgpu import nets
    wl = nets.workload(wid)
    X = nets.centres(wl, B)
    y = nets.labels(wl, X)
    l0, u0 = nets.input_box(X, wl.eps, wl.dataset)
    W = nets.spec_weight(y)
    dev = torch.device("cuda:0")
    eng = _engine(wl)
    l0d, u0d, Wd = l0.to(dev), u0.to(dev), W.to(dev)
    lb, ub, sl, su = eng.run(l0d, u0d, Wd, want_state=True, check_device=True)
    monkeypatch.setenv("CF_CONV_IMPL", "simt")
    lb2, ub2, sl2, su2 = eng.run(l0d, u0d, Wd, want_state=True, check_device=True, replay=(sl, su))
    n0 = wl.input_size
    sizes = [L.n_out for L in wl.layers] + [9]
    x = sl.cpu().numpy()[:, n0:], su.cpu().numpy()[:, n0:]
    r = sl2.cpu().numpy()[:, n0:], su2.cpu().numpy()[:, n0:]
    worst, where = parity.continuous_errors(x[0], x[1], r[0], r[1], sizes,
                                            label=(f"w{wid}_b{B}", "tensor-core vs CUDA-core conv"))
    assert worst <= 1.0, f"workload {wid}: tensor-core conv vs CUDA-core conv {worst:.3g}x tolerance at {where}"
    assert np.isfinite(x[0]).all() and np.isfinite(x[1]).all()
