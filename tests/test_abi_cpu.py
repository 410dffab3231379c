"""The C ABI without a GPU: the library loads, exports every declared symbol, plans
networks, and rejects bad input with the reference's error types before any launch."""
import ctypes
import os
import re

import pytest

from cfgpu import _lib, nets

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "cfgpu.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(cf_[a-z0-9_]+)\s*\(", src)))


def test_every_declared_symbol_is_exported():
    names = declared_functions()
    assert len(names) >= 13
    for n in names:
        assert hasattr(_lib.lib, n), f"{n} declared in include/cfgpu.h but not exported"
    assert set(_lib.EXPORTED) == set(names)


def test_version():
    assert b"sm_100a" in _lib.lib.cf_version()


def _net(wl, fake_ptr=256):
    descs = []
    for L in wl.layers:
        d = _lib.CfLayer()
        if L.kind == "relu":
            d.kind, d.n_in, d.n_out = _lib.CF_LAYER_RELU, L.n_in, L.n_out
        else:
            d.kind = _lib.CF_LAYER_LINEAR if L.kind == "linear" else _lib.CF_LAYER_CONV
            d.n_in, d.n_out = L.n_in, L.n_out
            d.W_dev = d.b_dev = fake_ptr
            if L.kind == "conv":
                d.cout, d.cin, d.kh, d.kw = L.W.shape
                _, d.ih, d.iw = L.in_shape
                _, d.oh, d.ow = L.out_shape
                d.stride, d.pad = L.stride, L.pad
        descs.append(d)
    arr = (_lib.CfLayer * len(descs))(*descs)
    return _lib.CfNetwork(len(descs), arr, wl.input_size, 9, 0), arr


@pytest.mark.parametrize("wid,N", [(0, 1103), (1, 2003), (2, 4403)])
def test_neuron_count_matches_reference_layout(wid, N):
    wl = nets.workload(wid)
    net, keep = _net(wl)
    assert _lib.lib.cf_network_neurons(ctypes.byref(net)) == N
    layout = nets.neuron_layout(wl)
    assert layout[-1][2] == N


def test_workspace_grows_linearly_in_chunk():
    wl = nets.workload(2)
    net, keep = _net(wl)
    w1 = _lib.lib.cf_deeppoly_workspace_bytes(ctypes.byref(net), 1)
    w8 = _lib.lib.cf_deeppoly_workspace_bytes(ctypes.byref(net), 8)
    w64 = _lib.lib.cf_deeppoly_workspace_bytes(ctypes.byref(net), 64)
    assert 0 < w1 < w8 < w64
    assert abs((w64 - w8) / 56 - (w8 - w1) / 7) < 1024


def test_bad_networks_are_rejected():
    wl = nets.workload(0)
    net, keep = _net(wl)
    keep[0].n_in = 783  # width mismatch with the input
    assert _lib.lib.cf_network_neurons(ctypes.byref(net)) == -1
    st = _lib.lib.cf_deeppoly_run(ctypes.byref(net), 1, 8, 8, 8, None, None, 8, 8, 8, 1 << 20, None)
    assert st == _lib.CF_ERR_SHAPE
    with pytest.raises(Exception, match="SHAPE MISMATCH"):
        _lib.check(st)
    keep[0].n_in = 784
    keep[1].kind = _lib.CF_LAYER_LINEAR  # ReLU turned into a weightless linear layer
    keep[1].W_dev = None
    st = _lib.lib.cf_deeppoly_run(ctypes.byref(net), 1, 8, 8, 8, None, None, 8, 8, 8, 1 << 20, None)
    assert st == _lib.CF_ERR_NULL


def test_workspace_too_small_is_reported():
    wl = nets.workload(0)
    net, keep = _net(wl)
    need = _lib.lib.cf_deeppoly_workspace_bytes(ctypes.byref(net), 1)
    st = _lib.lib.cf_deeppoly_run(ctypes.byref(net), 4, 8, 8, 8, None, None, 8, 8, 8, need - 1, None)
    assert st == _lib.CF_ERR_WORKSPACE
    assert b"workspace" in _lib.lib.cf_last_error()


def test_host_fault_injection(monkeypatch):
    """CF_FAULT makes the host wrapper fail before any launch (no GPU involved)."""
    monkeypatch.setenv("CF_FAULT", "relu_relax,deeppoly_run")
    st = _lib.lib.cf_relu_relax(1, 4, 8, 8, 4, 8, 8, 4, 8, 8, 8, 0, None)
    assert st == _lib.CF_ERR_INJECTED
    wl = nets.workload(0)
    net, keep = _net(wl)
    st = _lib.lib.cf_deeppoly_run(ctypes.byref(net), 1, 8, 8, 8, None, None, 8, 8, 8, 1 << 30, None)
    assert st == _lib.CF_ERR_INJECTED
    with pytest.raises(_lib.CfError):
        _lib.check(st)
    monkeypatch.setenv("CF_FAULT", "")


def test_argument_validation_without_launch():
    assert _lib.lib.cf_backsub_step(1, 1, 0, 4, 8, 0, 0, 4, None, 0, 0, None, None, None, 8, None, 8, 8, None) \
        == _lib.CF_ERR_SHAPE
    assert _lib.lib.cf_backsub_step(1, 1, 4, 4, 8, 0, 0, 4, None, 0, 0, 8, None, None, 8, None, 8, 8, None) \
        == _lib.CF_ERR_NULL
    assert _lib.lib.cf_relu_relax(1, 4, 8, 8, 4, 8, 8, 4, 8, 8, 8, 7, None) == _lib.CF_ERR_UNSUPPORTED
    shape = _lib.i64_array([2, 3])
    assert _lib.lib.cf_ew_binary(99, 2, shape, 8, 0, None, 8, 0, None, 8, 0, None) == _lib.CF_ERR_UNSUPPORTED
    assert _lib.lib.cf_ew_binary(0, 9, shape, 8, 0, None, 8, 0, None, 8, 0, None) == _lib.CF_ERR_SHAPE
    # empty problems are no-ops that touch nothing
    assert _lib.lib.cf_relu_relax(0, 4, None, None, 4, None, None, 4, None, None, None, 0, None) == _lib.CF_OK


@pytest.mark.parametrize("relax", [2, 3])
def test_forward_programs_plan_without_device(relax):
    """zono.cf / ibp.cf networks: same neuron layout and a workspace linear in the chunk;
    a workspace too small for one region is refused before any launch."""
    assert (_lib.CF_RELAX_ZONO, _lib.CF_RELAX_IBP) == (2, 3)
    wl = nets.workload(2)
    net, keep = _net(wl)
    net.relaxation = relax
    assert _lib.lib.cf_network_neurons(ctypes.byref(net)) == 4403
    w1 = _lib.lib.cf_deeppoly_workspace_bytes(ctypes.byref(net), 1)
    w8 = _lib.lib.cf_deeppoly_workspace_bytes(ctypes.byref(net), 8)
    w15 = _lib.lib.cf_deeppoly_workspace_bytes(ctypes.byref(net), 15)
    assert 0 < w1 < w8 < w15 and abs((w15 - w8) / 7 - (w8 - w1) / 7) < 4096
    st = _lib.lib.cf_deeppoly_run(ctypes.byref(net), 4, 8, 8, 8, None, None, 8, 8, 8, w1 - 1, None)
    assert st == _lib.CF_ERR_WORKSPACE
    conv, keep2 = _net(nets.workload(3))
    conv.relaxation = relax
    assert _lib.lib.cf_network_neurons(ctypes.byref(conv)) == 8011
    assert _lib.lib.cf_deeppoly_workspace_bytes(ctypes.byref(conv), 2) > 0
    net.relaxation = 7
    assert _lib.lib.cf_network_neurons(ctypes.byref(net)) == -1
