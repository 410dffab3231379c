"""cf_deeppoly_run_static: certification without any device allocation by the caller.

Callers such as a plugin running inside another framework's allocator, or a service
that must not touch the allocator while serving, cannot pass a workspace.  This entry
point uses a fixed device array inside libcfgpu instead.  The test calls it through the
C ABI twice in a row and checks both results against cf_deeppoly_run with a caller
workspace: bit for bit, since the region chunking of the driver does not change any
region's arithmetic; after each call cf_deeppoly_check_static reports the device status of
the fixed array.  It also checks that a network too large for the fixed array, and a CROWN
batch that does not fit it in one chunk, are rejected with a clear error.

The file name sorts last so that a run stopping at the first failure has already run
every other test; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

import parity

pytestmark = pytest.mark.gpu


def _inputs(wl, B, dev):
    from cfgpu import nets
    X = nets.centres(wl, B)
    y = nets.labels(wl, X)
    l0, u0 = nets.input_box(X, wl.eps, wl.dataset)
    return l0.to(dev), u0.to(dev), nets.spec_weight(y).to(dev)


@pytest.mark.parametrize("wid,B", [(2, 256), (1, 64)])
def test_static_scratch_matches_workspace_entry_point(wid, B):
    from cfgpu import _lib, nets
    from cfgpu.engine import DeepPolyEngine
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    wl = nets.workload(wid)
    eng = DeepPolyEngine(wl.layers, wl.input_size, dev)
    l0, u0, W = _inputs(wl, B, dev)
    lb_ref, ub_ref, sl_ref, su_ref = eng.run(l0, u0, W, want_state=True, check_device=True)
    torch.cuda.synchronize()
    sizes = [L.n_out for L in wl.layers] + [9]
    n0 = wl.input_size
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call in range(2):
        lb = torch.full((B, 9), float("nan"), dtype=torch.float64, device=dev)
        ub = torch.full_like(lb, float("nan"))
        sl = torch.full((B, eng.N), float("nan"), dtype=torch.float32, device=dev)
        su = torch.full_like(sl, float("nan"))
        st = _lib.lib.cf_deeppoly_run_static(ctypes.byref(eng.net), B, l0.data_ptr(), u0.data_ptr(), W.data_ptr(),
                                             sl.data_ptr(), su.data_ptr(), lb.data_ptr(), ub.data_ptr(), stream)
        _lib.check(st, f"cf_deeppoly_run_static call {call}")
        _lib.check(_lib.lib.cf_deeppoly_check_static(stream), f"device status after static call {call}")
        torch.cuda.synchronize()
        x_l, x_u = sl.cpu().numpy(), su.cpu().numpy()
        r_l, r_u = sl_ref.cpu().numpy(), su_ref.cpu().numpy()
        assert np.isfinite(x_l).all() and np.isfinite(x_u).all(), f"call {call}: unwritten outputs"
        worst, where = parity.continuous_errors(x_l[:, n0:], x_u[:, n0:], r_l[:, n0:], r_u[:, n0:], sizes)
        assert worst <= 1.0, f"call {call}: static vs workspace entry point {worst:.3g}x tolerance at {where}"
        # chunking does not change a region's arithmetic: the same bits
        assert np.array_equal(x_l, r_l) and np.array_equal(x_u, r_u), f"call {call}: state differs"
        assert np.array_equal(lb.cpu().numpy(), lb_ref.cpu().numpy())
        assert np.array_equal(ub.cpu().numpy(), ub_ref.cpu().numpy())


def test_static_scratch_rejects_crown_batch_beyond_one_chunk():
    """CROWN decides each ReLU branch over the whole batch, so its batch must fit the fixed
    array in one chunk; a larger batch is refused before any launch."""
    from cfgpu import _lib, nets
    from cfgpu.engine import DeepPolyEngine
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    wl = nets.workload(2)
    eng = DeepPolyEngine(wl.layers, wl.input_size, dev, certifier="crown")
    B = 1024
    assert eng.workspace_bytes(B) > _lib.CF_STATIC_SCRATCH_BYTES >= eng.workspace_bytes(1)
    l0 = torch.zeros(B, wl.input_size, device=dev)
    W = torch.zeros(B, 9, 10, device=dev)
    lb = torch.zeros(B, 9, dtype=torch.float64, device=dev)
    st = _lib.lib.cf_deeppoly_run_static(ctypes.byref(eng.net), B, l0.data_ptr(), l0.data_ptr(), W.data_ptr(),
                                         None, None, lb.data_ptr(), lb.data_ptr(),
                                         torch.cuda.current_stream(dev).cuda_stream)
    assert st == _lib.CF_ERR_WORKSPACE
    assert b"whole batch" in _lib.lib.cf_last_error()


def test_static_scratch_rejects_oversized_network():
    from cfgpu import _lib
    from cfgpu.nets import Layer
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    # one region of this network needs far more than the fixed array (weight images alone)
    n_in, n_hidden = 4096, 4096
    layers = [Layer("linear", np.zeros((n_hidden, n_in), np.float32), np.zeros(n_hidden, np.float32),
                    in_shape=(n_in, 1, 1), out_shape=(n_hidden, 1, 1)),
              Layer("relu", in_shape=(n_hidden, 1, 1), out_shape=(n_hidden, 1, 1)),
              Layer("linear", np.zeros((10, n_hidden), np.float32), np.zeros(10, np.float32),
                    in_shape=(n_hidden, 1, 1), out_shape=(10, 1, 1))]
    from cfgpu.engine import DeepPolyEngine
    eng = DeepPolyEngine(layers, n_in, dev)
    assert eng.workspace_bytes(1) > _lib.CF_STATIC_SCRATCH_BYTES
    dummy = torch.zeros(16, device=dev)
    st = _lib.lib.cf_deeppoly_run_static(ctypes.byref(eng.net), 1, dummy.data_ptr(), dummy.data_ptr(),
                                         dummy.data_ptr(), None, None, dummy.data_ptr(), dummy.data_ptr(),
                                         torch.cuda.current_stream(dev).cuda_stream)
    assert st == _lib.CF_ERR_WORKSPACE
    assert b"fixed" in _lib.lib.cf_last_error()
