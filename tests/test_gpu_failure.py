"""Failure detection on the GPU without a fault: a bounded device wait that runs out.

The chain kernel's waits on its mbarriers are bounded.  With a short poll limit
(CF_WAIT_POLLS) and one arrival withheld (CF_FAULT=chain_withhold_acc: the MMA issuer does
not signal that the first substitution's accumulator is ready), the transform warps' wait
gives up, the error word records the site, every role of the kernel unwinds (in-flight bulk
copies and MMAs are awaited before shared memory and tensor memory are released), later
launches of the pass exit early, and cf_deeppoly_check reports CF_ERR_TIMEOUT.  The context
stays usable: the next pass, without the fault, gives the usual bounds.
"""
import re

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

# k_chain's bounded waits (constraintflow-gpu_b200/csrc/cf_chain.cu): weight producer 11, 13;
# MMA issuer 21, 22; transform / drain warps 31-35.  With the accumulator commit withheld,
# whichever of them has waited longest gives up first -- all are downstream of it.
K_CHAIN_SITES = {11, 13, 21, 22, 31, 32, 33, 34, 35}


def _inputs(wl, B, dev):
    from cfgpu import nets
    X = nets.centres(wl, B)
    y = nets.labels(wl, X)
    l0, u0 = nets.input_box(X, wl.eps, wl.dataset)
    return l0.to(dev), u0.to(dev), nets.spec_weight(y).to(dev)


def test_withheld_arrival_times_out_and_context_recovers(monkeypatch):
    from cfgpu import _lib, nets
    from cfgpu.engine import DeepPolyEngine
    dev = torch.device("cuda:0")
    wl = nets.workload(0)          # 784-50-50-50-10: every layer bound by the chain kernel
    eng = DeepPolyEngine(wl.layers, wl.input_size, dev)
    l0, u0, W = _inputs(wl, 2, dev)
    lb_ok, ub_ok = eng.run(l0, u0, W, check_device=True)
    torch.cuda.synchronize()
    monkeypatch.setenv("CF_WAIT_POLLS", "65536")
    monkeypatch.setenv("CF_FAULT", "chain_withhold_acc")
    eng.run(l0, u0, W)
    st = _lib.lib.cf_deeppoly_check(eng._ws.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    msg = _lib.lib.cf_last_error()
    assert st == _lib.CF_ERR_TIMEOUT, (st, msg)
    m = re.search(rb"gave up \(site (\d+)\)", msg)
    assert m is not None, msg
    assert int(m.group(1)) in K_CHAIN_SITES, msg
    monkeypatch.delenv("CF_FAULT")
    monkeypatch.delenv("CF_WAIT_POLLS")
    lb, ub = eng.run(l0, u0, W, check_device=True)
    torch.cuda.synchronize()
    assert np.array_equal(lb.cpu().numpy(), lb_ok.cpu().numpy())
    assert np.array_equal(ub.cpu().numpy(), ub_ok.cpu().numpy())
