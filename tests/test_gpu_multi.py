"""Two ranks on two GPUs over NCCL: the sharded certification equals the single-GPU run.

Each rank (one process per GPU) certifies its contiguous shard of the regions with its own
DeepPolyEngine; cfgpu.dist all-gathers the per-region bounds over NCCL.  Regions are
independent, so every rank's gathered bounds and verdicts must equal, bit for bit, one
GPU's run over the whole batch.  Skipped when fewer than two GPUs are visible.
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

N_REGIONS = 37          # uneven shards: 19 + 18
WID = 2                 # the 784-(200x9)-10 MLP


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bounds_single():
    from cfgpu import nets
    from cfgpu.engine import DeepPolyEngine
    wl = nets.workload(WID)
    X = nets.centres(wl, N_REGIONS)
    y = nets.labels(wl, X)
    dev = torch.device("cuda:0")
    eng = DeepPolyEngine(wl.layers, wl.input_size, dev)
    lb, ub = eng.certify(X.to(dev), y.to(dev), wl.eps, wl.dataset)
    return lb.cpu().numpy(), ub.cpu().numpy()


def _worker(rank, world, port, q):
    import datetime
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    for p in (os.path.dirname(here), os.path.join(os.path.dirname(here), "constraintflow-gpu_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    from cfgpu import dist as cdist
    from cfgpu import nets
    from cfgpu.engine import DeepPolyEngine
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        wl = nets.workload(WID)
        X = nets.centres(wl, N_REGIONS)
        y = nets.labels(wl, X)
        eng = DeepPolyEngine(wl.layers, wl.input_size, dev)

        def certify(Xs, ys):
            return eng.certify(Xs.to(dev), ys.to(dev), wl.eps, wl.dataset)

        lb, ub, cert = cdist.certify_sharded(certify, X, y, rank, world)
        torch.cuda.synchronize()
        q.put((rank, lb.cpu().numpy(), ub.cpu().numpy(), cert.cpu().numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_sharded_bounds_equal_single_gpu():
    import torch.multiprocessing as mp
    lb1, ub1 = _bounds_single()
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    os.environ.update(env)
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, lb, ub, cert in res:
        assert lb.shape == (N_REGIONS, 9)
        assert np.array_equal(lb, lb1) and np.array_equal(ub, ub1), f"rank {rank}: gathered bounds differ"
        assert np.array_equal(cert, (lb1 >= 0).all(axis=1))
