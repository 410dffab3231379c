"""Host logic of the multi-GPU path on CPU: world_size-2 gloo ranks shard the regions,
certify their shard (here with the CPU oracle standing in for the GPU engine) and
all-gather; the result must equal the single-process run, region for region."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cfgpu import dist as cdist
from cfgpu import nets


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_certify(wl):
    from oracle import deeppoly_oracle as O

    def fn(X, y):
        l0, u0 = nets.input_box(X, wl.eps, wl.dataset)
        W = nets.spec_weight(y).numpy()
        _, lb, ub = O.deeppoly(wl.layers, l0.numpy(), u0.numpy(), W)
        return torch.from_numpy(lb), torch.from_numpy(ub)
    return fn


def _worker(rank, world, port, n, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        wl = nets.workload(1)
        X = nets.centres(wl, n)
        y = nets.labels(wl, X)
        lb, ub, cert = cdist.certify_sharded(_oracle_certify(wl), X, y, rank, world)
        q.put((rank, lb.numpy(), ub.numpy(), cert.numpy()))
    finally:
        dist.destroy_process_group()


def test_shard_range_covers_exactly():
    for n in (0, 1, 5, 64, 1023):
        for world in (1, 2, 3, 8):
            parts = [cdist.shard_range(n, r, world) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(parts[i][1] == parts[i + 1][0] for i in range(world - 1))
            sizes = [hi - lo for lo, hi in parts]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        cdist.shard_range(4, 2, 2)


def test_sharded_certification_matches_single_process():
    n, world = 7, 2   # uneven shards (4 + 3)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    wl = nets.workload(1)
    X = nets.centres(wl, n)
    y = nets.labels(wl, X)
    lb1, ub1 = _oracle_certify(wl)(X, y)
    for rank, lb, ub, cert in res:
        assert lb.shape == (n, 9)
        scale = float(np.abs(lb1.numpy()).max())
        np.testing.assert_allclose(lb, lb1.numpy(), rtol=1e-5, atol=1e-4 * scale)
        np.testing.assert_allclose(ub, ub1.numpy(), rtol=1e-5, atol=1e-4 * scale)
        np.testing.assert_array_equal(cert, (lb1.numpy() >= 0).all(axis=1))
