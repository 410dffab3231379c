"""Multi-GPU certification: input regions sharded over ranks (one process per GPU).

Regions are independent (every bound of a region depends only on that region's input
box), so a batch is split into contiguous shards, each rank certifies its shard with
its own DeepPolyEngine, and the only collective is one all-gather of the per-region
bounds at the end (NCCL on GPUs; gloo in the CPU tests of this host logic).
"""
import torch
import torch.distributed as dist


def shard_range(n_regions, rank, world):
    """Contiguous [lo, hi) of rank's regions; the first n % world ranks get one extra."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(int(n_regions), world)
    lo = rank * base + min(rank, extra)
    hi = lo + base + (1 if rank < extra else 0)
    return lo, hi


def gather_bounds(lb_local, ub_local, n_regions, rank, world, group=None):
    """All-gather per-region bounds [n_local, k] into [n_regions, k] on every rank.

    Shards may differ by one region; they are padded to the largest shard for the
    collective and the padding is dropped.  Every rank takes the same collective steps.
    """
    k = lb_local.shape[1]
    sizes = [shard_range(n_regions, r, world) for r in range(world)]
    cap = max(hi - lo for lo, hi in sizes)
    packed = torch.zeros(cap, 2 * k, dtype=lb_local.dtype, device=lb_local.device)
    n_local = lb_local.shape[0]
    packed[:n_local, :k] = lb_local
    packed[:n_local, k:] = ub_local
    out = [torch.empty_like(packed) for _ in range(world)]
    dist.all_gather(out, packed, group=group)
    lb = torch.cat([o[:hi - lo, :k] for o, (lo, hi) in zip(out, sizes)])
    ub = torch.cat([o[:hi - lo, k:] for o, (lo, hi) in zip(out, sizes)])
    return lb, ub


def certify_sharded(certify_fn, X, y, rank, world, group=None):
    """Run certify_fn(X_shard, y_shard) -> (lb, ub) on this rank's shard and gather.

    Returns (lb, ub, certified) for the whole batch on every rank; certified is the
    reference's verdict rule (all property lower bounds >= 0, constraintflow/cli.py:118-121).
    """
    n = int(X.shape[0])
    lo, hi = shard_range(n, rank, world)
    lb_l, ub_l = certify_fn(X[lo:hi], y[lo:hi])
    lb, ub = gather_bounds(lb_l, ub_l, n, rank, world, group)
    return lb, ub, (lb >= 0).all(dim=1)
