"""Point-sharded CPA transformations over several GPUs (one process per GPU).

Points are independent given theta, so each rank integrates a contiguous
slice of the points and the only exchange is one sum-allreduce of the
projected gradient dtheta (B^T is linear, so projecting local moments and then
summing equals projecting the summed moments).  theta and the basis are
replicated; outputs stay sharded.

    grid_r = shard_points(grid)                 # this rank's slice
    out_r = transform_grid_sharded(T, grid_r, theta)
    loss_r(out_r).backward()                    # theta.grad = sum over ranks
"""
import torch
import torch.distributed as dist

from .pytorch.transformer import transform


def shard_bounds(n_points, rank, world_size):
    """[lo, hi) of rank's contiguous share of n_points (sizes differ by <= 1)."""
    base, extra = divmod(int(n_points), int(world_size))
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def shard_points(points, rank=None, world_size=None):
    """This rank's slice of points [.., ndim, n_points] along the last axis."""
    if rank is None:
        rank = dist.get_rank() if dist.is_initialized() else 0
    if world_size is None:
        world_size = dist.get_world_size() if dist.is_initialized() else 1
    lo, hi = shard_bounds(points.shape[-1], rank, world_size)
    return points[..., lo:hi].contiguous()


def transform_grid_sharded(cpab, grid_shard, theta, group=None, compute_points_grad=True):
    """Cpab.transform_grid on this rank's points; backward sums dtheta over
    ``group`` (default: the world) with one allreduce per call."""
    if group is None and dist.is_initialized():
        group = dist.group.WORLD
    if group is not None and dist.get_world_size(group) == 1:
        group = None
    return transform(grid_shard, theta, cpab.params, compute_points_grad, group)


def allreduce_theta_grad(theta, group=None):
    """Register a hook summing theta's gradient over ``group`` once per
    backward (use with transform_grid_chain on sharded points: one
    allreduce of the whole [n_stages, d] gradient).  Returns the hook handle."""
    def hook(g):
        g = g.contiguous()
        dist.all_reduce(g, group=group)
        return g
    return theta.register_hook(hook)
