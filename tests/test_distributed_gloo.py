"""Multi-process host logic on CPU (gloo, world size 2): sharding the points
and summing the projected gradient over ranks equals the unsharded gradient;
the theta-gradient hook sums once per backward; a rank that leaves before the
collective makes the other rank's collective fail with an error (no hang).

The per-rank gradients come from the CPU oracle, which computes the same
quantities the GPU path computes on each rank (the GPU-side sharded path is
tested in tests/test_gpu_api.py)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

NC = [6, 6]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _inputs():
    from helpers import cpab, rand_points, rand_theta
    C = cpab(tuple(NC))
    pts = rand_points(2, 1001, 5)
    th = rand_theta(3, C.params.d, 6, 0.7)
    w = rand_points(2, 3 * 1001, 7, -1, 1).reshape(2, 3, 1001).transpose(1, 0, 2).copy()
    return C, pts, th, w


def _sharded_gradient(rank, world, port, q):
    try:
        _init(rank, world, port)
        from cpab.distributed import shard_points
        from oracle import oracle as O
        C, pts, th, w = _inputs()
        p_r = shard_points(torch.from_numpy(pts), rank, world).numpy()
        w_r = shard_points(torch.from_numpy(w), rank, world).numpy()
        _, As, _ = O.transform(NC, C.params.basis, p_r, th)
        dth, _ = O.gradient(NC, C.params.basis, p_r, As, w_r)
        t = torch.from_numpy(dth)
        dist.all_reduce(t)
        q.put((rank, t.numpy()))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))


def _hook_sum(rank, world, port, q):
    try:
        _init(rank, world, port)
        from cpab.distributed import allreduce_theta_grad
        theta = torch.zeros(4, 5, requires_grad=True)
        allreduce_theta_grad(theta)
        ((theta * (rank + 1)).sum() + (theta * 2.0).sum()).backward()
        q.put((rank, theta.grad.numpy().copy()))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))


def _node_hook_sum(rank, world, port, q):
    """The C++ transform node's sharded form: a hook on an identity view of
    theta sums only the gradient that flows through the view."""
    try:
        _init(rank, world, port)
        from cpab.pytorch.transformer import _allreduce_grad
        theta = torch.zeros(4, 5, requires_grad=True)
        view = theta.view_as(theta)
        view.register_hook(_allreduce_grad(None))
        ((view * (rank + 1)).sum() + (theta * 2.0).sum()).backward()
        q.put((rank, theta.grad.numpy().copy()))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))


def _one_rank_leaves(rank, world, port, q):
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        q.put((rank, "left"))
        q.close()
        q.join_thread()      # flush the message, then leave between steps,
        os._exit(0)          # before the collective
    try:
        dist.all_reduce(torch.ones(3))
        q.put((rank, "no error"))
    except Exception as e:
        q.put((rank, "error: " + type(e).__name__))


def _run(fn, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=90) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def test_sharded_gradient_equals_full_gradient():
    from oracle import oracle as O
    from helpers import rel_l2
    out = _run(_sharded_gradient)
    assert all(isinstance(v, np.ndarray) for v in out.values()), out
    C, pts, th, w = _inputs()
    _, As, _ = O.transform(NC, C.params.basis, pts, th)
    full, _ = O.gradient(NC, C.params.basis, pts, As, w)
    for r in (0, 1):
        assert rel_l2(out[r], full) < 1e-5
    np.testing.assert_array_equal(out[0], out[1])


def test_theta_gradient_hook_sums_over_ranks():
    out = _run(_hook_sum)
    for r in (0, 1):
        np.testing.assert_allclose(out[r], np.full((4, 5), (1 + 2) + 2 * 2.0))


def test_node_gradient_hook_sums_only_the_node_contribution():
    out = _run(_node_hook_sum)
    for r in (0, 1):
        # the view's gradient (rank + 1) is summed over ranks, the rest is not
        np.testing.assert_allclose(out[r], np.full((4, 5), (1 + 2) + 2.0))


def test_rank_leaving_turns_into_an_error_not_a_hang():
    out = _run(_one_rank_leaves)
    assert out[1] == "left"
    assert out[0].startswith("error"), out[0]
