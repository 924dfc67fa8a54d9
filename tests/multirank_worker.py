"""Worker for tests/test_gpu_multirank.py (one process per GPU, NCCL).

Each rank integrates its shard of the points; transform_grid_sharded sums
dtheta over ranks with one allreduce.  Rank 0 also computes the unsharded
gradient on its own GPU and checks that the two agree."""
import datetime
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [os.path.join(ROOT, "fg-cpab_b200"), ROOT, os.path.dirname(os.path.abspath(__file__))]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main(out_path):
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", local))
    from cpab import Cpab
    from cpab.distributed import shard_points, transform_grid_sharded
    C = Cpab([12, 12])
    g = torch.Generator().manual_seed(0)
    theta = torch.randn(4, C.params.d, generator=g).cuda()
    pts = torch.rand(2, 50001, generator=g).cuda()
    w = torch.randn(4, 2, 50001, generator=g).cuda()
    t = theta.clone().requires_grad_(True)
    out = transform_grid_sharded(C, shard_points(pts), t)
    (out * shard_points(w)).sum().backward()
    ok, err = True, 0.0
    if rank == 0:
        t_full = theta.clone().requires_grad_(True)
        (C.transform_grid(pts, t_full) * w).sum().backward()
        err = float((t.grad - t_full.grad).norm() / t_full.grad.norm())
        ok = err < 1e-5
    flag = torch.tensor([0.0 if ok else 1.0], device="cuda")
    dist.all_reduce(flag)
    dist.destroy_process_group()
    if rank == 0:
        with open(out_path, "w") as f:
            json.dump({"world": world, "rel_err": err, "ok": flag.item() == 0.0}, f)


if __name__ == "__main__":
    main(sys.argv[1])
