"""Point-sharded transform_grid over 2 GPUs with NCCL (one process per GPU,
launched with torch.distributed.run): the allreduced dtheta equals the
single-GPU gradient.  Skipped on machines with fewer than 2 GPUs."""
import json
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]

HERE = os.path.dirname(os.path.abspath(__file__))


def test_sharded_gradient_over_two_gpus(tmp_path):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = tmp_path / "result.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1",
           "--master-port=%d" % port, os.path.join(HERE, "multirank_worker.py"), str(out)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    res = json.loads(out.read_text())
    assert res["ok"] and res["world"] == 2, res
