#!/usr/bin/env python
"""Benchmark of the FG-CPAB hot path on B200: fwd+grad warped points/s.

Workload: Cpab([20, 20], zero_boundary=True),
batch 16, theta ~ N(0, 1), 125,000 points ~ U[0,1]^2 per GPU, nstepsolver 50;
one step = transform_grid forward + MSE(x_t, x) + backward to theta, through
the public API.  With N GPUs (torchrun, one process per GPU) every rank
integrates its own 125,000 points (weak scaling) and the gradient is summed
with one NCCL allreduce of dtheta per step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line on rank 0.  `value` is the device-resident throughput
(CUDA events around every step, L2 flushed between steps, max over ranks);
`e2e` is the same step with pinned-host inputs copied in and the loss and
gradient copied out inside the timed region.  `--impl reference` times the
CPU restatement of the reference kernels (oracle/, all host threads) on a
bounded sample of the same workload.
"""
import argparse
import datetime
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (os.path.join(ROOT, "fg-cpab_b200"), ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402
import torch.nn.functional as F  # noqa: E402

TESS = [20, 20]
BATCH = 16
N_POINTS = 125_000
NSTEP = 50
METRIC = "fwd+grad warped points/sec"
UNIT = "points/s"
L2_FLUSH_BYTES = 256 << 20


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


PROFILE = os.path.join(ROOT, "profiles", "k_backward_2d_20x20_b16_125k.md")


def profiled(key):
    """A number recorded in the committed ncu summary of k_backward on this
    workload (profiles/k_backward_2d_20x20_b16_125k.md), or None."""
    try:
        for line in open(PROFILE):
            if line.startswith(key + ":"):
                return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


def profiled_str(key):
    """A text field of the committed ncu summary, or None."""
    try:
        for line in open(PROFILE):
            if line.startswith(key + ":"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


ORDER_NOTE = "points sorted by cell inside every timed step (no order kept across steps)"
MESH_ORDER_NOTE = ("meshgrid points generated in the kernels and visited in a cell order "
                   "that depends only on the tessellation and output size, computed once")


def config(world):
    return {
        "workload": "2D Cpab([20,20], zero_boundary=True): batch 16, 125,000 U[0,1]^2 points per "
                    "GPU, theta~N(0,1), nstepsolver 50; transform_grid + MSE(x_t, x) + backward "
                    "to theta",
        "tess": TESS, "batch": BATCH, "points_per_gpu": N_POINTS, "nstepsolver": NSTEP,
        "global_batch": BATCH * N_POINTS * world,
        "parallelism": "points sharded over %d GPU(s), dtheta allreduce" % world,
        "l2": "flushed between timed steps (%d MiB write)" % (L2_FLUSH_BYTES >> 20),
        "point_order": ORDER_NOTE,
    }


# NVML sampling period.
CLOCK_INTERVAL_S = 0.002

_SAMPLER = r"""
import json, os, select, sys
import pynvml
pynvml.nvmlInit()
h = pynvml.nvmlDeviceGetHandleByIndex(int(sys.argv[1]))
out = {"max": pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM), "s": []}
def sample():
    try:
        out["s"].append((pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
                         int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(h))))
    except Exception:
        pass
print("idle", flush=True)
# commands on stdin: "g" start/resume sampling, "p" pause, "s" stop and report
cmd = os.read(0, 1)
while cmd == b"g":
    sample()
    print("ready", flush=True)
    while not select.select([0], [], [], float(sys.argv[2]))[0]:
        sample()
    sample()
    cmd = os.read(0, 1)
    if cmd == b"p":
        print("paused", flush=True)
        cmd = os.read(0, 1)
print(json.dumps(out), flush=True)
"""


class Clocks:
    """SM clock and throttle-reason samples (NVML, every CLOCK_INTERVAL_S, plus
    one at each end of every sampled stretch) taken while the timed regions
    run: the device-resident steps, the end-to-end steps and the graph
    replays, paused in between (a default run's regions last ~12 ms each).
    The sampler is a child process, so that it takes no time from this
    process's Python thread (the 1D step is bound by host time), and it is
    started before the warm-up steps and only told when to sample: a process
    spawned right before the timed steps measurably slowed their launches
    (~5% of a 2D step)."""
    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4}

    def __init__(self, index):
        import subprocess
        self.proc = None
        try:
            self.proc = subprocess.Popen([sys.executable, "-c", _SAMPLER, str(index),
                                          str(CLOCK_INTERVAL_S)],
                                         stdin=subprocess.PIPE, stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            if self.proc.stdout.readline().strip() != "idle":
                raise RuntimeError("clock sampler did not start")
        except Exception:
            self._kill()

    def _kill(self):
        if self.proc is not None:
            self.proc.kill()
            self.proc.wait()
        self.proc = None

    def _send(self, cmd, reply):
        if self.proc is None:
            return
        try:
            self.proc.stdin.write(cmd)
            self.proc.stdin.flush()
            if self.proc.stdout.readline().strip() != reply:
                raise RuntimeError("clock sampler did not answer %r" % cmd)
        except Exception:
            self._kill()

    def start(self):
        """Start (or resume) sampling."""
        self._send("g", "ready")

    def pause(self):
        self._send("p", "paused")

    def stop(self):
        if self.proc is None:
            return None
        try:
            out, _ = self.proc.communicate("s", timeout=30)
            d = json.loads(out.strip().splitlines()[-1])
        except Exception:
            self._kill()
            return None
        samples = d["s"]
        if not samples:
            return None
        mask = 0
        for _, r in samples:
            mask |= int(r)
        return {"sm_mhz": statistics.median(m for m, _ in samples),
                "sm_max_mhz": d["max"],
                "reasons": sorted(n for n, bit in self.REASONS.items() if mask & bit),
                "samples": len(samples)}


def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return rank, world, local


def max_over_ranks(x, world):
    t = torch.tensor([float(x)], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# CPU arm: the oracle restatement of the reference kernels.
# ---------------------------------------------------------------------------

def cpu_step(O, basis, pts, theta):
    """One fwd+grad of the reference composition on CPU; returns dtheta."""
    x, As, _ = O.transform(TESS, basis, pts, theta, NSTEP)
    gout = (2.0 / x.size) * (x - pts[None])
    mom, _ = O.adjoint(TESS, pts, As, gout.astype(np.float32), NSTEP, False, want_points=False)
    return O.project(basis, mom)


def cpu_sample_points(O, basis, theta, target_s):
    """Points per sample so that one sample takes about target_s seconds."""
    probe = 2048
    pts = np.random.default_rng(1).random((2, probe), dtype=np.float32)
    t0 = time.perf_counter()
    cpu_step(O, basis, pts, theta)
    dt = time.perf_counter() - t0
    n = int(probe * target_s / max(dt, 1e-6))
    return max(1024, min(N_POINTS, n))


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_baseline(basis, theta_np, target_s=10.0):
    """The oracle port on all host threads: repeated fwd+grad steps on (a
    sample of) the workload until about target_s seconds have passed."""
    from oracle import oracle as O
    O.set_num_threads(host_threads())   # torchrun sets OMP_NUM_THREADS=1
    n = cpu_sample_points(O, basis, theta_np, target_s)
    pts = np.random.default_rng(1).random((2, n), dtype=np.float32)
    reps, t0 = 0, time.perf_counter()
    while True:
        cpu_step(O, basis, pts, theta_np)
        reps += 1
        dt = time.perf_counter() - t0
        if dt >= target_s or reps >= 100:
            break
    return {"value": reps * n * BATCH / dt, "unit": UNIT, "cores": O.num_threads(), "kind": "port",
            "sample": "%d of the %d points x batch %d, %d fwd+grad steps (A-build, expm, "
                      "integrate, adjoint, projection) in %.1f s" % (n, N_POINTS, BATCH, reps, dt)}


def run_reference(args, rank, world):
    if rank != 0:
        return
    from cpab import Cpab
    from oracle import oracle as O
    O.set_num_threads(host_threads())   # torchrun sets OMP_NUM_THREADS=1
    C = Cpab(TESS, zero_boundary=True)
    theta = torch.randn(BATCH, C.params.d, generator=torch.Generator().manual_seed(0)).numpy()
    n = cpu_sample_points(O, C.params.basis, theta, 3.0)
    pts = np.random.default_rng(1).random((2, n), dtype=np.float32)
    for _ in range(args.warmup):
        cpu_step(O, C.params.basis, pts, theta)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_step(O, C.params.basis, pts, theta)
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    value = n * BATCH / dt
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config(world), "impl": "reference",
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": O.num_threads(), "kind": "port",
                         "sample": "%d of %d points x batch %d per step" % (n, N_POINTS, BATCH)},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


# ---------------------------------------------------------------------------
# GPU arm.
# ---------------------------------------------------------------------------

class Workload:
    """One benchmark configuration: inputs, one fwd+grad step, work counted."""

    def __init__(self, name, desc, tess, zero_boundary, batch, stages, scaling, parallelism):
        self.name, self.desc = name, desc
        self.tess, self.zero_boundary = tess, zero_boundary
        self.batch, self.stages = batch, stages
        self.scaling, self.parallelism = scaling, parallelism


def make_workload(name, rank, world, dev, unfused=False):
    """Build (workload, host inputs, step function, pairs per step on this rank)."""
    from cpab import Cpab
    from cpab.distributed import allreduce_theta_grad, shard_points, transform_grid_sharded
    gen = lambda seed: torch.Generator().manual_seed(seed)  # noqa: E731
    group = dist.group.WORLD if world > 1 else None

    if name in ("2d", "2d12", "2d30", "1d"):
        tess = {"2d": [20, 20], "2d12": [12, 12], "2d30": [30, 30], "1d": [50]}[name]
        nd = len(tess)
        B, nP = (8, 100_000) if nd == 1 else (BATCH, N_POINTS)
        w = Workload(name, "%dD Cpab(%s, zero_boundary=True): batch %d, %d U[0,1]^%d points per GPU, "
                     "theta~N(0,1), nstepsolver 50; transform_grid + %s + backward to theta"
                     % (nd, tess, B, nP, nd, "sum((x_t-x)^2)" if nd == 1 else "MSE(x_t, x)"),
                     tess, True, B, 1, "weak", "points sharded over %d GPU(s), dtheta allreduce" % world)
        C = Cpab(tess, zero_boundary=True)
        host = {"theta": torch.randn(B, C.params.d, generator=gen(0)),
                "points": torch.rand(nd, nP, generator=gen(1 + rank))}

        def step(x):
            t = x["theta"].requires_grad_(True)
            pts = x["points"]
            out = C.transform_grid(pts, t) if group is None else transform_grid_sharded(C, pts, t, group)
            ref = pts.expand_as(out)
            loss = F.mse_loss(out, ref, reduction="sum" if nd == 1 else "mean")
            loss.backward()
            return loss, t.grad
        return w, C, host, step, B * nP

    if name in ("dense2d", "3d"):
        if name == "dense2d":
            tess, zb, B, shape, scale = [30, 30], False, 32, [3, 512, 512], 0.5
        else:
            tess, zb, B, shape, scale = [10, 10, 10], True, 4, [1, 128, 128, 128], 1.0
        nd = len(tess)
        w = Workload(name, "%dD Cpab(%s, zero_boundary=%s): transform_data of %d x %s, theta~N(0,%g^2), "
                     "MSE to a second %s, backward to theta; each GPU its own batch"
                     % (nd, tess, zb, B, shape, scale, "image" if nd == 2 else "volume"),
                     tess, zb, B, 1, "weak", "batch-parallel over %d GPU(s), no collective" % world)
        C = Cpab(tess, zero_boundary=zb)
        w.fused_data = (shape[0], int(np.prod(shape[1:])))  # channels, input plane
        g = gen(2 + 10 * rank)
        if nd == 2:
            data = torch.rand(B, *shape, generator=g)
            target = torch.rand(B, *shape, generator=g)
        else:
            data = torch.stack([blobs(shape[1:], g) for _ in range(B)])[:, None]
            target = torch.stack([blobs(shape[1:], g) for _ in range(B)])[:, None]
        host = {"theta": torch.randn(B, C.params.d, generator=gen(0)) * scale, "data": data,
                "target": target}
        outsize = shape[1:]

        if unfused:
            # the reference's composition (cpab/cpab.py:306-308) through the
            # same library: meshgrid, transform_grid, interpolate
            del w.fused_data
            w.desc += " (unfused: uniform_meshgrid + transform_grid + interpolate)"
            # a fixed meshgrid keeps its sort order, as the fused path keeps
            # its meshgrid's processing order
            w.keep_order = True
            grid = C.uniform_meshgrid(outsize, device=dev)

            def step(x):
                t = x["theta"].requires_grad_(True)
                out = C.interpolate(x["data"], C.transform_grid(grid, t), outsize)
                loss = F.mse_loss(out, x["target"])
                loss.backward()
                return loss, t.grad
            return w, C, host, step, B * int(np.prod(outsize))

        def step(x):
            t = x["theta"].requires_grad_(True)
            out = C.transform_data(x["data"], t, outsize)
            loss = F.mse_loss(out, x["target"])
            loss.backward()
            return loss, t.grad
        return w, C, host, step, B * int(np.prod(outsize))

    if name in ("stn2d", "stn3d"):
        from cpab.pytorch.warp import CpabWarp, warp_composed
        if name == "stn2d":   # the layer of the reference's stn/demos/demo_2d.py
            tess, pad, B, shape, scale = (3, 3), "border", 32, [3, 128, 128], 0.7
        else:                 # and of stn/demos/demo_3d.py
            tess, pad, B, shape, scale = (4, 4, 4), "zeros", 32, [1, 32, 32, 32], 1.0
        K = 2
        nd = len(tess)
        layer = CpabWarp(tess, padding_mode=pad)
        w = Workload(name, "%dD CpabWarp(%s, padding_mode=%r): %d images %s, the composition "
                     "T_1 o T_2 of %d transformations theta~N(0,%g^2) (stn/stn.py:58-86), MSE to "
                     "a second batch, backward to both thetas; each GPU its own batch"
                     % (nd, tess, pad, B, shape, K, scale),
                     list(tess), True, B, K, "weak", "batch-parallel over %d GPU(s), no collective"
                     % world)
        C = layer.cpab
        w.warp_data = (shape[0], int(np.prod(shape[1:])))  # channels, image plane
        g = gen(2 + 10 * rank)
        host = {"theta": torch.randn(K, B, C.params.d, generator=gen(0)) * scale,
                "data": torch.rand(B, *shape, generator=g),
                "target": torch.rand(B, *shape, generator=g)}
        if unfused:
            del w.warp_data
            w.desc += " (unfused: the reference layer's CPAB_transformer calls + F.grid_sample)"

        def step(x):
            t = x["theta"].requires_grad_(True)
            out = (warp_composed(x["data"], list(t), C.params, pad) if unfused
                   else layer(x["data"], t))
            loss = F.mse_loss(out, x["target"])
            loss.backward()
            return loss, t.grad
        return w, C, host, step, B * int(np.prod(shape[1:])) * K

    if name == "chain3d":
        tess, K, grid_n = [16, 16, 16], 4, [160, 192, 160]
        w = Workload(name, "3D Cpab([16,16,16], zero_boundary=True): transform_grid_chain, 4 stages, "
                     "scale_by_dt, theta_chain~N(0,0.5^2), 160x192x160 meshgrid (4,915,200 points) "
                     "sharded over the GPUs, sum((x_t-x)^2) + backward to theta_chain",
                     tess, True, 1, K, "strong",
                     "meshgrid sharded over %d GPU(s), one dtheta allreduce" % world)
        C = Cpab(tess, zero_boundary=True)
        grid = shard_points(C.uniform_meshgrid(grid_n, device="cpu"), rank, world)
        host = {"theta": torch.randn(K, C.params.d, generator=gen(0)) * 0.5, "points": grid}

        def step(x):
            t = x["theta"].requires_grad_(True)
            if group is not None:
                allreduce_theta_grad(t, group)
            out = C.transform_grid_chain(x["points"], t, scale_by_dt=True)
            loss = F.mse_loss(out, x["points"].expand_as(out), reduction="sum")
            loss.backward()
            return loss, t.grad
        return w, C, host, step, grid.shape[1] * K
    raise ValueError("unknown config " + name)


def blobs(shape, g, n=20):
    """Sum of n Gaussian blobs (sigma ~ U[4,16] voxels, centres ~ U over the
    volume, unit amplitude) on a grid of the given shape."""
    axes = [torch.arange(s, dtype=torch.float32) for s in shape]
    zz, yy, xx = torch.meshgrid(*axes, indexing="ij")
    vol = torch.zeros(shape)
    for _ in range(n):
        c = [torch.rand(1, generator=g).item() * s for s in shape]
        sig = 4 + 12 * torch.rand(1, generator=g).item()
        vol += torch.exp(-((zz - c[0]) ** 2 + (yy - c[1]) ** 2 + (xx - c[2]) ** 2) / (2 * sig * sig))
    return vol


def graph_replay(step, resident, C, flush, steps, warmup, clocks=None):
    """ms per replay of the device-resident step captured in one CUDA graph."""
    from cpab.pytorch.transformer import clear_order_cache

    theta = resident["theta"].detach().clone().requires_grad_(True)
    static = dict(resident, theta=theta)

    def call():
        clear_order_cache(C.params)   # the sort is recorded into the graph
        theta.grad = None
        return step(static)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            call()
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        call()
    for _ in range(max(warmup, 1)):
        g.replay()
    torch.cuda.synchronize()
    if clocks is not None:
        clocks.start()
    ms = timed_steps(g.replay, steps, flush, 1)
    if clocks is not None:
        clocks.pause()
    del g
    return ms


# Native calls of the library timed per phase (CUDA events on the stream each
# is enqueued on) and the kernels each launches.
KERNELS_PER_CALL = {"build_A": 1, "build_A_tt": 1, "order_points": 3, "project": 1,
                    "project_tt": 1, "interpolate": 1,
                    "interpolate_backward": 1, "expm": 1, "forward": 1, "backward": 1,
                    "transform_data": 1, "transform_data_backward": 1, "forward_chain": 1,
                    "backward_chain": 1, "warp": 1, "warp_backward": 1}


class PhaseTimer:
    """Wraps the library's native calls (and torch.distributed.all_reduce)
    with CUDA events while `rec` names a dict to record into; also counts the
    kernels of this library that the recorded calls launch."""

    def __init__(self, native):
        self.rec = None
        self.only = None       # names to time (None: all); the others are only counted
        self.capture = False
        self.launches = 0
        for name in KERNELS_PER_CALL:
            setattr(native, name, self._wrap(name, getattr(native, name), True))
        dist.all_reduce = self._wrap("allreduce", dist.all_reduce, False)

    def _wrap(self, name, fn, ours):
        def call(*a, **k):
            rec = self.rec
            if rec is None or self.capture:
                return fn(*a, **k)
            if ours:
                self.launches += KERNELS_PER_CALL[name]
            if self.only is not None and name not in self.only:
                return fn(*a, **k)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            r = fn(*a, **k)
            e.record()
            rec.setdefault(name, []).append((s, e))
            return r
        return call


def phase_ms(rec, steps, world):
    """Mean ms per step of every recorded phase, max over ranks."""
    names = sorted(rec)
    if world > 1:  # every rank reports the same phases, in the same order
        names = sorted(set(names) | {"allreduce"})
    return {n: max_over_ranks(sum(s.elapsed_time(e) for s, e in rec.get(n, [])) / steps, world)
            for n in names}


E2E_NOTE = ("every step copies its inputs from pinned host memory and its loss and dtheta "
            "back; the faster of two loops: serial (copy, compute, read-back in sequence, "
            "CUDA events per step, the 256 MiB L2 flush between steps untimed) and overlapped "
            "(step j+1's inputs go in on a second stream, after a timed 256 MiB L2 flush on "
            "that stream, into the other of two input buffers while step j computes, and "
            "step j's loss and dtheta come back on that stream; CUDA events around the whole "
            "loop)")


def timed_e2e_overlapped(step, pinned, template, steps, warmup, flush, world, loss_pin,
                         grad_pin):
    """ms per step of the end-to-end loop with each step's input copy
    overlapped with the previous step's compute (double-buffered inputs, copies
    on a second stream), barrier + synchronize on both sides, max over ranks."""
    main = torch.cuda.current_stream()
    side = torch.cuda.Stream()
    bufs = [{k: torch.empty_like(v) for k, v in template.items()} for _ in range(2)]
    ready = [torch.cuda.Event(), torch.cuda.Event()]
    done = [torch.cuda.Event(), torch.cuda.Event()]

    def load(b):
        side.wait_event(done[b])  # the step that last read buffer b has finished
        with torch.cuda.stream(side):
            flush.zero_()
            for k in pinned:
                bufs[b][k].copy_(pinned[k], non_blocking=True)
        ready[b].record(side)

    def run(n):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(main)
        side.wait_event(start)
        load(0)
        for j in range(n):
            b = j % 2
            if j + 1 < n:
                load(1 - b)
            main.wait_event(ready[b])
            loss, grad = step(dict(bufs[b], theta=bufs[b]["theta"].detach()))
            done[b].record(main)
            # the read-back on the second stream too, so that the next step's
            # launches do not wait for it
            side.wait_event(done[b])
            loss, grad = loss.detach(), grad.detach()
            loss.record_stream(side)
            grad.record_stream(side)
            with torch.cuda.stream(side):
                loss_pin.copy_(loss.reshape(1), non_blocking=True)
                grad_pin.copy_(grad, non_blocking=True)
        main.wait_stream(side)
        end.record(main)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        return start.elapsed_time(end) / n

    run(max(warmup, 1))
    return max_over_ranks(run(steps), world)


def timed_steps(fn, steps, flush, world):
    """ms per step of fn() over `steps` calls: CUDA events per step, L2
    flushed before each (untimed), barrier + synchronize on both sides, max
    over ranks."""
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev = []
    for _ in range(steps):
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        ev.append((s, e))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    return max_over_ranks(sum(s.elapsed_time(e) for s, e in ev), world) / steps


def source_sha():
    """Hash of the sources of the integration kernels (k_forward, k_backward):
    profiles/ summaries record it, so a figure profiled from other sources is
    not reported as this build's."""
    import hashlib
    h = hashlib.sha256()
    for f in ("cpab_device.cuh", "integrate_body.cuh", "integrate.cu", "launch.h"):
        with open(os.path.join(ROOT, "fg-cpab_b200", "csrc", f), "rb") as fh:
            h.update(fh.read())
    return h.hexdigest()[:16]


def profile_record():
    """(traffic bytes, warp instructions, provenance) of the committed ncu
    summary of k_backward on the bench workload; the figures are None when
    the summary was made from other kernel sources than these."""
    sha = profiled_str("source_sha")
    prov = {"file": os.path.relpath(PROFILE, ROOT), "source_sha": sha,
            "commit": profiled_str("commit"), "current_source_sha": source_sha()}
    if sha is None or sha != prov["current_source_sha"]:
        prov["stale"] = True
        return None, None, prov
    return profiled("traffic_bytes_per_launch"), profiled("warp_instructions_per_launch"), prov


def breakdown(fn, steps, flush, world, timer):
    """(per-phase ms, kernels of this library per step) of fn: every native
    call and allreduce bracketed by CUDA events, in a pass of its own so that
    the events' host time does not enter the step times reported beside it.
    The pass takes the Python autograd node, whose C ABI calls the timer
    wraps; the C++ node (the default path) issues the same calls."""
    from cpab import _ext
    rec = {}
    timer.rec, timer.only = rec, None
    n0 = timer.launches
    with _ext.python_path():
        timed_steps(fn, steps, flush, world)
    timer.rec = None
    per_step = (timer.launches - n0) / steps
    timer.launches = n0
    return phase_ms(rec, steps, world), per_step


def strong_scaling(C, steps, warmup, flush, rank, world, timer):
    """The fixed 2D problem (125,000 points x batch 16) split over the ranks
    two ways: points sharded with one dtheta allreduce per step, and the batch
    sharded (16 / world transformations per rank, no collective).  Returns
    one record per way with the per-phase breakdown of rank max times."""
    from cpab.distributed import shard_points, transform_grid_sharded
    from cpab.pytorch.transformer import clear_order_cache
    dev = torch.device("cuda", torch.cuda.current_device())
    group = dist.group.WORLD
    theta = torch.randn(BATCH, C.params.d, generator=torch.Generator().manual_seed(0)).to(dev)
    pts = torch.rand(2, N_POINTS, generator=torch.Generator().manual_seed(1))
    mine = shard_points(pts, rank, world).to(dev)
    full = pts.to(dev)
    n_total = BATCH * N_POINTS * 2
    out = {}

    def points_step():
        clear_order_cache(C.params)
        t = theta.detach().requires_grad_(True)
        o = transform_grid_sharded(C, mine, t, group)
        # the global mean over all ranks' points, as one process would compute it
        (((o - mine) ** 2).sum() / n_total).backward()

    lo, hi = BATCH * rank // world, BATCH * (rank + 1) // world

    def batch_step():
        clear_order_cache(C.params)
        t = theta[lo:hi].detach().requires_grad_(True)
        o = C.transform_grid(full, t)
        (((o - full) ** 2).sum() / n_total).backward()

    for name, fn in (("points_sharded", points_step), ("batch_sharded", batch_step)):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        ms = timed_steps(fn, steps, flush, world)
        out[name] = {"value": BATCH * N_POINTS / (ms * 1e-3), "unit": UNIT, "ms_per_step": ms,
                     "phase_ms": breakdown(fn, steps, flush, world, timer)[0]}
        gms = graph_steps(fn, steps, flush, world, timer)
        if gms is not None:
            out[name]["graph_replay"] = {
                "value": BATCH * N_POINTS / (gms * 1e-3), "unit": UNIT, "ms_per_step": gms,
                "note": "each rank's step (sort, forward, loss, backward, projection and, "
                        "points sharded, the dtheta allreduce) captured once in a CUDA graph "
                        "and replayed: no host issue time, no rank drift from it"}
    out["points_sharded"]["how"] = ("the 125,000 points split over the ranks, all 16 "
                                    "transformations on every rank, one dtheta allreduce")
    out["batch_sharded"]["how"] = ("all 125,000 points on every rank, %d of the 16 "
                                   "transformations per rank, no collective"
                                   % (BATCH // world))
    out["problem"] = "fixed: 125,000 points x batch 16 (2,000,000 pairs) whatever the GPU count"
    return out


def graph_steps(fn, steps, flush, world, timer):
    """ms per replay of fn() captured in one CUDA graph on every rank (its NCCL
    allreduce included), max over ranks; None on every rank when any rank
    could not capture it (agreed on before any replay, so that no rank
    replays a collective the others never launch)."""
    g, ok = None, 1.0
    timer.capture = True
    try:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
    except Exception as e:  # noqa: BLE001 -- reported, and agreed on below
        print("graph capture failed: %r" % (e,), file=sys.stderr)
        g, ok = None, 0.0
    finally:
        timer.capture = False
    torch.cuda.synchronize()
    flag = torch.tensor([ok], device="cuda")
    if world > 1:
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    if flag.item() < 1.0:
        return None
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    ms = timed_steps(g.replay, steps, flush, world)
    del g  # before the process group goes: a graph holding NCCL calls must not outlive it
    return ms


REF_KERNELS = os.path.join(ROOT, "oracle", "_ref", "libcpab_ref.so")


def ref_gpu_kernels(C, host, steps, warmup, flush):
    """Baseline leg: the reference's own CUDA kernels (cpab/core/cpab_ops_2d.cu,
    compiled unmodified for sm_100a into oracle/_ref) and torch.sparse.mm for
    the projection, as the reference's transformer.py composes them, timed
    with CUDA events on the bench inputs (A from this library's build_A).
    Not part of the measured product; None when that build is absent."""
    if not os.path.exists(REF_KERNELS):
        return None
    import ctypes
    L = ctypes.CDLL(REF_KERNELS)
    i, f, p = ctypes.c_int, ctypes.c_float, ctypes.c_void_p
    L.ref_expm.argtypes = [i, p, i, f, p]
    L.ref_forward.argtypes = [i, i, i, i, p, i, i, p, p, i, i, i, p]
    L.ref_backward.argtypes = [i, i, i, i, i, p, i, i, p, i, p, i, i, p, p]
    from cpab import _native
    from cpab.pytorch.transformer import device_basis
    dev = torch.device("cuda", torch.cuda.current_device())
    nx, ny = TESS
    theta = host["theta"].to(dev)
    pts = host["points"].to(dev)
    nP = pts.shape[1]
    nC = C.params.nC
    basis = device_basis(C.params, dev)
    As, _ = _native.build_A(2, nC, basis, theta, 1.0 / NSTEP)
    g = torch.randn(BATCH, 2, nP, generator=torch.Generator().manual_seed(3)).to(dev)
    Bt = C._get_basis_sparse_gpu(device=dev).transpose(0, 1).coalesce()
    trels = torch.zeros_like(As)
    out = torch.zeros((BATCH, 2, nP), device=dev)
    mom = torch.zeros((BATCH, nC, 6), device=dev)
    gp = torch.zeros((BATCH, 2, nP), device=dev)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    torch.cuda.synchronize()
    # the reference's launchers run on the legacy default stream; torch's
    # default stream is that stream, so events recorded on it bracket them
    calls = {
        "expm": lambda: L.ref_expm(2, P(As), BATCH * nC, 1.0 / NSTEP, P(trels)),
        "forward": lambda: L.ref_forward(2, nx, ny, 1, P(pts), nP, 0, P(trels), P(As), BATCH,
                                         NSTEP, 0, P(out)),
        "backward": lambda: L.ref_backward(2, nx, ny, 1, nC, P(pts), nP, 0, P(As), BATCH, P(g),
                                           NSTEP, 0, P(mom), P(gp)),
        "project": lambda: torch.sparse.mm(Bt, mom.reshape(BATCH, -1).t()).t().contiguous(),
    }
    res = {}
    with torch.cuda.stream(torch.cuda.default_stream(dev)):
        for name, fn in calls.items():
            for _ in range(warmup):
                fn()
            torch.cuda.synchronize()
            ts = []
            for _ in range(steps):
                flush.zero_()
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                fn()
                e.record()
                torch.cuda.synchronize()
                ts.append(s.elapsed_time(e))
            res[name] = statistics.median(ts)
    res["fwd_grad_ms"] = res["expm"] + res["forward"] + res["backward"] + res["project"]
    return res


def run_ours(args, rank, world, local):
    from cpab import _native

    dev = torch.device("cuda", local)
    # rank 0 samples the clocks; its sampler process starts now, long before
    # the timed steps, and idles until they begin
    clocks = Clocks(local) if rank == 0 else None
    w, C, host, step, pairs_rank = make_workload(args.config, rank, world, dev, args.unfused)
    default = args.config == "2d"

    fused = getattr(w, "fused_data", None) is not None
    warped = getattr(w, "warp_data", None) is not None
    stn = args.config.startswith("stn")
    # one launch through all stages (the unfused STN runs one call per stage)
    chain = w.stages > 1 and C.params.ndim in (2, 3) and not stn
    # the integration calls of this workload (for transform_data and the STN
    # warp the fused resample-integration kernels)
    names = (("transform_data", "transform_data_backward") if fused else
             ("warp", "warp_backward") if warped else
             ("forward_chain", "backward_chain") if chain else ("forward", "backward"))
    timer = PhaseTimer(_native)

    resident = {k: v.to(dev) for k, v in host.items()}
    flush = torch.empty(L2_FLUSH_BYTES // 4, device=dev)

    from cpab.pytorch.transformer import clear_order_cache

    keep_order = getattr(w, "keep_order", False)

    def dev_step():
        # Every step sorts its points again, as a step on a new batch would
        # (the library would otherwise keep the order of the unchanged points).
        if not keep_order:
            clear_order_cache(C.params)
        return step(dict(resident, theta=resident["theta"].detach()))

    for _ in range(args.warmup):
        dev_step()
    torch.cuda.synchronize()

    if clocks is not None:
        clocks.start()
    # The step as a user runs it: no events but the step's own.
    ms_step = timed_steps(dev_step, args.steps, flush, world)
    if clocks is not None:
        clocks.pause()
    # Per-call CUDA events (and the kernel count) from a pass of the same steps.
    phases, launches_per_step = breakdown(dev_step, args.steps, flush, world, timer)
    launches = int(round(launches_per_step * args.steps))
    kern = {k: phases.get(n, 0.0) for k, n in (("forward", names[0]), ("backward", names[1]))}
    pairs_step = pairs_rank * world
    value = pairs_step / (ms_step * 1e-3)

    # End to end: pinned host inputs in, loss and gradient out, every step.
    pinned = {k: v.pin_memory() for k, v in host.items()}
    on_dev = {k: torch.empty_like(v) for k, v in resident.items()}
    loss_pin = torch.empty(1, pin_memory=True)
    grad_pin = torch.empty_like(host["theta"]).pin_memory()

    def e2e_step():
        for k in pinned:
            on_dev[k].copy_(pinned[k], non_blocking=True)
        loss, grad = step(dict(on_dev, theta=on_dev["theta"].detach()))
        loss_pin.copy_(loss.detach().reshape(1), non_blocking=True)
        grad_pin.copy_(grad, non_blocking=True)

    for _ in range(max(args.warmup, 1)):
        e2e_step()
    torch.cuda.synchronize()
    if clocks is not None:
        clocks.start()
    e2e_serial_ms = timed_steps(e2e_step, args.steps, flush, world)
    e2e_overlap_ms = timed_e2e_overlapped(step, pinned, resident, args.steps, args.warmup, flush,
                                          world, loss_pin, grad_pin)
    # Both loops are ways a user runs the step; the faster one is reported
    # (overlap wins where the copies are large, the serial loop where the
    # step is bound by host time and the second stream's bookkeeping adds to it).
    e2e_ms = min(e2e_serial_ms, e2e_overlap_ms)
    if clocks is not None:
        clocks.pause()

    # One GPU: the same device-resident step captured once in a CUDA graph
    # (sort, forward, loss, backward, projection recorded; every replay runs
    # them all), which removes the host launch gaps between its kernels.
    graph_ms = None
    if world == 1 and not args.no_graph:
        timer.capture = True
        graph_ms = graph_replay(step, resident, C, flush, args.steps, args.warmup, clocks)
        timer.capture = False
    clk = clocks.stop() if clocks is not None else None

    # N > 1, 2D 20x20: the fixed problem split over the ranks (strong scaling).
    strong = None
    if world > 1 and default and not args.no_strong:
        strong = strong_scaling(C, args.steps, args.warmup, flush, rank, world, timer)

    h2d = sum(v.numel() * v.element_size() for v in host.values())
    d2h = 4 + host["theta"].numel() * 4

    # N = 1: the reference's own GPU kernels on the same inputs (baseline leg).
    ref_kernels = None
    if world == 1 and default and not args.no_ref_kernels:
        ref_kernels = ref_gpu_kernels(C, host, args.steps, args.warmup, flush)
        if ref_kernels is not None:
            ours = {k: phases.get(k, 0.0) for k in ("build_A", "build_A_tt", "order_points",
                                                    "forward", "backward", "project",
                                                    "project_tt") if k in phases}
            ours["fwd_grad_ms"] = sum(ours.values())
            ref_kernels = {
                "what": "the reference's own CUDA kernels (cpab_ops_2d.cu, unmodified, sm_100a) "
                        "+ torch.sparse.mm projection, CUDA-event medians on the bench inputs",
                "reference_ms": ref_kernels, "ours_ms": ours,
                "speedup_fwd_grad": ref_kernels["fwd_grad_ms"] / ours["fwd_grad_ms"]}

    if rank == 0:
        hbm, peak_kind = peaks()
        p = C.params
        nd, ppc = p.ndim, p.params_pr_cell
        # Algorithmic bytes of one backward launch: the points, the upstream
        # gradient, cell matrices in and moments out (per stage).  The fused
        # transform_data backward reads the saved grid, the output gradient
        # and the image instead (its points are generated).
        pts_per_launch = pairs_rank // (w.batch * w.stages)
        if fused:
            ch, plane = w.fused_data
            bwd_bytes = (w.batch * (nd + ch) * pts_per_launch + w.batch * ch * plane
                         + 2 * w.batch * p.nC * ppc) * 4
        elif warped:  # sampled grid, stage inputs, output gradient, images, tables
            ch, plane = w.warp_data
            K = w.stages
            bwd_bytes = (w.batch * (K * nd + ch) * pts_per_launch + w.batch * ch * plane
                         + 2 * K * w.batch * p.nC * ppc) * 4
        elif chain:  # all stages: saved stage inputs instead of recomputed ones
            K = w.stages
            bwd_bytes = (nd * pts_per_launch + w.batch * nd * pts_per_launch
                         + (K - 1) * w.batch * nd * pts_per_launch
                         + 2 * K * w.batch * p.nC * ppc) * 4
        else:
            bwd_bytes = (nd * pts_per_launch + w.batch * nd * pts_per_launch
                         + 2 * w.batch * p.nC * ppc) * 4
        ach = bwd_bytes / (kern["backward"] * 1e-3) / 1e9
        traffic, inst, prov = profile_record() if default else (None, None, None)
        clk_mhz = (clk or {}).get("sm_mhz") or 1965.0
        issue_peak = 4 * 148 * clk_mhz * 1e6
        issue = None
        if inst:
            # The kernel is bound by instruction issue (4 schedulers x 148 SMs,
            # one warp instruction per scheduler per clock); the profiled
            # instruction count over the live launch time gives its fraction.
            issue_ach = inst / (kern["backward"] * 1e-3)
            issue = {"bound": "issue", "achieved": issue_ach, "peak": issue_peak,
                     "unit": "warp-inst/s", "frac": issue_ach / issue_peak,
                     "inst_per_launch": inst, "sm_mhz": clk_mhz, "profile": prov}
        cfg = config(world) if default else {
            "workload": w.desc, "tess": w.tess, "batch": w.batch, "stages": w.stages,
            "nstepsolver": NSTEP, "global_batch": pairs_step, "parallelism": w.parallelism,
            "l2": "flushed between timed steps (%d MiB write)" % (L2_FLUSH_BYTES >> 20),
            "point_order": (MESH_ORDER_NOTE if fused or warped else
                            "fixed meshgrid: its sort order is computed once and kept"
                            if keep_order else ORDER_NOTE)}
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": w.scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": cfg,
            "e2e": {"value": pairs_step / (e2e_ms * 1e-3), "unit": UNIT, "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "how": E2E_NOTE, "serial_ms_per_step": e2e_serial_ms,
                    "overlapped_ms_per_step": e2e_overlap_ms},
            "roofline": {"bound": "hbm",
                         "kernel": "k_backward_mesh (fused resample + adjoint)" if fused
                         else "k_backward_warp (fused grid_sample + adjoint, all stages)"
                         if warped
                         else "k_backward (fused adjoint, all chain stages)" if chain
                         else "k_backward (fused adjoint)",
                         "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                         "peak_kind": peak_kind, "traffic": traffic,
                         "algorithmic_bytes_per_launch": bwd_bytes, "profile": prov},
            "issue_roofline": issue,
            "kernel_ms": kern,
            "phase_ms": phases,
            "phase_note": "mean ms per step of each native call (and allreduce), CUDA events "
                          "in a separate pass of the same steps (kernel_ms and the roofline "
                          "use these); the remainder of a step is torch's loss kernels and "
                          "launch gaps",
            "graph_replay": None if graph_ms is None else {
                "value": pairs_step / (graph_ms * 1e-3), "unit": UNIT, "ms_per_step": graph_ms,
                "note": "the value step captured once in a CUDA graph and replayed; "
                        "value and e2e above are eager"},
            "gpu_launches": launches,
            "clocks": clk,
        }
        if strong is not None:
            line["strong"] = strong
        if ref_kernels is not None:
            line["ref_kernels"] = ref_kernels
        if default and world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(C.params.basis, host["theta"].numpy())
        emit(line)


_JSON_OUT = None


def emit(line):
    """Print the result line on the real stdout (everything else, including
    what NCCL or CUDA libraries print, goes to stderr)."""
    out = _JSON_OUT or sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def main():
    global _JSON_OUT
    sys.stdout.flush()
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)            # stdout of this process (and its libraries) -> stderr
    sys.stdout = sys.stderr
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true",
                    help="skip the one-GPU CUDA graph replay measurement")
    ap.add_argument("--no-strong", action="store_true",
                    help="skip the strong-scaling figures of the N>1 default run")
    ap.add_argument("--no-ref-kernels", action="store_true",
                    help="skip timing the reference's own GPU kernels at N=1")
    ap.add_argument("--unfused", action="store_true",
                    help="dense2d / 3d: time the unfused composition (meshgrid, transform_grid, "
                         "interpolate) instead of the fused transform_data kernels; stn2d / "
                         "stn3d: the reference layer's composition (a CPAB_transformer call per "
                         "transformation, then F.grid_sample) instead of the fused warp")
    ap.add_argument("--config", default="2d",
                    choices=["2d", "2d12", "2d30", "1d", "dense2d", "3d", "chain3d", "stn2d",
                             "stn3d"],
                    help="workload (default: BASELINE configs[1], 2D 20x20)")
    args = ap.parse_args()
    if args.impl == "reference":
        # CPU only: no process group; under torchrun rank 0 alone runs it.
        run_reference(args, int(os.environ.get("RANK", "0")),
                      int(os.environ.get("WORLD_SIZE", "1")))
        return
    rank, world, local = init_dist()
    try:
        run_ours(args, rank, world, local)
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
