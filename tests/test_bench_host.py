"""Host-side pieces of bench.py that need no GPU: the clock sampler (a child
process reading NVML, here a fake NVML module) and the config record."""
import os
import sys
import time

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402

FAKE_NVML = """
NVML_CLOCK_SM = 1
def nvmlInit(): pass
def nvmlDeviceGetHandleByIndex(i): return i
def nvmlDeviceGetMaxClockInfo(h, k): return 1965
def nvmlDeviceGetClockInfo(h, k): return 1800
def nvmlDeviceGetCurrentClocksEventReasons(h): return 0x4 | 0x40
"""


def test_clock_sampler_child_process(tmp_path, monkeypatch):
    (tmp_path / "pynvml.py").write_text(FAKE_NVML)
    monkeypatch.setenv("PYTHONPATH", str(tmp_path))
    c = bench.Clocks(0)
    c.start()
    assert c.proc is not None
    time.sleep(0.05)
    r = c.stop()
    assert r["sm_mhz"] == 1800 and r["sm_max_mhz"] == 1965
    assert r["reasons"] == ["hw_thermal_slowdown", "sw_power_cap"]
    assert r["samples"] >= 2
    assert c.proc.returncode == 0


def test_clock_sampler_pauses_between_timed_regions(tmp_path, monkeypatch):
    """Sampling covers several timed regions: start, pause, start again, stop."""
    (tmp_path / "pynvml.py").write_text(FAKE_NVML)
    monkeypatch.setenv("PYTHONPATH", str(tmp_path))
    c = bench.Clocks(0)
    c.start()
    time.sleep(0.02)
    c.pause()
    assert c.proc is not None
    time.sleep(0.02)
    c.start()
    time.sleep(0.02)
    r = c.stop()
    assert r is not None and r["samples"] >= 4 and r["sm_mhz"] == 1800
    assert c.proc.returncode == 0


def test_clock_sampler_without_nvml_reports_nothing(tmp_path, monkeypatch):
    (tmp_path / "pynvml.py").write_text("raise ImportError('no NVML here')\n")
    monkeypatch.setenv("PYTHONPATH", str(tmp_path))
    c = bench.Clocks(0)
    c.start()
    assert c.proc is None and c.stop() is None


@pytest.mark.parametrize("world", [1, 8])
def test_default_config_record(world):
    cfg = bench.config(world)
    assert cfg["global_batch"] == bench.BATCH * bench.N_POINTS * world
    assert cfg["point_order"] == bench.ORDER_NOTE
    assert "flushed" in cfg["l2"]


def _run_reference_arm(env_extra):
    import json
    import subprocess
    env = dict(os.environ, **env_extra)
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--steps", "1", "--warmup", "1"], capture_output=True, text=True,
                       env=env, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    return [json.loads(ln) for ln in lines]


def test_reference_arm_prints_one_line_on_rank0():
    """The CPU reference arm (the oracle port on host threads) prints one JSON
    line with the same metric/config as our arm, and e2e without copies."""
    (line,) = _run_reference_arm({"RANK": "0", "WORLD_SIZE": "1"})
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC
    assert line["config"] == bench.config(1) and line["higher_is_better"] is True
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"],
                           "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert line["cpu_baseline"]["kind"] in ("port", "reference") and line["value"] > 0


def test_reference_arm_other_ranks_do_nothing():
    assert _run_reference_arm({"RANK": "1", "WORLD_SIZE": "2"}) == []
