"""Clock sampling during a timed region, against a fake ``nvidia-smi`` on PATH (no GPU): the
median SM clock, the maximum clock, the throttle reasons seen and the peak power are read from
its CSV lines; without nvidia-smi the sampler says so instead of failing."""
import os
import stat
import time

from nanovllm_self_b200.utils.clocks import ClockSampler

LINES = [
    "0, 1965, 1965, 400.5, 0x0, Not Active, Not Active, Not Active, Not Active",
    "0, 1800, 1965, 990.0, 0x4, Not Active, Not Active, Not Active, Active",
    "0, 1750, 1965, 1001.2, 0x4, Not Active, Not Active, Not Active, Active",
    "garbage line",
    "0, 1850, 1965, 870.0, 0x0, Not Active, Not Active, Not Active, Not Active",
]


def _fake_smi(tmp_path, lines):
    exe = tmp_path / "nvidia-smi"
    body = "".join(f"echo '{ln}'\n" for ln in lines)
    exe.write_text("#!/bin/sh\n" + body + "exec sleep 30\n")
    exe.chmod(exe.stat().st_mode | stat.S_IEXEC)
    return str(tmp_path)


def test_sampler_summarises_the_fake_samples(tmp_path, monkeypatch):
    monkeypatch.setenv("PATH", _fake_smi(tmp_path, LINES) + os.pathsep + os.environ["PATH"])
    s = ClockSampler(0)
    s.start()
    deadline = time.time() + 10
    while len(s.lines) < len(LINES) and time.time() < deadline:
        time.sleep(0.01)
    r = s.stop()
    assert r["samples"] == 4 and r["sm_max_mhz"] == 1965.0
    assert r["sm_mhz"] == 1850.0  # median of 1750, 1800, 1850, 1965 (upper middle)
    assert r["reasons"] == ["sw_power_cap"] and r["power_w_max"] == 1001.2


def test_sampler_without_nvidia_smi(tmp_path, monkeypatch):
    monkeypatch.setenv("PATH", str(tmp_path))
    s = ClockSampler(0)
    s.start()
    assert s.stop()["reasons"] == ["nvidia-smi unavailable"]
