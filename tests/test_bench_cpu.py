"""bench.py on the CPU: the clock sampler that goes beside every bench line (parsing
nvidia-smi's CSV, reasons, its bounded start) and the JSON line of the reference
arm (`--impl reference`, the reference's CPU path on the host cores)."""
import json
import subprocess
import sys
import time

import pytest

import bench


def sample(sm, mx=1965, power_cap="Not Active", hw="Not Active"):
    return f"0, {sm}, {mx}, 900.1, 0x4, {hw}, Not Active, Not Active, {power_cap}"


def test_clock_sampler_summary():
    s = bench.ClockSampler("GPU-0")
    s.lines = [sample(1800), sample(1900, power_cap="Active"), sample(1965),
               "0, [N/A], 1965, 1, 0, a, b, c, d", "garbage", ""]
    out = s.stop()
    assert out["samples"] == 3
    assert out["sm_mhz"] == 1900
    assert out["sm_max_mhz"] == 1965
    assert out["reasons"] == ["sw_power_cap"]


def test_clock_sampler_reports_a_slowdown():
    s = bench.ClockSampler("GPU-0")
    s.lines = [sample(1200, hw="Active"), sample(1250)]
    out = s.stop()
    assert out["reasons"] == ["hw_slowdown"] and out["samples"] == 2


def test_clock_sampler_without_nvidia_smi(monkeypatch):
    def missing(*a, **k):
        raise FileNotFoundError("nvidia-smi")

    monkeypatch.setattr(bench.subprocess, "Popen", missing)
    out = bench.ClockSampler("GPU-0").start().stop()
    assert out == {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                   "device": "GPU-0"}


class FakeUUID:
    def __init__(self, raw: bytes):
        self.bytes = raw


class FakeProps:
    def __init__(self, raw: bytes, bus: int):
        self.uuid = FakeUUID(raw)
        self.pci_domain_id, self.pci_bus_id, self.pci_device_id = 0, bus, 0


def test_clock_sampler_names_the_visible_gpu_not_the_local_ordinal(monkeypatch):
    """With CUDA_VISIBLE_DEVICES=3 the process's cuda:0 is the machine's GPU 3;
    nvidia-smi ignores the variable, so the sampler must name the device by its
    UUID (here the fake UUID of the machine's GPU 3), never by --id=0."""
    import torch
    machine = {i: FakeProps(bytes([i]) * 16, 0x10 + i) for i in range(8)}
    visible = [3]
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "3")
    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda d: machine[visible[d]])
    dev_id = bench.smi_device_id(0)
    assert dev_id == "GPU-03030303-0303-0303-0303-030303030303"
    cmd = bench.ClockSampler(dev_id).command()
    assert f"--id={dev_id}" in cmd and "--id=0" not in cmd
    # without a UUID the PCI bus id names it
    props = FakeProps(b"", 0x13)
    props.uuid = None
    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda d: props)
    assert bench.smi_device_id(0) == "00000000:13:00.0"


class SlowSmi:
    """A stand-in for nvidia-smi -lms: its first line comes after `delay` seconds."""

    def __init__(self, delay, lines):
        self.delay, self.rows = delay, lines
        self.stdout = self
        self.ended = False

    def __iter__(self):
        time.sleep(self.delay)
        for ln in self.rows:
            if self.ended:
                return
            yield ln + "\n"
            time.sleep(0.01)

    def poll(self):
        return 0 if self.ended else None

    def terminate(self):
        self.ended = True

    def wait(self, timeout=None):
        return 0

    def kill(self):
        self.ended = True


def test_clock_sampler_start_waits_for_the_first_sample(monkeypatch):
    monkeypatch.setattr(bench.subprocess, "Popen",
                        lambda *a, **k: SlowSmi(0.3, [sample(1965)] * 50))
    t0 = time.monotonic()
    s = bench.ClockSampler("GPU-0").start()
    waited = time.monotonic() - t0
    assert s.lines, "start() returned before nvidia-smi produced a sample"
    assert 0.25 <= waited < 5.0
    assert s.stop()["samples"] >= 1


def test_clock_sampler_start_is_bounded(monkeypatch):
    monkeypatch.setattr(bench.subprocess, "Popen", lambda *a, **k: SlowSmi(30.0, []))
    t0 = time.monotonic()
    s = bench.ClockSampler("GPU-0").start()
    assert time.monotonic() - t0 < 6.0
    s.proc.terminate()


@pytest.mark.slow
def test_reference_arm_prints_the_contract_line():
    """The reference arm on this machine's cores (about a minute): one JSON line with
    impl "reference", a positive value, its cpu_baseline and a zero-copy e2e."""
    r = subprocess.run([sys.executable, str(bench.__file__), "--impl", "reference", "--steps", "1",
                        "--warmup", "3"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    for key in ("metric", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "config"):
        assert key in line, key
    assert line["value"] > 0 and line["steps"] == 1 and line["warmup"] == 3
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["kind"] in ("reference", "port")
    assert cb["cores"] >= 1 and cb["sample"]
    assert line["e2e"]["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
