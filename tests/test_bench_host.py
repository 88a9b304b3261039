"""Host-side logic of bench.py that needs no GPU: the clock sampler that
accompanies every timed region, and the CPU placement of a rank."""
import os
import stat
import sys
import time

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
import bench  # noqa: E402


@pytest.fixture
def slow_nvidia_smi(tmp_path, monkeypatch):
    """An nvidia-smi stand-in that, like the real one, takes a while before
    its first sample (0.4 s here), then reports every 50 ms."""
    exe = tmp_path / "nvidia-smi"
    exe.write_text("#!/bin/bash\nsleep 0.4\ni=0\nwhile true; do\n"
                   "  echo \"0, $((1800 + i)), 1965, 500, 0x0, Not Active, Not Active, Not Active, Active\"\n"
                   "  i=$((i+1)); sleep 0.05\ndone\n")
    exe.chmod(exe.stat().st_mode | stat.S_IXUSR)
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")


def test_short_region_gets_samples(slow_nvidia_smi):
    """A timed region shorter than nvidia-smi's start-up still gets samples,
    and only its own: the sampler is ready before the region starts."""
    c = bench.ClockSampler("0").start()
    assert c.lines, "start() returns once the first sample is in"
    c.mark()
    time.sleep(0.12)
    c.stop()
    s = c.summary()
    assert s["samples"] >= 2
    assert s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"]
    # the samples before mark() are not the region's
    assert s["samples"] == len(c.lines[c.i0:c.i1])


def test_sampler_without_nvidia_smi(tmp_path, monkeypatch):
    monkeypatch.setenv("PATH", str(tmp_path))  # no nvidia-smi anywhere
    c = bench.ClockSampler("0").start(ready_timeout=0.2)
    c.mark()
    c.stop()
    assert c.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}


def test_cpu_placement_without_nvml_changes_nothing():
    before = os.sched_getaffinity(0)
    n = bench.bind_to_gpu_cpus("0", "00000000:00:00.0")
    if n is None:  # no NVML or no such GPU here: the process keeps its CPUs
        assert os.sched_getaffinity(0) == before
    else:
        os.sched_setaffinity(0, before)


@pytest.mark.skipif(not os.path.exists(bench.REF_PROGRAM), reason="reference program not built")
def test_reference_program_sample(synth_model_path):
    """The reference arm's bounded sample: one reference program on the first
    workload sentence, encode then a 1 s window of beam-search steps; its
    rate is a whole-sentence rate below the window's step rate."""
    rate, per = bench.reference_program_rate(synth_model_path, bench.reference_sample(0, 1), 1.0, 1)
    assert len(per) == 1 and per[0]["steps_in_window"] >= 2
    assert 0 < rate < per[0]["step_rate"]
    assert per[0]["n_src"] == len(bench.reference_sample(0, 1)[0])
