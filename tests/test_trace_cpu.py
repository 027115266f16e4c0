"""Phase tracing (foundry_b200/utils/trace.py) on CPU: durations are kept per
phase (also when the body raises), ``timings(reset=True)`` clears them, and
FOUNDRY_TRACE=1 prints one ``[foundry TIMING]`` line per phase."""

import os
import subprocess
import sys
import time

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_phase_timings_and_reset():
    from foundry_b200.utils.trace import phase, timings

    timings(reset=True)
    with phase("unit.a"):
        time.sleep(0.01)
    with phase("unit.a"):
        pass
    with pytest.raises(ValueError):
        with phase("unit.b"):
            raise ValueError("boom")
    t = timings(reset=True)
    assert t["unit.a"]["n"] == 2 and t["unit.a"]["total_s"] >= 0.01
    assert t["unit.b"]["n"] == 1
    assert timings() == {}


def test_verbose_lines():
    code = ("import sys; sys.path.insert(0, %r)\n"
            "from foundry_b200.utils.trace import phase\n"
            "with phase('unit.verbose'):\n    pass\n") % ROOT
    r = subprocess.run([sys.executable, "-c", code], env=dict(os.environ, FOUNDRY_TRACE="1", CUDA_VISIBLE_DEVICES=""),
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and "[foundry TIMING] unit.verbose:" in r.stderr, r.stderr
