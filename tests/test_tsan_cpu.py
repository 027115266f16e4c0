"""Race detection: the host libraries built with ThreadSanitizer run the
mock-driver SAVE and LOAD scenarios (region allocations, module registry,
parallel file reads and the background template-build thread of the restore)
with halt_on_error; any reported race fails the test."""

import os
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIBTSAN = "/usr/lib/x86_64-linux-gnu/libtsan.so.2"


@pytest.mark.skipif(not os.path.exists(LIBTSAN), reason="libtsan not available")
def test_persistence_stack_under_thread_sanitizer(tmp_path):
    sys.path.insert(0, ROOT)
    from foundry_b200._build import build_tsan

    pkg_root = str(build_tsan(tmp_path / "tsan"))
    mock = os.path.join(pkg_root, "foundry_b200", "lib", "libfoundry_mockcuda.so")
    env = dict(os.environ, FOUNDRY_CUDA_DRIVER=mock, FOUNDRY_PKG_ROOT=pkg_root, PYTHONPATH=pkg_root,
               CUDA_VISIBLE_DEVICES="", LD_PRELOAD=LIBTSAN, FOUNDRY_TEST_REGION_BASE="0x7c0000000000",
               TSAN_OPTIONS="halt_on_error=1 exitcode=66 report_signal_unsafe=0")
    wd = str(tmp_path / "work")
    os.makedirs(wd)
    for scenario in ("save", "load"):
        r = subprocess.run([sys.executable, os.path.join(HERE, "mock_scenarios.py"), scenario, wd], env=env,
                           capture_output=True, text=True, timeout=600)
        assert "ThreadSanitizer" not in r.stderr, r.stderr[-6000:]
        assert r.returncode == 0, f"{scenario}: rc={r.returncode}\n{r.stdout[-2000:]}\n{r.stderr[-4000:]}"
        assert f"{scenario.upper()} OK" in r.stdout
