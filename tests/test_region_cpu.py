"""Region helpers on CPU: ``parse_size`` formats (the reference's
tests/test_preallocation.py size-parsing check) and the ``allocation_region``
context manager on the mock driver (allocations inside the block land in
the region, the preallocated window is used first, the region is stopped at
exit)."""

import os
import subprocess
import sys

import pytest

from foundry_b200 import parse_size

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
MOCK = os.path.join(ROOT, "foundry_b200", "lib", "libfoundry_mockcuda.so")


@pytest.mark.parametrize("text,value", [
    ("1GB", 1 << 30), ("1.5GB", 3 << 29), ("16MB", 16 << 20), ("24KB", 24 << 10), ("512", 512), ("2TB", 2 << 40),
    (" 64mb ", 64 << 20), ("8GiB", 8 << 30), ("3B", 3), (4096, 4096), (0, 0),
])
def test_parse_size(text, value):
    assert parse_size(text) == value


@pytest.mark.parametrize("bad", ["", "GB", "1.5", "1.5.0GB", "-1GB", "12 parsecs", "0x100"])
def test_parse_size_rejects(bad):
    if bad == "1.5":  # a bare decimal is bytes (floored), like the reference
        assert parse_size(bad) == 1
        return
    with pytest.raises(ValueError):
        parse_size(bad)


def test_parse_size_rejects_negative_int():
    with pytest.raises(ValueError):
        parse_size(-1)


CTX = r"""
import sys
sys.path.insert(0, ROOT)
import foundry_b200 as fb
c = fb.core()
assert c.driver_is_mock()
base, size = 0x610000000000, 4 << 30
with fb.allocation_region(base, "4GB", prealloc_size="256MB"):
    assert c.region_active()
    a = c.region_alloc(8 << 20)
    b = c.region_alloc(100 << 20)
    assert base <= a < b < base + (256 << 20), (hex(a), hex(b))   # inside the preallocated window
    big = c.region_alloc(512 << 20)                                 # past the window: still in the region
    assert base + (256 << 20) <= big < base + size, hex(big)
    off = fb.get_current_alloc_offset()
    assert off >= (256 << 20) + (512 << 20)
assert not c.region_active()
print("CTX_OK")
"""


def test_allocation_region_context_manager_on_mock():
    env = dict(os.environ, FOUNDRY_CUDA_DRIVER=MOCK, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, "-c", f"ROOT={ROOT!r}\n" + CTX], env=env, capture_output=True, text=True,
                       timeout=180)
    assert r.returncode == 0 and "CTX_OK" in r.stdout, r.stdout + r.stderr[-3000:]
