"""The runner's static arena on the mock driver: large tensors take exactly
sized region allocations, so the mapped total stays within the 2 MiB rounding
of the requested bytes (no stranded chunk tails), and the layout is the same
in two processes (SAVE == LOAD addresses)."""

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
MOCK = os.path.join(ROOT, "foundry_b200", "lib", "libfoundry_mockcuda.so")

BODY = r"""
import sys
sys.path.insert(0, ROOT)
from foundry_b200 import core, get_current_alloc_offset
from foundry_b200.runner.arena import Arena
a = Arena(0x600000000000, "64GB", device="cpu")
ptrs = []
for i in range(20):                      # KV-cache-like 605 MB layers mixed with small tensors
    ptrs.append(a.alloc_bytes(605 << 20))
    ptrs.append(a.alloc_bytes(4096))
mapped = get_current_alloc_offset()
want = 20 * (606 << 20) + (2 << 20)       # 2 MiB rounding per layer + the small-tensor chunk(s)
assert mapped <= want + (1 << 30), (mapped, want)
print("LAYOUT", ptrs[0], ptrs[-1], mapped)
"""


def _run():
    env = dict(os.environ, FOUNDRY_CUDA_DRIVER=MOCK, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, "-c", f"ROOT={ROOT!r}\n" + BODY], env=env, capture_output=True, text=True,
                       timeout=180)
    assert r.returncode == 0, r.stdout + r.stderr[-3000:]
    return [l for l in r.stdout.splitlines() if l.startswith("LAYOUT")][0]


def test_large_tensors_do_not_strand_chunk_tails_and_layout_is_deterministic():
    assert _run() == _run()
