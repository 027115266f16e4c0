"""Repository hygiene checker (foundry_b200/utils/lint.py): SPDX header status
and --fix for Python and CUDA sources, shebang/encoding lines kept first,
empty files passing, whitespace in file names rejected."""

import os
import subprocess
import sys

from foundry_b200.utils import lint

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIC, COP = lint.header_lines("#", "MIT", "Copyright the authors")


def _write(tmp_path, name, text):
    p = tmp_path / name
    p.write_text(text)
    return str(p)


def test_status_and_fix_python(tmp_path):
    both = _write(tmp_path, "a.py", "#!/usr/bin/env python\n# -*- coding: utf-8 -*-\nx = 1\n")
    only_lic = _write(tmp_path, "b.py", f'"""doc"""\n{LIC}\ny = 2')
    only_cop = _write(tmp_path, "c.py", f"{COP}\n")
    done = _write(tmp_path, "d.py", f"{LIC}\n{COP}\nz = 3\n")
    empty = _write(tmp_path, "__init__.py", "")
    res = lint.check_spdx([both, only_lic, only_cop, done, empty], "MIT", "Copyright the authors")
    S = lint.Status
    assert res == {both: S.MISSING_BOTH, only_lic: S.MISSING_COPYRIGHT, only_cop: S.MISSING_LICENSE,
                   done: S.COMPLETE, empty: S.EMPTY}
    lint.check_spdx([both, only_lic, only_cop], "MIT", "Copyright the authors", fix=True)
    lines = open(both).read().splitlines()
    assert lines[:4] == ["#!/usr/bin/env python", "# -*- coding: utf-8 -*-", LIC, COP] and lines[4] == "x = 1"
    assert open(only_lic).read().splitlines() == ['"""doc"""', LIC, COP, "y = 2"]
    assert open(only_cop).read().splitlines() == [LIC, COP]
    again = lint.check_spdx([both, only_lic, only_cop], "MIT", "Copyright the authors")
    assert set(again.values()) == {S.COMPLETE}


def test_cuda_sources_use_slash_comments_and_unknown_types_are_skipped(tmp_path):
    cu = _write(tmp_path, "k.cu", "__global__ void k() {}\n")
    md = _write(tmp_path, "notes.md", "text\n")
    res = lint.check_spdx([cu, md], "MIT", "Copyright the authors", fix=True)
    assert list(res) == [cu]
    lic, cop = lint.header_lines("//", "MIT", "Copyright the authors")
    assert open(cu).read().splitlines()[:2] == [lic, cop]


def test_cli_exit_codes_and_file_names(tmp_path):
    good = _write(tmp_path, "ok.py", f"{LIC}\n{COP}\n")
    bad = _write(tmp_path, "has space.py", "x = 1\n")
    env = dict(os.environ, PYTHONPATH=ROOT)
    run = lambda *a: subprocess.run([sys.executable, "-m", "foundry_b200.utils.lint", *a], env=env,  # noqa: E731
                                    capture_output=True, text=True, timeout=120)
    assert run("spdx", "--license", "MIT", "--owner", "Copyright the authors", good).returncode == 0
    r = run("spdx", "--license", "MIT", "--owner", "Copyright the authors", bad)
    assert r.returncode == 1 and "missing both lines" in r.stdout
    assert run("names", good).returncode == 0
    r = run("names", good, bad)
    assert r.returncode == 1 and "has space.py" in r.stdout
    assert lint.bad_names(["a/b c/ok.py", "x\ty.py", "a/b/ok.py"]) == ["a/b c/ok.py", "x\ty.py"]
