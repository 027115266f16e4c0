"""Repository hygiene checks run as pre-commit hooks (``.pre-commit-config.yaml``).

    python -m foundry_b200.utils.lint spdx [--fix] [--license ID] [--owner TEXT] FILE...
    python -m foundry_b200.utils.lint names FILE...

``spdx``: every source file carries the two SPDX lines (license identifier
and file copyright text) near its top, in the file's comment syntax (``#``
for Python/shell/TOML/YAML, ``//`` for C, C++ and CUDA). A shebang and a
Python encoding line stay first. With ``--fix`` the missing line(s) are
inserted: both after the shebang/encoding lines, a lone missing line beside
its partner. Empty files (e.g. an empty ``__init__.py``) pass. Exit status 1
when any file was missing a line (fixed or not), as pre-commit expects.

``names``: no whitespace in file paths (tools and shells split on it).

Parity: reference tools/pre_commit/check_spdx_header.py:1-121 (Python files
only, fixed header) and .pre-commit-config.yaml:41-63 (filename check); this
version also covers C/C++/CUDA sources and takes the license and owner as
arguments.
"""

from __future__ import annotations

import argparse
import enum
import os
import re
import sys
from typing import Iterable

DEFAULT_LICENSE = "Apache-2.0"
DEFAULT_OWNER = "Copyright contributors to the foundry_b200 project"
HEADER_SCAN_LINES = 12  # the SPDX lines must appear within this many lines of the top

_SLASH_EXT = {".c", ".cc", ".cpp", ".cxx", ".h", ".hh", ".hpp", ".cu", ".cuh"}
_HASH_EXT = {".py", ".pyi", ".sh", ".bash", ".toml", ".yaml", ".yml", ".cmake"}
_CODING = re.compile(r"^[ \t\f]*#.*?coding[:=][ \t]*[-\w.]+")


class Status(enum.Enum):
    EMPTY = "empty"
    COMPLETE = "complete"
    MISSING_LICENSE = "missing license line"
    MISSING_COPYRIGHT = "missing copyright line"
    MISSING_BOTH = "missing both lines"


def comment_prefix(path: str) -> str | None:
    """The line-comment marker for ``path``, or None for file types not checked."""
    ext = os.path.splitext(path)[1].lower()
    if ext in _SLASH_EXT:
        return "//"
    if ext in _HASH_EXT or os.path.basename(path) in ("CMakeLists.txt", "Makefile"):
        return "#"
    return None


def header_lines(prefix: str, license_id: str, owner: str) -> tuple[str, str]:
    return (f"{prefix} SPDX-License-Identifier: {license_id}", f"{prefix} SPDX-FileCopyrightText: {owner}")


def _preamble_len(lines: list[str]) -> int:
    """Lines that must stay above the header: a shebang, then a coding line."""
    n = 0
    if lines and lines[0].startswith("#!"):
        n = 1
    if len(lines) > n and _CODING.match(lines[n]):
        n += 1
    return n


def status_of(lines: list[str], license_line: str, copyright_line: str) -> Status:
    if not any(line.strip() for line in lines):
        return Status.EMPTY
    top = [line.strip() for line in lines[:HEADER_SCAN_LINES]]
    has_l, has_c = license_line in top, copyright_line in top
    if has_l and has_c:
        return Status.COMPLETE
    if has_l:
        return Status.MISSING_COPYRIGHT
    if has_c:
        return Status.MISSING_LICENSE
    return Status.MISSING_BOTH


def fixed(lines: list[str], status: Status, license_line: str, copyright_line: str) -> list[str]:
    """``lines`` with the missing SPDX line(s) inserted (lines keep their newlines)."""
    out = list(lines)
    top = [line.strip() for line in out[:HEADER_SCAN_LINES]]
    if status is Status.MISSING_BOTH:
        at = _preamble_len(out)
        out[at:at] = [license_line + "\n", copyright_line + "\n"]
    elif status is Status.MISSING_COPYRIGHT:
        i = top.index(license_line)
        out.insert(i + 1, copyright_line + "\n")
    elif status is Status.MISSING_LICENSE:
        i = top.index(copyright_line)
        out.insert(i, license_line + "\n")
    return out


def check_spdx(paths: Iterable[str], license_id: str = DEFAULT_LICENSE, owner: str = DEFAULT_OWNER,
               fix: bool = False) -> dict[str, Status]:
    """Status of every checked file (files of unknown type are skipped)."""
    result: dict[str, Status] = {}
    for path in paths:
        prefix = comment_prefix(path)
        if prefix is None:
            continue
        lic, cop = header_lines(prefix, license_id, owner)
        with open(path, encoding="utf-8", newline="") as f:
            lines = f.readlines()
        st = status_of(lines, lic, cop)
        result[path] = st
        if fix and st not in (Status.EMPTY, Status.COMPLETE):
            if lines and not lines[-1].endswith("\n"):
                lines[-1] += "\n"
            with open(path, "w", encoding="utf-8", newline="") as f:
                f.writelines(fixed(lines, st, lic, cop))
    return result


def bad_names(paths: Iterable[str]) -> list[str]:
    return [p for p in paths if any(c.isspace() for c in p)]


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(prog="python -m foundry_b200.utils.lint")
    sub = ap.add_subparsers(dest="cmd", required=True)
    sp = sub.add_parser("spdx", help="check (or --fix) SPDX header lines")
    sp.add_argument("--fix", action="store_true")
    sp.add_argument("--license", default=DEFAULT_LICENSE)
    sp.add_argument("--owner", default=DEFAULT_OWNER)
    sp.add_argument("files", nargs="*")
    nm = sub.add_parser("names", help="reject whitespace in file names")
    nm.add_argument("files", nargs="*")
    args = ap.parse_args(argv)
    if args.cmd == "names":
        bad = bad_names(args.files)
        for p in bad:
            print(f"file name contains whitespace: {p!r}")
        return 1 if bad else 0
    res = check_spdx(args.files, args.license, args.owner, fix=args.fix)
    missing = {p: s for p, s in res.items() if s not in (Status.EMPTY, Status.COMPLETE)}
    for p, s in missing.items():
        print(f"{p}: {s.value}{' (fixed)' if args.fix else ''}")
    return 1 if missing else 0


if __name__ == "__main__":
    sys.exit(main())
