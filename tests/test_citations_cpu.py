"""Every reference citation `file:N-M` in the boundary header, the oracle and
the kernel sources points inside the cited reference file.

The citations are how a reader checks parity against the reference, so each
one must name a file of the reference tree and lines that exist in it.  The
reference tree is read from $DS_REFERENCE_ROOT (default: the path where this
repository's build reads it); the test is skipped where it is absent.
"""
import os
import re

import pytest

from conftest import ROOT

REF = os.environ.get("DS_REFERENCE_ROOT", "/root/reference")

SCANNED = ["include", "oracle", "ds-experiment_b200/csrc", "ds-experiment_b200/ds_b200",
           "tests/golden"]
SUFFIXES = (".h", ".c", ".cu", ".cuh", ".py")

# path:lines, where path is relative to the reference root or a bare file name
CITE = re.compile(r"(?<![\w/.])((?:[\w.-]+/)*[\w.-]+\.(?:cpp|cu|h|py|md|txt)|Dockerfile)"
                  r":(\d+(?:-\d+)?(?:,\s?\d+(?:-\d+)?)*)")


def _sources():
    for d in SCANNED:
        base = os.path.join(ROOT, d)
        for dirpath, _, files in os.walk(base):
            for f in files:
                if f.endswith(SUFFIXES):
                    yield os.path.join(dirpath, f)


def _reference_index():
    by_rel, by_name = {}, {}
    for dirpath, dirs, files in os.walk(REF):
        dirs[:] = [d for d in dirs if not d.startswith(".")]
        for f in files:
            p = os.path.join(dirpath, f)
            rel = os.path.relpath(p, REF)
            by_rel[rel] = p
            by_name.setdefault(f, []).append(p)
    return by_rel, by_name


def _line_count(path):
    with open(path, "rb") as f:
        return f.read().count(b"\n") + 1


@pytest.mark.skipif(not os.path.isdir(REF), reason="reference tree not present")
def test_reference_citations_point_inside_their_files():
    by_rel, by_name = _reference_index()
    checked, bad = 0, []
    for src in _sources():
        text = open(src, encoding="utf-8", errors="replace").read()
        for m in CITE.finditer(text):
            cited, ranges = m.group(1), m.group(2)
            if cited in by_rel:
                target = by_rel[cited]
            elif "/" not in cited and len(by_name.get(cited, [])) == 1:
                target = by_name[cited][0]
            else:
                continue  # one of this repository's own files, not a reference citation
            n = _line_count(target)
            for part in ranges.replace(" ", "").split(","):
                lo, _, hi = part.partition("-")
                lo, hi = int(lo), int(hi or lo)
                checked += 1
                if not (1 <= lo <= hi <= n):
                    line = text.count("\n", 0, m.start()) + 1
                    bad.append(f"{os.path.relpath(src, ROOT)}:{line} cites {cited}:{part} "
                               f"({n} lines)")
    assert checked > 50, checked
    assert not bad, "\n".join(bad)
