"""Every reference citation (file.py:line[-line]) in the shipped sources points
at lines that exist, and where a citation names a function or class right
before it ("Name.method -- file.py:a-b", "method (file.py:a-b)"), that
definition starts inside the cited range.

Reads the reference source tree, so it runs only where that tree is mounted
(the build container); elsewhere it is skipped.
"""

import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = "/root/reference"
SEARCH = ("helix_online_kv", "tools", "tests", "")

SOURCES = ["include/hokv.h", "bench.py", "__graft_entry__.py"]
for root in ("helix-online-kv_b200", "oracle", "tests"):
    for dirpath, _, files in os.walk(os.path.join(REPO, root)):
        if "__pycache__" in dirpath or "_build" in dirpath:
            continue
        for f in files:
            if f.endswith((".py", ".h", ".cu", ".cuh")):
                SOURCES.append(os.path.relpath(os.path.join(dirpath, f), REPO))

CITE = re.compile(r"([A-Za-z_][\w.]*)?(\s*(?:--|\()\s*)?((?:[\w]+/)*\w+\.py):(\d+)(?:-(\d+))?((?:,\d+-\d+)*)")

pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "helix_online_kv")),
                                reason="reference source tree not mounted")


def _ref_lines(name):
    for sub in SEARCH:
        p = os.path.join(REF, sub, name)
        if os.path.isfile(p):
            with open(p) as f:
                return f.read().splitlines()
    return None


def _def_spans(lines, name):
    """(first, last) line of every def/class `name`: up to the next line at the
    same or a lower indentation that starts a definition or a decorator."""
    spans = []
    for i, l in enumerate(lines):
        m = re.match(rf"(\s*)(def|class)\s+{re.escape(name)}\b", l)
        if not m:
            continue
        ind, end = len(m.group(1)), len(lines)
        for j in range(i + 1, len(lines)):
            t = lines[j]
            if t.strip() and len(t) - len(t.lstrip()) <= ind and re.match(r"\s*(def |class |@)", t):
                end = j
                break
        spans.append((i + 1, end))
    return spans


def _citations():
    for rel in SOURCES:
        if rel.endswith("test_citations.py"):
            continue
        with open(os.path.join(REPO, rel)) as f:
            text = f.read()
        for m in CITE.finditer(text):
            sym, sep, path, a, b, more = m.groups()
            ranges = [(int(a), int(b or a))]
            for extra in re.findall(r"(\d+)-(\d+)", more or ""):
                ranges.append((int(extra[0]), int(extra[1])))
            line = text.count("\n", 0, m.start()) + 1
            yield rel, line, (sym if sep else None), path, ranges


def test_cited_ranges_exist():
    bad, n = [], 0
    for rel, line, _, path, ranges in _citations():
        lines = _ref_lines(os.path.basename(path) if path.count("/") == 0 else path)
        if lines is None and "/" in path:
            lines = _ref_lines(path.split("/", 1)[1])
        if lines is None:
            continue   # a file of this repository (e.g. hokv_lib.cu), not the reference's
        for a, b in ranges:
            n += 1
            if not (1 <= a <= b <= len(lines)):
                bad.append(f"{rel}:{line}: {path}:{a}-{b} outside 1..{len(lines)}")
    assert n > 50, n
    assert not bad, "\n".join(bad)


def test_named_definitions_inside_cited_ranges():
    bad, n = [], 0
    for rel, line, sym, path, ranges in _citations():
        if not sym:
            continue
        lines = _ref_lines(os.path.basename(path))
        if lines is None:
            continue
        name = sym.rstrip(".").split(".")[-1]
        spans = _def_spans(lines, name)
        if not spans:
            continue   # prose before the citation, not a definition of that file
        n += 1
        if not any(a <= e and s <= b for s, e in spans for a, b in ranges):
            bad.append(f"{rel}:{line}: {sym} spans {spans} of {path}, cited {ranges}")
    assert n >= 10, n
    assert not bad, "\n".join(bad)
