"""Every reference citation in the boundary, the docs, the package and the oracle resolves.

A citation is ``namitorch/<path>.py:N`` or ``namitorch/<path>.py:N-M``. Each must name a
file of the reference checkout and lie inside it. The C ABI header's citations of the
GradScaler stages must also land on the methods they name. Skipped without a reference
checkout ($NAMITORCH_REFERENCE, or ``reference`` beside this repository).
"""
import re
from pathlib import Path

import pytest

from conftest import REPO, reference_root

CITATION = re.compile(r"(namitorch/[\w/]+\.py):(\d+)(?:-(\d+))?")
SOURCES = ["include", "INTEGRATION.md", "DESIGN.md", "README.md", "namitorch_b200", "oracle", "bench.py",
           "__graft_entry__.py"]


def _files():
    for name in SOURCES:
        path = REPO / name
        if path.is_file():
            yield path
        elif path.is_dir():
            yield from sorted(p for p in path.rglob("*") if p.suffix in (".py", ".h", ".cu", ".cuh", ".md"))


def _citations():
    for path in _files():
        for number, line in enumerate(path.read_text().splitlines(), 1):
            for match in CITATION.finditer(line):
                first = int(match.group(2))
                last = int(match.group(3)) if match.group(3) else first
                yield path.relative_to(REPO), number, match.group(1), first, last


@pytest.fixture(scope="module")
def reference():
    root = reference_root()
    if root is None:
        pytest.skip("reference checkout not available")
    return root


def test_there_are_citations_to_check():
    assert sum(1 for _ in _citations()) > 100


def test_every_citation_lies_inside_its_reference_file(reference):
    bad = []
    lengths = {}
    for where, number, target, first, last in _citations():
        file = reference / target
        if target not in lengths:
            lengths[target] = len(file.read_text().splitlines()) if file.is_file() else None
        n = lengths[target]
        if n is None or not 1 <= first <= last <= n:
            bad.append(f"{where}:{number}: {target}:{first}-{last} (file has {n} lines)")
    assert not bad, "\n".join(bad)


@pytest.mark.parametrize("method", ["_finite", "unscale_", "step", "update"])
def test_header_lands_on_the_gradscaler_stages(reference, method):
    """The header cites GradScaler's stages by range; each range must start on the method's def
    (or contain it, for a range that covers several methods)."""
    amp = (reference / "namitorch" / "amp.py").read_text().splitlines()
    header = (REPO / "include" / "namitorch_b200.h").read_text()
    defline = next(i for i, line in enumerate(amp, 1) if line.strip().startswith(f"def {method}("))
    ranges = [(int(a), int(b or a)) for a, b in re.findall(r"namitorch/amp\.py:(\d+)(?:-(\d+))?", header)]
    assert any(a <= defline <= b for a, b in ranges), (method, defline, ranges)
    for a, b in ranges:
        assert amp[a - 1].strip(), f"amp.py:{a} is a blank line"
