"""Every `file:line` citation of the reference resolves inside the cited file.

Headers, integration notes, design notes, the package, the oracle and the tests
cite the reference (KristiTopollai/stochastic-rounding-pytorch) as
`path:first-last`.  A citation is checked when a checkout of the reference is
available (``$SR_STATES_REFERENCE``, else the conventional checkout location):
the file must exist, at the cited path or under its ``sr_states/`` package,
and the line range must lie inside it.  Without a checkout the test is skipped.
"""

import os
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
REFERENCE = Path(os.environ.get("SR_STATES_REFERENCE", "/root/reference"))
CITATION = re.compile(r"([A-Za-z0-9_./-]+\.(?:py|md|toml|c|h|cu))[:](\d+)(?:-(\d+))?")


def _cited_files():
    files = sorted(ROOT.glob("include/*.h")) + [ROOT / "INTEGRATION.md", ROOT / "DESIGN.md",
                                                  ROOT / "bench.py", ROOT / "__graft_entry__.py"]
    for tree, suffixes in (("stochastic-rounding-pytorch_b200", (".py", ".cu", ".cuh", ".cpp")),
                           ("oracle", (".py", ".c")), ("tests", (".py",))):
        files += sorted(p for p in (ROOT / tree).rglob("*")
                        if p.suffix in suffixes and "_build" not in p.parts)
    return files


def _resolve(path):
    for candidate in (REFERENCE / path, REFERENCE / "sr_states" / path):
        if candidate.is_file():
            return candidate
    return None


@pytest.mark.skipif(not (REFERENCE / "sr_states").is_dir(), reason="no reference checkout")
def test_every_reference_citation_resolves_inside_the_cited_file():
    lengths, problems, checked = {}, [], 0
    for source in _cited_files():
        for match in CITATION.finditer(source.read_text()):
            cited, first = match.group(1), int(match.group(2))
            last = int(match.group(3) or first)
            target = _resolve(cited)
            where = f"{source.relative_to(ROOT)}: {match.group(0)}"
            if target is None:
                # Citations of this repository's own files are not reference citations.
                if (ROOT / cited).is_file() or (ROOT / "stochastic-rounding-pytorch_b200" /
                                                cited).is_file():
                    continue
                problems.append(f"{where} (no such file in the reference)")
                continue
            if target not in lengths:
                lengths[target] = len(target.read_text().splitlines())
            checked += 1
            if not 1 <= first <= last <= lengths[target]:
                problems.append(f"{where} (the file has {lengths[target]} lines)")
    assert checked > 50
    assert not problems, "\n".join(problems)
