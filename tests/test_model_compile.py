"""The model compiler in the library (geo_b200_model_compile, the
`geo_cycle_b200 compile | validate` commands) against the reference's compiler
(tools/geo_model.py) on edge-case documents: JSON syntax errors with their
positions, Python-number quirks (8.0 as a version, true as a signature entry,
integers of any length), every initialiser form and its failures, unicode
escapes, CRLF text, invalid UTF-8 and every validation rule. For each document
the exit status, stdout, stderr and the IR bytes must equal what the reference
compiler produced (tests/golden/model, made by tests/golden/make_model_golden.py).
"""
from __future__ import annotations

import json
import pathlib
import subprocess

import pytest

from geometricelementaryoperators_b200 import build

CASES = pathlib.Path(__file__).resolve().parent / "golden" / "model"
NAMES = sorted(p.stem for p in CASES.glob("*.json"))


@pytest.mark.parametrize("name", NAMES)
def test_compile_matches_reference_compiler(name, tmp_path):
    expect = json.loads((CASES / f"{name}.expect").read_text())
    src, ir = CASES / f"{name}.json", tmp_path / f"{name}.geoir"
    res = subprocess.run([str(build.CLI), "compile", str(src), str(ir)], capture_output=True, text=True,
                         timeout=60)
    assert res.returncode == expect["status"], res.stderr
    assert res.stdout.replace(str(ir), "<ir>").replace(str(src), "<model>") == expect["stdout"]
    assert res.stderr.replace(str(ir), "<ir>").replace(str(src), "<model>") == expect["stderr"]
    assert (ir.read_text() if ir.exists() else "") == expect["ir"]


def test_cases_cover_acceptance_and_rejection():
    status = [json.loads((CASES / f"{n}.expect").read_text())["status"] for n in NAMES]
    assert len(NAMES) >= 80 and status.count(0) >= 20 and status.count(1) >= 60
