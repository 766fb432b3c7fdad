"""The model front end (geometricelementaryoperators_b200.model_ir) against the
reference's compiler (tools/geo_model.py): identical IR bytes and PASS lines for
every fixture document, and the same rejections with the same messages
(fixtures made by tests/golden/make_cycle_golden.py)."""
from __future__ import annotations

import pathlib
import subprocess
import sys

import pytest

from geometricelementaryoperators_b200 import model_ir

CYCLE = pathlib.Path(__file__).resolve().parent / "golden" / "cycle"
ROOT = pathlib.Path(__file__).resolve().parent.parent
DOCS = sorted(p.stem for p in CYCLE.glob("*.json"))
INVALID = sorted(p.stem for p in (CYCLE / "invalid").glob("*.json"))


@pytest.mark.parametrize("name", DOCS)
def test_compiled_ir_is_the_reference_compilers(name, tmp_path):
    out = tmp_path / f"{name}.geoir"
    res = subprocess.run([sys.executable, "-m", "geometricelementaryoperators_b200.model_ir", "compile",
                          str(CYCLE / f"{name}.json"), str(out)], capture_output=True, text=True, cwd=ROOT)
    assert res.returncode == 0, res.stderr
    assert out.read_bytes() == (CYCLE / f"{name}.geoir").read_bytes()
    assert res.stdout.replace(str(out), f"{name}.geoir") == (CYCLE / f"{name}.compile.txt").read_text()


@pytest.mark.parametrize("name", INVALID)
def test_rejections_match(name, capsys):
    assert model_ir.main(["validate", str(CYCLE / "invalid" / f"{name}.json")]) == 1
    err = capsys.readouterr().err.replace(str(CYCLE / "invalid" / f"{name}.json"), f"{name}.json")
    assert err == (CYCLE / "invalid" / f"{name}.stderr.txt").read_text()


def test_validate_summary():
    lines, summary = model_ir.compile_file(CYCLE / "all_ops.json")
    assert lines[0] == "geo_model_ir=8" and lines[-1] == "end=1"
    assert summary == {"nodes": 18, "parameters": 2, "inputs": 1, "targets": 1, "states": 0, "blade_count": 64,
                       "batch_size": 16}
