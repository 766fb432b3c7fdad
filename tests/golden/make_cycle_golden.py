"""Fixtures for the geo_cycle model runner and its model front end.

Writes, under tests/golden/cycle/, a set of model documents (JSON), their IR as
compiled by the reference's own compiler (tools/geo_model.py), seeded CSV
datasets, and what the reference's own runner (tools/geo_cycle*.c, built by
`make -C oracle ref` into oracle/_ref/geo_cycle) produces from them: trained
checkpoints, predictions, exported C headers and its printed PASS lines. The
tests compare this library's front end (model_ir.py, CPU) and runner
(geo_cycle_b200, GPU) against these files.

Usage: python tests/golden/make_cycle_golden.py --reference <reference tree>
"""
from __future__ import annotations

import json
import pathlib
import shutil
import subprocess
import sys

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from geometricelementaryoperators_b200.synthetic import splitmix_uniform  # noqa: E402

REF: pathlib.Path | None = None  # the reference tree, from --reference
RUNNER = ROOT / "oracle" / "_ref" / "geo_cycle"
OUT = pathlib.Path(__file__).resolve().parent / "cycle"


def tail(prediction: str, target: str) -> list[dict]:
    return [{"name": "negative_target", "op": "scale", "input": target, "scalar": -1.0},
            {"name": "residual", "op": "add", "inputs": [prediction, "negative_target"]},
            {"name": "loss", "op": "squared_norm", "input": "residual"}]


def model(n, sig, nodes, output, optimizer, lr, epochs, batch, **extra) -> dict:
    doc = {"version": 8, "dimension": n, "signature": sig, "nodes": nodes + tail(output, "target"), "loss": "loss",
           "output": output, "optimizer": {"type": optimizer, "learning_rate": lr},
           "training": {"epochs": epochs, "batch_size": batch}}
    doc.update(extra)
    return doc


def documents() -> dict[str, dict]:
    docs = {}
    # W recovery: Cl(2,0), y = x w, SGD
    docs["gp_exact"] = model(2, [1, 1], [{"name": "x", "op": "input"}, {"name": "target", "op": "target"},
                                         {"name": "w", "op": "parameter", "init": "zeros"},
                                         {"name": "prediction", "op": "gp", "inputs": ["x", "w"]}],
                             "prediction", "sgd", 0.5, 40, 4)
    # two parameters with a tanh layer, Cl(3,1), Adam
    docs["mlp"] = model(4, [1, 1, 1, -1], [
        {"name": "x", "op": "input"}, {"name": "target", "op": "target"},
        {"name": "w1", "op": "parameter", "init": "random:3:0.3"},
        {"name": "w2", "op": "parameter", "init": "random:4:0.3"},
        {"name": "bias", "op": "constant", "init": "scalar:0.25"},
        {"name": "hidden", "op": "gp", "inputs": ["x", "w1"]},
        {"name": "act", "op": "tanh", "input": "hidden"},
        {"name": "shifted", "op": "add", "inputs": ["act", "bias"]},
        {"name": "prediction", "op": "gp", "inputs": ["w2", "shifted"]}],
        "prediction", "adam", 0.02, 3, 8)
    # every op kind, Cl(6,0), Adam (the batched path of the runner)
    docs["all_ops"] = model(6, [1] * 6, [
        {"name": "x", "op": "input"}, {"name": "target", "op": "target"},
        {"name": "w1", "op": "parameter", "init": "random:11:0.2"},
        {"name": "w2", "op": "parameter", "init": "basis:3:0.75"},
        {"name": "c", "op": "constant", "init": "scalar:1.25"},
        {"name": "gp", "op": "gp", "inputs": ["x", "w1"]},
        {"name": "act", "op": "tanh", "input": "gp"},
        {"name": "gate", "op": "sigmoid", "input": "w2"},
        {"name": "gated", "op": "hadamard", "inputs": ["act", "gate"]},
        {"name": "rev", "op": "reverse", "input": "gated"},
        {"name": "inv", "op": "grade_involution", "input": "rev"},
        {"name": "conj", "op": "clifford_conjugate", "input": "inv"},
        {"name": "proj", "op": "grade_project", "input": "conj", "grade": 2},
        {"name": "shift", "op": "add", "inputs": ["proj", "c"]},
        {"name": "prediction", "op": "normalize", "input": "shift"}],
        "prediction", "adam", 0.01, 2, 16)
    # a unit-norm parameter (constraint), Cl(3,0), Adam
    docs["constraint"] = model(3, [1, 1, 1], [
        {"name": "x", "op": "input"}, {"name": "target", "op": "target"},
        {"name": "r", "op": "parameter", "init": "basis:0:1.0", "constraint": "unit_euclidean"},
        {"name": "prediction", "op": "gp", "inputs": ["x", "r"]}],
        "prediction", "adam", 0.05, 2, 5)
    # recurrence: h = tanh(x w + state u), reset column, SGD (the per-row path)
    docs["recurrent"] = model(2, [1, -1], [
        {"name": "x", "op": "input"}, {"name": "target", "op": "target"},
        {"name": "h", "op": "state", "init": "zeros"},
        {"name": "w", "op": "parameter", "init": "random:5:0.5"},
        {"name": "u", "op": "parameter", "init": "random:6:0.5"},
        {"name": "xw", "op": "gp", "inputs": ["x", "w"]},
        {"name": "hu", "op": "gp", "inputs": ["h", "u"]},
        {"name": "pre", "op": "add", "inputs": ["xw", "hu"]},
        {"name": "prediction", "op": "tanh", "input": "pre"}],
        "prediction", "sgd", 0.05, 2, 3, state_updates={"h": "prediction"})
    # the same MLP at 1 and 2 epochs: continuous vs resumed training
    for epochs in (1, 2):
        d = json.loads(json.dumps(docs["mlp"]))
        d["training"]["epochs"] = epochs
        docs[f"resume{epochs}"] = d
    return docs


def invalid_documents() -> dict[str, object]:
    """Documents the compiler must reject (one rule each)."""
    good = documents()["gp_exact"]

    def edit(fn):
        d = json.loads(json.dumps(good))
        fn(d)
        return d

    return {
        "bad_version": edit(lambda d: d.update(version=7)),
        "bad_signature": edit(lambda d: d.update(signature=[1, 2])),
        "unknown_root": edit(lambda d: d.update(extra=1)),
        "duplicate_name": edit(lambda d: d["nodes"].append({"name": "x", "op": "input"})),
        "forward_input": edit(lambda d: d["nodes"].insert(3, {"name": "early", "op": "gp", "inputs": ["x", "late"]})),
        "bad_op": edit(lambda d: d["nodes"].append({"name": "odd", "op": "cube", "input": "x"})),
        "scalar_on_gp": edit(lambda d: d["nodes"][3].update(scalar=2.0)),
        "leaf_constraint": edit(lambda d: d["nodes"][0].update(constraint="unit_euclidean")),
        "bad_init": edit(lambda d: d["nodes"][2].update(init="gaussian")),
        "short_init": edit(lambda d: d["nodes"][2].update(init=[1.0, 2.0])),
        "missing_loss": edit(lambda d: d.update(loss="nothing")),
        "bad_lr": edit(lambda d: d["optimizer"].update(learning_rate=0.0)),
        "bad_beta": edit(lambda d: d["optimizer"].update(beta1=1.0)),
        "bool_epochs": edit(lambda d: d["training"].update(epochs=True)),
        "not_an_object": [1, 2, 3],
    }


def dataset(name: str, doc: dict, rows: int, seed: int, with_target: bool) -> np.ndarray:
    n = doc["dimension"]
    N = 1 << n
    inputs = sum(1 for nd in doc["nodes"] if nd["op"] == "input")
    targets = sum(1 for nd in doc["nodes"] if nd["op"] == "target") if with_target else 0
    reset = doc.get("dataset", {}).get("reset_column", any(nd["op"] == "state" for nd in doc["nodes"]))
    data = splitmix_uniform(seed, (rows, (inputs + targets) * N))
    if name == "gp_exact" and with_target:
        # targets are exact products with a hidden multivector
        truth = np.array([0.75, -1.25, 0.5, 1.0])
        sig = doc["signature"]
        for r in range(rows):
            x = data[r, :N]
            y = np.zeros(N)
            for a in range(N):
                for b in range(N):
                    s = 1
                    for axis in range(n):
                        if (a >> axis) & 1:
                            if bin(b & ((1 << axis) - 1)).count("1") & 1:
                                s = -s
                            if (b >> axis) & 1:
                                s *= sig[axis]
                    y[a ^ b] += x[a] * truth[b] * s
            data[r, N:2 * N] = y
    if reset:
        flags = np.zeros((rows, 1))
        flags[::7] = 1.0
        data = np.concatenate([flags, data], axis=1)
    return data


def write_csv(path: pathlib.Path, data: np.ndarray) -> None:
    path.write_text("\n".join(",".join(format(float(v), ".17g") for v in row) for row in data) + "\n")


def run(cmd: list[str]) -> subprocess.CompletedProcess:
    return subprocess.run(cmd, capture_output=True, text=True)


def main() -> None:
    global REF, COMPILER
    import argparse

    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", required=True, type=pathlib.Path, help="root of the reference source tree")
    REF = ap.parse_args().reference.resolve()
    COMPILER = REF / "tools" / "geo_model.py"
    if not COMPILER.exists():
        raise SystemExit(f"{COMPILER} not found: --reference must name the reference tree")
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), "ref", f"REF={REF}"], check=True)
    if OUT.exists():
        shutil.rmtree(OUT)
    (OUT / "invalid").mkdir(parents=True)
    docs = documents()
    for i, (name, doc) in enumerate(docs.items()):
        js = OUT / f"{name}.json"
        js.write_text(json.dumps(doc, indent=2, sort_keys=True) + "\n")
        ir = OUT / f"{name}.geoir"
        res = run([sys.executable, str(COMPILER), "compile", str(js), str(ir)])
        assert res.returncode == 0, res.stderr
        (OUT / f"{name}.compile.txt").write_text(res.stdout.replace(str(ir), f"{name}.geoir"))
        base = name if not name.startswith("resume") else "resume"
        rows = {"gp_exact": 8, "mlp": 48, "all_ops": 48, "constraint": 21, "recurrent": 30, "resume": 48}[base]
        seed = 1000 + (i if not name.startswith("resume") else 99)
        train = OUT / f"{base}.csv"
        pred_in = OUT / f"{base}.predict_in.csv"
        if not train.exists():
            write_csv(train, dataset(base, doc, rows, seed, True))
            write_csv(pred_in, dataset(base, doc, 6, seed + 500, False))
        ckpt = OUT / f"{name}.checkpoint"
        res = run([str(RUNNER), "train", str(ir), str(train), str(ckpt)])
        assert res.returncode == 0, (name, res.stderr)
        (OUT / f"{name}.train.txt").write_text(res.stdout.replace(str(ckpt), f"{name}.checkpoint"))
        pred = OUT / f"{name}.predict.csv"
        res = run([str(RUNNER), "predict", str(ir), str(ckpt), str(pred_in), str(pred)])
        assert res.returncode == 0, (name, res.stderr)
        header = OUT / f"{name}.h"
        res = run([str(RUNNER), "export-c", str(ir), str(ckpt), str(header), name])
        assert res.returncode == 0, (name, res.stderr)
        res = run([str(RUNNER), "check", str(ir)])
        assert res.returncode == 0, (name, res.stderr)
        (OUT / f"{name}.check.txt").write_text(res.stdout)
    for name, doc in invalid_documents().items():
        js = OUT / "invalid" / f"{name}.json"
        js.write_text(json.dumps(doc, indent=2, sort_keys=True) + "\n")
        res = run([sys.executable, str(COMPILER), "validate", str(js)])
        assert res.returncode == 1, name
        (OUT / "invalid" / f"{name}.stderr.txt").write_text(res.stderr.replace(str(js), f"{name}.json"))
    size = sum(p.stat().st_size for p in OUT.rglob("*") if p.is_file())
    print(f"wrote {OUT} ({size} bytes)")


if __name__ == "__main__":
    main()
