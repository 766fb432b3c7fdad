"""JSON model documents -> geo_cycle model IR ("geo_model_ir=8").

The front end of the geo_cycle runner (geo/geo_cycle_b200.h, the
``geo_cycle_b200`` command): it accepts the model documents of the reference's
compiler (tools/geo_model.py: root keys, node ops, initializers, optimizer,
training and dataset sections) with the same validation rules, and writes the
same IR text, so models move between the two unchanged.

    python -m geometricelementaryoperators_b200.model_ir validate model.json
    python -m geometricelementaryoperators_b200.model_ir compile model.json model.geoir
"""
from __future__ import annotations

import argparse
import json
import math
import os
import pathlib
import random
import re
import sys
import tempfile
from typing import Any

IR_VERSION = 8
NO_NODE = 2**32 - 1
NAME_PATTERN = re.compile(r"^[A-Za-z_][A-Za-z0-9_]{0,62}$")

OP_KINDS = {"input": 1, "target": 2, "parameter": 3, "constant": 4, "state": 5, "add": 6, "scale": 7, "gp": 8,
            "reverse": 9, "grade_project": 10, "grade_involution": 11, "clifford_conjugate": 12, "hadamard": 13,
            "tanh": 14, "sigmoid": 15, "normalize": 16, "squared_norm": 17}
LEAF_OPS = frozenset(("input", "target", "parameter", "constant", "state"))
ONE_INPUT_OPS = frozenset(("scale", "reverse", "grade_project", "grade_involution", "clifford_conjugate", "tanh",
                           "sigmoid", "normalize", "squared_norm"))
TWO_INPUT_OPS = frozenset(("add", "gp", "hadamard"))
CONSTRAINT_CODES = {"none": 0, "unit_euclidean": 1, "unit_vector_metric": 2, "even_versor": 3}
OPTIMIZER_CODES = {"sgd": 1, "adam": 2}
ROOT_KEYS = frozenset(("version", "dimension", "signature", "seed", "nodes", "loss", "output", "state_updates",
                       "optimizer", "training", "dataset", "metadata"))
NODE_KEYS = frozenset(("name", "op", "inputs", "input", "scalar", "grade", "constraint", "requires_grad", "init"))


class ModelError(ValueError):
    """A document the compiler rejects."""


def _number(value: Any, what: str) -> float:
    if isinstance(value, bool) or not isinstance(value, (int, float)):
        raise ModelError(f"{what} must be a number")
    out = float(value)
    if not math.isfinite(out):
        raise ModelError(f"{what} must be finite")
    return out


def _positive(value: Any, what: str) -> float:
    out = _number(value, what)
    if out <= 0.0:
        raise ModelError(f"{what} must be positive")
    return out


def _count(value: Any, what: str) -> int:
    if isinstance(value, bool) or not isinstance(value, int) or value <= 0:
        raise ModelError(f"{what} must be a positive integer")
    return value


def initial_value(spec: Any, blades: int, seed: int, name: str) -> tuple[float, ...]:
    """Initial coefficients of a node: a list, "zeros", "ones", "scalar:v",
    "basis:i:v" or "random[:seed[:scale]]" (uniform in [-scale, scale] from
    Python's Mersenne Twister seeded with (seed << 32) ^ sum of the name's code
    points; scale 0.1 by default)."""
    if isinstance(spec, list):
        if len(spec) != blades:
            raise ModelError(f"initializer for {name} must contain {blades} coefficients")
        return tuple(_number(v, f"initializer {name}[{i}]") for i, v in enumerate(spec))
    if spec is None or spec == "zeros":
        return (0.0,) * blades
    if spec == "ones":
        return (1.0,) * blades
    if not isinstance(spec, str):
        raise ModelError(f"invalid initializer for {name}")
    kind, *args = spec.split(":")
    if kind == "scalar" and len(args) == 1:
        out = [0.0] * blades
        out[0] = _number(float(args[0]), f"initializer {name}")
        return tuple(out)
    if kind == "basis" and len(args) == 2:
        blade = int(args[0])
        if not 0 <= blade < blades:
            raise ModelError(f"basis index for {name} is out of range")
        out = [0.0] * blades
        out[blade] = _number(float(args[1]), f"initializer {name}")
        return tuple(out)
    if kind == "random" and len(args) <= 2:
        stream_seed = int(args[0]) if args and args[0] else seed
        scale = _positive(float(args[1]), f"random scale for {name}") if len(args) == 2 else 0.1
        rng = random.Random((stream_seed << 32) ^ sum(ord(c) for c in name))
        return tuple(rng.uniform(-scale, scale) for _ in range(blades))
    raise ModelError(f"unsupported initializer '{spec}' for {name}")


def _section(document: dict, key: str) -> dict:
    value = document.get(key, {})
    if not isinstance(value, dict):
        raise ModelError(f"{key} must be an object")
    return value


def compile_document(document: Any) -> tuple[list[str], dict[str, int]]:
    """IR lines and a summary for a model document; ModelError when it is rejected."""
    if not isinstance(document, dict):
        raise ModelError("model root must be an object")
    extra = sorted(set(document) - ROOT_KEYS)
    if extra:
        raise ModelError(f"unknown root keys: {', '.join(extra)}")
    if document.get("version") != IR_VERSION:
        raise ModelError("version must be 8")
    n = document.get("dimension")
    if isinstance(n, bool) or not isinstance(n, int) or not 1 <= n <= 6:
        raise ModelError("dimension must be an integer from 1 through 6")
    signature = document.get("signature")
    if not isinstance(signature, list) or len(signature) != n or any(v not in (-1, 1) for v in signature):
        raise ModelError("signature must contain exactly dimension entries, each +1 or -1")
    seed = document.get("seed", 1)
    if isinstance(seed, bool) or not isinstance(seed, int) or seed < 0:
        raise ModelError("seed must be a nonnegative integer")
    raw_nodes = document.get("nodes")
    if not isinstance(raw_nodes, list) or not raw_nodes:
        raise ModelError("nodes must be a nonempty array")
    optimizer = _section(document, "optimizer")
    training = _section(document, "training")
    dataset = _section(document, "dataset")
    blades = 1 << n

    index_of: dict[str, int] = {}
    nodes: list[dict[str, Any]] = []
    for position, raw in enumerate(raw_nodes):
        if not isinstance(raw, dict):
            raise ModelError(f"node {position} must be an object")
        extra = sorted(set(raw) - NODE_KEYS)
        if extra:
            raise ModelError(f"node {position} has unknown keys: {', '.join(extra)}")
        name, op = raw.get("name"), raw.get("op")
        if not isinstance(name, str) or not NAME_PATTERN.fullmatch(name):
            raise ModelError(f"node {position} has an invalid name")
        if name in index_of:
            raise ModelError(f"duplicate node name '{name}'")
        if op not in OP_KINDS:
            raise ModelError(f"node {name} has unsupported op '{op}'")
        scalar = _number(raw.get("scalar", 0.0), f"node {name} scalar")
        grade = raw.get("grade", 0)
        if isinstance(grade, bool) or not isinstance(grade, int) or not 0 <= grade <= n:
            raise ModelError(f"node {name} grade is invalid")
        constraint_name = raw.get("constraint", "none")
        if constraint_name not in CONSTRAINT_CODES:
            raise ModelError(f"node {name} has invalid constraint")
        constraint = CONSTRAINT_CODES[constraint_name]
        grad = raw.get("requires_grad", op == "parameter")
        if not isinstance(grad, bool):
            raise ModelError(f"node {name} requires_grad must be boolean")
        value = initial_value(raw.get("init", "zeros"), blades, seed, name)
        left = right = NO_NODE
        if op in LEAF_OPS:
            if raw.get("inputs") is not None or raw.get("input") is not None:
                raise ModelError(f"leaf node {name} cannot have inputs")
            if op != "parameter" and constraint != 0:
                raise ModelError(f"constraint is valid only on parameter node {name}")
        elif op in ONE_INPUT_OPS:
            source = raw.get("input")
            if not isinstance(source, str) or source not in index_of:
                raise ModelError(f"node {name} must reference one earlier input")
            left = index_of[source]
            value, constraint, grad = (0.0,) * blades, 0, False
        else:
            sources = raw.get("inputs")
            if not isinstance(sources, list) or len(sources) != 2 or any(not isinstance(v, str) for v in sources):
                raise ModelError(f"node {name} must have two inputs")
            if any(v not in index_of for v in sources):
                raise ModelError(f"node {name} references an unknown or forward input")
            left, right = index_of[sources[0]], index_of[sources[1]]
            value, constraint, grad = (0.0,) * blades, 0, False
        if op == "normalize" and scalar == 0.0:
            scalar = 1e-12
        if op != "grade_project" and "grade" in raw:
            raise ModelError(f"grade is only valid for grade_project node {name}")
        if op not in ("scale", "normalize") and "scalar" in raw:
            raise ModelError(f"scalar is not valid for node {name}")
        index_of[name] = position
        nodes.append({"name": name, "op": op, "left": left, "right": right, "scalar": scalar, "grade": grade,
                      "constraint": constraint, "grad": int(grad), "value": value})

    loss, output = document.get("loss"), document.get("output")
    if not isinstance(loss, str) or loss not in index_of:
        raise ModelError("loss must name an existing node")
    if not isinstance(output, str) or output not in index_of:
        raise ModelError("output must name an existing node")
    updates = document.get("state_updates", {})
    if not isinstance(updates, dict):
        raise ModelError("state_updates must be an object")
    bindings = []
    for state, source in sorted(updates.items()):
        if state not in index_of or source not in index_of:
            raise ModelError("state update references an unknown node")
        if nodes[index_of[state]]["op"] != "state":
            raise ModelError(f"state update key '{state}' is not a state")
        bindings.append((index_of[state], index_of[source]))
    states = {i for i, node in enumerate(nodes) if node["op"] == "state"}
    bound = {s for s, _ in bindings}
    if states != bound:
        missing = [nodes[i]["name"] for i in sorted(states - bound)]
        raise ModelError(f"every state requires an update binding: {', '.join(missing)}")

    kind = optimizer.get("type", "adam")
    if kind not in OPTIMIZER_CODES:
        raise ModelError("optimizer.type must be sgd or adam")
    lr = _positive(optimizer.get("learning_rate", 0.01), "optimizer.learning_rate")
    beta1 = _number(optimizer.get("beta1", 0.9), "optimizer.beta1")
    beta2 = _number(optimizer.get("beta2", 0.999), "optimizer.beta2")
    eps = _positive(optimizer.get("epsilon", 1e-8), "optimizer.epsilon")
    if not (0.0 <= beta1 < 1.0 and 0.0 <= beta2 < 1.0):
        raise ModelError("optimizer beta values must be in [0,1)")
    epochs = _count(training.get("epochs", 1), "training.epochs")
    batch = _count(training.get("batch_size", 1), "training.batch_size")
    reset_each_epoch = training.get("reset_state_each_epoch", True)
    if not isinstance(reset_each_epoch, bool):
        raise ModelError("training.reset_state_each_epoch must be boolean")
    reset_column = dataset.get("reset_column", bool(states))
    if not isinstance(reset_column, bool):
        raise ModelError("dataset.reset_column must be boolean")

    g17 = "{:.17g}".format
    lines = ["geo_model_ir=8", f"dimension={n}", "signature=" + ",".join(str(v) for v in signature),
             f"optimizer={OPTIMIZER_CODES[kind]}", f"learning_rate={g17(lr)}", f"beta1={g17(beta1)}",
             f"beta2={g17(beta2)}", f"epsilon={g17(eps)}", f"epochs={epochs}", f"batch_size={batch}",
             f"reset_state_each_epoch={int(reset_each_epoch)}", f"reset_column={int(reset_column)}",
             f"node_count={len(nodes)}", f"loss={index_of[loss]}", f"output={index_of[output]}"]
    for i, node in enumerate(nodes):
        fields = [str(i), str(OP_KINDS[node["op"]]), node["name"], str(node["left"]), str(node["right"]),
                  g17(node["scalar"]), str(node["grade"]), str(node["constraint"]), str(node["grad"])]
        lines.append("node=" + ",".join(fields))
        lines.append("value=" + ",".join(g17(v) for v in node["value"]))
    lines.extend(f"state_update={s},{src}" for s, src in bindings)
    lines.append("end=1")
    summary = {"nodes": len(nodes), "parameters": sum(nd["op"] == "parameter" for nd in nodes),
               "inputs": sum(nd["op"] == "input" for nd in nodes), "targets": sum(nd["op"] == "target" for nd in nodes),
               "states": len(states), "blade_count": blades, "batch_size": batch}
    return lines, summary


def compile_file(path: pathlib.Path) -> tuple[list[str], dict[str, int]]:
    try:
        document = json.loads(pathlib.Path(path).read_text(encoding="utf-8"))
    except (OSError, json.JSONDecodeError) as exc:
        raise ModelError(str(exc)) from exc
    return compile_document(document)


def write_ir(path: pathlib.Path, lines: list[str]) -> None:
    """Writes the IR through a temporary file in the same directory, then renames it."""
    path = pathlib.Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    fd, tmp = tempfile.mkstemp(prefix=path.name + ".", suffix=".tmp", dir=path.parent)
    try:
        with os.fdopen(fd, "w", encoding="utf-8", newline="\n") as out:
            out.write("\n".join(lines) + "\n")
            out.flush()
            os.fsync(out.fileno())
        os.replace(tmp, path)
    except BaseException:
        try:
            os.unlink(tmp)
        except FileNotFoundError:
            pass
        raise


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description="Compile GEO V8 JSON model documents into geo_cycle model IR.")
    commands = parser.add_subparsers(dest="command", required=True)
    commands.add_parser("validate").add_argument("model", type=pathlib.Path)
    c = commands.add_parser("compile")
    c.add_argument("model", type=pathlib.Path)
    c.add_argument("output", type=pathlib.Path)
    args = parser.parse_args(argv)
    try:
        lines, summary = compile_file(args.model)
        info = " ".join(f"{k}={v}" for k, v in summary.items())
        if args.command == "compile":
            write_ir(args.output, lines)
            print(f"GEO_MODEL_COMPILE: PASS output={args.output} {info}")
        else:
            print(f"GEO_MODEL_VALIDATE: PASS {info}")
        return 0
    except (ModelError, OSError, ValueError) as exc:
        print(f"geo_model: {exc}", file=sys.stderr)
        return 1


if __name__ == "__main__":
    raise SystemExit(main())
