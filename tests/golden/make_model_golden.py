"""Generate tests/golden/model/: edge-case model documents and what the
reference's own compiler (tools/geo_model.py) does with each.

For every case this writes <case>.json (the document bytes, written verbatim so
syntax errors and line endings survive) and <case>.expect, which holds the
compiler's exit status, its stdout and stderr with the paths replaced by
placeholders, and the IR it wrote (empty when it rejected the document).
tests/test_model_compile.py runs this library's compiler on the same documents
and requires the same four things.

Usage: python tests/golden/make_model_golden.py --reference <reference tree>
"""
from __future__ import annotations

import argparse
import json
import pathlib
import shutil
import subprocess
import sys
import tempfile

OUT = pathlib.Path(__file__).resolve().parent / "model"


def base(**over) -> dict:
    doc = {"version": 8, "dimension": 2, "signature": [1, -1], "seed": 3,
           "nodes": [{"name": "x", "op": "input"}, {"name": "t", "op": "target"},
                     {"name": "w", "op": "parameter", "init": "random"},
                     {"name": "p", "op": "gp", "inputs": ["x", "w"]},
                     {"name": "nt", "op": "scale", "input": "t", "scalar": -1.0},
                     {"name": "r", "op": "add", "inputs": ["p", "nt"]},
                     {"name": "loss", "op": "squared_norm", "input": "r"}],
           "loss": "loss", "output": "p"}
    doc.update(over)
    return doc


def with_node(index: int, **fields) -> dict:
    doc = base()
    doc["nodes"][index] = {**doc["nodes"][index], **fields}
    return doc


def js(doc) -> str:
    return json.dumps(doc, indent=1)


def cases() -> dict[str, str]:
    c: dict[str, str] = {}
    # accepted documents with Python-number and JSON quirks
    c["version_float"] = js(base(version=8.0))
    c["signature_bool_and_float"] = js(base(signature=[True, -1.0]))
    c["huge_seed"] = js(base(seed=2**70 + 12345))
    c["seed_zero"] = js(base(seed=0))
    c["no_seed"] = js({k: v for k, v in base().items() if k != "seed"})
    c["random_negative_seed"] = js(with_node(2, init="random:-5:0.5"))
    c["random_empty_seed"] = js(with_node(2, init="random::0.3"))
    c["random_seed_only"] = js(with_node(2, init="random:77"))
    c["random_huge_seed"] = js(with_node(2, init="random:123456789012345678901234567890:2"))
    c["random_underscore_seed"] = js(with_node(2, init="random:1_000: 0.25 "))
    c["scalar_spaced_exponent"] = js(with_node(2, init="scalar: 2.5e-3 "))
    c["scalar_underscores"] = js(with_node(2, init="scalar:1_000.5"))
    c["basis_plus_sign"] = js(with_node(2, init="basis:+3:-0.0"))
    c["ones_and_list"] = js({**base(), "nodes": base()["nodes"][:2] + [
        {"name": "w", "op": "parameter", "init": [1, 2.5, -3e-7, 0]}] + base()["nodes"][3:]})
    c["constant_ones"] = js({**base(), "nodes": base()["nodes"] + [{"name": "k", "op": "constant", "init": "ones"}]})
    c["normalize_default_scalar"] = js({**base(), "nodes": base()["nodes"] + [
        {"name": "nrm", "op": "normalize", "input": "p"},
        {"name": "g1", "op": "grade_project", "input": "nrm", "grade": 1}]})
    c["metadata_nested_unicode"] = js(base(metadata={"note": "café ☃", "list": [1, {"a": None}]}))
    c["duplicate_root_key"] = '{"version": 7, "version": 8, ' + js(base())[1:]
    c["escaped_name"] = js(base()).replace('"name": "x"', '"name": "\\u0078x"').replace('"x", "w"', '"xx", "w"')
    c["crlf_lines"] = js(base()).replace("\n", "\r\n")
    c["state_model"] = js(base(nodes=base()["nodes"] + [{"name": "s", "op": "state"},
                                                        {"name": "s2", "op": "add", "inputs": ["s", "p"]}],
                               state_updates={"s": "s2"}, training={"epochs": 3, "batch_size": 2**70},
                               dataset={"reset_column": False}, optimizer={"type": "sgd", "beta2": 0.5}))
    c["adam_all_fields"] = js(base(optimizer={"type": "adam", "learning_rate": 1e-3, "beta1": 0, "beta2": 0.25,
                                              "epsilon": 1}, training={"reset_state_each_epoch": False}))
    c["requires_grad_false"] = js(with_node(2, requires_grad=False, constraint="unit_euclidean"))
    # JSON syntax errors
    c["syntax_missing_comma"] = '{"version": 8 "dimension": 2}'
    c["syntax_trailing_comma_object"] = '{"version": 8,}'
    c["syntax_trailing_comma_array"] = '{"signature": [1, -1,]}'
    c["syntax_unterminated_string"] = '{"version": 8, "nam'
    c["syntax_bad_escape"] = '{"version": "\\q"}'
    c["syntax_bad_unicode_escape"] = '{"version": "\\u12g4"}'
    c["syntax_extra_data"] = '{"version": 8}\n\n  {}'
    c["syntax_empty"] = ''
    c["syntax_control_char"] = '{"version": "a\tb"}'
    c["syntax_missing_colon"] = '{\n  "version" 8}'
    c["syntax_single_quotes"] = "{'version': 8}"
    c["nan_scalar"] = js(base()).replace('"scalar": -1.0', '"scalar": NaN')
    c["infinity_lr"] = js(base()).replace('"loss": "loss"', '"loss": "loss", "optimizer": {"learning_rate": Infinity}')
    # rule failures not covered by the runner fixtures
    c["dimension_float"] = js(base(dimension=2.0))
    c["dimension_seven"] = js(base(dimension=7))
    c["seed_negative"] = js(base(seed=-1))
    c["seed_bool"] = js(base(seed=True))
    c["nodes_empty"] = js(base(nodes=[]))
    c["node_not_object"] = js(base(nodes=[5]))
    c["node_unknown_keys"] = js(with_node(0, colour="red", alpha=1))
    c["name_digit_first"] = js(with_node(0, name="1x"))
    c["name_too_long"] = js(with_node(0, name="a" * 64))
    c["op_number"] = js(with_node(0, op=5))
    c["op_null"] = js(with_node(0, op=None))
    c["op_float"] = js(with_node(0, op=1.5e20))
    c["op_missing"] = js(base(nodes=[{"name": "x"}]))
    c["scalar_bool"] = js(with_node(4, scalar=True))
    c["scalar_string"] = js(with_node(4, scalar="1"))
    c["grade_too_big"] = js(with_node(0, grade=3))
    c["grade_on_input"] = js(with_node(0, grade=1))
    c["constraint_unknown"] = js(with_node(2, constraint="spherical"))
    c["requires_grad_int"] = js(with_node(2, requires_grad=1))
    c["leaf_with_input"] = js(with_node(0, input="t"))
    c["unary_missing_input"] = js(with_node(4, input="nope"))
    c["binary_one_input"] = js(with_node(3, inputs=["x"]))
    c["binary_forward_input"] = js(with_node(3, inputs=["x", "r"]))
    c["init_bad_kind"] = js(with_node(2, init=5))
    c["init_scalar_text"] = js(with_node(2, init="scalar:abc"))
    c["init_scalar_nan"] = js(with_node(2, init="scalar:nan"))
    c["init_scalar_inf"] = js(with_node(2, init="scalar:-Infinity"))
    c["init_basis_hex"] = js(with_node(2, init="basis:0x3:1"))
    c["init_basis_range"] = js(with_node(2, init="basis:4:1"))
    c["init_basis_negative"] = js(with_node(2, init="basis:-1:1"))
    c["init_random_zero_scale"] = js(with_node(2, init="random:1:0"))
    c["init_random_empty_scale"] = js(with_node(2, init="random:1:"))
    c["init_random_bad_seed"] = js(with_node(2, init="random:1.5"))
    c["init_random_four_parts"] = js(with_node(2, init="random:1:2:3"))
    c["init_list_entry"] = js(with_node(2, init=[1, "2", 3, 4]))
    c["init_on_unary_ignored_but_checked"] = js(with_node(4, init="scalar:zz"))
    c["output_missing"] = js({k: v for k, v in base().items() if k != "output"})
    c["state_unbound"] = js(base(nodes=base()["nodes"] + [{"name": "s", "op": "state"}, {"name": "s9", "op": "state"}]))
    c["state_update_not_state"] = js(base(state_updates={"x": "p"}))
    c["state_update_unknown"] = js(base(state_updates={"q": "p"}))
    c["state_updates_list"] = js(base(state_updates=[]))
    c["optimizer_list"] = js(base(optimizer=[]))
    c["optimizer_type_bad"] = js(base(optimizer={"type": "rmsprop"}))
    c["epsilon_zero"] = js(base(optimizer={"epsilon": 0}))
    c["beta2_one"] = js(base(optimizer={"beta2": 1}))
    c["training_string"] = js(base(training="fast"))
    c["batch_zero"] = js(base(training={"batch_size": 0}))
    c["reset_each_epoch_int"] = js(base(training={"reset_state_each_epoch": 0}))
    c["dataset_reset_string"] = js(base(dataset={"reset_column": "yes"}))
    c["not_utf8"] = None  # written as bytes below
    return c


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", required=True, type=pathlib.Path, help="root of the reference source tree")
    compiler = ap.parse_args().reference.resolve() / "tools" / "geo_model.py"
    if not compiler.exists():
        raise SystemExit(f"{compiler} not found: --reference must name the reference tree")
    if OUT.exists():
        shutil.rmtree(OUT)
    OUT.mkdir(parents=True)
    with tempfile.TemporaryDirectory() as tmp:
        for name, text in cases().items():
            src = OUT / f"{name}.json"
            if text is None:
                src.write_bytes(b'{"version": 8, "metadata": "\xff"}')
            else:
                src.write_bytes(text.encode("utf-8"))
            ir = pathlib.Path(tmp) / f"{name}.geoir"
            res = subprocess.run([sys.executable, str(compiler), "compile", str(src), str(ir)], capture_output=True,
                                 text=True)
            expect = {"status": res.returncode,
                      "stdout": res.stdout.replace(str(ir), "<ir>").replace(str(src), "<model>"),
                      "stderr": res.stderr.replace(str(ir), "<ir>").replace(str(src), "<model>"),
                      "ir": ir.read_text() if ir.exists() else ""}
            (OUT / f"{name}.expect").write_text(json.dumps(expect, indent=1) + "\n")
    print(f"wrote {len(cases())} cases to {OUT}")


if __name__ == "__main__":
    main()
