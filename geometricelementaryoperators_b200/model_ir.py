"""JSON model documents -> geo_cycle model IR ("geo_model_ir=8"), from Python.

The compiler itself is native: geo_b200_model_compile_text in libgeo_b200.so
(geo/geo_cycle_b200.h), the same code behind ``geo_cycle_b200 compile`` and
``geo_cycle_b200 validate``. This module only hands it the document text and
returns what it produced.

    python -m geometricelementaryoperators_b200.model_ir validate model.json
    python -m geometricelementaryoperators_b200.model_ir compile model.json model.geoir
"""
from __future__ import annotations

import ctypes
import pathlib
import sys

from . import abi


class ModelError(ValueError):
    """A document the compiler rejects (the message is the compiler's)."""


def _lib() -> ctypes.CDLL:
    lib = abi.lib()
    fn = lib.geo_b200_model_compile_text
    if fn.argtypes is None:
        fn.argtypes = [ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p,
                       ctypes.c_size_t, ctypes.c_char_p, ctypes.c_size_t]
        fn.restype = ctypes.c_int
        lib.geo_b200_model_free_text.argtypes = [ctypes.c_void_p]
        lib.geo_b200_model_free_text.restype = None
        lib.geo_b200_model_compile.argtypes = [ctypes.c_char_p, ctypes.c_char_p]
        lib.geo_b200_model_compile.restype = ctypes.c_int
    return lib


def compile_bytes(document: bytes) -> tuple[list[str], dict[str, int]]:
    """IR lines and the summary counts of a document given as UTF-8 bytes."""
    lib = _lib()
    ir = ctypes.c_void_p()
    summary = ctypes.create_string_buffer(512)
    error = ctypes.create_string_buffer(2048)
    if not lib.geo_b200_model_compile_text(document, len(document), ctypes.byref(ir), summary, len(summary), error,
                                           len(error)):
        raise ModelError(error.value.decode("utf-8", "replace"))
    try:
        text = ctypes.string_at(ir.value).decode("utf-8")
    finally:
        lib.geo_b200_model_free_text(ir)
    counts = {k: int(v) for k, v in (item.split("=") for item in summary.value.decode().split())}
    return text.splitlines(), counts


def compile_file(path) -> tuple[list[str], dict[str, int]]:
    try:
        data = pathlib.Path(path).read_bytes()
    except OSError as exc:
        raise ModelError(str(exc)) from exc
    return compile_bytes(data)


def main(argv: list[str] | None = None) -> int:
    args = list(sys.argv[1:] if argv is None else argv)
    if len(args) == 3 and args[0] == "compile":
        sys.stdout.flush()
        return 0 if _lib().geo_b200_model_compile(args[1].encode(), args[2].encode()) else 1
    if len(args) == 2 and args[0] == "validate":
        try:
            _, counts = compile_file(args[1])
        except ModelError as exc:
            print(f"geo_model: {exc}", file=sys.stderr)
            return 1
        print("GEO_MODEL_VALIDATE: PASS " + " ".join(f"{k}={v}" for k, v in counts.items()))
        return 0
    print("usage: model_ir validate <model.json> | compile <model.json> <model.geoir>", file=sys.stderr)
    return 2


if __name__ == "__main__":
    raise SystemExit(main())
