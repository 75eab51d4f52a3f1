"""Writes tests/golden/ref_ctypes_signatures.json.

The reference's Python binding declares the C ABI to ctypes in
python/ndtensors_rs/src/ndtensors_rs/_lib.py (_declare_functions, :58-206):
for every symbol an argtypes list and a restype.  This script reads that file
as text (its syntax tree; nothing of it is imported or executed) and records
each declaration as data: the symbol, the ctypes spelling of every argument
and of the result.  The tests bind libndtensors_capi.so with exactly these
declarations, as the reference's binding would, and run the reference's
known answers through them.  Run here (where the reference is present):
    python tests/golden/make_ref_ctypes_fixture.py
"""

from __future__ import annotations

import ast
import json
from pathlib import Path

REF = Path("/root/reference/python/ndtensors_rs/src/ndtensors_rs/_lib.py")
OUT = Path(__file__).resolve().parent / "ref_ctypes_signatures.json"


def spell(node) -> str:
    """ctypes.c_size_t -> 'c_size_t'; ctypes.POINTER(ctypes.c_int) -> 'POINTER(c_int)'; None -> 'None'."""
    if isinstance(node, ast.Constant) and node.value is None:
        return "None"
    if isinstance(node, ast.Attribute):
        return node.attr
    if isinstance(node, ast.Call):
        return f"{spell(node.func)}({', '.join(spell(a) for a in node.args)})"
    raise ValueError(ast.dump(node))


def main() -> None:
    tree = ast.parse(REF.read_text())
    sigs = {}
    for node in ast.walk(tree):
        if not isinstance(node, ast.Assign) or len(node.targets) != 1:
            continue
        tgt = node.targets[0]
        if not (isinstance(tgt, ast.Attribute) and isinstance(tgt.value, ast.Attribute)):
            continue
        name, field = tgt.value.attr, tgt.attr
        if not name.startswith("ndt_") or field not in ("argtypes", "restype"):
            continue
        entry = sigs.setdefault(name, {})
        if field == "argtypes":
            entry["argtypes"] = [spell(e) for e in node.value.elts]
        else:
            entry["restype"] = spell(node.value)
        entry["line"] = node.lineno
    out = {"generated_by": "tests/golden/make_ref_ctypes_fixture.py",
           "source": "python/ndtensors_rs/src/ndtensors_rs/_lib.py (_declare_functions)",
           "functions": dict(sorted(sigs.items()))}
    OUT.write_text(json.dumps(out, indent=1) + "\n")
    print(f"{len(sigs)} declarations -> {OUT}")


if __name__ == "__main__":
    main()
