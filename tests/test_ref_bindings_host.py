"""The reference binding's ctypes declarations (tests/golden/
ref_ctypes_signatures.json, from python/ndtensors_rs/src/ndtensors_rs/_lib.py)
against this library, without a device: every declared symbol is exported,
the C header declares it with the same parameter types in the same order and
the same result type, and the host-side calls (creation, queries, element
access, NULL handling) behave as the reference's tests expect."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

import refbind

HEADER = Path(__file__).resolve().parent.parent / "include" / "ndtensors_capi.h"

# ctypes spelling -> the C parameter types it may marshal
C_OF = {
    "c_void_p": {"ndt_tensor_f64*", "const ndt_tensor_f64*"},
    "POINTER(c_size_t)": {"const size_t*", "size_t*"},
    "c_size_t": {"size_t"},
    "POINTER(c_int)": {"int*"},
    "POINTER(c_long)": {"const long*"},
    "POINTER(c_double)": {"const double*", "double*"},
    "c_double": {"double"},
    "POINTER(c_void_p)": {"ndt_tensor_f64**"},
    "c_int": {"int"},
    "None": {"void"},
}


def header_prototypes():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    protos = {}
    for m in re.finditer(r"([A-Za-z_][\w\s\*]*?)\b(ndt_\w+)\s*\(([^;{]*?)\)\s*;", text, flags=re.S):
        ret = " ".join(m.group(1).split()).replace(" *", "*")
        params = []
        for p in m.group(3).split(","):
            p = " ".join(p.split())
            if not p or p == "void":
                continue
            toks = p.replace("*", " * ").split()
            # drop the parameter name
            toks = toks[:-1] if toks and toks[-1] not in ("*",) and len(toks) > 1 else toks
            params.append(" ".join(toks).replace(" *", "*").replace("* ", "*"))
        protos[m.group(2)] = (ret.split()[-1] if ret.split() else ret, params, ret)
    return protos


def test_every_reference_declaration_matches_the_header():
    protos = header_prototypes()
    for name, sig in refbind.declarations().items():
        assert name in protos, f"{name} not declared in the header"
        ret_full, params = protos[name][2], protos[name][1]
        assert len(params) == len(sig["argtypes"]), (name, params, sig["argtypes"])
        for c, p in zip(sig["argtypes"], params):
            assert p in C_OF[c], (name, c, p)
        assert ret_full.replace("const ", "const ") in C_OF[sig["restype"]] or \
            (sig["restype"] == "c_void_p" and ret_full.endswith("*")), (name, sig["restype"], ret_full)


def test_reference_binding_loads_and_binds_every_symbol():
    lib = refbind.load()
    for name in refbind.declarations():
        assert getattr(lib, name) is not None


def test_host_calls_through_reference_declarations():
    lib = refbind.load()
    st = ctypes.c_int(-999)
    shape = (ctypes.c_size_t * 3)(2, 3, 4)
    t = lib.ndt_tensor_f64_zeros(shape, 3, ctypes.byref(st))
    assert st.value == 0 and t
    assert lib.ndt_tensor_f64_ndim(t) == 3 and lib.ndt_tensor_f64_len(t) == 24
    out = (ctypes.c_size_t * 3)()
    assert lib.ndt_tensor_f64_shape(t, out) == 0 and list(out) == [2, 3, 4]
    v = ctypes.c_double()
    assert lib.ndt_tensor_f64_get_linear(t, 99, ctypes.byref(v)) == -3  # out of bounds
    c = lib.ndt_tensor_f64_clone(t)
    assert c
    lib.ndt_tensor_f64_release(c)
    lib.ndt_tensor_f64_release(t)
    lib.ndt_tensor_f64_release(None)  # NULL-safe
    assert lib.ndt_tensor_f64_ndim(None) == 0 and lib.ndt_tensor_f64_len(None) == 0
    # shape == NULL with ndim > 0 -> NDT_INVALID_ARGUMENT; a NULL status pointer -> NULL
    assert not lib.ndt_tensor_f64_zeros(None, 2, ctypes.byref(st)) and st.value == -1
    assert not lib.ndt_tensor_f64_zeros(shape, 3, None)
    data = (ctypes.c_double * 5)(*range(5))
    assert not lib.ndt_tensor_f64_from_data(data, 5, shape, 3, ctypes.byref(st)) and st.value == -2


@pytest.mark.parametrize("missing", ["ndt_tensor_f64_data_mut", "ndt_tensor_f64_contract_jvp"])
def test_reference_binding_leaves_out_what_it_leaves_out(missing):
    """The reference binding declares neither data_mut nor contract_jvp; the
    library still exports both (the Julia binding and C callers use them)."""
    assert missing not in refbind.declarations()
    assert hasattr(ctypes.CDLL(str(refbind.LIB)), missing)
