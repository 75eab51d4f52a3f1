"""libndtensors_capi.so bound the way the reference's Python binding binds it.

TEST INFRASTRUCTURE.  tests/golden/ref_ctypes_signatures.json holds the
ctypes declarations of python/ndtensors_rs/src/ndtensors_rs/_lib.py
(_declare_functions, :58-206), read from that file as data.  `load()` opens
a fresh handle on this library and applies exactly those argtypes and
restypes, so calls go through the same marshalling the reference's binding
uses; `RefEngine` drives the reference's f64 C ABI through it with nothing
of this repository's Python package in between.
"""

from __future__ import annotations

import ctypes
import json
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
FIXTURE = ROOT / "tests" / "golden" / "ref_ctypes_signatures.json"
LIB = ROOT / "ndtensors-rs_b200" / "lib" / "libndtensors_capi.so"


def ctype(spelling: str):
    """'c_size_t' -> ctypes.c_size_t, 'POINTER(c_int)' -> POINTER(c_int), 'None' -> None."""
    if spelling == "None":
        return None
    if spelling.startswith("POINTER(") and spelling.endswith(")"):
        return ctypes.POINTER(ctype(spelling[8:-1]))
    return getattr(ctypes, spelling)


def declarations():
    return json.loads(FIXTURE.read_text())["functions"]


def load(path: Path = LIB) -> ctypes.CDLL:
    lib = ctypes.CDLL(str(path))
    for name, sig in declarations().items():
        f = getattr(lib, name)
        f.argtypes = [ctype(a) for a in sig["argtypes"]]
        f.restype = ctype(sig["restype"])
    return lib


class RefEngine:
    """permutedims / contract / contract_vjp of f64 tensors through the
    reference's declarations (tensor.py / ops.py of the reference binding do
    the same calls: from_data on Fortran-ordered data, the operation, then
    shape + data to read the result)."""

    name = "reference-binding"

    def __init__(self, lib: ctypes.CDLL):
        self.lib = lib

    def _new(self, a: np.ndarray):
        a = np.asarray(a, dtype=np.float64)
        flat = np.ascontiguousarray(a.ravel(order="F"))
        if flat.size == 0:
            flat = np.zeros(1)
        shape = (ctypes.c_size_t * max(a.ndim, 1))(*a.shape)
        st = ctypes.c_int(-999)
        h = self.lib.ndt_tensor_f64_from_data(flat.ctypes.data_as(ctypes.POINTER(ctypes.c_double)), flat.size,
                                              shape, a.ndim, ctypes.byref(st))
        assert st.value == 0 and h, st.value
        return h

    def _take(self, h) -> np.ndarray:
        nd = self.lib.ndt_tensor_f64_ndim(h)
        shape = (ctypes.c_size_t * max(nd, 1))()
        assert self.lib.ndt_tensor_f64_shape(h, shape) == 0
        sh = tuple(shape[i] for i in range(nd))
        n = self.lib.ndt_tensor_f64_len(h)
        p = self.lib.ndt_tensor_f64_data(h)
        out = np.ctypeslib.as_array(p, shape=(n,)).copy()
        self.lib.ndt_tensor_f64_release(h)
        return out[: int(np.prod(sh))].reshape(sh, order="F") if sh else out[:1].reshape(())

    def permutedims(self, a, perm):
        h = self._new(a)
        st = ctypes.c_int(-999)
        p = (ctypes.c_size_t * max(len(perm), 1))(*perm)
        r = self.lib.ndt_tensor_f64_permutedims(h, p, len(perm), ctypes.byref(st))
        self.lib.ndt_tensor_f64_release(h)
        return (st.value, None) if st.value != 0 else (0, self._take(r))

    def contract(self, a, la, b, lb):
        ha, hb = self._new(a), self._new(b)
        l1 = (ctypes.c_long * max(len(la), 1))(*la)
        l2 = (ctypes.c_long * max(len(lb), 1))(*lb)
        st = ctypes.c_int(-999)
        r = self.lib.ndt_tensor_f64_contract(ha, l1, len(la), hb, l2, len(lb), ctypes.byref(st))
        self.lib.ndt_tensor_f64_release(ha)
        self.lib.ndt_tensor_f64_release(hb)
        return (st.value, None) if st.value != 0 else (0, self._take(r))

    def vjp(self, a, la, b, lb, g):
        ha, hb, hg = self._new(a), self._new(b), self._new(g)
        l1 = (ctypes.c_long * max(len(la), 1))(*la)
        l2 = (ctypes.c_long * max(len(lb), 1))(*lb)
        ga, gb = ctypes.c_void_p(), ctypes.c_void_p()
        st = ctypes.c_int(-999)
        self.lib.ndt_tensor_f64_contract_vjp(ha, l1, len(la), hb, l2, len(lb), hg, ctypes.byref(ga),
                                             ctypes.byref(gb), ctypes.byref(st))
        for h in (ha, hb, hg):
            self.lib.ndt_tensor_f64_release(h)
        if st.value != 0:
            return st.value, None, None
        return 0, self._take(ga.value), self._take(gb.value)
