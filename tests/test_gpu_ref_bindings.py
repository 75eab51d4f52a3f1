"""The reference's known answers through the reference binding's own ctypes
declarations (python/ndtensors_rs/src/ndtensors_rs/_lib.py, kept as data in
tests/golden/ref_ctypes_signatures.json), computing on the GPU.

This is the drop-in check for the reference's Python binding: its _lib.py
declares 17 functions; bound with exactly those declarations, this library
must answer every f64 known-answer case of the reference's tests (naive.rs,
permutedims.rs, the C ABI's lib.rs tests, the Python suite's test_contract.py
and test_tensor.py) as the reference does, and the VJP cases within 1e-12.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import refbind
from golden_runner import load_cases, run_case

pytestmark = pytest.mark.gpu

CASES = [c for c in load_cases()
         if c["op"] in ("permutedims", "contract", "vjp")
         and all(c.get(k, {}).get("dtype", "f64") == "f64" for k in ("a", "b", "grad"))]


@pytest.fixture(scope="module")
def engine(gpu):
    return refbind.RefEngine(refbind.load())


@pytest.mark.parametrize("case", CASES, ids=[c["id"] for c in CASES])
def test_known_answer_through_reference_declarations(engine, case):
    assert run_case(engine, case) != "skip"


def test_reference_binding_roundtrip_and_elements(engine):
    """tensor.py's from_numpy / to_numpy / __getitem__ / fill paths."""
    lib = engine.lib
    rng = np.random.default_rng(3)
    a = rng.standard_normal((3, 4, 5))
    h = engine._new(a)
    v = ctypes.c_double()
    assert lib.ndt_tensor_f64_get_linear(h, 7, ctypes.byref(v)) == 0 and v.value == a.ravel(order="F")[7]
    assert lib.ndt_tensor_f64_set_linear(h, 7, 42.0) == 0
    assert lib.ndt_tensor_f64_fill(h, 2.5) == 0
    back = engine._take(h)
    assert back.shape == a.shape and np.all(back == 2.5)
    st = ctypes.c_int(-999)
    shape = (ctypes.c_size_t * 2)(64, 32)
    for fn in (lib.ndt_tensor_f64_ones, lib.ndt_tensor_f64_rand, lib.ndt_tensor_f64_randn):
        t = fn(shape, 2, ctypes.byref(st))
        assert st.value == 0 and t
        x = engine._take(t)
        assert x.shape == (64, 32) and np.all(np.isfinite(x))
