"""The reference's known-answer tests, run through the C ABI on the GPU."""

from __future__ import annotations

import pytest

from golden_runner import CapiEngine, OracleEngine, load_cases, run_case

CASES = [c for c in load_cases() if c["op"] not in ("strides", "cart_to_lin", "lin_to_cart", "properties")]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=[c["id"] for c in CASES])
def test_capi_known_answer(case, gpu, oracle):
    eng = CapiEngine(gpu)
    op = case["op"]
    if op == "from_data":
        import ctypes

        import numpy as np

        lib = gpu.get_lib()
        a = case["a"]
        data = (ctypes.c_double * len(a["data"]))(*a["data"])
        shape = (ctypes.c_size_t * len(a["shape"]))(*a["shape"])
        st = ctypes.c_int(-999)
        t = lib.ndt_tensor_f64_from_data(data, len(a["data"]), shape, len(a["shape"]), ctypes.byref(st))
        assert st.value == case["expect"]["status"]
        if st.value == 0:
            v = ctypes.c_double()
            for i, x in case["expect"]["index"]:
                assert lib.ndt_tensor_f64_get_linear(t, i, ctypes.byref(v)) == 0 and v.value == x
            lib.ndt_tensor_f64_release(t)
        return
    if op == "ones":
        t = gpu.TensorF64.ones(tuple(case["shape"]))
        assert t.ndim == case["expect"]["ndim"] and len(t) == case["expect"]["len"]
        for i, x in case["expect"]["index"]:
            assert t[i] == x
        return
    assert run_case(eng, case, OracleEngine(oracle)) == "ok"
