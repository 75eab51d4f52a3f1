"""contract_gemm_shard's argument checks through the C ABI (no device needed:
they come before any computation)."""

from __future__ import annotations

import ctypes

import numpy as np


def test_contract_gemm_shard_rejects_bad_arguments(ndt):
    lib = ndt.get_lib()
    a = ndt.TensorF64.from_numpy(np.ones((3, 4)))
    b = ndt.TensorF64.from_numpy(np.ones((4, 5)))
    la = (ctypes.c_long * 2)(1, -1)
    lb = (ctypes.c_long * 2)(-1, 2)
    st = ctypes.c_int(-999)
    for label, rank, nranks in [(1, 2, 2), (1, -1, 2), (1, 0, 0)]:
        p = lib.ndt_tensor_f64_contract_gemm_shard(a._ptr, la, 2, b._ptr, lb, 2, label, rank, nranks,
                                                   ctypes.byref(st))
        assert not p and st.value == -1
    p = lib.ndt_tensor_f64_contract_gemm_shard(None, la, 2, b._ptr, lb, 2, 1, 0, 1, ctypes.byref(st))
    assert not p and st.value == -1
    assert lib.ndt_tensor_f64_contract_gemm_shard(a._ptr, la, 2, b._ptr, lb, 2, 1, 0, 1, None) is None
