"""C-ABI host-side behaviour that needs no GPU.

Covers: the library loads and exports every symbol include/ndtensors_capi.h
declares; argument checks and status codes of crates/ndtensors-capi/src/lib.rs
(NULL handling, length checks, index bounds, permutation validation, label
validation); handle bookkeeping (shape / len / clone with copy on write /
fill / set_linear / data / data_mut).  Without a CUDA device, storage stays
on the host and every computation fails loudly with NDT_INTERNAL_ERROR.
"""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "ndtensors_capi.h"

SZ = ctypes.c_size_t


def declared_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ndt_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_reference_abi():
    names = declared_symbols()
    reference_19 = [
        "ndt_tensor_f64_zeros", "ndt_tensor_f64_ones", "ndt_tensor_f64_rand", "ndt_tensor_f64_randn",
        "ndt_tensor_f64_from_data", "ndt_tensor_f64_release", "ndt_tensor_f64_clone", "ndt_tensor_f64_ndim",
        "ndt_tensor_f64_len", "ndt_tensor_f64_shape", "ndt_tensor_f64_data", "ndt_tensor_f64_data_mut",
        "ndt_tensor_f64_get_linear", "ndt_tensor_f64_set_linear", "ndt_tensor_f64_fill",
        "ndt_tensor_f64_permutedims", "ndt_tensor_f64_contract", "ndt_tensor_f64_contract_vjp",
        "ndt_tensor_f64_contract_jvp",
    ]
    for n in reference_19:
        assert n in names, n


def test_library_exports_every_declared_symbol(ndt):
    lib_path = ndt.lib_path()
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib_path)], capture_output=True, text=True, check=True)
    exported = set(re.findall(r"\bT (ndt_[a-z0-9_]+)$", out.stdout, flags=re.M))
    missing = [n for n in declared_symbols() if n not in exported]
    assert not missing, missing
    # and nothing but the C ABI leaks out
    assert all(n.startswith("ndt_") for n in exported)


def test_every_declared_symbol_has_ctypes_signature(ndt):
    from ndtensors_b200._lib import SIGNATURES

    bound = {s[0] for s in SIGNATURES}
    missing = [n for n in declared_symbols() if n not in bound]
    assert not missing, missing


def _shape(lib, t):
    n = lib.ndt_tensor_f64_ndim(t)
    out = (SZ * max(n, 1))()
    assert lib.ndt_tensor_f64_shape(t, out) == 0
    return tuple(out[i] for i in range(n))


def test_creation_and_queries(ndt):
    lib = ndt.get_lib()
    st = ctypes.c_int(-999)
    shape = (SZ * 3)(2, 3, 4)
    t = lib.ndt_tensor_f64_zeros(shape, 3, ctypes.byref(st))
    assert st.value == 0 and t
    assert lib.ndt_tensor_f64_ndim(t) == 3
    assert lib.ndt_tensor_f64_len(t) == 24
    assert _shape(lib, t) == (2, 3, 4)
    v = ctypes.c_double(-1)
    assert lib.ndt_tensor_f64_get_linear(t, 23, ctypes.byref(v)) == 0 and v.value == 0.0
    assert lib.ndt_tensor_f64_get_linear(t, 24, ctypes.byref(v)) == -3
    lib.ndt_tensor_f64_release(t)
    # rank 0 holds one element (tensor.rs:45-54)
    t0 = lib.ndt_tensor_f64_ones(None, 0, ctypes.byref(st))
    assert st.value == 0 and lib.ndt_tensor_f64_len(t0) == 1 and lib.ndt_tensor_f64_ndim(t0) == 0
    assert lib.ndt_tensor_f64_get_linear(t0, 0, ctypes.byref(v)) == 0 and v.value == 1.0
    lib.ndt_tensor_f64_release(t0)
    # zero extent: storage still holds max(1, 0) = 1 element
    z = lib.ndt_tensor_f64_zeros((SZ * 2)(2, 0), 2, ctypes.byref(st))
    assert st.value == 0 and lib.ndt_tensor_f64_len(z) == 1
    lib.ndt_tensor_f64_release(z)


def test_null_handling(ndt):
    lib = ndt.get_lib()
    st = ctypes.c_int(-999)
    # NULL status -> NULL result, status untouched
    assert not lib.ndt_tensor_f64_zeros((SZ * 1)(2), 1, None)
    # NULL shape with ndim > 0 -> INVALID_ARGUMENT (capi/lib.rs:90-95, :1417-1421)
    assert not lib.ndt_tensor_f64_randn(None, 2, ctypes.byref(st)) and st.value == -1
    assert not lib.ndt_tensor_f64_from_data(None, 1, None, 0, ctypes.byref(st)) and st.value == -1
    lib.ndt_tensor_f64_release(None)
    assert not lib.ndt_tensor_f64_clone(None)
    assert lib.ndt_tensor_f64_ndim(None) == 0 and lib.ndt_tensor_f64_len(None) == 0
    assert lib.ndt_tensor_f64_shape(None, (SZ * 1)()) == -1
    assert not lib.ndt_tensor_f64_data(None)
    assert lib.ndt_tensor_f64_fill(None, 1.0) == -1
    assert lib.ndt_tensor_f64_set_linear(None, 0, 1.0) == -1
    assert not lib.ndt_tensor_f64_permutedims(None, (SZ * 1)(0), 1, ctypes.byref(st)) and st.value == -1
    one = (ctypes.c_long * 1)(1)
    assert not lib.ndt_tensor_f64_contract(None, one, 1, None, one, 1, ctypes.byref(st)) and st.value == -1
    ga, gb = ctypes.c_void_p(), ctypes.c_void_p()
    lib.ndt_tensor_f64_contract_vjp(None, one, 1, None, one, 1, None, ctypes.byref(ga), ctypes.byref(gb),
                                    ctypes.byref(st))
    assert st.value == -1


def test_from_data_length_check(ndt):
    lib = ndt.get_lib()
    st = ctypes.c_int(-999)
    data = (ctypes.c_double * 2)(1.0, 2.0)
    assert not lib.ndt_tensor_f64_from_data(data, 2, (SZ * 2)(2, 3), 2, ctypes.byref(st))
    assert st.value == -2


def test_clone_is_copy_on_write(ndt):
    a = ndt.TensorF64.from_numpy(np.arange(6.0).reshape(2, 3))
    b = a.copy()
    b[0] = 42.0
    assert a[0] == 0.0 and b[0] == 42.0
    c = a.copy()
    c.fill(7.0)
    assert a[1] == 3.0 and c[5] == 7.0
    np.testing.assert_array_equal(a.to_numpy(), np.arange(6.0).reshape(2, 3))


def test_data_mut_roundtrip(ndt):
    lib = ndt.get_lib()
    t = ndt.TensorF64.zeros((2, 2))
    p = lib.ndt_tensor_f64_data_mut(t._ptr)
    for i in range(4):
        p[i] = float(i + 1)
    assert [t[i] for i in range(4)] == [1.0, 2.0, 3.0, 4.0]
    q = lib.ndt_tensor_f64_data(t._ptr)
    assert q[3] == 4.0


def test_rand_ranges(ndt):
    t = ndt.TensorF64.rand((1000,))
    a = t.to_numpy()
    assert np.all((a >= 0) & (a < 1))
    n = ndt.TensorF64.randn((4000,)).to_numpy()
    assert abs(n.mean()) < 0.1 and abs(n.std() - 1.0) < 0.1


def test_complex_handles(ndt):
    z = np.array([[1 + 2j, 3 - 1j], [0.5j, -2.0]])
    t = ndt.TensorC64.from_numpy(z)
    assert t.shape == (2, 2) and len(t) == 4
    assert t[1] == 0.5j
    np.testing.assert_array_equal(t.to_numpy(), z)
    t[0] = 9 + 9j
    assert t[0] == 9 + 9j


def test_validation_precedes_compute(ndt):
    """Errors the reference reports before computing are reported the same
    way here, device or not."""
    lib = ndt.get_lib()
    st = ctypes.c_int(-999)
    t = ndt.TensorF64.zeros((2, 3))
    for perm in ([0], [0, 1, 2], [0, 2], [0, 0]):
        arr = (SZ * len(perm))(*perm)
        assert not lib.ndt_tensor_f64_permutedims(t._ptr, arr, len(perm), ctypes.byref(st))
        assert st.value == -5
    a, b = ndt.TensorF64.ones((2, 3)), ndt.TensorF64.ones((4, 5))
    la, lb = (ctypes.c_long * 2)(1, -1), (ctypes.c_long * 2)(-1, 2)
    assert not lib.ndt_tensor_f64_contract(a._ptr, la, 2, b._ptr, lb, 2, ctypes.byref(st))
    assert st.value == -2  # shape mismatch (naive.rs:72-77)
    assert not lib.ndt_tensor_f64_contract(a._ptr, la, 1, b._ptr, lb, 2, ctypes.byref(st))
    assert st.value == -2  # wrong number of labels
    with pytest.raises(ValueError):
        ndt.contract(a, (1, -1), b, (-1, 2))


@pytest.mark.skipif("__import__('ndtensors_b200').device_available()", reason="a CUDA device is present")
def test_compute_without_device_fails_loudly(ndt):
    lib = ndt.get_lib()
    st = ctypes.c_int(-999)
    t = ndt.TensorF64.ones((2, 3))
    assert not lib.ndt_tensor_f64_permutedims(t._ptr, (SZ * 2)(1, 0), 2, ctypes.byref(st))
    assert st.value == -4
    assert "no CUDA device" in ndt.last_error()
    with pytest.raises(ndt.NDTensorsError):
        ndt.contract(ndt.TensorF64.ones((2, 3)), (1, -1), ndt.TensorF64.ones((3, 4)), (-1, 2))


@pytest.mark.skipif("__import__('ndtensors_b200').device_available()", reason="a CUDA device is present")
def test_torch_contract_has_no_cpu_path(ndt):
    """torch_contract resolves lazily from the package, as the reference
    binding's does, and without a device it raises instead of computing."""
    import torch

    from ndtensors_b200.torch_ops import TORCH_AVAILABLE

    assert TORCH_AVAILABLE
    tc = ndt.torch_contract
    with pytest.raises(ndt.NDTensorsError):
        tc(torch.ones((2, 3)), (1, -1), torch.ones((3, 4)), (-1, 2))


def test_from_torch_cpu_tensor_with_grad(ndt):
    """A CPU tensor that requires grad enters the library like any other
    (host bookkeeping; no device needed)."""
    import torch

    x = torch.arange(6, dtype=torch.float64).reshape(2, 3).requires_grad_()
    t = ndt.TensorF64.from_torch(x)
    assert t.shape == (2, 3)
    np.testing.assert_array_equal(t.to_numpy(), x.detach().numpy())
