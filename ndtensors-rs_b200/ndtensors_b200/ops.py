"""Contractions over the C ABI.

``contract`` / ``contract_vjp`` / ``contract_jvp`` keep the behaviour of the
reference's Python binding (python/ndtensors_rs/src/ndtensors_rs/ops.py):
negative labels are contracted, positive labels are kept, the output axes are
A's positive labels then B's (the C ABI's naive-loop order), and a shape
mismatch raises ``ValueError``.  ``contract_gemm`` is the TTGT form with
label-sorted output (crates/ndtensors/src/contract/gemm.rs:47-95).
"""

from __future__ import annotations

import ctypes
from typing import Optional, Sequence, Tuple

from ._lib import get_lib
from .tensor import NDTensorsError, StatusCode, TensorC64, TensorF64, check_status


def _labels(ls: Sequence[int]):
    n = len(ls)
    return (ctypes.c_long * max(n, 1))(*ls), n


def _contract(fname: str, a, labels_a, b, labels_b):
    if type(a) is not type(b):
        raise TypeError("operands must have the same element type")
    la, na = _labels(labels_a)
    lb, nb = _labels(labels_b)
    status = ctypes.c_int(-999)
    ptr = getattr(get_lib(), f"ndt_tensor_{a._prefix}_{fname}")(
        a._ptr, la, na, b._ptr, lb, nb, ctypes.byref(status)
    )
    if status.value == StatusCode.SHAPE_MISMATCH:
        raise ValueError("Contracted dimensions must have matching sizes")
    check_status(status.value, fname)
    return type(a)(ptr)


def contract(a, labels_a: Sequence[int], b, labels_b: Sequence[int]):
    """C ABI contraction (ndt_tensor_*_contract)."""
    return _contract("contract", a, labels_a, b, labels_b)


def contract_gemm(a, labels_a: Sequence[int], b, labels_b: Sequence[int]):
    """TTGT contraction with output axes sorted by label."""
    return _contract("contract_gemm", a, labels_a, b, labels_b)


def contract_gemm_shard(a, labels_a: Sequence[int], b, labels_b: Sequence[int], axis_label: int, rank: int,
                        nranks: int):
    """This rank's slab of contract_gemm(a, labels_a, b, labels_b), split
    along the free axis labelled `axis_label` into `nranks` near-equal ranges
    (no collective: the slabs of all ranks are the whole result)."""
    if type(a) is not type(b):
        raise TypeError("operands must have the same element type")
    la, na = _labels(labels_a)
    lb, nb = _labels(labels_b)
    status = ctypes.c_int(-999)
    ptr = getattr(get_lib(), f"ndt_tensor_{a._prefix}_contract_gemm_shard")(
        a._ptr, la, na, b._ptr, lb, nb, int(axis_label), int(rank), int(nranks), ctypes.byref(status))
    if status.value == StatusCode.SHAPE_MISMATCH:
        raise ValueError("Contracted dimensions must have matching sizes")
    check_status(status.value, "contract_gemm_shard")
    return type(a)(ptr)


def contract_vjp(a: TensorF64, labels_a: Sequence[int], b: TensorF64, labels_b: Sequence[int],
                 grad_output: TensorF64) -> Tuple[TensorF64, TensorF64]:
    la, na = _labels(labels_a)
    lb, nb = _labels(labels_b)
    ga, gb = ctypes.c_void_p(), ctypes.c_void_p()
    status = ctypes.c_int(-999)
    get_lib().ndt_tensor_f64_contract_vjp(
        a._ptr, la, na, b._ptr, lb, nb, grad_output._ptr, ctypes.byref(ga), ctypes.byref(gb), ctypes.byref(status)
    )
    if status.value == StatusCode.SHAPE_MISMATCH:
        raise ValueError("Shape mismatch in contract_vjp")
    check_status(status.value, "contract_vjp")
    return TensorF64(ga.value), TensorF64(gb.value)


def contract_jvp(a: TensorF64, labels_a: Sequence[int], b: TensorF64, labels_b: Sequence[int],
                 tangent_a: Optional[TensorF64] = None,
                 tangent_b: Optional[TensorF64] = None) -> Tuple[TensorF64, Optional[TensorF64]]:
    la, na = _labels(labels_a)
    lb, nb = _labels(labels_b)
    po, to = ctypes.c_void_p(), ctypes.c_void_p()
    status = ctypes.c_int(-999)
    get_lib().ndt_tensor_f64_contract_jvp(
        a._ptr, la, na, b._ptr, lb, nb,
        tangent_a._ptr if tangent_a is not None else None,
        tangent_b._ptr if tangent_b is not None else None,
        ctypes.byref(po), ctypes.byref(to), ctypes.byref(status),
    )
    if status.value == StatusCode.SHAPE_MISMATCH:
        raise ValueError("Shape mismatch in contract_jvp")
    check_status(status.value, "contract_jvp")
    return TensorF64(po.value), (TensorF64(to.value) if to.value else None)


__all__ = ["contract", "contract_gemm", "contract_vjp", "contract_jvp", "NDTensorsError", "TensorC64"]
