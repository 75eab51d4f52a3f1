"""ctypes front end of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and the CPU
baseline leg of bench.py as the reference answer.  The product never imports it.

Arrays are numpy arrays in column-major (Fortran) order, float64 or
complex128.  Every function returns (status, result) with status one of the
NDO_* values of ndt_oracle.h.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path
from typing import List, Sequence, Tuple

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"

OK, WRONG_NUM, SHAPE_MISMATCH, INVALID_PERM, BLOCK_NOT_FOUND, CAPACITY, PANIC = 0, 1, 2, 3, 4, 8, 9

_lib = None
S = ctypes.c_size_t
SP = ctypes.POINTER(ctypes.c_size_t)
I32P = ctypes.POINTER(ctypes.c_int32)
VP = ctypes.c_void_p


class BsDesc(ctypes.Structure):
    _fields_ = [("ndim", S), ("nblk", SP), ("bsz", SP), ("nnzb", S), ("coords", SP)]


def build() -> None:
    subprocess.check_call(["make", "-s", "-C", str(HERE)])


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        _lib = ctypes.CDLL(str(LIB))
    return _lib


def _sz(v: Sequence[int]):
    v = list(v)
    return (S * max(len(v), 1))(*v)


def _i32(v: Sequence[int]):
    v = list(v)
    return (ctypes.c_int32 * max(len(v), 1))(*v)


def _dt(a: np.ndarray) -> int:
    return 1 if np.iscomplexobj(a) else 0


def _flat(a: np.ndarray) -> np.ndarray:
    """Column-major storage with the reference's max(1, prod) rule."""
    f = np.asarray(a).ravel(order="F")
    if f.size == 0:
        f = np.zeros(1, dtype=np.asarray(a).dtype)
    return np.ascontiguousarray(f)


def _p(a: np.ndarray):
    return a.ctypes.data_as(VP)


def compute_strides(shape):
    out = _sz([0] * len(shape))
    lib().ndo_compute_strides(_sz(shape), S(len(shape)), out)
    return [out[i] for i in range(len(shape))]


def linear_to_cartesian(linear, shape):
    out = _sz([0] * len(shape))
    st = lib().ndo_linear_to_cartesian(S(linear), _sz(shape), S(len(shape)), out)
    return st, [out[i] for i in range(len(shape))]


def cartesian_to_linear(idx, strides):
    f = lib().ndo_cartesian_to_linear
    f.restype = S
    return f(_sz(idx), _sz(strides), S(len(idx)))


def permutedims(a: np.ndarray, perm: Sequence[int], shape=None):
    shape = tuple(a.shape) if shape is None else tuple(shape)
    src = _flat(a)
    dst = np.zeros_like(src)
    st = lib().ndo_permutedims(_dt(src), _p(src), _sz(shape), S(len(shape)), _sz(perm), S(len(perm)), _p(dst))
    if st != OK:
        return st, None
    new_shape = tuple(shape[p] for p in perm)
    n = int(np.prod(new_shape, dtype=np.int64))
    return st, (dst[:n].reshape(new_shape, order="F") if n == dst.size else dst)


def permutedims_range(a: np.ndarray, perm, lo: int, hi: int, dst: np.ndarray):
    src = _flat(a)
    return lib().ndo_permutedims_range(_dt(src), _p(src), _sz(a.shape), S(a.ndim), _sz(perm), _p(dst), S(lo), S(hi))


def _contract(fn_shape, fn, a, la, b, lb, shape_a=None, shape_b=None):
    sa = tuple(a.shape) if shape_a is None else tuple(shape_a)
    sb = tuple(b.shape) if shape_b is None else tuple(shape_b)
    A, B = _flat(a), _flat(b)
    out_shape = _sz([0] * (len(sa) + len(sb) + 1))
    ond = S(0)
    st = fn_shape(_sz(sa), S(len(sa)), _i32(la), S(len(la)), _sz(sb), S(len(sb)), _i32(lb), S(len(lb)),
                  out_shape, ctypes.byref(ond))
    if st != OK:
        return st, None
    oshape = tuple(out_shape[i] for i in range(ond.value))
    n = max(1, int(np.prod(oshape, dtype=np.int64)))
    out = np.zeros(n, dtype=np.result_type(A, B))
    st = fn(_dt(out), _p(A), S(A.size), _sz(sa), S(len(sa)), _i32(la), S(len(la)),
            _p(B), S(B.size), _sz(sb), S(len(sb)), _i32(lb), S(len(lb)), _p(out), S(n))
    if st != OK:
        return st, None
    m = int(np.prod(oshape, dtype=np.int64))
    return st, (out.reshape(oshape, order="F") if m == n else out)


def contract_naive(a, la, b, lb, shape_a=None, shape_b=None):
    """The C ABI's contraction (contract/naive.rs:45-187)."""
    L = lib()
    return _contract(L.ndo_contract_naive_outshape, L.ndo_contract_naive, a, la, b, lb, shape_a, shape_b)


def contract_gemm(a, la, b, lb, shape_a=None, shape_b=None):
    """contract_gemm (contract/gemm.rs:47-236)."""
    L = lib()
    return _contract(L.ndo_contract_gemm_outshape, L.ndo_contract_gemm, a, la, b, lb, shape_a, shape_b)


def properties(la, sa, lb, sb) -> dict:
    na, nb = len(la), len(lb)
    npairs, nua, nub = S(0), S(0), S(0)
    pa, pb = _sz([0] * max(na, 1)), _sz([0] * max(na, 1))
    ua, ub = _sz([0] * max(na, 1)), _sz([0] * max(nb, 1))
    perm_a, perm_b, perm_c = _sz([0] * max(na, 1)), _sz([0] * max(nb + na, 1)), _sz([0] * max(na + nb, 1))
    olab = _i32([0] * max(na + nb, 1))
    dims = _sz([0, 0, 0])
    flags = (ctypes.c_int * 3)()
    st = lib().ndo_contract_properties(_i32(la), _sz(sa), S(na), _i32(lb), _sz(sb), S(nb), ctypes.byref(npairs), pa,
                                       pb, ctypes.byref(nua), ua, ctypes.byref(nub), ub, perm_a, perm_b, perm_c, olab,
                                       dims, flags)
    assert st == OK
    np_ = npairs.value
    nout = nua.value + nub.value
    return {
        "contracted_pairs": [(pa[i], pb[i]) for i in range(np_)],
        "uncontracted_a": [ua[i] for i in range(nua.value)],
        "uncontracted_b": [ub[i] for i in range(nub.value)],
        "perm_a": [perm_a[i] for i in range(na)],
        "perm_b": [perm_b[i] for i in range(np_ + nub.value)],
        "perm_c": [perm_c[i] for i in range(nout)],
        "output_labels": [olab[i] for i in range(nout)],
        "dleft": dims[0],
        "dmid": dims[1],
        "dright": dims[2],
        "permute_a": bool(flags[0]),
        "permute_b": bool(flags[1]),
        "permute_c": bool(flags[2]),
    }


# ---------------------------------------------------------------- block sparse
class BlockSparse:
    """Block-sparse tensor in the reference's storage model: per-axis block
    sizes, stored block coordinates (storage order) and packed data."""

    def __init__(self, block_sizes: List[List[int]], coords: List[Tuple[int, ...]], data: np.ndarray):
        self.block_sizes = [list(map(int, b)) for b in block_sizes]
        self.coords = [tuple(map(int, c)) for c in coords]
        self.data = np.ascontiguousarray(data)

    @property
    def ndim(self):
        return len(self.block_sizes)

    def block_shape(self, c):
        return tuple(self.block_sizes[ax][c[ax]] for ax in range(self.ndim))

    def offsets(self):
        off, o = [], 0
        for c in self.coords:
            off.append(o)
            o += int(np.prod(self.block_shape(c), dtype=np.int64))
        return off, o

    def block(self, c):
        off, _ = self.offsets()
        i = self.coords.index(tuple(c))
        shp = self.block_shape(c)
        n = int(np.prod(shp, dtype=np.int64))
        return self.data[off[i]:off[i] + n].reshape(shp, order="F")

    def desc(self):
        self._keep = (
            _sz([len(b) for b in self.block_sizes]),
            _sz([x for b in self.block_sizes for x in b]),
            _sz([x for c in self.coords for x in c]),
        )
        return BsDesc(self.ndim, self._keep[0], self._keep[1], len(self.coords), self._keep[2])

    def dense_shape(self):
        return tuple(sum(b) for b in self.block_sizes)


def bs_contract(A: BlockSparse, la, B: BlockSparse, lb):
    """contract_blocksparse (contract/blocksparse.rs:87-183)."""
    L = lib()
    da, db = A.desc(), B.desc()
    ond, nnzb, total = S(0), S(0), S(0)
    nbmax = sum(len(b) for b in A.block_sizes) + sum(len(b) for b in B.block_sizes) + 1
    nblk, bsz = _sz([0] * (A.ndim + B.ndim + 1)), _sz([0] * nbmax)
    st = L.ndo_bs_contract_plan(ctypes.byref(da), _i32(la), S(len(la)), ctypes.byref(db), _i32(lb), S(len(lb)),
                                ctypes.byref(ond), nblk, bsz, ctypes.byref(nnzb), None, ctypes.byref(total))
    if st != OK:
        return st, None
    nb_out = nnzb.value
    coords = _sz([0] * max(1, nb_out * ond.value))
    cap = S(nb_out)
    st = L.ndo_bs_contract_plan(ctypes.byref(da), _i32(la), S(len(la)), ctypes.byref(db), _i32(lb), S(len(lb)),
                                ctypes.byref(ond), nblk, bsz, ctypes.byref(cap), coords, ctypes.byref(total))
    if st != OK:
        return st, None
    nd = ond.value
    sizes, k = [], 0
    for ax in range(nd):
        sizes.append([bsz[k + i] for i in range(nblk[ax])])
        k += nblk[ax]
    oc = [tuple(coords[b * nd + i] for i in range(nd)) for b in range(nb_out)]
    dt = np.result_type(A.data, B.data)
    out = np.zeros(max(1, total.value), dtype=dt)
    st = L.ndo_bs_contract(_dt(out), ctypes.byref(da), _p(A.data), _i32(la), S(len(la)), ctypes.byref(db), _p(B.data),
                           _i32(lb), S(len(lb)), _p(out), S(out.size))
    if st != OK:
        return st, None
    return st, BlockSparse(sizes, oc, out[: total.value])


def bs_work(A: BlockSparse, la, B: BlockSparse, lb):
    npairs, mnk = S(0), ctypes.c_double(0)
    da, db = A.desc(), B.desc()
    st = lib().ndo_bs_contract_work(ctypes.byref(da), _i32(la), S(len(la)), ctypes.byref(db), _i32(lb), S(len(lb)),
                                    ctypes.byref(npairs), ctypes.byref(mnk))
    return st, npairs.value, mnk.value


def bs_permutedims(A: BlockSparse, perm):
    """permutedims_blocksparse (operations/blocksparse.rs:61-129)."""
    d = A.desc()
    nd = A.ndim
    nblk = _sz([0] * nd)
    bsz = _sz([0] * sum(len(b) for b in A.block_sizes))
    coords = _sz([0] * max(1, len(A.coords) * nd))
    out = np.zeros_like(A.data) if A.data.size else np.zeros(1, dtype=A.data.dtype)
    st = lib().ndo_bs_permutedims(_dt(A.data), ctypes.byref(d), _p(A.data), _sz(perm), S(len(perm)), nblk, bsz,
                                  coords, _p(out))
    if st != OK:
        return st, None
    sizes, k = [], 0
    for ax in range(nd):
        sizes.append([bsz[k + i] for i in range(nblk[ax])])
        k += nblk[ax]
    oc = [tuple(coords[b * nd + i] for i in range(nd)) for b in range(len(A.coords))]
    return st, BlockSparse(sizes, oc, out[: A.data.size])


def bs_to_dense(A: BlockSparse) -> np.ndarray:
    d = A.desc()
    shape = A.dense_shape()
    out = np.zeros(max(1, int(np.prod(shape, dtype=np.int64))), dtype=A.data.dtype)
    data = A.data if A.data.size else np.zeros(1, dtype=A.data.dtype)
    st = lib().ndo_bs_to_dense(_dt(out), ctypes.byref(d), _p(data), _p(out))
    assert st == OK
    n = int(np.prod(shape, dtype=np.int64))
    return out.reshape(shape, order="F") if n == out.size else out


def bs_from_dense(dense: np.ndarray, block_sizes, coords) -> BlockSparse:
    A = BlockSparse(block_sizes, coords, np.zeros(0, dtype=dense.dtype))
    _, total = A.offsets()
    out = np.zeros(max(1, total), dtype=dense.dtype)
    d = A.desc()
    src = _flat(dense)
    st = lib().ndo_bs_from_dense(_dt(out), ctypes.byref(d), _p(src), _p(out))
    assert st == OK
    return BlockSparse(block_sizes, coords, out[:total])


def diag_to_dense(block_sizes, coords, diag: np.ndarray) -> np.ndarray:
    """DiagBlockSparseTensor::to_dense (diagblocksparse_tensor.rs:399-426)."""
    S_ = BlockSparse(block_sizes, coords, diag)
    d = S_.desc()
    shape = S_.dense_shape()
    out = np.zeros(max(1, int(np.prod(shape, dtype=np.int64))), dtype=diag.dtype)
    data = diag if diag.size else np.zeros(1, dtype=diag.dtype)
    st = lib().ndo_diag_to_dense(_dt(out), ctypes.byref(d), _p(np.ascontiguousarray(data)), _p(out))
    assert st == OK
    n = int(np.prod(shape, dtype=np.int64))
    return out.reshape(shape, order="F") if n == out.size else out
