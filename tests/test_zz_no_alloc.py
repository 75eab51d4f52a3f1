"""The allocation-free contraction entry point, checked against the regular one.

ndt_b200_contract_f64_noalloc serves callers that may not allocate device
memory (allocation-free hot loops, hosts that own the memory budget): it packs
operands into a fixed scratch array compiled into the library instead of
calling cudaMalloc.  This test calls it through the C ABI on caller-owned
device buffers and compares the result with ndt_tensor_f64_contract on the
same inputs, on two calls in a row (the scratch array keeps the previous
call's contents, which must not leak into the next result).  The file name
makes pytest collect it last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SZ = ctypes.c_size_t
RTOL = 1e-12  # relative Frobenius error, as for every contraction test


def rel_fro(x, y):
    return np.linalg.norm((np.asarray(x) - np.asarray(y)).ravel()) / np.linalg.norm(np.asarray(y).ravel())


def _noalloc(lib, torch, a, la, b, lb, out_len):
    A = torch.from_numpy(np.asfortranarray(a).ravel(order="F").copy()).cuda()
    B = torch.from_numpy(np.asfortranarray(b).ravel(order="F").copy()).cuda()
    C = torch.full((out_len,), float("nan"), dtype=torch.float64, device="cuda")
    out_shape = (SZ * (a.ndim + b.ndim + 1))()
    out_ndim = SZ(0)
    st = lib.ndt_b200_contract_f64_noalloc(
        ctypes.c_void_p(A.data_ptr()), (SZ * a.ndim)(*a.shape), a.ndim, (ctypes.c_long * len(la))(*la),
        ctypes.c_void_p(B.data_ptr()), (SZ * b.ndim)(*b.shape), b.ndim, (ctypes.c_long * len(lb))(*lb),
        ctypes.c_void_p(C.data_ptr()), out_len, out_shape, ctypes.byref(out_ndim),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    shape = tuple(out_shape[i] for i in range(out_ndim.value))
    return st, C.cpu().numpy()[: int(np.prod(shape))].reshape(shape, order="F") if st == 0 else None


CASES = [
    # both operands need packing (permuted contracted axes)
    ((8, 7, 6), (-2, 1, -1), (6, 9, 8), (-1, 2, -2)),
    # no packing (plain MPS-style merge)
    ((16, 4, 32), (1, 2, -1), (32, 4, 16), (-1, 3, 4)),
    # unmatched negative label pinned at index 0, ragged sizes
    ((5, 3, 11), (1, -9, -1), (11, 13), (-1, 2)),
]


@pytest.mark.parametrize("sa,la,sb,lb", CASES)
def test_noalloc_matches_regular_entry_point(gpu, sa, la, sb, lb):
    import torch

    lib = gpu.get_lib()
    rng = np.random.default_rng(abs(hash((sa, la, sb, lb))) % (2**32))
    a, b = rng.standard_normal(sa), rng.standard_normal(sb)
    ref = gpu.contract(gpu.TensorF64.from_numpy(a), la, gpu.TensorF64.from_numpy(b), lb).to_numpy()
    for _ in range(2):  # two calls in a row share the scratch array
        st, got = _noalloc(lib, torch, a, list(la), b, list(lb), ref.size)
        assert st == 0, gpu.last_error()
        assert got.shape == ref.shape
        assert rel_fro(got, ref) <= RTOL


def test_noalloc_rejects_oversize_scratch(gpu):
    import torch

    lib = gpu.get_lib()
    # packing A (3M doubles = 24 MB) exceeds the fixed 16 MiB scratch
    a = np.zeros((3000, 1000))
    b = np.zeros((3000, 2))
    st, _ = _noalloc(lib, torch, a, [-1, 1], b, [-1, 2], 2000)
    assert st == -1
    assert "scratch" in gpu.last_error()
