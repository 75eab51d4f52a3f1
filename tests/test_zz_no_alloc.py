"""The allocation-free contraction entry point, checked against the regular one.

ndt_b200_contract_f64_noalloc serves callers that may not allocate device
memory (allocation-free hot loops, hosts that own the memory budget): it packs
operands into a fixed scratch array compiled into the library instead of
calling cudaMalloc.  This test calls it through the C ABI on caller-owned
device buffers and compares the result with ndt_tensor_f64_contract on the
same inputs, on two calls in a row (the scratch array keeps the previous
call's contents, which must not leak into the next result), and with the
oracle's restatement of the reference's naive contraction; it checks through
the device's default memory pool (the one the library allocates from) that a
call takes no memory from it.  Only operands that need packing count against
the scratch limit: a contraction whose operands are read in place runs at any
size.  The file name makes pytest collect it last.
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


def _device_operands(torch, a, b, out_len):
    A = torch.from_numpy(np.asfortranarray(a).ravel(order="F").copy()).cuda()
    B = torch.from_numpy(np.asfortranarray(b).ravel(order="F").copy()).cuda()
    C = torch.full((out_len,), float("nan"), dtype=torch.float64, device="cuda")
    return A, B, C


def _noalloc(lib, torch, a, la, b, lb, out_len, bufs=None):
    A, B, C = bufs if bufs is not None else _device_operands(torch, a, b, out_len)
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
    # long k over a small output: the regular entry point splits k, this one
    # runs one launch (scratch bound exactly 16 MiB)
    ((512, 2048), (1, -1), (2048, 512), (-1, 2)),
]


def _seed(*key):
    return int.from_bytes(repr(key).encode(), "little") % (2**32)


@pytest.mark.parametrize("sa,la,sb,lb", CASES)
def test_noalloc_matches_regular_entry_point(gpu, oracle, sa, la, sb, lb):
    import torch

    lib = gpu.get_lib()
    rng = np.random.default_rng(_seed(sa, la, sb, lb))
    a, b = rng.standard_normal(sa), rng.standard_normal(sb)
    ref = gpu.contract(gpu.TensorF64.from_numpy(a), la, gpu.TensorF64.from_numpy(b), lb).to_numpy()
    ost, oref = oracle.contract_naive(a, list(la), b, list(lb))
    assert ost == 0 and oref.shape == ref.shape
    for _ in range(2):  # two calls in a row share the scratch array
        st, got = _noalloc(lib, torch, a, list(la), b, list(lb), ref.size)
        assert st == 0, gpu.last_error()
        assert got.shape == ref.shape
        assert rel_fro(got, ref) <= RTOL
        assert rel_fro(got, oref) <= RTOL


def test_noalloc_unpacked_operands_have_no_size_limit(gpu):
    """A (2048 x 1024, 16 MiB) is read in place as an MN-major matrix and B
    (1024 x 96) as a K-major one: nothing is packed, so the call succeeds
    although the two operands together exceed the scratch array."""
    import torch

    lib = gpu.get_lib()
    rng = np.random.default_rng(11)
    a, b = rng.standard_normal((2048, 1024)), rng.standard_normal((1024, 96))
    ref = gpu.contract(gpu.TensorF64.from_numpy(a), [1, -1], gpu.TensorF64.from_numpy(b), [-1, 2]).to_numpy()
    want = a @ b
    assert a.nbytes + b.nbytes > 16 << 20
    for _ in range(2):
        st, got = _noalloc(lib, torch, a, [1, -1], b, [-1, 2], ref.size)
        assert st == 0, gpu.last_error()
        assert rel_fro(got, ref) <= RTOL
        assert rel_fro(got, want) <= RTOL


def test_noalloc_rejects_oversize_scratch(gpu):
    import torch

    lib = gpu.get_lib()
    # A's contracted axes (labels -2 on axis 0, -1 on axis 2) are not one
    # strided run in pair order, so A is packed: m * k = 300 * 10000 doubles
    # (24 MB), more than the fixed 16 MiB scratch.
    a = np.zeros((40, 300, 250))
    b = np.zeros((250, 40, 2))
    st, _ = _noalloc(lib, torch, a, [-2, 1, -1], b, [-1, -2, 2], 600)
    assert st == -1
    assert "scratch" in gpu.last_error()


def _pool_used(torch):
    """(current, high watermark) bytes in use from the device's default memory pool."""
    from cuda.bindings import runtime as rt

    err, pool = rt.cudaDeviceGetDefaultMemPool(torch.cuda.current_device())
    assert err == rt.cudaError_t.cudaSuccess, err
    err, cur = rt.cudaMemPoolGetAttribute(pool, rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemCurrent)
    assert err == rt.cudaError_t.cudaSuccess, err
    err, high = rt.cudaMemPoolGetAttribute(pool, rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemHigh)
    assert err == rt.cudaError_t.cudaSuccess, err
    return int(cur), int(high), pool


def _reset_pool_high(torch):
    from cuda.bindings import driver as dr
    from cuda.bindings import runtime as rt

    torch.cuda.synchronize()
    _, _, pool = _pool_used(torch)
    (err,) = rt.cudaMemPoolSetAttribute(pool, rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemHigh, dr.cuuint64_t(0))
    assert err == rt.cudaError_t.cudaSuccess, err
    cur, _, _ = _pool_used(torch)
    return cur


def test_noalloc_takes_no_pool_memory(gpu):
    """The regular entry point takes its output (and split-K workspace) from the
    pool; the allocation-free one must leave the pool's high watermark where it
    was, on the long-k shape where the regular GEMM would split k."""
    import torch

    lib = gpu.get_lib()
    rng = np.random.default_rng(7)
    a, b = rng.standard_normal((512, 2048)), rng.standard_normal((2048, 512))
    ta, tb = gpu.TensorF64.from_numpy(a), gpu.TensorF64.from_numpy(b)
    before = _reset_pool_high(torch)
    ref = gpu.contract(ta, [1, -1], tb, [-1, 2])
    torch.cuda.synchronize()
    assert _pool_used(torch)[1] > before, "the pool watermark does not see the library's allocations"
    ref = ref.to_numpy()
    bufs = _device_operands(torch, a, b, ref.size)
    for _ in range(2):
        before = _reset_pool_high(torch)
        st, got = _noalloc(lib, torch, a, [1, -1], b, [-1, 2], ref.size, bufs)
        assert st == 0, gpu.last_error()
        assert _pool_used(torch)[1] <= before
        assert rel_fro(got, ref) <= RTOL
