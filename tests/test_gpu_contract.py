"""Dense contraction on the GPU (DMMA GEMM + gather) vs the oracle.

Tolerance: relative Frobenius error <= 1e-12 for f64 and complex128 (the
parity bound of this contraction path); the oracle sums in a different order
(plain i-j-k loop) so bit equality is not expected.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL = 1e-12


def rel_fro(x, y):
    x, y = np.asarray(x), np.asarray(y)
    d = np.linalg.norm((x - y).ravel())
    n = np.linalg.norm(y.ravel())
    return d / n if n > 0 else d


def _rand(rng, shape, cplx):
    if cplx:
        return rng.standard_normal(shape) + 1j * rng.standard_normal(shape)
    return rng.standard_normal(shape)


def _cls(gpu, cplx):
    return gpu.TensorC64 if cplx else gpu.TensorF64


def _check_naive(gpu, oracle, a, la, b, lb):
    cls = _cls(gpu, np.iscomplexobj(a))
    got = gpu.contract(cls.from_numpy(a), la, cls.from_numpy(b), lb).to_numpy()
    st, ref = oracle.contract_naive(a, la, b, lb)
    assert st == 0
    assert got.shape == ref.shape
    assert rel_fro(got, ref) <= RTOL, rel_fro(got, ref)


def _check_gemm(gpu, oracle, a, la, b, lb):
    cls = _cls(gpu, np.iscomplexobj(a))
    got = gpu.contract_gemm(cls.from_numpy(a), la, cls.from_numpy(b), lb).to_numpy()
    st, ref = oracle.contract_gemm(a, la, b, lb)
    assert st == 0
    assert got.shape == ref.shape
    assert rel_fro(got, ref) <= RTOL, rel_fro(got, ref)


CASES = [
    # (shape_a, labels_a, shape_b, labels_b)
    ((7, 5), (1, -1), (5, 9), (-1, 2)),                    # matrix, ragged sizes
    ((5, 7), (-1, 1), (5, 9), (-1, 2)),                    # A transposed (K-major)
    ((7, 5), (1, -1), (9, 5), (2, -1)),                    # B transposed
    ((130, 67), (1, -1), (67, 129), (-1, 2)),              # edge tiles in m, n, k
    ((3, 4, 5), (1, -1, -2), (5, 2, 4), (-2, 2, -1)),      # permuted contracted axes -> pack
    ((6, 2, 3, 4), (-1, 1, -2, 2), (3, 5, 6), (-2, 3, -1)),
    ((2, 3, 4), (1, 2, -1), (4, 5), (-1, 3)),
    ((4,), (-1,), (4,), (-1,)),                            # scalar -> shape [1]
    ((3,), (1,), (4,), (2,)),                              # outer product
    ((2, 3), (1, 2), (), ()),                              # rank-0 operand
    ((3, 3), (-1, -1), (3,), (-1,)),                       # duplicate label: B follows first pair
    ((3, 4), (-7, 1), (5,), (2,)),                         # unmatched negative label pinned at 0
    ((3, 4), (0, 1), (4, 2), (-3, 2)),                     # label 0 pinned; B's -3 pinned
    ((8, 16, 24), (2, -1, 1), (24, 16, 5), (3, -1, -9)),   # unsorted output (naive order kept)
]


@pytest.mark.parametrize("cplx", [False, True])
@pytest.mark.parametrize("sa,la,sb,lb", CASES)
def test_contract_naive_semantics(gpu, oracle, sa, la, sb, lb, cplx):
    rng = np.random.default_rng(abs(hash((sa, la, sb, lb, cplx))) % (2**32))
    _check_naive(gpu, oracle, _rand(rng, sa, cplx), list(la), _rand(rng, sb, cplx), list(lb))


@pytest.mark.parametrize("cplx", [False, True])
def test_contract_gemm_semantics_sorted_output(gpu, oracle, cplx):
    rng = np.random.default_rng(11)
    a, b = _rand(rng, (6, 4, 5), cplx), _rand(rng, (5, 3, 4), cplx)
    _check_gemm(gpu, oracle, a, [3, -1, -2], b, [-2, 1, -1])
    _check_gemm(gpu, oracle, _rand(rng, (4, 5), cplx), [2, -1], _rand(rng, (5, 3), cplx), [-1, 1])


def test_contract_gemm_rejects_duplicate_pairs(gpu):
    a, b = gpu.TensorF64.ones((3, 3)), gpu.TensorF64.ones((3,))
    with pytest.raises(ValueError):
        gpu.contract_gemm(a, (-1, -1), b, (-1,))


def test_contract_zero_extent_is_internal_error(gpu):
    lib = gpu.get_lib()
    a, b = gpu.TensorF64.zeros((2, 0)), gpu.TensorF64.ones((3,))
    la, lb = (ctypes.c_long * 2)(1, 2), (ctypes.c_long * 1)(3)
    st = ctypes.c_int(-999)
    assert not lib.ndt_tensor_f64_contract(a._ptr, la, 2, b._ptr, lb, 1, ctypes.byref(st))
    assert st.value == -4


@pytest.mark.parametrize("m,n,k", [(1024, 512, 1025), (768, 512, 1537), (512, 512, 2049), (512, 512, 2048),
                                   (512, 512, 4095)])
def test_split_k_pieces_cover_k(gpu, m, n, k):
    """Grids with a mostly idle last wave and a long k run split-K (2, 3 and 4
    pieces for these shapes); k not a multiple of the piece count times 32
    must still be covered to its last index."""
    rng = np.random.default_rng(m + n + k)
    a, b = rng.standard_normal((m, k)), rng.standard_normal((k, n))
    got = gpu.contract(gpu.TensorF64.from_numpy(a), (1, -1), gpu.TensorF64.from_numpy(b), (-1, 2)).to_numpy()
    assert rel_fro(got, a @ b) <= RTOL


def test_split_k_pieces_cover_k_c128(gpu):
    """complex128 (3M kernel) through split-K: 512 x 512 x 1025 runs 2 pieces."""
    rng = np.random.default_rng(1025)
    a = rng.standard_normal((512, 1025)) + 1j * rng.standard_normal((512, 1025))
    b = rng.standard_normal((1025, 512)) + 1j * rng.standard_normal((1025, 512))
    got = gpu.contract(gpu.TensorC64.from_numpy(a), (1, -1), gpu.TensorC64.from_numpy(b), (-1, 2)).to_numpy()
    assert rel_fro(got, a @ b) <= RTOL


def test_mps_merge_full_size(gpu, oracle):
    """Dense f64 MPS two-site merge at full size: A[256,4,256] x B[256,4,256]
    contracting A's last with B's first -> C[256,4,4,256]; N(0,1) seed 1001."""
    rng = np.random.default_rng(1001)
    a = rng.standard_normal((256, 4, 256))
    b = rng.standard_normal((256, 4, 256))
    t = gpu.contract(gpu.TensorF64.from_numpy(a), (1, 2, -1), gpu.TensorF64.from_numpy(b), (-1, 3, 4))
    got = t.to_numpy()
    assert got.shape == (256, 4, 4, 256)
    ref = np.einsum("ijk,klm->ijlm", a, b, optimize=True)
    assert rel_fro(got, ref) <= RTOL
    # pin against the oracle's TTGT restatement on a slice
    st, oref = oracle.contract_gemm(a[:32], [1, 2, -1], b[:, :, :16], [-1, 3, 4])
    assert st == 0 and rel_fro(got[:32, :, :, :16], oref) <= RTOL


@pytest.mark.parametrize("dtype", [0, 1])
@pytest.mark.parametrize("ak,bk", [(0, 1), (1, 1), (0, 0), (1, 0)])
@pytest.mark.parametrize("m,n,k", [
    (1, 1, 1), (17, 9, 31), (128, 128, 16), (300, 200, 100), (1024, 64, 7),
    # multi-wave grids with partial last waves, odd k, a single k-step
    (1024, 1024, 256), (1000, 700, 1000), (777, 555, 333), (2048, 2048, 8),
    # split-K (a 3.4-wave grid over a long k): equal and ragged k splits
    (4096, 1024, 1024), (4000, 1000, 1500),
])
def test_raw_gemm(gpu, dtype, ak, bk, m, n, k):
    """ndt_b200_gemm_dev against numpy, all operand layouts, edge tiles."""
    import torch

    rng = np.random.default_rng(m * 7 + n * 3 + k + 100 * ak + 10 * bk + dtype)
    cplx = dtype == 1
    A = _rand(rng, (m, k), cplx)
    B = _rand(rng, (k, n), cplx)
    # storage: A MN-major -> column-major (m,k); K-major -> column-major (k,m)
    a_store = np.asfortranarray(A if not ak else A.T).ravel(order="F")
    b_store = np.asfortranarray(B if bk else B.T).ravel(order="F")
    lda = k if ak else m
    ldb = k if bk else n
    dt = torch.complex128 if cplx else torch.float64
    ta = torch.from_numpy(a_store.copy()).to("cuda", dt)
    tb = torch.from_numpy(b_store.copy()).to("cuda", dt)
    tc = torch.zeros(m * n, dtype=dt, device="cuda")
    lib = gpu.get_lib()
    st = lib.ndt_b200_gemm_dev(dtype, m, n, k, ctypes.c_void_p(ta.data_ptr()), lda, ak, ctypes.c_void_p(tb.data_ptr()),
                               ldb, bk, ctypes.c_void_p(tc.data_ptr()), m, 0,
                               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    torch.cuda.synchronize()
    C = tc.cpu().numpy().reshape((m, n), order="F")
    assert rel_fro(C, A @ B) <= RTOL
    # accumulate mode: C += A B
    st = lib.ndt_b200_gemm_dev(dtype, m, n, k, ctypes.c_void_p(ta.data_ptr()), lda, ak, ctypes.c_void_p(tb.data_ptr()),
                               ldb, bk, ctypes.c_void_p(tc.data_ptr()), m, 1,
                               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    C2 = tc.cpu().numpy().reshape((m, n), order="F")
    assert rel_fro(C2, 2 * (A @ B)) <= RTOL


def test_vjp_jvp_numerics(gpu):
    rng = np.random.default_rng(21)
    a, b, g = rng.standard_normal((4, 6)), rng.standard_normal((6, 5)), rng.standard_normal((4, 5))
    T = gpu.TensorF64
    ga, gb = gpu.contract_vjp(T.from_numpy(a), (1, -1), T.from_numpy(b), (-1, 2), T.from_numpy(g))
    assert rel_fro(ga.to_numpy(), g @ b.T) <= RTOL
    assert rel_fro(gb.to_numpy(), a.T @ g) <= RTOL
    da, db = rng.standard_normal((4, 6)), rng.standard_normal((6, 5))
    p, t = gpu.contract_jvp(T.from_numpy(a), (1, -1), T.from_numpy(b), (-1, 2), T.from_numpy(da), T.from_numpy(db))
    assert rel_fro(p.to_numpy(), a @ b) <= RTOL
    assert rel_fro(t.to_numpy(), da @ b + a @ db) <= RTOL


def test_torch_interop_device_roundtrip(gpu):
    import torch

    x = torch.randn(5, 6, 7, dtype=torch.float64, device="cuda")
    t = gpu.TensorF64.from_torch(x)
    assert t.shape == (5, 6, 7)
    np.testing.assert_array_equal(t.to_numpy(), x.cpu().numpy())


def test_device_ptr_mut_writes_are_the_tensor(gpu):
    """Writes through device_ptr_mut become the tensor's values: a zeros
    tensor (held as a uniform value until materialised) filled by torch reads
    back the written data on the host and in a contraction, and a clone that
    shared the storage keeps its old values (copy on write)."""
    import torch

    from ndtensors_b200.blocksparse import _DeviceSpan

    t = gpu.TensorF64.zeros((4, 3))
    t.device_ptr()  # materialised zeros, storage shared with the clone below
    keep = gpu.TensorF64(gpu.get_lib().ndt_tensor_f64_clone(t._ptr))
    dst = torch.as_tensor(_DeviceSpan(t.device_ptr_mut(), 12), device="cuda")
    src = torch.arange(12, dtype=torch.float64, device="cuda")
    dst.copy_(src)
    torch.cuda.synchronize()
    got = t.to_numpy()
    np.testing.assert_array_equal(got, np.arange(12.0).reshape(3, 4).T)  # column-major
    np.testing.assert_array_equal(keep.to_numpy(), np.zeros((4, 3)))
    e = gpu.contract(t, (1, -1), gpu.TensorF64.from_numpy(np.ones(3)), (-1,)).to_numpy()
    np.testing.assert_allclose(e, got.sum(axis=1), rtol=1e-15)
    bs = gpu.blocksparse
    b = bs.BlockSparseF64.zeros([[2, 3], [4]], [(1, 0), (0, 0)])
    view = torch.as_tensor(_DeviceSpan(b.device_ptr_mut(), b.nnz), device="cuda")
    view.copy_(torch.arange(b.nnz, dtype=torch.float64, device="cuda") + 1)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(b.to_numpy_data(), np.arange(b.nnz) + 1.0)
