"""Sizes past 2^31 elements (or doubles): 64-bit offsets in every kernel.

Each tensor here is about 17 GB.  Tensors are created in the library, filled
in place through device_ptr_mut by torch (no host copy), and checked on the
device: permutes bit-exactly against torch's own strided view of the source
(int64 views of the doubles), contractions against torch float64 matmul
(cuBLAS) at the contraction tolerance, relative Frobenius error <= 1e-12.

Column-major storage of shape S is row-major storage of reversed(S), so a
library tensor seen from torch is the reversed-axes view of the same bytes.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

RTOL = 1e-12
TWO31 = 1 << 31


def _view(t, shape, width=1):
    """torch view (reversed axes) of library tensor t's device data."""
    from ndtensors_b200.blocksparse import _DeviceSpan

    n = int(np.prod(shape, dtype=np.int64))
    flat = torch.as_tensor(_DeviceSpan(t.device_ptr(), n * width), device="cuda")
    if width == 2:
        flat = flat.view(torch.complex128)
    return flat.view(tuple(reversed(shape)))


def _filled(cls, shape, seed, width=1):
    """A library tensor of `shape` holding N(0, 1) values written by torch
    through device_ptr_mut (which returns once the zeros are in place)."""
    from ndtensors_b200.blocksparse import _DeviceSpan

    t = cls.zeros(shape)
    n = int(np.prod(shape, dtype=np.int64)) * width
    span = torch.as_tensor(_DeviceSpan(t.device_ptr_mut(), n), device="cuda")
    span.normal_(generator=torch.Generator(device="cuda").manual_seed(seed))
    torch.cuda.synchronize()
    return t


@pytest.fixture(autouse=True)
def _release(gpu):
    yield
    torch.cuda.synchronize()
    gpu.get_lib().ndt_b200_synchronize()
    gpu.get_lib().ndt_b200_empty_cache()
    torch.cuda.empty_cache()


def _check_permute(gpu, cls, shape, perm, torch_perm, width=1):
    assert int(np.prod(shape, dtype=np.int64)) * width > TWO31  # doubles of one tensor
    t = _filled(cls, shape, 11, width)
    n0 = gpu.launch_count()
    out = t.permutedims(perm)
    gpu.synchronize()
    assert gpu.launch_count() > n0  # the permute ran on the device
    assert out.shape == tuple(shape[p] for p in perm)
    src = _view(t, shape, width)
    got = _view(out, out.shape, width)
    assert bool(src.abs().amax() > 0)  # the source really holds the drawn values
    if width == 2:
        src, got = torch.view_as_real(src), torch.view_as_real(got)
        torch_perm = tuple(torch_perm) + (len(shape),)
    assert torch.equal(got.view(torch.int64), src.view(torch.int64).permute(torch_perm))


def test_permute_tiled_past_2pow31_elements(gpu):
    # 65536 x 32769 f64 = 2^31 + 65536 elements (17.2 GB): the tiled transpose
    _check_permute(gpu, gpu.TensorF64, (65536, 32769), (1, 0), (1, 0))


def test_permute_runs_past_2pow31_elements(gpu):
    # 256 x 4194305 x 2 f64 = 2^31 + 512 elements, perm (0, 2, 1): runs of 256
    # contiguous elements keep the source's stride-1 axis first
    _check_permute(gpu, gpu.TensorF64, (256, 4194305, 2), (0, 2, 1), (1, 0, 2))


def test_permute_c128_past_2pow31_doubles(gpu):
    # 32768 x 32769 complex128 = 1.07e9 elements, 2.15e9 doubles (17.2 GB)
    _check_permute(gpu, gpu.TensorC64, (32768, 32769), (1, 0), (1, 0), width=2)


def test_contract_operand_past_2pow31_elements(gpu):
    # A[65536, 32769] . B[32769, 8] (A: 2^31 + 65536 elements, odd k, split-K)
    m, k, n = 65536, 32769, 8
    a = _filled(gpu.TensorF64, (m, k), 21)
    b = _filled(gpu.TensorF64, (k, n), 22)
    c = gpu.contract(a, (1, -1), b, (-1, 2))
    gpu.synchronize()
    assert c.shape == (m, n)
    ref_t = _view(b, (k, n)) @ _view(a, (m, k))  # (A B)^T = B^T A^T, both as torch views
    got_t = _view(c, (m, n))
    err = float(torch.linalg.norm((got_t - ref_t).flatten()) / torch.linalg.norm(ref_t.flatten()))
    assert err <= RTOL



def test_blocksparse_block_offset_past_2pow31(gpu):
    """A's first block holds 46341^2 > 2^31 elements, so the block that the
    only matched pair reads starts past 2^31 in A's packed data.  The blocks
    are written through the library (insert_block)."""
    bs = gpu.blocksparse
    big = 46341
    assert big * big > TWO31
    A = bs.BlockSparseF64.zeros([[big, 8], [big, 8]], [(0, 0), (1, 1)])
    B = bs.BlockSparseF64.zeros([[big, 8], [4]], [(1, 0)])
    rng = np.random.default_rng(5)
    a11, b10 = rng.standard_normal((8, 8)), rng.standard_normal((8, 4))
    A.insert_block((1, 1), a11)
    B.insert_block((1, 0), b10)
    C = bs.contract(A, [1, -1], B, [-1, 2])
    assert C.coords == [(1, 0)]
    got = C.to_numpy_data().reshape((8, 4), order="F")
    ref = a11 @ b10
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) <= RTOL
