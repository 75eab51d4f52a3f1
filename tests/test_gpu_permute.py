"""permutedims on the GPU vs the oracle's restatement of
GenericBackend::permute_into (backend/generic.rs:15-39): bit-exact."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SZ = ctypes.c_size_t


def _rand(rng, shape, cplx):
    if cplx:
        return rng.standard_normal(shape) + 1j * rng.standard_normal(shape)
    return rng.standard_normal(shape)


def _bits(x):
    """Raw bit pattern in column-major order (bit-exact comparison)."""
    return np.ascontiguousarray(np.asarray(x).ravel(order="F")).view(np.uint64)


def _check(gpu, oracle, a, perm):
    cls = gpu.TensorC64 if np.iscomplexobj(a) else gpu.TensorF64
    got = cls.from_numpy(a).permutedims(perm).to_numpy()
    st, ref = oracle.permutedims(a, perm)
    assert st == 0
    assert got.shape == ref.shape
    assert np.array_equal(_bits(got), _bits(ref)), "permute must be bit-exact"


SHAPES = [
    ((3,), (0,)),
    ((17, 33), (1, 0)),
    ((1, 5, 1), (2, 0, 1)),
    ((2, 3, 4), (2, 0, 1)),
    ((33, 17, 3), (1, 2, 0)),
    ((5, 7, 11, 13), (3, 1, 0, 2)),
    ((16, 16, 16, 16), (3, 2, 1, 0)),
    ((8, 8, 8, 8, 8, 8), (5, 3, 1, 0, 4, 2)),
    ((2, 3, 5, 7, 3, 2), (4, 0, 5, 2, 1, 3)),
    ((64, 3, 65), (2, 1, 0)),
    ((1000, 3), (1, 0)),
    ((3, 1000), (1, 0)),
    ((2, 2, 2, 2, 2, 2, 2, 2), (7, 0, 6, 1, 5, 2, 4, 3)),
    ((40, 50, 2), (0, 2, 1)),  # stride-1 axis stays first: row gather
    ((4, 9, 100), (1, 0, 2)),
    # run copies (source stride-1 axis stays the destination's first axis)
    ((9, 5, 7), (0, 2, 1)),            # 72-byte runs: 8-byte copies (c128: 16-byte)
    ((64, 10, 33), (0, 2, 1)),         # 512-byte runs, 16-byte vectors
    ((3000, 3, 2), (0, 2, 1)),         # runs longer than one 16 KB chunk (c128)
    ((16, 2, 5, 2, 3), (0, 1, 4, 3, 2)),  # first two axes merge into one run
]


@pytest.mark.parametrize("cplx", [False, True])
def test_permute_run_copy_full_size(gpu, oracle, cplx):
    """The DMRG operand shape [1024, 10, 2048] with perm (0, 2, 1): 8 KB runs."""
    rng = np.random.default_rng(31)
    a = _rand(rng, (1024, 10, 256 if cplx else 2048), cplx)
    _check(gpu, oracle, a, (0, 2, 1))


@pytest.mark.parametrize("cplx", [False, True])
@pytest.mark.parametrize("shape,perm", SHAPES)
def test_permute_matches_oracle(gpu, oracle, shape, perm, cplx):
    rng = np.random.default_rng(abs(hash((shape, perm, cplx))) % (2**32))
    _check(gpu, oracle, _rand(rng, shape, cplx), perm)


def test_permute_random_ranks(gpu, oracle):
    rng = np.random.default_rng(1234)
    for trial in range(40):
        r = int(rng.integers(1, 7))
        shape = tuple(int(x) for x in rng.integers(1, 9, size=r))
        perm = tuple(int(x) for x in rng.permutation(r))
        _check(gpu, oracle, _rand(rng, shape, bool(trial % 2)), perm)


def test_permute_rank0_and_identity(gpu, oracle):
    t = gpu.TensorF64.from_numpy(np.array(3.5))
    out = t.permutedims(())
    assert out.shape == () and out[0] == 3.5
    a = np.random.default_rng(3).standard_normal((6, 7))
    _check(gpu, oracle, a, (0, 1))


def test_permute_zero_extent_is_internal_error(gpu):
    lib = gpu.get_lib()
    t = gpu.TensorF64.zeros((2, 0))
    st = ctypes.c_int(-999)
    assert not lib.ndt_tensor_f64_permutedims(t._ptr, (SZ * 2)(1, 0), 2, ctypes.byref(st))
    assert st.value == -4  # the reference panics in linear_to_cartesian


@pytest.mark.parametrize("cplx", [False, True])
def test_permute_16pow6_full_size(gpu, oracle, cplx):
    """The permutedims workload at full size: 16^6 elements, perm (5,3,1,0,4,2),
    bit-exact against the oracle, plus the inverse permutation round trip."""
    rng = np.random.default_rng(1002)
    shape, perm = (16,) * 6, (5, 3, 1, 0, 4, 2)
    a = _rand(rng, shape, cplx)
    cls = gpu.TensorC64 if cplx else gpu.TensorF64
    t = cls.from_numpy(a)
    p = t.permutedims(perm)
    got = p.to_numpy()
    st, ref = oracle.permutedims(a, perm)
    assert st == 0
    assert np.array_equal(_bits(got), _bits(ref))
    inv = tuple(int(i) for i in np.argsort(perm))
    back = p.permutedims(inv).to_numpy()
    assert np.array_equal(_bits(back), _bits(a))


def test_permute_raw_device_entry(gpu, oracle):
    """ndt_b200_permutedims_dev on caller-owned device buffers (torch)."""
    import torch

    rng = np.random.default_rng(5)
    shape, perm = (9, 10, 11, 12), (2, 3, 0, 1)
    a = rng.standard_normal(shape)
    src = torch.from_numpy(np.asfortranarray(a).ravel(order="F").copy()).cuda()
    dst = torch.empty_like(src)
    lib = gpu.get_lib()
    st = lib.ndt_b200_permutedims_dev(0, ctypes.c_void_p(src.data_ptr()), ctypes.c_void_p(dst.data_ptr()),
                                      (SZ * 4)(*shape), 4, (SZ * 4)(*perm), 4,
                                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    torch.cuda.synchronize()
    st2, ref = oracle.permutedims(a, perm)
    assert np.array_equal(dst.cpu().numpy(), ref.ravel(order="F"))
    bad = lib.ndt_b200_permutedims_dev(0, ctypes.c_void_p(src.data_ptr()), ctypes.c_void_p(dst.data_ptr()),
                                       (SZ * 4)(*shape), 4, (SZ * 4)(0, 0, 1, 2), 4, None)
    assert bad == -5


def test_abi_concurrent_host_threads(gpu, oracle):
    """Several host threads drive the C ABI at once (from_data -> permutedims
    -> data on their own handles): uploads, kernels and read-backs of
    different threads interleave on the library's streams, every result
    stays bit-exact."""
    import threading

    import torch

    lib = gpu.get_lib()
    dev = torch.cuda.current_device()
    shape, perm = (24, 7, 5, 33), (3, 1, 0, 2)
    rng = np.random.default_rng(77)
    inputs = [np.asfortranarray(rng.standard_normal(shape)) for _ in range(6)]
    refs = [oracle.permutedims(x, perm)[1] for x in inputs]
    shape_c, perm_c = (SZ * 4)(*shape), (SZ * 4)(*perm)
    bad = []

    def worker(idx):
        torch.cuda.set_device(dev)
        st = ctypes.c_int(-999)
        for rep in range(5):
            for i in idx:
                x = inputs[i]
                t = lib.ndt_tensor_f64_from_data(x.ctypes.data_as(ctypes.POINTER(ctypes.c_double)), x.size, shape_c,
                                                 4, ctypes.byref(st))
                p = lib.ndt_tensor_f64_permutedims(t, perm_c, 4, ctypes.byref(st))
                d = lib.ndt_tensor_f64_data(p)
                got = np.ctypeslib.as_array(d, shape=(x.size,)).copy() if d else None
                if st.value != 0 or got is None or not np.array_equal(_bits(got), _bits(refs[i])):
                    bad.append((i, rep, st.value))
                lib.ndt_tensor_f64_release(p)
                lib.ndt_tensor_f64_release(t)

    ths = [threading.Thread(target=worker, args=([0, 2, 4],)), threading.Thread(target=worker, args=([1, 3, 5],)),
           threading.Thread(target=worker, args=([5, 0, 3],))]
    for th in ths:
        th.start()
    for th in ths:
        th.join()
    assert not bad, bad[:5]
