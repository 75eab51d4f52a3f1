"""The multi-GPU C ABI's argument checks and NCCL loading, without a device:
the communicator calls reject bad arguments before touching NCCL or a GPU,
NCCL's unique id can be made on a host without a GPU, and the gathered
contractions reject a missing communicator."""

from __future__ import annotations

import ctypes


def test_comm_argument_checks(ndt):
    lib = ndt.get_lib()
    st = ctypes.c_int(-999)
    uid = ctypes.create_string_buffer(128)
    assert not lib.ndt_b200_comm_init(None, 2, 0, ctypes.byref(st)) and st.value == -1
    for nranks, rank in [(0, 0), (2, 2), (2, -1)]:
        assert not lib.ndt_b200_comm_init(uid, nranks, rank, ctypes.byref(st)) and st.value == -1
    assert not lib.ndt_b200_comm_init(uid, 2, 0, None)
    assert not lib.ndt_b200_comm_from_nccl(None, ctypes.byref(st)) and st.value == -1
    assert lib.ndt_b200_comm_rank(None) == -1 and lib.ndt_b200_comm_size(None) == 0
    lib.ndt_b200_comm_release(None)  # NULL-safe
    assert lib.ndt_b200_comm_unique_id(None) == -1


def test_unique_id_without_a_gpu(ndt):
    """NCCL's bootstrap id needs no device: 128 bytes, not all zero."""
    lib = ndt.get_lib()
    uid = ctypes.create_string_buffer(128)
    assert lib.ndt_b200_comm_unique_id(uid) == 0, ndt.last_error()
    assert any(uid.raw)


def test_gathered_contractions_need_a_communicator(ndt):
    lib = ndt.get_lib()
    bs = ndt.blocksparse
    a = bs.BlockSparseF64.from_blocks([[2], [3]], [(0, 0)], [1.0] * 6)
    la = (ctypes.c_long * 2)(1, -1)
    lb = (ctypes.c_long * 2)(-1, 2)
    st = ctypes.c_int(-999)
    assert not lib.ndt_blocksparse_f64_contract_gathered(a._ptr, la, 2, a._ptr, lb, 2, None, ctypes.byref(st))
    assert st.value == -1
    assert not lib.ndt_blocksparse_f64_allgather(a._ptr, None, ctypes.byref(st)) and st.value == -1
