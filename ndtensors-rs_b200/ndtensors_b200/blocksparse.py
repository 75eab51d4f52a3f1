"""Block-sparse and diag-block-sparse tensors over the C ABI.

Storage model of the reference (crates/ndtensors/src/blocksparse_tensor.rs,
storage/blocksparse/): per-axis block sizes, stored blocks packed in the
order given, each block column-major.  ``contract`` is contract_blocksparse
(contract/blocksparse.rs:87-183) run as one grouped FP64 tensor-core launch;
``contract_shard`` computes one rank's FLOP-balanced share of the output
blocks; ``contract_diag`` contracts with a diagonal block tensor.
"""

from __future__ import annotations

import ctypes
from typing import List, Sequence, Tuple

import numpy as np

from ._lib import c_double_p, get_lib, last_error
from .tensor import NDTensorsError, StatusCode, TensorC64, TensorF64, check_status

SZ = ctypes.c_size_t


def _structure_args(block_sizes, coords):
    ndim = len(block_sizes)
    nblk = (SZ * max(ndim, 1))(*[len(b) for b in block_sizes])
    flat = [int(x) for b in block_sizes for x in b]
    bsz = (SZ * max(len(flat), 1))(*flat)
    cflat = [int(x) for c in coords for x in c]
    cs = (SZ * max(len(cflat), 1))(*cflat)
    return ndim, nblk, bsz, len(coords), cs


def _raise(status, what, code_exc=StatusCode.SHAPE_MISMATCH, exc=ValueError):
    if status == code_exc:
        raise exc(f"{what}: {StatusCode(status).name} ({last_error()})")
    check_status(status, what)


class _BsBase:
    __slots__ = ("_ptr", "_lib")
    _prefix = ""
    _np_dtype = np.float64
    _width = 1
    _dense_cls = TensorF64

    def __init__(self, ptr):
        self._lib = get_lib()
        self._ptr = ptr

    def __del__(self):
        if getattr(self, "_ptr", None):
            getattr(self._lib, f"ndt_blocksparse_{self._prefix}_release")(self._ptr)
            self._ptr = None

    def _f(self, name):
        return getattr(self._lib, f"ndt_blocksparse_{self._prefix}_{name}")

    @classmethod
    def zeros(cls, block_sizes: Sequence[Sequence[int]], coords: Sequence[Sequence[int]]):
        ndim, nblk, bsz, nnzb, cs = _structure_args(block_sizes, coords)
        st = ctypes.c_int(-999)
        p = getattr(get_lib(), f"ndt_blocksparse_{cls._prefix}_zeros")(ndim, nblk, bsz, nnzb, cs, ctypes.byref(st))
        check_status(st.value, "blocksparse zeros")
        return cls(p)

    @classmethod
    def from_blocks(cls, block_sizes, coords, data):
        """Packed data (blocks in `coords` order, each column-major)."""
        ndim, nblk, bsz, nnzb, cs = _structure_args(block_sizes, coords)
        arr = np.ascontiguousarray(np.asarray(data, dtype=cls._np_dtype).ravel())
        buf = arr.view(np.float64) if arr.size else np.zeros(1)
        st = ctypes.c_int(-999)
        p = getattr(get_lib(), f"ndt_blocksparse_{cls._prefix}_from_data")(
            ndim, nblk, bsz, nnzb, cs, buf.ctypes.data_as(c_double_p), arr.size, ctypes.byref(st))
        _raise(st.value, "blocksparse from_data")
        return cls(p)

    @classmethod
    def from_torch(cls, block_sizes, coords, data):
        """Packed data from a CUDA torch tensor (copied device to device)."""
        import torch

        want = torch.complex128 if cls._width == 2 else torch.float64
        d = data.to(want).contiguous()
        ndim, nblk, bsz, nnzb, cs = _structure_args(block_sizes, coords)
        st = ctypes.c_int(-999)
        p = getattr(get_lib(), f"ndt_blocksparse_{cls._prefix}_from_device_ptr")(
            ndim, nblk, bsz, nnzb, cs, ctypes.c_void_p(d.data_ptr()), d.numel(), ctypes.byref(st))
        _raise(st.value, "blocksparse from_device_ptr")
        return cls(p)

    def device_ptr(self) -> int:
        return self._f("device_ptr")(self._ptr)

    @classmethod
    def from_dense(cls, dense, block_sizes, coords):
        ndim, nblk, bsz, nnzb, cs = _structure_args(block_sizes, coords)
        st = ctypes.c_int(-999)
        p = getattr(get_lib(), f"ndt_blocksparse_{cls._prefix}_from_dense")(
            dense._ptr, ndim, nblk, bsz, nnzb, cs, ctypes.byref(st))
        _raise(st.value, "blocksparse from_dense")
        return cls(p)

    @property
    def ndim(self) -> int:
        return int(self._f("ndim")(self._ptr))

    @property
    def nnzblocks(self) -> int:
        return int(self._f("nnzblocks")(self._ptr))

    @property
    def nnz(self) -> int:
        return int(self._f("nnz")(self._ptr))

    def _structure(self):
        nd, nb = self.ndim, self.nnzblocks
        nbt = int(self._f("nblocks_total")(self._ptr))
        nblk = (SZ * max(nd, 1))()
        bsz = (SZ * max(nbt, 1))()
        cs = (SZ * max(nb * nd, 1))()
        offs = (SZ * max(nb, 1))()
        check_status(self._f("structure")(self._ptr, nblk, bsz, cs, offs), "structure")
        sizes, k = [], 0
        for ax in range(nd):
            sizes.append([int(bsz[k + i]) for i in range(nblk[ax])])
            k += nblk[ax]
        coords = [tuple(int(cs[b * nd + i]) for i in range(nd)) for b in range(nb)]
        return sizes, coords, [int(offs[b]) for b in range(nb)]

    @property
    def block_sizes(self) -> List[List[int]]:
        return self._structure()[0]

    @property
    def coords(self) -> List[Tuple[int, ...]]:
        return self._structure()[1]

    @property
    def dense_shape(self) -> Tuple[int, ...]:
        return tuple(sum(b) for b in self.block_sizes)

    def to_numpy_data(self) -> np.ndarray:
        n = self.nnz
        if n == 0:
            return np.zeros(0, dtype=self._np_dtype)
        p = self._f("data")(self._ptr)
        if not p:
            raise NDTensorsError(f"data: {last_error()}")
        flat = np.ctypeslib.as_array(p, shape=(n * self._width,)).copy()
        return flat.view(np.complex128) if self._width == 2 else flat

    def block(self, coords) -> np.ndarray:
        sizes = self.block_sizes
        shape = tuple(sizes[ax][c] for ax, c in enumerate(coords))
        n = int(np.prod(shape, dtype=np.int64))
        out = np.zeros(max(n, 1) * self._width)
        st = self._f("get_block")(self._ptr, (SZ * len(coords))(*coords), out.ctypes.data_as(c_double_p), max(n, 1))
        if st == StatusCode.INDEX_OUT_OF_BOUNDS:
            raise KeyError(f"block {tuple(coords)} not stored")
        check_status(st, "get_block")
        v = out.view(np.complex128) if self._width == 2 else out
        return v[:n].reshape(shape, order="F")

    def insert_block(self, coords, data) -> None:
        arr = np.asfortranarray(np.asarray(data, dtype=self._np_dtype))
        flat = np.ascontiguousarray(arr.ravel(order="F"))
        buf = flat.view(np.float64)
        st = self._f("insert_block")(self._ptr, (SZ * len(coords))(*coords), buf.ctypes.data_as(c_double_p), flat.size)
        if st == StatusCode.INDEX_OUT_OF_BOUNDS:
            raise KeyError(f"block {tuple(coords)} not stored")
        _raise(st, "insert_block")

    def to_dense(self):
        st = ctypes.c_int(-999)
        p = self._f("to_dense")(self._ptr, ctypes.byref(st))
        check_status(st.value, "to_dense")
        return self._dense_cls(p)

    def permutedims(self, perm: Sequence[int]):
        st = ctypes.c_int(-999)
        p = self._f("permutedims")(self._ptr, (SZ * max(len(perm), 1))(*perm), len(perm), ctypes.byref(st))
        if st.value == StatusCode.INVALID_PERMUTATION:
            raise ValueError(f"Invalid permutation: {perm}")
        check_status(st.value, "permutedims")
        return type(self)(p)

    def __repr__(self):
        return f"{type(self).__name__}(dense_shape={self.dense_shape}, nnzblocks={self.nnzblocks})"


class BlockSparseF64(_BsBase):
    __slots__ = ()
    _prefix = "f64"
    _np_dtype = np.float64
    _width = 1
    _dense_cls = TensorF64


class BlockSparseC64(_BsBase):
    __slots__ = ()
    _prefix = "c64"
    _np_dtype = np.complex128
    _width = 2
    _dense_cls = TensorC64


class _DiagBase:
    __slots__ = ("_ptr", "_lib")
    _prefix = ""
    _np_dtype = np.float64
    _dense_cls = TensorF64
    _bs_cls = BlockSparseF64

    def __init__(self, ptr):
        self._lib = get_lib()
        self._ptr = ptr

    def __del__(self):
        if getattr(self, "_ptr", None):
            getattr(self._lib, f"ndt_diagblocksparse_{self._prefix}_release")(self._ptr)
            self._ptr = None

    @classmethod
    def from_blocks(cls, block_sizes, coords, diag):
        """Diagonal values of each listed block (min of its extents), packed in order."""
        ndim, nblk, bsz, nnzb, cs = _structure_args(block_sizes, coords)
        arr = np.ascontiguousarray(np.asarray(diag, dtype=cls._np_dtype).ravel())
        buf = arr.view(np.float64) if arr.size else np.zeros(1)
        st = ctypes.c_int(-999)
        p = getattr(get_lib(), f"ndt_diagblocksparse_{cls._prefix}_from_data")(
            ndim, nblk, bsz, nnzb, cs, buf.ctypes.data_as(c_double_p), arr.size, ctypes.byref(st))
        _raise(st.value, "diagblocksparse from_data")
        return cls(p)

    @property
    def nnz(self):
        return int(getattr(self._lib, f"ndt_diagblocksparse_{self._prefix}_nnz")(self._ptr))

    def to_dense(self):
        st = ctypes.c_int(-999)
        p = getattr(self._lib, f"ndt_diagblocksparse_{self._prefix}_to_dense")(self._ptr, ctypes.byref(st))
        check_status(st.value, "to_dense")
        return self._dense_cls(p)

    def to_blocksparse(self):
        st = ctypes.c_int(-999)
        p = getattr(self._lib, f"ndt_diagblocksparse_{self._prefix}_to_blocksparse")(self._ptr, ctypes.byref(st))
        check_status(st.value, "to_blocksparse")
        return self._bs_cls(p)


class DiagBlockSparseF64(_DiagBase):
    __slots__ = ()
    _prefix = "f64"
    _np_dtype = np.float64
    _dense_cls = TensorF64
    _bs_cls = BlockSparseF64


class DiagBlockSparseC64(_DiagBase):
    __slots__ = ()
    _prefix = "c64"
    _np_dtype = np.complex128
    _dense_cls = TensorC64
    _bs_cls = BlockSparseC64


def _labels(ls):
    return (ctypes.c_long * max(len(ls), 1))(*ls), len(ls)


def contract(a, labels_a, b, labels_b):
    """contract_blocksparse: sorted output blocks, one grouped GEMM launch."""
    if type(a) is not type(b):
        raise TypeError("operands must have the same element type")
    la, na = _labels(labels_a)
    lb, nb = _labels(labels_b)
    st = ctypes.c_int(-999)
    p = a._f("contract")(a._ptr, la, na, b._ptr, lb, nb, ctypes.byref(st))
    _raise(st.value, "blocksparse contract")
    return type(a)(p)


def contract_shard(a, labels_a, b, labels_b, rank: int, nranks: int):
    """This rank's FLOP-balanced share of the output blocks (no collective):
    output blocks go to ranks heaviest first, each to the least loaded rank,
    so every rank derives the same assignment from the same operands."""
    la, na = _labels(labels_a)
    lb, nb = _labels(labels_b)
    st = ctypes.c_int(-999)
    p = a._f("contract_shard")(a._ptr, la, na, b._ptr, lb, nb, int(rank), int(nranks), ctypes.byref(st))
    _raise(st.value, "blocksparse contract_shard")
    return type(a)(p)


def contract_select(a, labels_a, b, labels_b, out_coords):
    """Only the listed output blocks (natural order: A's free axes, then B's),
    computed from the blocks the operands hold."""
    la, na = _labels(labels_a)
    lb, nb = _labels(labels_b)
    flat = [int(x) for c in out_coords for x in c]
    cs = (SZ * max(len(flat), 1))(*flat)
    st = ctypes.c_int(-999)
    p = a._f("contract_select")(a._ptr, la, na, b._ptr, lb, nb, cs, len(out_coords), ctypes.byref(st))
    _raise(st.value, "blocksparse contract_select")
    return type(a)(p)


def shard_plan(a, labels_a, b, labels_b, nranks: int):
    """Output blocks and real flops per rank of contract_shard (host only)."""
    la, na = _labels(labels_a)
    lb, nb = _labels(labels_b)
    blocks = (SZ * nranks)()
    flops = (ctypes.c_double * nranks)()
    st = a._f("shard_plan")(a._ptr, la, na, b._ptr, lb, nb, int(nranks), blocks, flops)
    _raise(st, "blocksparse shard_plan")
    return [int(x) for x in blocks], [float(x) for x in flops]


class _DeviceSpan:
    """A raw device range exposed through __cuda_array_interface__ (zero copy)."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f8", "data": (int(ptr), False),
                                         "strides": None, "version": 2}


def allgather(shard, group=None):
    """Gather every rank's shard (disjoint output blocks of one contraction)
    into the full block-sparse tensor on all ranks, with torch.distributed.
    Blocks come out sorted, as contract_blocksparse orders them.

    Two collectives: the per-rank lengths, then one all_gather of every
    rank's [packed data, block coordinates] padded to the longest (on NCCL
    all links carry data at once and nothing leaves HBM but the
    coordinates).  Shards hold interleaved subsets of the sorted output
    block list (contract_shard assigns blocks by longest processing time),
    so one device concatenation of the received blocks, taken in sorted
    coordinate order, gives the packed data.  On gloo (CPU tests) the same
    steps run on host tensors."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    nccl = dist.get_backend(group) == "nccl"
    dev = torch.device("cuda", torch.cuda.current_device()) if nccl else torch.device("cpu")
    sizes, coords, _ = shard._structure()
    nd = len(sizes)
    width = shard._width
    nelem = shard.nnz
    nval = nelem * width                      # doubles of packed data
    ncrd = len(coords) * nd                   # int64 coordinates
    meta = torch.tensor([nval, ncrd], dtype=torch.int64, device=dev)
    metas = torch.empty(world * 2, dtype=torch.int64, device=dev)
    dist.all_gather_into_tensor(metas, meta, group=group)
    counts = metas.view(world, 2).tolist()
    pad = max(max(v + c for v, c in counts), 1)
    send = torch.empty(pad, dtype=torch.float64, device=dev)
    if nval:
        if nccl:
            # the shard was written on the library's stream
            if get_lib().ndt_b200_get_stream() != torch.cuda.current_stream().cuda_stream:
                check_status(get_lib().ndt_b200_synchronize(), "synchronize")
            own = torch.as_tensor(_DeviceSpan(shard.device_ptr(), nval), device=dev)
        else:
            own = torch.from_numpy(np.ascontiguousarray(shard.to_numpy_data()).view(np.float64))
        send[:nval].copy_(own)
    if ncrd:
        send[nval: nval + ncrd].view(torch.int64).copy_(
            torch.tensor([x for c in coords for x in c], dtype=torch.int64, device=dev))
    recv = torch.empty(world * pad, dtype=torch.float64, device=dev)
    dist.all_gather_into_tensor(recv, send, group=group)
    # every rank's blocks, as (coords, start in recv, doubles), in rank order
    blocks = []
    for r, (v, c) in enumerate(counts):
        if not c:
            continue
        flat_c = recv[r * pad + v: r * pad + v + c].view(torch.int64).tolist()
        start = r * pad
        for i in range(0, len(flat_c), nd):
            crd = tuple(flat_c[i: i + nd])
            n = width
            for ax, q in enumerate(crd):
                n *= sizes[ax][q]
            blocks.append((crd, start, n))
            start += n
    blocks.sort(key=lambda x: x[0])
    all_coords = [b[0] for b in blocks]
    # runs of blocks that are adjacent in recv become one slice each
    parts, run0, run1 = [], None, None
    for _, st_, n in blocks:
        if run1 is not None and st_ == run1:
            run1 += n
            continue
        if run1 is not None and run1 > run0:
            parts.append(recv[run0:run1])
        run0, run1 = st_, st_ + n
    if run1 is not None and run1 > run0:
        parts.append(recv[run0:run1])
    data = torch.cat(parts) if parts else torch.empty(0, dtype=torch.float64, device=dev)
    if nccl:
        torch.cuda.current_stream().synchronize()
        return type(shard).from_torch(sizes, all_coords, data.view(torch.complex128) if width == 2 else data)
    flat = data.numpy()
    return type(shard).from_blocks(sizes, all_coords, flat.view(np.complex128) if width == 2 else flat)


def contract_through_diag(a, labels_a, s, labels_s, b, labels_b, rank: int = 0, nranks: int = 1):
    """(A . S) . B with S a rank-2 DiagBlockSparse between A and B: S's first
    label is contracted with one axis of A, its second with one axis of B,
    and every other label of A and B is positive.  The result is
    contract(contract_diag(A, S), B): the free axes of A and B in label
    order.  Runs as one grouped launch that scales A's contracted index by
    S's diagonal while loading A (no A . S intermediate) when S's blocks are
    square and each coordinate of A's contracted axis meets one S block.
    rank / nranks: this rank's share of the output blocks (contract_shard's
    assignment)."""
    la, na = _labels(labels_a)
    ls, ns = _labels(labels_s)
    lb, nb = _labels(labels_b)
    st = ctypes.c_int(-999)
    p = a._f("contract_through_diag")(a._ptr, la, na, s._ptr, ls, ns, b._ptr, lb, nb, int(rank), int(nranks),
                                      ctypes.byref(st))
    _raise(st.value, "blocksparse contract_through_diag")
    return type(a)(p)


def contract_diag(a, labels_a, s, labels_s):
    """Block-sparse x diag-block-sparse (diagonal blocks as dense blocks)."""
    la, na = _labels(labels_a)
    ls, ns = _labels(labels_s)
    st = ctypes.c_int(-999)
    p = a._f("contract_diag")(a._ptr, la, na, s._ptr, ls, ns, ctypes.byref(st))
    _raise(st.value, "blocksparse contract_diag")
    return type(a)(p)


__all__ = ["BlockSparseF64", "BlockSparseC64", "DiagBlockSparseF64", "DiagBlockSparseC64", "contract",
           "contract_shard", "contract_select", "shard_plan", "allgather", "contract_diag", "contract_through_diag"]
