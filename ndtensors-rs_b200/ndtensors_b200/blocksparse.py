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
        if not d.is_cuda:
            return cls.from_blocks(block_sizes, coords, d.numpy())
        ndim, nblk, bsz, nnzb, cs = _structure_args(block_sizes, coords)
        # torch wrote d on its own stream; the library copies it on another
        torch.cuda.current_stream(d.device).synchronize()
        st = ctypes.c_int(-999)
        p = getattr(get_lib(), f"ndt_blocksparse_{cls._prefix}_from_device_ptr")(
            ndim, nblk, bsz, nnzb, cs, ctypes.c_void_p(d.data_ptr()), d.numel(), ctypes.byref(st))
        _raise(st.value, "blocksparse from_device_ptr")
        # the copy has read d before d (a temporary) goes back to torch
        check_status(get_lib().ndt_b200_synchronize(), "synchronize")
        return cls(p)

    @classmethod
    def from_device_blocks(cls, block_sizes, coords, src_offsets, src_ptr: int, src_len: int):
        """Blocks read from anywhere in device memory: block i of `coords` at
        element offset src_offsets[i] of the buffer at src_ptr (src_len
        elements); the result holds them sorted by coordinates, packed (one
        copy kernel)."""
        if isinstance(coords, np.ndarray):  # n x ndim array: no per-block Python objects
            ndim = len(block_sizes)
            flat = [int(x) for b in block_sizes for x in b]
            nblk = (SZ * max(ndim, 1))(*[len(b) for b in block_sizes])
            bsz = (SZ * max(len(flat), 1))(*flat)
            carr = np.ascontiguousarray(coords, dtype=np.uint64).ravel()
            nnzb = coords.shape[0]
            cs = carr.ctypes.data_as(ctypes.POINTER(SZ)) if carr.size else (SZ * 1)()
        else:
            ndim, nblk, bsz, nnzb, cs = _structure_args(block_sizes, coords)
        offs = np.ascontiguousarray(np.asarray(src_offsets, dtype=np.uint64))
        op = offs.ctypes.data_as(ctypes.POINTER(SZ)) if offs.size else (SZ * 1)()
        st = ctypes.c_int(-999)
        p = getattr(get_lib(), f"ndt_blocksparse_{cls._prefix}_from_device_blocks")(
            ndim, nblk, bsz, nnzb, cs, op, ctypes.c_void_p(int(src_ptr)), int(src_len), ctypes.byref(st))
        _raise(st.value, "blocksparse from_device_blocks")
        return cls(p)

    def _shard_layout(self):
        """(nranks, all output block coordinates (n x ndim, sorted), owner
        rank of each) for a shard of a sharded contraction, else None."""
        nr, nb = ctypes.c_int(0), SZ(0)
        if self._f("shard_layout")(self._ptr, ctypes.byref(nr), ctypes.byref(nb), None, None) != 0:
            return None
        nd = max(self.ndim, 1)
        crd = np.zeros(max(nb.value * nd, 1), dtype=np.uint64)
        own = np.zeros(max(nb.value, 1), dtype=np.int32)
        st = self._f("shard_layout")(self._ptr, ctypes.byref(nr), ctypes.byref(nb),
                                     crd.ctypes.data_as(ctypes.POINTER(SZ)),
                                     own.ctypes.data_as(ctypes.POINTER(ctypes.c_int)))
        check_status(st, "shard_layout")
        return nr.value, crd[: nb.value * nd].reshape(nb.value, nd).astype(np.int64), own[: nb.value]

    def device_ptr(self) -> int:
        return self._f("device_ptr")(self._ptr)

    def device_ptr_mut(self) -> int:
        """Device buffer of the packed data for writing from outside the
        library (copy on write if shared; the device copy then holds the
        values)."""
        p = self._f("device_ptr_mut")(self._ptr)
        if not p:
            raise NDTensorsError(f"device_ptr_mut: {last_error()}")
        return p

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
    """A raw device range exposed through __cuda_array_interface__ (zero copy).

    Version 3 with the library's compute stream as "stream": a consumer (torch)
    makes its own stream wait for the library's work on the range before it
    touches it.  device_ptr / device_ptr_mut already return with that work
    complete when the library runs on its own stream; with a caller stream
    installed (ndt_b200_set_stream) the key orders the two streams."""

    def __init__(self, ptr: int, n: int):
        lib_stream = get_lib().ndt_b200_get_stream() or 0
        cai = {"shape": (n,), "typestr": "<f8", "data": (int(ptr), False), "strides": None, "version": 3}
        if lib_stream:
            cai["stream"] = int(lib_stream)
        self.__cuda_array_interface__ = cai


_HOST_GROUPS = {}


def _host_group(group, dist):
    """A gloo group over the same ranks as `group` (created once, collectively
    on first use): host-side exchanges that must not queue behind the
    device collectives of the NCCL group."""
    key = id(group) if group is not None else None
    g = _HOST_GROUPS.get(key)
    if g is None:
        ranks = dist.get_process_group_ranks(group) if group is not None else list(range(dist.get_world_size()))
        g = _HOST_GROUPS[key] = dist.new_group(ranks=ranks, backend="gloo")
    return g


class Comm:
    """The library's NCCL communicator (ndt_comm) over the ranks of a job, one
    process per GPU.  ``Comm.from_group(group)`` builds it collectively over a
    torch.distributed group: rank 0 creates NCCL's unique id and the group
    broadcasts it.  Used by contract_gathered, contract_through_diag_gathered
    and allgather, which gather a sharded result in the library (an in-place
    NCCL all-gather, then one copy kernel into the sorted output)."""

    _by_group = {}

    def __init__(self, ptr: int):
        self._lib = get_lib()
        self._ptr = ptr

    def __del__(self):
        if getattr(self, "_ptr", None):
            self._lib.ndt_b200_comm_release(self._ptr)
            self._ptr = None

    release = __del__

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(128)
        check_status(get_lib().ndt_b200_comm_unique_id(buf), "comm_unique_id")
        return buf.raw

    @classmethod
    def init(cls, uid: bytes, nranks: int, rank: int) -> "Comm":
        st = ctypes.c_int(-999)
        p = get_lib().ndt_b200_comm_init(uid, int(nranks), int(rank), ctypes.byref(st))
        check_status(st.value, "comm_init")
        return cls(p)

    @classmethod
    def from_group(cls, group=None) -> "Comm":
        """Collective over `group` (default: the world); cached per group."""
        import torch.distributed as dist

        key = id(group) if group is not None else None
        c = cls._by_group.get(key)
        if c is None:
            obj = [cls.unique_id() if dist.get_rank(group) == 0 else None]
            src = dist.get_global_rank(group, 0) if group is not None else 0
            dist.broadcast_object_list(obj, src=src, group=group)
            c = cls._by_group[key] = cls.init(obj[0], dist.get_world_size(group), dist.get_rank(group))
        return c

    @property
    def rank(self) -> int:
        return int(self._lib.ndt_b200_comm_rank(self._ptr))

    @property
    def size(self) -> int:
        return int(self._lib.ndt_b200_comm_size(self._ptr))


def contract_gathered(a, labels_a, b, labels_b, comm: Comm):
    """contract() with the work split over the communicator's ranks and the
    result gathered on every rank (collective: every rank calls it with the
    same operands).  Each rank computes its share of the output blocks and
    stores every tile into every rank's output buffer as it computes it (the
    ranks map each other's buffers); when they cannot, each rank's blocks are
    gathered with an NCCL all-gather."""
    la, na = _labels(labels_a)
    lb, nb = _labels(labels_b)
    st = ctypes.c_int(-999)
    p = a._f("contract_gathered")(a._ptr, la, na, b._ptr, lb, nb, comm._ptr, ctypes.byref(st))
    _raise(st.value, "blocksparse contract_gathered")
    return type(a)(p)


def contract_through_diag_gathered(a, labels_a, s, labels_s, b, labels_b, comm: Comm):
    """contract_through_diag() split over the communicator's ranks (one
    grouped launch per chunk with S applied as the operands load) and gathered
    on every rank (collective)."""
    la, na = _labels(labels_a)
    ls, ns = _labels(labels_s)
    lb, nb = _labels(labels_b)
    st = ctypes.c_int(-999)
    p = a._f("contract_through_diag_gathered")(a._ptr, la, na, s._ptr, ls, ns, b._ptr, lb, nb, comm._ptr,
                                                 ctypes.byref(st))
    _raise(st.value, "blocksparse contract_through_diag_gathered")
    return type(a)(p)


def allgather(shard, group=None, comm: Comm = None):
    """Gather every rank's shard (disjoint output blocks of one contraction)
    into the full block-sparse tensor on all ranks, with torch.distributed.
    Blocks come out sorted, as contract_blocksparse orders them.

    The layout (which rank holds which blocks) comes with the shards of a
    sharded contraction (contract_shard, contract_through_diag): every rank
    derived the same assignment, so nothing is exchanged.  Other shards
    exchange their structure (packed length, block count, block
    coordinates) in one small all_gather over host memory; with NCCL it runs
    on a gloo group over the same ranks, so it neither waits for the kernel
    still computing the shard nor queues behind device collectives.  Then one
    all_gather moves every rank's packed data, padded to the longest, over
    NVLink, and the library assembles the sorted tensor from the gathered
    buffer with one copy kernel (from_device_blocks).  Nothing on the host
    waits for the device.  On gloo (CPU tests) the same steps run on host
    tensors.

    With `comm` (or on an NCCL group, for a shard that carries its layout)
    the library gathers the shard itself (ndt_blocksparse_*_allgather): one
    in-place NCCL all-gather of the shards, then one copy kernel into the
    sorted output, with no Python work per block."""
    import torch
    import torch.distributed as dist

    layout0 = shard._shard_layout()
    if comm is None and layout0 is not None and dist.get_backend(group) == "nccl" and \
            layout0[0] == dist.get_world_size(group):
        comm = Comm.from_group(group)
    if comm is not None:
        st = ctypes.c_int(-999)
        p = shard._f("allgather")(shard._ptr, comm._ptr, ctypes.byref(st))
        _raise(st.value, "blocksparse allgather")
        return type(shard)(p)
    world = dist.get_world_size(group)
    nccl = dist.get_backend(group) == "nccl"
    dev = torch.device("cuda", torch.cuda.current_device()) if nccl else torch.device("cpu")
    sizes, coords, _ = shard._structure()
    nd = max(len(sizes), 1)
    width = shard._width
    nval = shard.nnz * width  # doubles of packed data
    cap = 1
    for b in sizes:
        cap *= max(len(b), 1)

    # ---- structure: [packed length, block count, coordinates...] of every rank
    def exchange(cpad):
        mine = np.zeros(2 + cpad * nd, dtype=np.int64)
        mine[0], mine[1] = nval, len(coords)
        if coords:
            mine[2: 2 + len(coords) * nd] = np.asarray(coords, dtype=np.int64).ravel()
        outs = [torch.empty(mine.size, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(outs, torch.from_numpy(mine), group=hg)
        return torch.stack(outs).numpy()

    size_arr = [np.asarray(b, dtype=np.int64) for b in sizes]

    def elems_of(cr):
        e = np.ones(cr.shape[0], dtype=np.int64)
        for ax in range(len(sizes)):
            e *= size_arr[ax][cr[:, ax]]
        return e

    # every rank's blocks (each shard stores its blocks sorted) and packed length
    layout = shard._shard_layout()
    hg = (_host_group(group, dist) if nccl else group) if layout is None or layout[0] != world else None
    if layout is not None and layout[0] == world:
        # a shard of a sharded contraction: every rank knows the whole layout
        _, lc, lo = layout
        per_rank = [lc[lo == r] for r in range(world)]
        nvals = [int(elems_of(cr).sum()) * width for cr in per_rank]
    else:
        if cap * nd <= (1 << 19):
            table = exchange(cap)
        else:  # very many possible blocks: block counts first, then coordinates
            cnts = [torch.empty(1, dtype=torch.int64) for _ in range(world)]
            dist.all_gather(cnts, torch.tensor([len(coords)], dtype=torch.int64), group=hg)
            table = exchange(max(int(max(c.item() for c in cnts)), 1))
        nvals = [int(v) for v in table[:, 0]]
        per_rank = [table[r, 2: 2 + int(table[r, 1]) * nd].reshape(int(table[r, 1]), nd) for r in range(world)]
    # element offsets in the gathered buffer (rank r's data starts at r * pad doubles)
    pad = max(max(nvals), 1)
    pad += pad % width  # whole elements per rank
    all_c, all_off = [], []
    for r, cr in enumerate(per_rank):
        if not cr.shape[0]:
            continue
        e = elems_of(cr)
        all_c.append(cr)
        all_off.append(r * (pad // width) + np.concatenate(([0], np.cumsum(e)[:-1])))
    gathered_c = np.concatenate(all_c) if all_c else np.zeros((0, nd), dtype=np.int64)
    gathered_off = np.concatenate(all_off) if all_off else np.zeros(0, dtype=np.int64)

    # ---- data: one all_gather of the packed shards, padded to the longest
    if nccl and get_lib().ndt_b200_get_stream() != torch.cuda.current_stream().cuda_stream:
        check_status(get_lib().ndt_b200_synchronize(), "synchronize")  # shard written on another stream
    send = torch.empty(pad, dtype=torch.float64, device=dev)
    if nval:
        if nccl:
            own = torch.as_tensor(_DeviceSpan(shard.device_ptr(), nval), device=dev)
        else:
            own = torch.from_numpy(np.ascontiguousarray(shard.to_numpy_data()).view(np.float64))
        send[:nval].copy_(own)
    recv = torch.empty(world * pad, dtype=torch.float64, device=dev)
    dist.all_gather_into_tensor(recv, send, group=group)
    if not nccl:
        coord_list = [tuple(int(x) for x in row) for row in gathered_c] if len(sizes) else [() for _ in gathered_c]
        flat = recv.numpy().view(np.complex128) if width == 2 else recv.numpy()
        parts = [flat[o: o + int(np.prod([sizes[a][q] for a, q in enumerate(c)]))]
                 for c, o in zip(coord_list, gathered_off)]
        order = sorted(range(len(coord_list)), key=lambda i: coord_list[i])
        data = np.concatenate([parts[i] for i in order]) if order else flat[:0]
        return type(shard).from_blocks(sizes, [coord_list[i] for i in order], data)
    lib_stream = get_lib().ndt_b200_get_stream()
    if lib_stream != torch.cuda.current_stream().cuda_stream:
        torch.cuda.current_stream().synchronize()  # the library reads recv on its own stream
    out = type(shard).from_device_blocks(sizes, gathered_c, gathered_off, recv.data_ptr(), recv.numel() // width)
    if lib_stream != torch.cuda.current_stream().cuda_stream:
        check_status(get_lib().ndt_b200_synchronize(), "synchronize")  # before recv goes back to torch
    return out


def contract_through_diag(a, labels_a, s, labels_s, b, labels_b, rank: int = 0, nranks: int = 1):
    """(A . S) . B with S a rank-2 DiagBlockSparse between A and B: S's first
    label is contracted with one axis of A, its second with one axis of B,
    and every other label of A and B is positive.  The result is
    contract(contract_diag(A, S), B): the free axes of A and B in label
    order.  Sharded (nranks > 1), runs as one grouped launch that applies
    S's diagonal to the contracted index while loading the operands (no
    A . S intermediate) when S's blocks are square and each coordinate of
    A's contracted axis meets one S block; unsharded, the two contractions
    in turn (one pass over A costs less than the in-GEMM scaling when a rank
    does all the work).
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
