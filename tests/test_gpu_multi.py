"""Sharded block-sparse contraction on 2 to 8 GPUs over NCCL.

Each rank computes its cost-balanced share of the output blocks
(contract_shard, contract_through_diag) and the shards are gathered in HBM
by the library (allgather over the library's NCCL communicator: one in-place
all-gather, one copy kernel into the sorted output).  The gathered
contractions of the C ABI (contract_gathered, contract_through_diag_gathered:
each tile stored into every rank's mapped buffer as it is computed, or chunk
by chunk over NCCL when the buffers cannot be mapped) are checked the same way, and the c128
chain at bond 8192 block by block against the CPU block reference.  The
gathered tensor must equal the unsharded contraction on one GPU (relative
error 1e-12); every rank's gathered bytes must be identical.  Runs as one
spawned process per visible GPU (at most 8); skipped when fewer than two
devices are visible.
"""

from __future__ import annotations

import datetime
import hashlib
import os
import socket
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "ndtensors-rs_b200"))
    sys.path.insert(0, os.path.join(root, "tests"))
    import ndtensors_b200 as ndt
    from workloads import cfg4_tensors, cfg5_tensors

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    bs = ndt.blocksparse
    results = []
    try:
        # U(1) rank-4 x rank-4, sector dims / 8 (f64)
        (sa, ca, a), (sb, cb, b), la, lb = cfg4_tensors(scale=8)
        A = bs.BlockSparseF64.from_blocks(sa, ca, a)
        B = bs.BlockSparseF64.from_blocks(sb, cb, b)
        full = bs.contract(A, la, B, lb)
        shard = bs.contract_shard(A, la, B, lb, rank, world)
        gathered = bs.allgather(shard)
        ok = gathered.coords == full.coords and np.allclose(
            gathered.to_numpy_data(), full.to_numpy_data(), rtol=1e-12, atol=1e-12)
        results.append(("cfg4/8 f64", bool(ok), shard.nnzblocks, full.nnzblocks))
        # c128 two-site MPS chain with the diagonal bond tensor, bond 1024
        (sa, ca, a), (ss, cs_, sd), (sb, cb, b) = cfg5_tensors(bond=1024)
        A = bs.BlockSparseC64.from_blocks(sa, ca, a)
        S = bs.DiagBlockSparseC64.from_blocks(ss, cs_, sd)
        B = bs.BlockSparseC64.from_blocks(sb, cb, b)
        AS = bs.contract_diag(A, [1, 2, -1], S, [-1, 3])
        full = bs.contract(AS, [1, 2, -1], B, [-1, 3, 4])
        gathered = bs.allgather(bs.contract_shard(AS, [1, 2, -1], B, [-1, 3, 4], rank, world))
        ok = gathered.coords == full.coords and np.allclose(
            gathered.to_numpy_data(), full.to_numpy_data(), rtol=1e-12, atol=1e-12)
        results.append(("cfg5 bond 1024 c128", bool(ok), -1, full.nnzblocks))
        # the same chain through the diagonal as one launch per rank
        gathered = bs.allgather(bs.contract_through_diag(A, [1, 2, -1], S, [-1, -2], B, [-2, 3, 4], rank, world))
        ok = gathered.coords == full.coords and np.allclose(
            gathered.to_numpy_data(), full.to_numpy_data(), rtol=1e-12, atol=1e-12)
        results.append(("cfg5 bond 1024 c128 through diag", bool(ok), -1, full.nnzblocks))
        # the library's communicator and gathered contractions (C ABI)
        comm = bs.Comm.from_group()
        assert (comm.rank, comm.size) == (rank, world)
        gathered = bs.allgather(bs.contract_through_diag(A, [1, 2, -1], S, [-1, -2], B, [-2, 3, 4], rank, world),
                                comm=comm)
        ok = gathered.coords == full.coords and np.allclose(
            gathered.to_numpy_data(), full.to_numpy_data(), rtol=1e-12, atol=1e-12)
        results.append(("cfg5 bond 1024 allgather (library)", bool(ok), -1, full.nnzblocks))
        gathered = bs.contract_through_diag_gathered(A, [1, 2, -1], S, [-1, -2], B, [-2, 3, 4], comm)
        ok = gathered.coords == full.coords and np.allclose(
            gathered.to_numpy_data(), full.to_numpy_data(), rtol=1e-12, atol=1e-12)
        results.append(("cfg5 bond 1024 contract_through_diag_gathered", bool(ok), -1, full.nnzblocks))
        (sa, ca, a), (sb, cb, b), la, lb = cfg4_tensors(scale=8)
        A4 = bs.BlockSparseF64.from_blocks(sa, ca, a)
        B4 = bs.BlockSparseF64.from_blocks(sb, cb, b)
        full4 = bs.contract(A4, la, B4, lb)
        g4 = bs.contract_gathered(A4, la, B4, lb, comm)
        ok = g4.coords == full4.coords and np.array_equal(g4.to_numpy_data(), full4.to_numpy_data())
        results.append(("cfg4/8 f64 contract_gathered (bit-exact)", bool(ok), -1, full4.nnzblocks))
        # permuted operand blocks (strided plan: the tiles reach the peers
        # through the strided epilogue), f64 and c128, against the unsharded
        # natural-order contraction of the same data
        Ap4 = A4.permutedims([2, 0, 3, 1])  # labels (-1, 1, -2, 2)
        gp4 = bs.contract_gathered(Ap4, [-1, 1, -2, 2], B4, lb, comm)
        ok = gp4.coords == full4.coords and np.array_equal(gp4.to_numpy_data(), full4.to_numpy_data())
        results.append(("cfg4/8 f64 permuted A contract_gathered (bit-exact)", bool(ok), -1, full4.nnzblocks))
        AS1 = bs.contract_diag(A, [1, 2, -1], S, [-1, 3])
        full1 = bs.contract(AS1, [1, 2, -1], B, [-1, 3, 4])
        gp5 = bs.contract_gathered(AS1.permutedims([2, 0, 1]), [-1, 1, 2], B, [-1, 3, 4], comm)
        ok = gp5.coords == full1.coords and np.allclose(gp5.to_numpy_data(), full1.to_numpy_data(), rtol=1e-12,
                                                        atol=1e-12)
        results.append(("cfg5 bond 1024 c128 permuted A contract_gathered", bool(ok), -1, full1.nnzblocks))
        # bond 8192 (the benchmark's size), every block against the CPU reference
        from blockref import reference_blocks, rel_fro

        Ah, Sh, Bh = cfg5_tensors()
        A8 = bs.BlockSparseC64.from_blocks(*Ah)
        S8 = bs.DiagBlockSparseC64.from_blocks(*Sh)
        B8 = bs.BlockSparseC64.from_blocks(*Bh)
        for _ in range(2):  # twice in a row: the second call reuses the communicator
            g8 = bs.contract_through_diag_gathered(A8, [1, 2, -1], S8, [-1, -2], B8, [-2, 3, 4], comm)
        _, c8, o8 = g8._structure()
        d8 = g8.to_numpy_data()
        # every rank holds the same bytes (each block is computed by one rank
        # and stored to all); rank 0 checks them against the CPU reference
        digest = hashlib.sha256(np.ascontiguousarray(d8).tobytes()).hexdigest()
        digests = [None] * world
        dist.all_gather_object(digests, digest)
        results.append(("cfg5 bond 8192 gathered bytes identical on every rank",
                        all(d == digests[0] for d in digests), -1, 128))
        if rank == 0:
            ends = list(o8[1:]) + [len(d8)]
            got = {tuple(int(x) for x in c): d8[o:e] for c, o, e in zip(c8, o8, ends)}
            ref = reference_blocks(Ah, Bh, 2, 1, list(got), kscale=np.asarray(Sh[2]))
            err = max(rel_fro(got[c], ref[c]) for c in ref)
            results.append((f"cfg5 bond 8192 gathered vs CPU reference (max block err {err:.1e})",
                            bool(err <= 1e-12 and len(got) == 128), -1, 128))
        dist.barrier()
        del comm
        bs.Comm._by_group.clear()
        q.put((rank, results, None))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, results, repr(e)))
    finally:
        dist.destroy_process_group()


def test_sharded_contract_allgather_nccl_multi_gpu(gpu):
    """Every visible GPU (2 to 8) as one rank."""
    import multiprocessing as mp

    import torch

    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs two visible GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = [q.get(timeout=600) for _ in ps]
    for p in ps:
        p.join(timeout=60)
    for rank, results, err in out:
        assert err is None, f"rank {rank}: {err}"
        for name, ok, _, _ in results:
            assert ok, f"rank {rank}: {name} gathered shards differ from the unsharded contraction"
