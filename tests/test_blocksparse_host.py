"""Block-sparse host logic that needs no GPU: structure bookkeeping, error
codes, the FLOP-balanced shard plan, and the shard gather over
torch.distributed (gloo, world size 2)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from workloads import cfg4_tensors, flops_blocksparse


def test_structure_queries(ndt):
    bs = ndt.blocksparse
    t = bs.BlockSparseF64.from_blocks([[2, 3], [4, 5]], [(1, 1), (0, 0)], np.arange(15 + 8, dtype=float))
    assert t.ndim == 2 and t.nnzblocks == 2 and t.nnz == 23
    assert t.block_sizes == [[2, 3], [4, 5]]
    assert t.coords == [(1, 1), (0, 0)]  # storage order kept (BlockOffsets::from_blocks)
    assert t.dense_shape == (5, 9)
    np.testing.assert_array_equal(t.block((0, 0)), np.arange(15, 23, dtype=float).reshape((2, 4), order="F"))
    t.insert_block((0, 0), np.ones((2, 4)))
    np.testing.assert_array_equal(t.block((0, 0)), np.ones((2, 4)))
    with pytest.raises(ValueError):
        t.insert_block((0, 0), np.ones((3, 4)))  # wrong block shape (blocksparse_tensor.rs:218-223)
    with pytest.raises(KeyError):
        t.block((0, 1))


def test_structure_errors(ndt):
    bs = ndt.blocksparse
    with pytest.raises(ndt.NDTensorsError):
        bs.BlockSparseF64.zeros([[2, 3]], [(2,)])  # coordinate out of range
    with pytest.raises(ndt.NDTensorsError):
        bs.BlockSparseF64.zeros([[2, 3]], [(0,), (0,)])  # duplicate block
    with pytest.raises(ValueError):
        bs.BlockSparseF64.from_blocks([[2, 3]], [(0,)], np.zeros(3))  # length != 2


def test_shard_plan_is_flop_balanced(ndt):
    (sa, ca, a), (sb, cb, b), la, lb = cfg4_tensors(scale=8)
    bs = ndt.blocksparse
    A = bs.BlockSparseF64.from_blocks(sa, ca, a)
    B = bs.BlockSparseF64.from_blocks(sb, cb, b)
    total = flops_blocksparse((sa, ca, a), la, (sb, cb, b), lb, False)
    for n in (1, 2, 4, 8):
        blocks, flops = bs.shard_plan(A, la, B, lb, n)
        assert sum(blocks) == 489  # every output block in exactly one shard
        assert abs(sum(flops) - total) <= 1e-9 * total
        if n > 1:
            # longest processing time first never splits a block: the
            # heaviest block bounds both the excess over the mean and the
            # spread between ranks
            big = max_block_flops((sa, ca), la, (sb, cb), lb)
            assert max(flops) <= total / n + big + 1
            assert max(flops) - min(flops) <= big + 1


def max_block_flops(A, la, B, lb):
    sa, ca = A
    sb, cb = B
    per = {}
    for c in ca:
        for d in cb:
            if c[2] == d[0] and c[3] == d[1]:
                key = (c[0], c[1], d[2], d[3])
                m = sa[0][c[0]] * sa[1][c[1]]
                k = sa[2][c[2]] * sa[3][c[3]]
                n = sb[2][d[2]] * sb[3][d[3]]
                per[key] = per.get(key, 0) + 2.0 * m * n * k
    return max(per.values())


def _gather_worker(rank, world, port, q, cplx=False, interleaved=False):
    import sys

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import datetime

    import torch.distributed as dist

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "ndtensors-rs_b200"))
    import ndtensors_b200 as ndt

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        sizes = [[2, 3, 1], [4, 1]]
        all_coords = [(0, 0), (0, 1), (1, 0), (2, 1)]
        lens = [8, 2, 12, 1]
        offs = np.cumsum([0] + lens)
        data = np.arange(offs[-1], dtype=float) * 1.5
        if cplx:
            data = data - 0.5j * data[::-1]
        # shards of the sorted block list, contiguous or interleaved (as
        # contract_shard's heaviest-first assignment makes them); with 3
        # ranks the middle one holds no block (more ranks than output blocks)
        if world == 2:
            owned = [[0, 2], [1, 3]] if interleaved else [[0, 1], [2, 3]]
        else:
            owned = [[0, 3], [], [1, 2]] if interleaved else [[0, 1], [], [2, 3]]
        mine = owned[rank]
        cls = ndt.blocksparse.BlockSparseC64 if cplx else ndt.blocksparse.BlockSparseF64
        part = np.concatenate([data[offs[i]:offs[i + 1]] for i in mine]) if mine else data[:0]
        shard = cls.from_blocks(sizes, [all_coords[i] for i in mine], part)
        full = ndt.blocksparse.allgather(shard)
        ok = full.coords == all_coords and np.array_equal(full.to_numpy_data(), data)
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,cplx,interleaved", [(2, False, False), (3, True, False), (2, True, True),
                                                     (3, False, True)])
def test_allgather_shards_gloo(world, cplx, interleaved):
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ps = [ctx.Process(target=_gather_worker, args=(r, world, port, q, cplx, interleaved)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=60)
    assert sorted(res) == [(r, True) for r in range(world)]


def _gather_failure_worker(rank, world, port, q, mode):
    """Rank 1 fails before the gather: it exits ("exit") or stays alive but
    never joins the collective ("absent"); rank 0 must get an error from
    allgather within the process group's timeout, not hang."""
    import sys
    import time

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import datetime

    import torch.distributed as dist

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "ndtensors-rs_b200"))
    import ndtensors_b200 as ndt

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    shard = ndt.blocksparse.BlockSparseF64.from_blocks([[2, 3], [4]], [(rank, 0)], np.ones(8 if rank == 0 else 12))
    if rank == 1:
        if mode == "exit":
            os._exit(3)  # the process dies without a word to its peers
        time.sleep(8)  # alive past the 5 s timeout, but never reaches the gather
        q.put((rank, "absent"))
        q.close()
        q.join_thread()  # flush before the hard exit
        os._exit(0)
    t0 = time.monotonic()
    try:
        ndt.blocksparse.allgather(shard)
        q.put((rank, "no error", time.monotonic() - t0))
    except Exception as e:  # noqa: BLE001 - any error ends the wait, which is what is checked
        q.put((rank, type(e).__name__, time.monotonic() - t0))
    q.close()
    q.join_thread()
    os._exit(0)  # skip process-group teardown with a lost peer


@pytest.mark.parametrize("mode", ["exit", "absent"])
def test_allgather_fails_when_a_rank_is_lost(mode):
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ps = [ctx.Process(target=_gather_failure_worker, args=(r, 2, port, q, mode)) for r in range(2)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(2 if mode == "absent" else 1):
        r = q.get(timeout=60)
        res[r[0]] = r[1:]
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    outcome, waited = res[0]
    assert outcome != "no error"
    assert waited < 30  # bounded by the 5 s process-group timeout, not a hang
