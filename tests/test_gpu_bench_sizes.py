"""Parity at the sizes the benchmark reports.

The block-sparse configurations are checked here at the exact sizes whose
rates bench.py prints, block by block, against an independent CPU reference
(tests/blockref.py: the reference's per-output-block sum of pair GEMMs,
contract/blocksparse.rs:144-180, with torch's CPU matmul in float64 /
complex128 standing in for faer):

* U(1) rank-4 x rank-4 at half scale (sector dims [4,12,28,48,72,48,28,12,4],
  489 output blocks, 9.99e12 flop): every output block;
* the complex128 two-site MPS chain (A . S) . B at bond 8192 (33 sectors,
  4.52e10 flop), the path the benchmark times: unsharded (two contractions)
  and sharded over 2, 4 and 8 ranks (one grouped launch per rank that applies
  S's diagonal as B's fragments load); every output block of every shard.

Tolerance: relative Frobenius error 1e-12 per output block, and over the
whole output.  Block structure (coordinates, order, sizes) exactly.
"""

from __future__ import annotations

import numpy as np
import pytest

from blockref import reference_blocks, rel_fro
from workloads import cfg4_tensors, cfg5_tensors

pytestmark = pytest.mark.gpu
RTOL = 1e-12


def _blocks(t):
    """{coords: flat column-major block} of a library block-sparse tensor."""
    _, coords, offs = t._structure()
    data = t.to_numpy_data()
    ends = list(offs[1:]) + [len(data)]
    return {tuple(int(x) for x in c): data[o:e] for c, o, e in zip(coords, offs, ends)}


def _check_all(got_blocks, ref):
    assert set(got_blocks) == set(ref)
    num = den = 0.0
    for c, r in ref.items():
        g = got_blocks[c]
        assert g.shape == r.shape, c
        e = rel_fro(g, r)
        assert e <= RTOL, (c, e)
        num += float(np.linalg.norm(g - r) ** 2)
        den += float(np.linalg.norm(r) ** 2)
    assert (num / den) ** 0.5 <= RTOL


def test_cfg4_half_scale_every_block(gpu):
    (sa, ca, a), (sb, cb, b), la, lb = cfg4_tensors(scale=2)
    bs = gpu.blocksparse
    A, B = bs.BlockSparseF64.from_blocks(sa, ca, a), bs.BlockSparseF64.from_blocks(sb, cb, b)
    C = bs.contract(A, la, B, lb)
    assert C.nnzblocks == 489 and C.coords == sorted(C.coords)
    got = _blocks(C)
    del C
    ref = reference_blocks((sa, ca, a), (sb, cb, b), 2, 2, list(got))
    _check_all(got, ref)


@pytest.fixture(scope="module")
def cfg5(gpu):
    A, S, B = cfg5_tensors()  # bond 8192
    bs = gpu.blocksparse
    tA = bs.BlockSparseC64.from_blocks(*A)
    tS = bs.DiagBlockSparseC64.from_blocks(*S)
    tB = bs.BlockSparseC64.from_blocks(*B)
    return A, S, B, tA, tS, tB


def _cfg5_reference(A, S, B, coords):
    return reference_blocks(A, B, 2, 1, coords, kscale=np.asarray(S[2]))


def test_cfg5_bond8192_unsharded_every_block(gpu, cfg5):
    A, S, B, tA, tS, tB = cfg5
    C = gpu.blocksparse.contract_through_diag(tA, [1, 2, -1], tS, [-1, -2], tB, [-2, 3, 4])
    assert C.coords == sorted(C.coords)
    got = _blocks(C)
    _check_all(got, _cfg5_reference(A, S, B, list(got)))


@pytest.mark.parametrize("nranks", [2, 4, 8])
def test_cfg5_bond8192_sharded_every_block(gpu, cfg5, nranks):
    A, S, B, tA, tS, tB = cfg5
    bs = gpu.blocksparse
    full = bs.contract_through_diag(tA, [1, 2, -1], tS, [-1, -2], tB, [-2, 3, 4])
    got = {}
    for r in range(nranks):
        shard = bs.contract_through_diag(tA, [1, 2, -1], tS, [-1, -2], tB, [-2, 3, 4], r, nranks)
        part = _blocks(shard)
        assert not (set(part) & set(got)), "output blocks owned by two ranks"
        got.update(part)
    assert sorted(got) == full.coords  # the shards partition the output blocks
    _check_all(got, _cfg5_reference(A, S, B, list(got)))
