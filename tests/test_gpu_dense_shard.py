"""Dense contraction split along a free index (contract_gemm_shard).

Each rank's slab of contract_gemm's result, along the free axis a chosen
label marks, comes from reading the operand in place over the rank's range
(the dense multi-GPU scheme: no reduction).  The slabs of all ranks, joined
along that axis, must equal the unsplit contract_gemm (relative Frobenius
error 1e-12) and the oracle's restatement of contract_gemm (gemm.rs:47-236).
All ranks' slabs are computed here on one GPU.
"""

from __future__ import annotations

import numpy as np
import pytest

from workloads import CFG3_STEPS, cfg3_tensors

pytestmark = pytest.mark.gpu
RTOL = 1e-12


def rel_fro(x, y):
    return np.linalg.norm((np.asarray(x) - np.asarray(y)).ravel()) / np.linalg.norm(np.asarray(y).ravel())


def _out_axis(la, lb, label):
    """Position of `label` among contract_gemm's output axes (unpaired labels, sorted)."""
    paired = {l for l in la if l < 0 and l in lb}
    out = sorted([l for l in la if l not in paired] + [l for l in lb if l not in paired])
    return out.index(label)


CASES = [
    # (shape_a, la, shape_b, lb, split label): DMRG step 1 split on L's a (A's
    # stride-1 axis), on psi's last axis (B's slowest), a permuted operand pair,
    # complex, and an outer product
    ((64, 5, 64), (1, 2, -1), (64, 2, 2, 64), (-1, 3, 4, 5), 1, False),
    ((64, 5, 64), (1, 2, -1), (64, 2, 2, 64), (-1, 3, 4, 5), 5, False),
    ((7, 9, 11, 5), (-2, 3, -1, 1), (11, 7, 13), (-1, -2, 2), 3, False),
    ((7, 9, 11, 5), (-2, 3, -1, 1), (11, 7, 13), (-1, -2, 2), 2, True),
    ((33, 4), (2, 1), (5, 6), (4, 3), 2, False),
]


@pytest.mark.parametrize("nranks", [1, 2, 3, 8])
@pytest.mark.parametrize("sa,la,sb,lb,label,cplx", CASES)
def test_shards_join_to_contract_gemm(gpu, oracle, sa, la, sb, lb, label, cplx, nranks):
    rng = np.random.default_rng(int.from_bytes(repr((sa, la, sb, lb, cplx)).encode(), "little") % 2**32)

    def r(shape):
        x = rng.standard_normal(shape)
        return x + 1j * rng.standard_normal(shape) if cplx else x

    a, b = r(sa), r(sb)
    T = gpu.TensorC64 if cplx else gpu.TensorF64
    ta, tb = T.from_numpy(a), T.from_numpy(b)
    full = gpu.contract_gemm(ta, list(la), tb, list(lb)).to_numpy()
    st, ref = oracle.contract_gemm(a, list(la), b, list(lb))
    assert st == 0
    ax = _out_axis(la, lb, label)
    ext = full.shape[ax]
    parts = []
    for rank in range(nranks):
        s = gpu.contract_gemm_shard(ta, list(la), tb, list(lb), label, rank, nranks).to_numpy()
        lo, hi = ext * rank // nranks, ext * (rank + 1) // nranks
        want_shape = list(full.shape)
        want_shape[ax] = hi - lo
        assert list(s.shape) == want_shape
        if hi > lo:
            parts.append(s)
    joined = np.concatenate(parts, axis=ax)
    assert rel_fro(joined, full) <= RTOL
    assert rel_fro(joined, ref) <= RTOL


def test_dmrg_chain_split_along_a_matches_unsplit(gpu):
    """The DMRG environment chain at bond 256 with step 1 split along a (the
    chain's other steps keep a as a free axis): every rank's result is its
    rows of the unsplit chain."""
    host = cfg3_tensors(256)
    T = gpu.TensorF64
    ts = [T.from_numpy(x) for x in host]

    def chain(first):
        cur = first
        for (la, lb), t in zip(CFG3_STEPS[1:], ts[2:]):
            cur = gpu.contract_gemm(cur, la, t, lb)
        return cur.to_numpy()

    full = chain(gpu.contract_gemm(ts[0], CFG3_STEPS[0][0], ts[1], CFG3_STEPS[0][1]))
    rows = []
    for rank in range(4):
        rows.append(chain(gpu.contract_gemm_shard(ts[0], CFG3_STEPS[0][0], ts[1], CFG3_STEPS[0][1], 1, rank, 4)))
    assert rel_fro(np.concatenate(rows, axis=0), full) <= RTOL


def test_shard_argument_errors(gpu):
    a = gpu.TensorF64.from_numpy(np.ones((3, 4)))
    b = gpu.TensorF64.from_numpy(np.ones((4, 5)))
    for label, rank, nranks in [(-1, 0, 2), (7, 0, 2), (1, 2, 2), (1, 0, 0)]:
        with pytest.raises(Exception):
            gpu.contract_gemm_shard(a, [1, -1], b, [-1, 2], label, rank, nranks)
