"""The CPU block reference used at benchmark sizes (tests/blockref.py) agrees
with the oracle's restatement of contract_blocksparse on reduced sizes of the
same configurations (block structure and values)."""

from __future__ import annotations

import numpy as np

from blockref import reference_blocks, rel_fro
from workloads import cfg4_tensors, cfg5_tensors


def test_blockref_cfg4_eighth_scale_matches_oracle(oracle):
    (sa, ca, a), (sb, cb, b), la, lb = cfg4_tensors(scale=8)
    st, ref = oracle.bs_contract(oracle.BlockSparse(sa, ca, a), la, oracle.BlockSparse(sb, cb, b), lb)
    assert st == 0
    got = reference_blocks((sa, ca, a), (sb, cb, b), 2, 2, ref.coords)
    assert rel_fro(np.concatenate([got[tuple(c)] for c in ref.coords]), ref.data) <= 1e-13


def test_blockref_cfg5_bond64_with_diagonal_matches_oracle(oracle):
    A, S, B = cfg5_tensors(bond=64)
    sd = oracle.diag_to_dense(*S)
    st, AS = oracle.bs_contract(oracle.BlockSparse(*A), [1, 2, -1], oracle.bs_from_dense(sd, S[0], S[1]), [-1, 3])
    assert st == 0
    st, ref = oracle.bs_contract(AS, [1, 2, -1], oracle.BlockSparse(*B), [-1, 3, 4])
    assert st == 0
    got = reference_blocks(A, B, 2, 1, ref.coords, kscale=np.asarray(S[2]))
    assert rel_fro(np.concatenate([got[tuple(c)] for c in ref.coords]), ref.data) <= 1e-13
