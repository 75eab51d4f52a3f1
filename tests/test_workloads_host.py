"""The synthetic workload generators reproduce their configurations' stated
structure (host only, no GPU; structure is computed without drawing data
except for the two-site MPS, about 0.2 GB).

U(1) rank-4 x rank-4 (9 sectors, dims [8,24,56,96,144,96,56,24,8]): 489
stored blocks per operand, 8.505e9 elements (68.0 GB) per operand, 3321
matched pairs, 489 output blocks, 6.39e14 flop, the total-charge-0 sector
(M_0 = 46720) carrying 31.9 % of it; half scale 0.532e9 elements and
9.99e12 flop; quarter scale 0.27 GB and 1.56e11 flop.  c128 two-site MPS at
bond 8192 (33 Gaussian sectors): 65 blocks per operand, 6.36e6 elements,
128 pairs, 4.52e10 real flop, 12.6e6 output elements.  DMRG update at bond
1024: 8.67e10 flop over the four steps.
"""

from __future__ import annotations

import pytest

import workloads as W

LA, LB = [1, 2, -1, -2], [-1, -2, 3, 4]


def _cfg4(scale):
    sizes, coords = W.cfg4_structure(W.cfg4_dims(scale))
    pairs = [(x, y) for x in coords for y in coords if x[2] == y[0] and x[3] == y[1]]
    outs = {(x[0], x[1], y[2], y[3]) for x, y in pairs}
    flop = W.flops_blocksparse((sizes, coords, None), LA, (sizes, coords, None), LB, False)
    return sizes, coords, pairs, outs, flop


@pytest.mark.parametrize("scale,elems,flop", [(1, 8_505_335_808, 6.3938e14), (2, 531_583_488, 9.9902e12),
                                              (4, 33_223_968, 1.5610e11)])
def test_u1_rank4_structure(scale, elems, flop):
    sizes, coords, pairs, outs, f = _cfg4(scale)
    assert len(coords) == 489 and coords == sorted(coords)
    assert sum(W.block_elems(sizes, coords)) == elems
    assert len(pairs) == 3321 and len(outs) == 489
    assert f == pytest.approx(flop, rel=1e-4)


def test_u1_rank4_charge_zero_sector_share():
    q, d = W.CFG4_SECTORS, W.cfg4_dims(1)
    m0 = sum(d[a] * d[b] for a in range(9) for b in range(9) if q[a] + q[b] == 0)
    assert m0 == 46720
    total = _cfg4(1)[4]
    assert 2.0 * m0 ** 3 / total == pytest.approx(0.319, abs=5e-4)


def test_mps_sector_dims_are_the_rounded_gaussian():
    assert sum(W.CFG5_DIMS_8192) == 8192 and len(W.CFG5_DIMS_8192) == 33
    assert W.gaussian_sector_dims(8192) == W.CFG5_DIMS_8192
    assert sum(W.gaussian_sector_dims(1024)) == 1024


def test_mps_two_site_structure():
    A, S, B = W.cfg5_tensors()
    assert len(A[1]) == 65 and len(B[1]) == 65
    assert sum(W.block_elems(A[0], A[1])) == 6_362_194
    pairs = [(x, y) for x in A[1] for y in B[1] if x[2] == y[0]]
    outs = {(x[0], x[1], y[1], y[2]) for x, y in pairs}
    assert len(pairs) == 128 and len(outs) == 128
    assert sum(A[0][0][o[0]] * B[0][2][o[3]] for o in outs) == 12_636_474
    assert W.flops_blocksparse(A, [1, 2, -1], B, [-1, 3, 4], True) == pytest.approx(4.5175e10, rel=1e-4)
    # S: 33 diagonal blocks over the whole bond, values exp(-k/400)
    assert len(S[1]) == 33 and len(S[2]) == 8192
    assert abs(S[2][400] - 2.718281828459045 ** -1) < 1e-15


def test_dmrg_update_flop():
    f = W.cfg3_flops(1024)
    assert f[0] == f[3] == 2.0 * 5 * 1024 * 1024 * 4 * 1024
    assert sum(f) == pytest.approx(8.67e10, rel=1e-3)
