"""The oracle on seeded random cases against numpy (host only).

The known-answer tests pin the oracle to the reference's own values; these
widen its coverage to random ranks, shapes and label patterns:
- permutedims equals numpy's transpose bit for bit (f64 and complex128);
- contract_gemm equals einsum with the open labels ascending, contract_naive
  einsum with A's open labels then B's in their own order (relative
  Frobenius error <= 1e-12, scalar results of shape (1,));
- block-sparse contraction equals the dense contraction of the to_dense
  operands, with output blocks sorted; block-sparse permutedims equals the
  dense transpose, with blocks re-sorted.
"""

from __future__ import annotations

import itertools
import random
import string

import numpy as np
import pytest

RTOL = 1e-12


def _rel(x, y):
    x, y = np.asarray(x).ravel(), np.asarray(y).ravel()
    ny = np.linalg.norm(y)
    return np.linalg.norm(x - y) / ny if ny else np.linalg.norm(x)


def _draw(rng, shape, cplx):
    x = rng.standard_normal(shape)
    return x + 1j * rng.standard_normal(shape) if cplx else x


@pytest.mark.parametrize("seed", range(6))
def test_permutedims_random_vs_numpy(oracle, seed):
    r = random.Random(seed)
    rng = np.random.default_rng(seed)
    for _ in range(20):
        nd = r.randrange(1, 6)
        shape = tuple(r.randrange(1, 5) for _ in range(nd))
        perm = list(range(nd))
        r.shuffle(perm)
        a = _draw(rng, shape, seed % 2 == 1)
        st, got = oracle.permutedims(a, perm)
        assert st == 0
        np.testing.assert_array_equal(got, np.transpose(a, perm))


def _label_case(r):
    """Open labels 1, 2, ... split between A and B, contracted labels -1, -2,
    ...; axes shuffled within each tensor; extents 1..4."""
    nfa, nfb, nc = r.randrange(0, 3), r.randrange(0, 3), r.randrange(0, 3)
    if nfa + nc == 0:
        nfa = 1
    if nfb + nc == 0:
        nfb = 1
    opens = list(range(1, nfa + nfb + 1))
    r.shuffle(opens)
    la = opens[:nfa] + [-(i + 1) for i in range(nc)]
    lb = opens[nfa:] + [-(i + 1) for i in range(nc)]
    r.shuffle(la)
    r.shuffle(lb)
    ext = {x: r.randrange(1, 5) for x in la + lb}
    return la, lb, ext


def _einsum(a, la, b, lb, out):
    letters = {x: string.ascii_letters[i] for i, x in enumerate(sorted(set(la + lb)))}
    spec = "".join(letters[x] for x in la) + "," + "".join(letters[x] for x in lb) + "->" + \
        "".join(letters[x] for x in out)
    return np.einsum(spec, a, b)


@pytest.mark.parametrize("seed", range(8))
def test_contractions_random_vs_einsum(oracle, seed):
    r = random.Random(100 + seed)
    rng = np.random.default_rng(100 + seed)
    cplx = seed % 2 == 1
    for _ in range(25):
        la, lb, ext = _label_case(r)
        a = _draw(rng, tuple(ext[x] for x in la), cplx)
        b = _draw(rng, tuple(ext[x] for x in lb), cplx)
        sorted_out = sorted(x for x in la + lb if x > 0)
        naive_out = [x for x in la if x > 0] + [x for x in lb if x > 0]
        for fn, out in ((oracle.contract_gemm, sorted_out), (oracle.contract_naive, naive_out)):
            st, got = fn(a, la, b, lb)
            assert st == 0, (la, lb)
            ref = _einsum(a, la, b, lb, out)
            if not out:
                assert got.shape == (1,)
                ref = np.reshape(ref, (1,))
            else:
                assert got.shape == ref.shape
            assert _rel(got, ref) <= RTOL


def _random_bs(r, rng, sizes, cplx, keep=0.6):
    coords = [c for c in itertools.product(*[range(len(s)) for s in sizes]) if r.random() < keep]
    if not coords:
        coords = [tuple(0 for _ in sizes)]
    n = sum(int(np.prod([sizes[ax][c] for ax, c in enumerate(cc)])) for cc in coords)
    return coords, _draw(rng, n, cplx)


@pytest.mark.parametrize("seed", range(6))
def test_blocksparse_contract_random_vs_dense(oracle, seed):
    """A(1, -1[, 2]) x B(-1, 3) with random block structures and stored
    subsets: to_dense of the result equals the dense contraction."""
    r = random.Random(200 + seed)
    rng = np.random.default_rng(200 + seed)
    cplx = seed % 2 == 1
    for _ in range(10):
        sz = lambda: [r.randrange(1, 4) for _ in range(r.randrange(1, 4))]  # noqa: E731
        s_free, s_k, s_free2, s_b = sz(), sz(), sz(), sz()
        three = r.random() < 0.5
        sa = [s_free, s_k] + ([s_free2] if three else [])
        la = [1, -1] + ([2] if three else [])
        sb, lb = [s_k, s_b], [-1, 3]
        ca, da = _random_bs(r, rng, sa, cplx)
        cb, db = _random_bs(r, rng, sb, cplx)
        A, B = oracle.BlockSparse(sa, ca, da), oracle.BlockSparse(sb, cb, db)
        st, C = oracle.bs_contract(A, la, B, lb)
        assert st == 0
        assert C.coords == sorted(C.coords)
        ref = _einsum(oracle.bs_to_dense(A), la, oracle.bs_to_dense(B), lb, [1, 2, 3] if three else [1, 3])
        got = oracle.bs_to_dense(C) if C.coords else np.zeros_like(ref)
        assert got.shape == ref.shape
        assert _rel(got, ref) <= RTOL


@pytest.mark.parametrize("seed", range(4))
def test_blocksparse_permutedims_random_vs_dense(oracle, seed):
    r = random.Random(300 + seed)
    rng = np.random.default_rng(300 + seed)
    for _ in range(10):
        nd = r.randrange(2, 5)
        sizes = [[r.randrange(1, 4) for _ in range(r.randrange(1, 4))] for _ in range(nd)]
        coords, data = _random_bs(r, rng, sizes, seed % 2 == 1)
        A = oracle.BlockSparse(sizes, coords, data)
        perm = list(range(nd))
        r.shuffle(perm)
        st, P = oracle.bs_permutedims(A, perm)
        assert st == 0
        assert P.coords == sorted(P.coords)
        np.testing.assert_array_equal(oracle.bs_to_dense(P), np.transpose(oracle.bs_to_dense(A), perm))
