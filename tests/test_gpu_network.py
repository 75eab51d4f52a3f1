"""contract_network on the GPU: the DMRG environment update as one network
(greedy order fuses W1.W2 into one operator, applied in one skinny pass) and
random networks, against the oracle's pairwise chain and numpy's einsum.
Tolerance: relative Frobenius error <= 1e-12."""

from __future__ import annotations

import numpy as np
import pytest

from workloads import CFG3_STEPS, cfg3_tensors

pytestmark = pytest.mark.gpu

RTOL = 1e-12
# L(a, w, x) psi(x, s1, s2, b) W1(w, w', s1, s1') W2(w', w'', s2, s2') R(r, w'', b) -> E(a, s1', s2', r)
DMRG_LABELS = [[1, -1, -2], [-2, -3, -4, -5], [-1, -6, -3, 2], [-6, -7, -4, 3], [4, -7, -5]]


def rel_fro(x, y):
    d = np.linalg.norm((np.asarray(x) - np.asarray(y)).ravel())
    n = np.linalg.norm(np.asarray(y).ravel())
    return d / n if n > 0 else d


def test_dmrg_network_vs_oracle_chain(gpu, oracle):
    L, psi, W1, W2, R = cfg3_tensors(bond=64)
    T = gpu.TensorF64
    got = gpu.contract_network([T.from_numpy(x) for x in (L, psi, W1, W2, R)], DMRG_LABELS).to_numpy()
    cur = L
    for (la, lb), b in zip(CFG3_STEPS, [psi, W1, W2, R]):
        st, cur = oracle.contract_gemm(cur, la, b, lb)
        assert st == 0
    assert got.shape == cur.shape == (64, 2, 2, 64)
    assert rel_fro(got, cur) <= RTOL


def test_dmrg_network_full_bond_vs_chain(gpu):
    L, psi, W1, W2, R = cfg3_tensors(bond=1024)
    T = gpu.TensorF64
    ts = [T.from_numpy(x) for x in (L, psi, W1, W2, R)]
    cur = ts[0]
    for (la, lb), b in zip(CFG3_STEPS, ts[1:]):
        cur = gpu.contract_gemm(cur, la, b, lb)
    got = gpu.contract_network(ts, DMRG_LABELS)
    assert got.shape == cur.shape
    assert rel_fro(got.to_numpy(), cur.to_numpy()) <= RTOL


def _letters(labels):
    names = {}
    for ls in labels:
        for x in ls:
            names.setdefault(x, chr(ord("a") + len(names)))
    return names


@pytest.mark.parametrize("seed", range(6))
@pytest.mark.parametrize("cplx", [False, True])
def test_random_networks_vs_einsum(gpu, seed, cplx):
    rng = np.random.default_rng(seed)
    # a ring of 3-5 tensors with one or two open legs each and random extents
    n = int(rng.integers(3, 6))
    ext = {}
    labels = [[] for _ in range(n)]
    nxt_open = 1
    for i in range(n):
        c = -(i + 1)
        ext[c] = int(rng.integers(2, 9))
        labels[i].append(c)
        labels[(i + 1) % n].append(c)
        for _ in range(int(rng.integers(1, 3))):
            labels[i].append(nxt_open)
            ext[nxt_open] = int(rng.integers(1, 6))
            nxt_open += 1
    for ls in labels:
        rng.shuffle(ls)
    arrs = []
    for ls in labels:
        shp = tuple(ext[x] for x in ls)
        a = rng.standard_normal(shp) + (1j * rng.standard_normal(shp) if cplx else 0)
        arrs.append(a)
    cls = gpu.TensorC64 if cplx else gpu.TensorF64
    got = gpu.contract_network([cls.from_numpy(a) for a in arrs], labels).to_numpy()
    nm = _letters(labels)
    spec = ",".join("".join(nm[x] for x in ls) for ls in labels) + "->" + "".join(
        nm[x] for x in sorted(x for x in ext if x > 0))
    ref = np.einsum(spec, *arrs)
    assert got.shape == ref.shape
    assert rel_fro(got, ref) <= RTOL
