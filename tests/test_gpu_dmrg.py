"""DMRG environment-update chain and the skinny contraction kernel.

The chain L.psi -> .W1 -> .W2 -> .R runs through contract_gemm (TTGT
semantics, output sorted by label): steps 1 and 4 are DMMA GEMMs, steps 2 and
3 (k = n = 10 against 2 D^2 rows) run on the skinny kernel, which reads the
permuted operand through its strides.

Parity: the oracle's contract_gemm at bond 64 (every step), and torch's
float64 einsum (cuBLAS) at the full bond 1024, each step fed the library's
own previous output.  Tolerance: relative Frobenius error <= 1e-12.
"""

from __future__ import annotations

import numpy as np
import pytest

from workloads import CFG3_STEPS, cfg3_tensors

pytestmark = pytest.mark.gpu

RTOL = 1e-12
EINSUM = ["awx,xpqb->awpqb", "awpqb,wvpr->aqbvr", "aqbvr,vuqt->abrut", "abrut,zub->artz"]


def rel_fro(x, y):
    x, y = np.asarray(x), np.asarray(y)
    d = np.linalg.norm((x - y).ravel())
    n = np.linalg.norm(y.ravel())
    return d / n if n > 0 else d


def _rand(rng, shape, cplx):
    if cplx:
        return rng.standard_normal(shape) + 1j * rng.standard_normal(shape)
    return rng.standard_normal(shape)


def test_dmrg_chain_vs_oracle_bond64(gpu, oracle):
    L, psi, W1, W2, R = cfg3_tensors(bond=64)
    T = gpu.TensorF64
    cur = L
    for (la, lb), b in zip(CFG3_STEPS, [psi, W1, W2, R]):
        got = gpu.contract_gemm(T.from_numpy(cur), la, T.from_numpy(b), lb).to_numpy()
        st, ref = oracle.contract_gemm(cur, la, b, lb)
        assert st == 0 and got.shape == ref.shape
        assert rel_fro(got, ref) <= RTOL, (la, rel_fro(got, ref))
        cur = got
    assert cur.shape == (64, 2, 2, 64)


def test_dmrg_chain_full_bond_vs_torch(gpu):
    import torch

    L, psi, W1, W2, R = cfg3_tensors(bond=1024)
    T = gpu.TensorF64
    cur = T.from_numpy(L)
    shapes = [(1024, 5, 2, 2, 1024), (1024, 2, 1024, 5, 2), (1024, 1024, 2, 5, 2), (1024, 2, 2, 1024)]
    for (la, lb), b, eq, shp in zip(CFG3_STEPS, [psi, W1, W2, R], EINSUM, shapes):
        nxt = gpu.contract_gemm(cur, la, T.from_numpy(b), lb)
        x = torch.from_numpy(cur.to_numpy()).cuda()
        y = torch.from_numpy(np.ascontiguousarray(b)).cuda()
        ref = torch.einsum(eq, x, y).cpu().numpy()
        got = nxt.to_numpy()
        assert got.shape == shp == ref.shape
        assert rel_fro(got, ref) <= RTOL, (eq, rel_fro(got, ref))
        cur = nxt


SKINNY = [
    # (shape_a, labels_a, shape_b, labels_b): gemm semantics
    ((4096, 32), (1, -1), (32, 32), (-1, 2)),                       # k = n = 32 (largest f64 bucket)
    ((2049, 7), (1, -1), (7, 3), (-1, 2)),                          # ragged row count
    ((64, 5, 2, 2, 64), (1, -1, -2, 3, 4), (5, 5, 2, 2), (-1, 5, -2, 6)),   # DMRG step 2 shape
    ((5, 5, 2, 2), (2, -1, 3, -2), (64, 5, 2, 2, 64), (1, -1, -2, 4, 5)),   # small m, permuted C
    ((3000, 1), (1, -1), (1, 9), (-1, 2)),                          # k = 1 (outer product)
    ((2049,), (1,), (5,), (2,)),                                    # no contracted axis, odd rows (half pair)
    ((1024, 10, 6), (1, -1, 2), (10, 10), (-1, 3)),                 # 16-byte pair copies, two row axes
    ((9, 4096), (-1, 1), (9, 16), (-1, 2)),                         # A K-major (strided rows)
    ((4096, 17), (1, -1), (17, 33), (-1, 2)),                       # n = 33: GEMM path, same answer
]


@pytest.mark.parametrize("sa,la,sb,lb", SKINNY)
@pytest.mark.parametrize("cplx", [False, True])
def test_skinny_contract_gemm(gpu, oracle, sa, la, sb, lb, cplx):
    rng = np.random.default_rng(hash((sa, sb, cplx)) % 2**32)
    a = _rand(rng, sa, cplx)
    b = _rand(rng, sb, cplx)
    cls = gpu.TensorC64 if cplx else gpu.TensorF64
    got = gpu.contract_gemm(cls.from_numpy(a), la, cls.from_numpy(b), lb).to_numpy()
    st, ref = oracle.contract_gemm(a, la, b, lb)
    assert st == 0 and got.shape == ref.shape
    assert rel_fro(got, ref) <= RTOL, rel_fro(got, ref)


@pytest.mark.parametrize("sa,la,sb,lb", [
    ((4096, 3, 3), (1, -1, -2), (3, 3, 5), (-1, -2, 2)),           # two contracted axes
    ((4096, 4, 3), (1, -3, -1), (3, 5), (-1, 2)),                  # unmatched -3 pinned at index 0
    ((3, 4096), (-1, 1), (3, 3, 2), (-1, -1, 2)),                  # duplicate B label: first pair
])
def test_skinny_contract_naive(gpu, oracle, sa, la, sb, lb):
    rng = np.random.default_rng(7)
    a = rng.standard_normal(sa)
    b = rng.standard_normal(sb)
    got = gpu.contract(gpu.TensorF64.from_numpy(a), la, gpu.TensorF64.from_numpy(b), lb).to_numpy()
    st, ref = oracle.contract_naive(a, la, b, lb)
    assert st == 0 and got.shape == ref.shape
    assert rel_fro(got, ref) <= RTOL, rel_fro(got, ref)


def test_skinny_launches_one_kernel(gpu):
    """DMRG step 2 is a single launch: no packing of the permuted operand."""
    L, psi, W1, W2, R = cfg3_tensors(bond=64)
    T = gpu.TensorF64
    T1 = gpu.contract_gemm(T.from_numpy(L), CFG3_STEPS[0][0], T.from_numpy(psi), CFG3_STEPS[0][1])
    w = T.from_numpy(W1)
    T1.device_ptr()
    w.device_ptr()
    gpu.synchronize()
    n0 = gpu.launch_count()
    out = gpu.contract_gemm(T1, CFG3_STEPS[1][0], w, CFG3_STEPS[1][1])
    gpu.synchronize()
    assert gpu.launch_count() - n0 == 1
    assert out.shape == (64, 2, 64, 5, 2)


@pytest.mark.parametrize("nranks", [2, 4])
def test_dmrg_chain_split_along_free_index(gpu, nranks):
    """The multi-GPU split of the chain: rank r runs all four steps on its
    slab L[a0:a1] of the free index a (axis 0 of L and of every intermediate,
    never contracted), with no collective.  Each slab's result equals the
    matching rows of the unsplit chain."""
    D = 256
    L, psi, W1, W2, R = cfg3_tensors(bond=D)
    T = gpu.TensorF64
    rhs = [T.from_numpy(x) for x in (psi, W1, W2, R)]

    def chain(l0):
        cur = T.from_numpy(l0)
        for (la, lb), b in zip(CFG3_STEPS, rhs):
            cur = gpu.contract_gemm(cur, la, b, lb)
        return cur.to_numpy()

    full = chain(L)
    for r in range(nranks):
        a0, a1 = r * D // nranks, (r + 1) * D // nranks
        part = chain(np.asfortranarray(L[a0:a1]))
        assert part.shape == (a1 - a0,) + full.shape[1:]
        assert rel_fro(part, full[a0:a1]) <= RTOL
