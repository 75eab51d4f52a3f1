"""Seeded synthetic inputs of the benchmark configurations.

Used by the tests and by bench.py.  The generator is numpy's PCG64 seeded
per configuration (seed = 1000 + configuration number); entries are N(0,1)
(complex: independent real and imaginary parts) unless stated.

U(1) block structures (the reference has no charges: block-sparse structure
is whatever blocks a caller stores, storage/blocksparse/block.rs): a block
is stored iff the charges of its sectors balance under the index arrows.
"""

from __future__ import annotations

import itertools
from typing import List, Tuple

import numpy as np

# U(1) rank-4 block-sparse: 9 charge sectors q = -4..4 per index
CFG4_SECTORS = list(range(-4, 5))
CFG4_DIMS_FULL = [8, 24, 56, 96, 144, 96, 56, 24, 8]


def cfg4_dims(scale: int = 2) -> List[int]:
    """Sector dims divided by `scale` (1 = the literal config: 68 GB per
    operand, does not fit one GPU; 2 = the primary single-GPU scale)."""
    return [max(1, d // scale) for d in CFG4_DIMS_FULL]


def cfg4_structure(dims: List[int]):
    """Rank-4, arrows (in, in, out, out): blocks with q0 + q1 - q2 - q3 = 0,
    in lexicographic order.  Returns (block_sizes, coords)."""
    n = len(dims)
    q = CFG4_SECTORS
    coords = [c for c in itertools.product(range(n), repeat=4) if q[c[0]] + q[c[1]] - q[c[2]] - q[c[3]] == 0]
    return [list(dims)] * 4, coords


def block_elems(sizes, coords):
    return [int(np.prod([sizes[ax][c] for ax, c in enumerate(cc)])) for cc in coords]


def cfg4_tensors(scale: int = 2, seed: int = 1004):
    """A(1,2,-1,-2) x B(-1,-2,3,4), f64."""
    dims = cfg4_dims(scale)
    sizes, coords = cfg4_structure(dims)
    total = sum(block_elems(sizes, coords))
    rng = np.random.default_rng(seed)
    a = rng.standard_normal(total)
    b = rng.standard_normal(total)
    return (sizes, coords, a), (sizes, coords, b), [1, 2, -1, -2], [-1, -2, 3, 4]


# c128 two-site MPS: bond 8192 in 33 sectors q = -16..16, Gaussian profile (sigma 6
# sectors), largest-remainder rounding to the bond dimension; phys {0, 1}
CFG5_DIMS_8192 = [16, 24, 36, 52, 74, 102, 137, 178, 225, 278, 332, 387, 439, 484, 518, 540, 548, 540, 518, 484,
                  439, 387, 332, 278, 225, 178, 137, 102, 74, 52, 36, 24, 16]


def gaussian_sector_dims(bond: int, nsec: int = 33, sigma: float = 6.0) -> List[int]:
    q = np.arange(nsec) - nsec // 2
    w = np.exp(-(q.astype(float) ** 2) / (2 * sigma * sigma))
    raw = w / w.sum() * bond
    base = np.floor(raw).astype(int)
    rem = bond - base.sum()
    order = np.argsort(-(raw - base), kind="stable")
    base[order[:rem]] += 1
    return [int(x) for x in base]


def cfg5_tensors(bond: int = 8192, seed: int = 1005):
    """A[l,s1,m] (q_l + q_s1 = q_m), S diag on m (blocks (q,q), values
    exp(-k/400) with k the global diagonal index), B[m,s2,r]
    (q_m + q_s2 = q_r); complex128.  Returns (A, S, B) as (sizes, coords, data)."""
    dims = CFG5_DIMS_8192 if bond == 8192 else gaussian_sector_dims(bond)
    nsec = len(dims)
    q = [i - nsec // 2 for i in range(nsec)]
    phys = [1, 1]  # charges 0 and 1, one state each
    rng = np.random.default_rng(seed)

    def mps(first_bond_dims):
        sizes = [list(dims), list(phys), list(dims)]
        coords = []
        for il in range(nsec):
            for s in range(2):
                qm = q[il] + s
                if -(nsec // 2) <= qm <= nsec // 2:
                    coords.append((il, s, qm + nsec // 2))
        n = sum(block_elems(sizes, coords))
        data = rng.standard_normal(n) + 1j * rng.standard_normal(n)
        return sizes, coords, data

    A = mps(dims)
    B = mps(dims)
    s_sizes = [list(dims), list(dims)]
    s_coords = [(i, i) for i in range(nsec)]
    diag = np.exp(-np.arange(sum(dims)) / 400.0).astype(np.complex128)
    return A, (s_sizes, s_coords, diag), B


def flops_blocksparse(Asp, la, Bsp, lb, complex_: bool) -> float:
    """Sum over matched block pairs of 2mnk (8mnk complex)."""
    sa, ca, _ = Asp
    sb, cb, _ = Bsp
    pa, pb = [], []
    for i, l in enumerate(la):
        if l < 0 and l in lb:
            pa.append(i)
            pb.append(lb.index(l))
    ua = [i for i in range(len(la)) if i not in pa]
    ub = [j for j in range(len(lb)) if j not in pb]
    byk = {}
    for c in cb:
        byk.setdefault(tuple(c[j] for j in pb), []).append(c)
    tot = 0.0
    for c in ca:
        for d in byk.get(tuple(c[i] for i in pa), []):
            m = np.prod([sa[i][c[i]] for i in ua]) if ua else 1
            k = np.prod([sa[i][c[i]] for i in pa]) if pa else 1
            n = np.prod([sb[j][d[j]] for j in ub]) if ub else 1
            tot += (8.0 if complex_ else 2.0) * m * n * k
    return tot


# DMRG environment-update chain, bond D (1024 in the benchmark),
# MPO bond 5, physical dimension 2.  Entries N(0,1)/sqrt(fan-in), the fan-in
# being the product of the axes the tensor contracts in its step.
CFG3_STEPS = [
    # (A labels, B labels): T1 = L.psi, T2 = T1.W1, T3 = T2.W2, E = T3.R
    ([1, 2, -1], [-1, 3, 4, 5]),
    ([1, -1, -2, 3, 4], [-1, 5, -2, 6]),
    ([1, -2, 3, -1, 4], [-1, 5, -2, 6]),
    ([1, -1, 2, -2, 3], [4, -2, -1]),
]


def cfg3_tensors(bond: int = 1024, seed: int = 1003):
    """L[D,5,D], psi[D,2,2,D], W1, W2 [5,5,2,2], R[D,5,D] (column-major numpy)."""
    rng = np.random.default_rng(seed)
    D = bond

    def t(shape, fan_in):
        return np.asfortranarray(rng.standard_normal(shape) / np.sqrt(fan_in))

    L = t((D, 5, D), D)
    psi = t((D, 2, 2, D), D)
    W1 = t((5, 5, 2, 2), 10)
    W2 = t((5, 5, 2, 2), 10)
    R = t((D, 5, D), 5 * D)
    return L, psi, W1, W2, R


def cfg3_flops(bond: int = 1024) -> List[float]:
    """Real flop (2mnk) of the four steps."""
    D = bond
    return [2.0 * (5 * D) * D * (4 * D), 2.0 * (2 * D * D) * 10 * 10, 2.0 * (2 * D * D) * 10 * 10,
            2.0 * (4 * D) * (5 * D) * D]
