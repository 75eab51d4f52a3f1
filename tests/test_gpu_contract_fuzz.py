"""Seeded random contractions around the planner's branch boundaries.

The contraction planner picks between the skinny kernel (k <= 32 and one
side <= 32 against >= 2048 rows), the tiled DMMA GEMM, split-K (long k over a
grid whose last wave is mostly idle), and packing an operand whose axes do
not form a strided matrix.  Each case below draws sizes from one of those
regions (and from small ragged sizes), an operand layout, and f64 or
complex128, and compares the C ABI's contract with numpy einsum at the
contraction tolerance (relative Frobenius error <= 1e-12).
"""

from __future__ import annotations

import random

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL = 1e-12


def _cases(count=40, seed=2024):
    rng = random.Random(seed)
    out = []
    for i in range(count):
        region = ("split_k", "skinny", "ragged", "mid")[i % 4]
        if region == "split_k":
            m = rng.choice([64, 100, 257, 512, 640, 1000])
            n = rng.choice([8, 33, 64, 200, 512])
            k = rng.randrange(1024, 4200)
        elif region == "skinny":
            m, n, k = rng.randrange(2040, 5000), rng.randrange(1, 34), rng.randrange(1, 34)
        elif region == "ragged":
            m, n, k = rng.randrange(1, 70), rng.randrange(1, 70), rng.randrange(1, 70)
        else:
            m, n, k = rng.randrange(100, 1100), rng.randrange(100, 1100), rng.randrange(30, 700)
        layout = rng.choice(["mk,kn", "km,nk", "split_m"])
        if layout == "split_m":
            m1 = rng.choice([2, 3])
            m = max(m1, m - m % m1)
        cplx = rng.random() < 0.35
        out.append((region, m, n, k, layout, cplx))
    return out


CASES = _cases()


@pytest.mark.parametrize("region,m,n,k,layout,cplx", CASES,
                         ids=[f"{c[0]}-{c[1]}x{c[2]}x{c[3]}-{c[4]}-{'c128' if c[5] else 'f64'}" for c in CASES])
def test_contract_random_vs_einsum(gpu, region, m, n, k, layout, cplx):
    rng = np.random.default_rng(m * 1000003 + n * 1009 + k)

    def draw(shape):
        x = rng.standard_normal(shape)
        return x + 1j * rng.standard_normal(shape) if cplx else x

    T = gpu.TensorC64 if cplx else gpu.TensorF64
    if layout == "mk,kn":
        a, b = draw((m, k)), draw((k, n))
        la, lb, eq = (1, -1), (-1, 2), "ik,kj->ij"
    elif layout == "km,nk":
        a, b = draw((k, m)), draw((n, k))
        la, lb, eq = (-1, 1), (2, -1), "ki,jk->ij"
    else:  # A's free axis split around the contracted one: A is packed first
        m1 = 2 if m % 2 == 0 else 3
        a, b = draw((m1, k, m // m1)), draw((k, n))
        la, lb, eq = (1, -1, 2), (-1, 3), "akb,kj->abj"
    got = gpu.contract(T.from_numpy(a), la, T.from_numpy(b), lb).to_numpy()
    ref = np.einsum(eq, a, b)
    assert got.shape == ref.shape
    err = np.linalg.norm((got - ref).ravel()) / np.linalg.norm(ref.ravel())
    assert err <= RTOL, f"relative Frobenius error {err:.3e}"
