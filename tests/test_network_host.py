"""contract_network's label validation (host only, no GPU needed)."""

from __future__ import annotations

import numpy as np
import pytest


def _t(ndt, *shape):
    return ndt.TensorF64.from_numpy(np.zeros(shape))


def test_network_rejects_bad_labels(ndt):
    a, b = _t(ndt, 2, 3), _t(ndt, 3, 4)
    with pytest.raises(ValueError, match="labels for a rank"):
        ndt.contract_network([a, b], [[1, -1, 5], [-1, 2]])
    with pytest.raises(ValueError, match="extents"):
        ndt.contract_network([a, _t(ndt, 4, 4)], [[1, -1], [-1, 2]])
    with pytest.raises(ValueError, match="exactly 2"):
        ndt.contract_network([a, b, _t(ndt, 3)], [[1, -1], [-1, 2], [-1]])
    with pytest.raises(ValueError, match="open label"):
        ndt.contract_network([a, _t(ndt, 3, 2)], [[1, -1], [-1, 1]])
    with pytest.raises(ValueError, match="repeated"):
        ndt.contract_network([_t(ndt, 3, 3)], [[-1, -1]])
    with pytest.raises(ValueError, match="label 0"):
        ndt.contract_network([a, b], [[0, -1], [-1, 2]])
    with pytest.raises(ValueError, match="one label list"):
        ndt.contract_network([a, b], [[1, -1]])


def test_plan_dmrg_update_combines_the_operators_first():
    """The greedy order on the DMRG environment update L.psi.W1.W2.R (bond
    1024): W1.W2 first (a 400-entry operator), then L.psi, then one pass of
    the intermediate against W1W2 with k = n = 20, then R."""
    from math import prod

    from ndtensors_b200.network import _plan

    d = 1024
    labels = [[1, -1, -2], [-2, -3, -4, -5], [-1, -6, -3, 2], [-6, -7, -4, 3], [4, -7, -5]]
    shapes = [(d, 5, d), (d, 2, 2, d), (5, 5, 2, 2), (5, 5, 2, 2), (d, 5, d)]
    ext = {x: n for shp, ls in zip(shapes, labels) for x, n in zip(ls, shp)}
    steps = _plan(shapes, labels)
    assert [(s[0], s[1]) for s in steps] == [(2, 3), (0, 1), (5, 6), (4, 7)]
    assert prod(ext[x] for x in steps[0][3]) == 400
    i, j, shared, keep, _, _ = steps[2]
    w_keep = [x for x in steps[0][3] if x in keep]
    assert prod(ext[x] for x in shared) == 20 and prod(ext[x] for x in w_keep) == 20
    assert sorted(steps[-1][3]) == [1, 2, 3, 4]


def _random_network(rng):
    """A ring of 3..6 tensors (neighbours share one contracted label), each
    with 0..2 open labels; extents 1..6."""
    import random

    assert isinstance(rng, random.Random)
    n = rng.randrange(3, 7)
    labels = [[] for _ in range(n)]
    ext = {}
    for i in range(n):
        c = -(i + 1)
        ext[c] = rng.randrange(1, 7)
        labels[i].append(c)
        labels[(i + 1) % n].append(c)
    nxt = 1
    for i in range(n):
        for _ in range(rng.randrange(0, 3)):
            ext[nxt] = rng.randrange(1, 7)
            labels[i].append(nxt)
            nxt += 1
    for ls in labels:
        rng.shuffle(ls)
    shapes = [tuple(ext[x] for x in ls) for ls in labels]
    return shapes, labels


def test_plan_random_networks_are_complete_orders():
    """Every plan is n - 1 pairwise steps over live operands; each step
    contracts exactly the labels its two operands share; the last step
    leaves exactly the open labels."""
    import random

    from ndtensors_b200.network import _plan

    rng = random.Random(7)
    for _ in range(50):
        shapes, labels = _random_network(rng)
        steps = _plan(shapes, labels)
        assert len(steps) == len(labels) - 1
        live = {i: list(ls) for i, ls in enumerate(labels)}
        for i, j, shared, keep, _, out in steps:
            assert i in live and j in live and out not in live
            assert sorted(shared) == sorted(x for x in live[i] if x in live[j])
            assert sorted(keep) == sorted([x for x in live[i] + live[j] if x not in shared])
            del live[i], live[j]
            live[out] = keep
        (final,) = live.values()
        assert sorted(final) == sorted(x for ls in labels for x in ls if x > 0)


def test_plan_disconnected_parts_meet_in_an_outer_product():
    from ndtensors_b200.network import _plan

    steps = _plan([(2, 3), (3, 4), (5,)], [[1, -1], [-1, 2], [3]])
    assert steps[0][:3] == (0, 1, [-1])
    assert steps[1][2] == [] and sorted(steps[1][3]) == [1, 2, 3]
