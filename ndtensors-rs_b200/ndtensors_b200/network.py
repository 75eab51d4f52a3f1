"""Contraction of a tensor network on the GPU, pair by pair.

Beyond the reference, which contracts two tensors at a time and leaves the
order to the caller.  Labels follow the reference's convention: a negative
label names an index contracted between exactly two tensors, a positive label
an open index; the result's axes are the open labels in ascending order (as
contract_gemm orders them).

Order: greedy, each step contracting the pair of connected tensors whose
result is smallest (then the fewest flops, then the earliest pair).  Small
operators therefore combine first: in a DMRG environment update
L.psi.W1.W2.R the two MPO tensors W1.W2 become one 400-entry operator, and
the two bandwidth-bound passes over the 168 MB intermediate collapse into
one skinny contraction (k = n = 20).

The whole order is planned before anything runs; the steps are then issued
largest first among those whose operands exist, so the GPU is busy with a
long GEMM while the host issues the small steps.  Every pairwise step runs
contract_gemm with internal labels chosen so that
its output is already in natural TTGT order (A's kept axes, then B's), so no
intermediate pays for a sort permute; only the final result is permuted, if
its natural order is not ascending in the open labels.
"""

from __future__ import annotations

from collections import OrderedDict
from math import prod
from typing import Sequence

from .ops import contract_gemm


def _pair_cost(la, lb, ext):
    shared = [x for x in la if x < 0 and x in lb]
    keep = [x for x in la if x not in shared] + [x for x in lb if x not in shared]
    size = prod(ext[x] for x in keep)
    return size, size * prod(ext[x] for x in shared), shared, keep


_PLANS: "OrderedDict[tuple, list]" = OrderedDict()
_PLAN_CACHE_SIZE = 64


def contract_network(tensors: Sequence, labels: Sequence[Sequence[int]]):
    """Contract all `tensors` (TensorF64 or TensorC64, one element type);
    `labels[i]` labels the axes of tensors[i].  Returns the tensor over the
    open labels, ascending.  Plans are cached by (labels, shapes), so a
    network contracted again (every sweep step of a DMRG run) issues its first
    kernel without planning."""
    if len(tensors) != len(labels) or not tensors:
        raise ValueError("one label list per tensor, at least one tensor")
    shapes = tuple(tuple(t.shape) for t in tensors)
    key = (tuple(tuple(ls) for ls in labels), shapes)
    steps = _PLANS.get(key)
    if steps is None:
        steps = _plan(shapes, labels)
        _PLANS[key] = steps
        if len(_PLANS) > _PLAN_CACHE_SIZE:
            _PLANS.popitem(last=False)
    else:
        _PLANS.move_to_end(key)
    return _execute(tensors, labels, steps)


def _plan(shapes, labels):
    ext, seen = {}, {}
    for shp, ls in zip(shapes, labels):
        if len(ls) != len(shp):
            raise ValueError(f"{len(ls)} labels for a rank-{len(shp)} tensor")
        if len(set(ls)) != len(ls):
            raise ValueError(f"repeated label within one tensor: {list(ls)}")
        for x, n in zip(ls, shp):
            if x == 0:
                raise ValueError("label 0 is neither open nor contracted")
            if x in ext and ext[x] != n:
                raise ValueError(f"label {x}: extents {ext[x]} and {n} differ")
            ext[x] = n
            seen[x] = seen.get(x, 0) + 1
    for x, c in seen.items():
        if x < 0 and c != 2:
            raise ValueError(f"contracted label {x} appears in {c} tensors (needs exactly 2)")
        if x > 0 and c != 1:
            raise ValueError(f"open label {x} appears in {c} tensors")

    # greedy pairwise order over symbolic operands
    live = {i: list(ls) for i, ls in enumerate(labels)}
    steps = []  # (id_a, id_b, shared, keep, flops, id_out)
    nid = len(shapes)
    while len(live) > 1:
        ids = sorted(live)
        best = None
        for x in range(len(ids)):
            for y in range(x + 1, len(ids)):
                i, j = ids[x], ids[y]
                size, flops, shared, keep = _pair_cost(live[i], live[j], ext)
                if not shared:
                    continue
                key = (size, flops, x, y)
                if best is None or key < best[0]:
                    best = (key, i, j, shared, keep, flops)
        if best is None:  # disconnected: outer product of the two smallest
            i, j = sorted(sorted(ids, key=lambda k: prod(ext[v] for v in live[k]))[:2])
            _, flops, shared, keep = _pair_cost(live[i], live[j], ext)
        else:
            _, i, j, shared, keep, flops = best
        steps.append((i, j, shared, keep, flops, nid))
        del live[i], live[j]
        live[nid] = keep
        nid += 1
    return steps


def _execute(tensors, labels, steps):
    # any order that respects the dependencies is valid; ready steps go
    # largest first, so a long GEMM is on the GPU while the host issues the
    # small ones
    vals = {i: (t, list(ls)) for i, (t, ls) in enumerate(zip(tensors, labels))}
    pending = list(steps)
    while pending:
        ready = [st for st in pending if st[0] in vals and st[1] in vals]
        st = max(ready, key=lambda z: z[4])
        pending.remove(st)
        i, j, shared, keep, _, out_id = st
        (ta, la), (tb, lb) = vals.pop(i), vals.pop(j)
        # internal labels: contracted pairs negative, kept axes 1, 2, ... in
        # natural order, so contract_gemm's sorted output is the natural one
        code = {x: -(k + 1) for k, x in enumerate(shared)}
        code.update({x: k + 1 for k, x in enumerate(keep)})
        vals[out_id] = (contract_gemm(ta, [code[x] for x in la], tb, [code[x] for x in lb]), keep)
    (t, ls), = vals.values()
    perm = sorted(range(len(ls)), key=lambda k: ls[k])
    if perm != list(range(len(ls))):
        t = t.permutedims(perm)
    return t


__all__ = ["contract_network"]
