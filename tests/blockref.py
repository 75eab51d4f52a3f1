"""Independent CPU reference for block-sparse contractions at benchmark sizes.

TEST INFRASTRUCTURE ONLY (tests and bench.py's self-check): it computes
chosen output blocks of a block-sparse contraction the way the reference's
contract_blocksparse does (contract/blocksparse.rs:144-180: for each output
block, the sum over its matched block pairs of the pair's GEMM), with
torch's CPU float64 / complex128 matmul standing in for faer.  The oracle's
plain i-j-k loops are too slow at these sizes (1e10 - 1e13 flop); this
restatement covers the label pattern of the benchmark configurations:
A's axes are [free..., contracted...] and B's are [contracted..., free...]
with the contracted axes in the same order, so every block pair is one
column-major GEMM with no permutation.  An optional diagonal `kscale` on the
contracted index (one contracted axis) gives (A . diag(s)) . B.
"""

from __future__ import annotations

from math import prod
from typing import Dict, Iterable, Optional, Sequence, Tuple

import numpy as np


def block_offsets(sizes, coords):
    """Packed offsets of the blocks in storage order (block_offsets.rs:76-90)."""
    offs, o = {}, 0
    for c in coords:
        offs[tuple(c)] = o
        o += prod(sizes[ax][x] for ax, x in enumerate(c))
    return offs


def reference_blocks(A, B, nfree_a: int, nc: int, out_coords: Iterable[Sequence[int]],
                     kscale: Optional[np.ndarray] = None) -> Dict[Tuple[int, ...], np.ndarray]:
    """Output blocks `out_coords` of A . B (or (A . diag(kscale)) . B), each as
    a flat column-major array.  A, B are (sizes, coords, data) with packed
    column-major blocks in storage order (numpy arrays, or torch tensors on
    any device: only the blocks a pair uses are copied to the host); A has
    nfree_a free axes followed by nc contracted ones, B has the nc contracted
    axes followed by its free axes.  kscale (nc == 1 only) holds the diagonal over the whole contracted
    index, in the index's natural order."""
    import torch

    sa, ca, da = A
    sb, cb, db = B
    offa, offb = block_offsets(sa, ca), block_offsets(sb, cb)

    def as_torch(d):
        return d if isinstance(d, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(d))

    ta, tb = as_torch(da), as_torch(db)
    ks = None
    if kscale is not None:
        assert nc == 1, "a diagonal on the contracted index needs one contracted axis"
        ks = torch.from_numpy(np.ascontiguousarray(kscale))
        cum = np.concatenate([[0], np.cumsum(sa[nfree_a])]).astype(int)
    by_key = {}
    for c in ca:
        by_key.setdefault(tuple(c[:nfree_a]), []).append(tuple(c))
    bset = set(tuple(d) for d in cb)
    out = {}
    for oc in out_coords:
        oc = tuple(int(x) for x in oc)
        fa, fb = oc[:nfree_a], oc[nfree_a:]
        m = prod(sa[i][fa[i]] for i in range(nfree_a))
        n = prod(sb[nc + j][fb[j]] for j in range(len(fb)))
        acc = None
        for c in by_key.get(fa, []):
            kc = c[nfree_a:]
            d = kc + fb
            if d not in bset:
                continue
            k = prod(sa[nfree_a + i][kc[i]] for i in range(nc))
            x = ta[offa[c]:offa[c] + m * k].cpu().view(k, m)  # row-major (k, m) == column-major A block (m, k)
            if ks is not None:
                s0 = int(cum[kc[0]])
                x = x * ks[s0:s0 + k].view(k, 1)
            y = tb[offb[d]:offb[d] + k * n].cpu().view(n, k)  # column-major B block (k, n)
            p = y @ x  # row-major (n, m) == column-major C block (m, n)
            acc = p if acc is None else acc + p
        if acc is None:
            acc = torch.zeros(n, m, dtype=ta.dtype)
        out[oc] = acc.reshape(-1).numpy()
    return out


def output_coords(A, B, nfree_a: int, nc: int):
    """Sorted output block coordinates of A . B for the label pattern above
    (compute_block_contributions, contract/blocksparse.rs:216-275)."""
    _, ca, _ = A
    _, cb, _ = B
    by_k = {}
    for d in cb:
        by_k.setdefault(tuple(d[:nc]), []).append(tuple(d[nc:]))
    out = set()
    for c in ca:
        for fb in by_k.get(tuple(c[nfree_a:]), []):
            out.add(tuple(c[:nfree_a]) + fb)
    return sorted(out)


def pair_flops(A, B, nfree_a: int, nc: int, out_coords, complex_: bool = False):
    """{output block: 2mnk (8mnk complex) summed over its pairs}."""
    sa, ca, _ = A
    sb, cb, _ = B
    bset = set(tuple(d) for d in cb)
    by_free = {}
    for c in ca:
        by_free.setdefault(tuple(c[:nfree_a]), []).append(tuple(c))
    f = 8.0 if complex_ else 2.0
    res = {}
    for oc in out_coords:
        oc = tuple(oc)
        fa, fb = oc[:nfree_a], oc[nfree_a:]
        m = prod(sa[i][fa[i]] for i in range(nfree_a))
        n = prod(sb[nc + j][fb[j]] for j in range(len(fb)))
        tot = 0.0
        for c in by_free.get(fa, []):
            kc = c[nfree_a:]
            if kc + fb in bset:
                tot += f * m * n * prod(sa[nfree_a + i][kc[i]] for i in range(nc))
        res[oc] = tot
    return res


def rel_fro(x, y) -> float:
    x, y = np.asarray(x).ravel(), np.asarray(y).ravel()
    n = np.linalg.norm(y)
    return float(np.linalg.norm(x - y) / n) if n > 0 else float(np.linalg.norm(x - y))
