"""Block-sparse contraction on the GPU (one grouped DMMA launch) vs the
oracle's restatement of contract_blocksparse (contract/blocksparse.rs:87-275).

Block structure (output coordinates, order, block sizes, packed offsets) must
match exactly; values within relative Frobenius error 1e-12."""

from __future__ import annotations

import numpy as np
import pytest

from workloads import cfg4_tensors, cfg5_tensors

pytestmark = pytest.mark.gpu
RTOL = 1e-12


def rel_fro(x, y):
    x, y = np.asarray(x).ravel(), np.asarray(y).ravel()
    n = np.linalg.norm(y)
    return np.linalg.norm(x - y) / n if n > 0 else np.linalg.norm(x - y)


def _cls(gpu, cplx):
    return gpu.blocksparse.BlockSparseC64 if cplx else gpu.blocksparse.BlockSparseF64


def _check(gpu, oracle, A, la, B, lb):
    cplx = np.iscomplexobj(A[2])
    cls = _cls(gpu, cplx)
    got = gpu.blocksparse.contract(cls.from_blocks(*A), la, cls.from_blocks(*B), lb)
    st, ref = oracle.bs_contract(oracle.BlockSparse(*A), la, oracle.BlockSparse(*B), lb)
    assert st == 0
    assert got.block_sizes == ref.block_sizes
    assert got.coords == ref.coords  # sorted output blocks, packed offsets
    assert rel_fro(got.to_numpy_data(), ref.data) <= RTOL
    return got, ref


def random_bs(rng, sizes, density, cplx):
    coords = []
    import itertools

    for c in itertools.product(*[range(len(s)) for s in sizes]):
        if rng.random() < density:
            coords.append(c)
    rng.shuffle(coords)  # arbitrary storage order
    n = sum(int(np.prod([sizes[a][x] for a, x in enumerate(c)])) for c in coords)
    data = rng.standard_normal(n) + (1j * rng.standard_normal(n) if cplx else 0)
    return sizes, [tuple(c) for c in coords], data


PATTERNS = [
    # (sizes_a, la, sizes_b, lb)
    ([[3, 5], [4, 2, 6]], [1, -1], [[4, 2, 6], [7, 1]], [-1, 2]),  # matmul, in place
    ([[4, 2, 6], [3, 5]], [-1, 1], [[4, 2, 6], [7, 1]], [-1, 2]),  # A K-major
    ([[3, 5], [4, 2, 6]], [1, -1], [[7, 1], [4, 2, 6]], [2, -1]),  # B MN-major
    ([[2, 3], [3, 1], [2, 2]], [1, -1, -2], [[2, 2], [3, 1], [4, 1]], [-2, -1, 2]),  # permuted -> block packing
    ([[2, 3], [3, 1]], [-1, -2], [[2, 3], [3, 1]], [-1, -2]),  # full contraction -> scalar block
    ([[2, 3]], [1], [[4, 1]], [2]),  # outer product of block vectors
    ([[3, 2], [2, 4], [5]], [1, -1, 2], [[2, 4], [3, 3]], [-1, 3]),  # middle contracted axis
]


@pytest.mark.parametrize("cplx", [False, True])
@pytest.mark.parametrize("sa,la,sb,lb", PATTERNS)
def test_blocksparse_contract_matches_oracle(gpu, oracle, sa, la, sb, lb, cplx):
    # a seed that does not depend on PYTHONHASHSEED (str hashes do)
    rng = np.random.default_rng(int.from_bytes(repr((sa, la, sb, cplx)).encode(), "little") % (2**32))
    A = random_bs(rng, sa, 0.7, cplx)
    B = random_bs(rng, sb, 0.7, cplx)
    _check(gpu, oracle, A, la, B, lb)


def test_blocksparse_unsorted_output_labels(gpu, oracle):
    """Output labels not ascending: the reference stores contract_gemm's
    label-sorted block data under the unsorted block coordinates when the
    block shapes agree (square blocks here), and fails otherwise."""
    rng = np.random.default_rng(77)
    A = random_bs(rng, [[3, 3], [4, 2]], 1.0, False)  # every output block is 3 x 3
    B = random_bs(rng, [[4, 2], [3, 3]], 1.0, False)
    _check(gpu, oracle, A, [2, -1], B, [-1, 1])
    A2 = random_bs(rng, [[3, 2], [4, 2]], 1.0, False)
    B2 = random_bs(rng, [[4, 2], [5, 1]], 1.0, False)
    st, _ = oracle.bs_contract(oracle.BlockSparse(*A2), [2, -1], oracle.BlockSparse(*B2), [-1, 1])
    assert st == oracle.SHAPE_MISMATCH
    with pytest.raises(ValueError):
        gpu.blocksparse.contract(gpu.blocksparse.BlockSparseF64.from_blocks(*A2), [2, -1],
                                 gpu.blocksparse.BlockSparseF64.from_blocks(*B2), [-1, 1])


def test_blocksparse_no_matching_pairs_and_empty(gpu, oracle):
    A = ([[2, 3], [4, 5]], [(0, 0)], np.ones(8))
    B = ([[4, 5], [2, 2]], [(1, 0)], np.ones(10))
    got, ref = _check(gpu, oracle, A, [1, -1], B, [-1, 2])
    assert got.nnzblocks == 0
    E = ([[2, 3], [4, 5]], [], np.zeros(0))
    _check(gpu, oracle, E, [1, -1], B, [-1, 2])


def merge_shards(shards):
    """Blocks of all shards in sorted coordinate order: (coords, packed data)."""
    items = []
    for s in shards:
        _, coords, offs = s._structure()
        d = s.to_numpy_data()
        ends = list(offs[1:]) + [len(d)]
        items += [(c, d[o:e]) for c, o, e in zip(coords, offs, ends)]
    items.sort(key=lambda x: x[0])
    data = np.concatenate([x[1] for x in items]) if items else np.zeros(0)
    return [x[0] for x in items], data


@pytest.mark.parametrize("nranks", [2, 3, 4])
def test_shards_reassemble_full_result(gpu, oracle, nranks):
    (sa, ca, a), (sb, cb, b), la, lb = cfg4_tensors(scale=8)
    cls = gpu.blocksparse.BlockSparseF64
    A, B = cls.from_blocks(sa, ca, a), cls.from_blocks(sb, cb, b)
    full = gpu.blocksparse.contract(A, la, B, lb)
    shards = [gpu.blocksparse.contract_shard(A, la, B, lb, r, nranks) for r in range(nranks)]
    for s in shards:
        assert s.coords == sorted(s.coords)  # each shard's blocks sorted
    coords, data = merge_shards(shards)
    assert coords == full.coords
    assert np.array_equal(data, full.to_numpy_data())  # same kernel, same bits
    # heaviest-first assignment: the shards' FLOPs differ by at most one block's
    blocks, flops = gpu.blocksparse.shard_plan(A, la, B, lb, nranks)
    assert blocks == [s.nnzblocks for s in shards]
    # every shard carries the same layout: all output blocks and their owners
    lays = [s._shard_layout() for s in shards]
    for n, lc, lo in lays:
        assert n == nranks and [tuple(int(x) for x in c) for c in lc] == full.coords
        assert np.array_equal(lo, lays[0][2])
    for r, s in enumerate(shards):
        assert [tuple(int(x) for x in c) for c in lays[0][1][lays[0][2] == r]] == s.coords
    assert full._shard_layout() is None  # an unsharded result has none


def test_permuted_shards_reassemble_full_result(gpu):
    """Shards of a contraction whose A blocks are read in place through their
    strides (labels (-1, 1, -2, 2)) reassemble into the full result, which
    equals the natural-order contraction of the same data bit for bit."""
    (sa, ca, a), (sb, cb, b), la, lb = cfg4_tensors(scale=8)
    cls = gpu.blocksparse.BlockSparseF64
    A, B = cls.from_blocks(sa, ca, a), cls.from_blocks(sb, cb, b)
    Ap, lap = A.permutedims([2, 0, 3, 1]), [-1, 1, -2, 2]
    full = gpu.blocksparse.contract(Ap, lap, B, lb)
    natural = gpu.blocksparse.contract(A, la, B, lb)
    assert full.coords == natural.coords
    assert np.array_equal(full.to_numpy_data(), natural.to_numpy_data())
    for nranks in (2, 3):
        shards = [gpu.blocksparse.contract_shard(Ap, lap, B, lb, r, nranks) for r in range(nranks)]
        coords, data = merge_shards(shards)
        assert coords == full.coords
        assert np.array_equal(data, full.to_numpy_data())


def test_cfg4_small_scale_vs_oracle(gpu, oracle):
    """U(1) rank-4 x rank-4 over 2 shared indices, 9 sectors, dims / 8."""
    A, B, la, lb = cfg4_tensors(scale=8)
    _check(gpu, oracle, A, la, B, lb)


def test_cfg4_half_scale_block_spot_checks(gpu):
    """The primary configuration (sector dims halved, 4.25 GB per operand):
    structure checked in full, block values against numpy on a sample of
    output blocks (size-independent check of the full-size run)."""
    (sa, ca, a), (sb, cb, b), la, lb = cfg4_tensors(scale=2)
    cls = gpu.blocksparse.BlockSparseF64
    A, B = cls.from_blocks(sa, ca, a), cls.from_blocks(sb, cb, b)
    C = gpu.blocksparse.contract(A, la, B, lb)
    assert C.coords == sorted(C.coords) and C.nnzblocks == 489
    offs = np.cumsum([0] + [int(np.prod([sa[i][c[i]] for i in range(4)])) for c in ca])
    amap = {c: i for i, c in enumerate(ca)}
    bmap = {c: i for i, c in enumerate(cb)}
    rng = np.random.default_rng(3)
    coords = C.coords
    for idx in rng.choice(len(coords), size=6, replace=False):
        oc = coords[idx]
        shape = (sa[0][oc[0]], sa[1][oc[1]], sb[2][oc[2]], sb[3][oc[3]])
        ref = np.zeros(shape)
        for (c, i) in amap.items():
            if c[0] != oc[0] or c[1] != oc[1]:
                continue
            d = (c[2], c[3], oc[2], oc[3])
            if d not in bmap:
                continue
            ash = tuple(sa[k][c[k]] for k in range(4))
            bsh = tuple(sb[k][d[k]] for k in range(4))
            ab = a[offs[i]:offs[i] + int(np.prod(ash))].reshape(ash, order="F")
            j = bmap[d]
            bb = b[offs[j]:offs[j] + int(np.prod(bsh))].reshape(bsh, order="F")
            ref += np.einsum("ijkl,klmn->ijmn", ab, bb, optimize=True)
        assert rel_fro(C.block(oc), ref) <= RTOL


def test_permutedims_and_dense_roundtrip(gpu, oracle):
    rng = np.random.default_rng(9)
    for cplx in (False, True):
        A = random_bs(rng, [[2, 3], [1, 4, 2], [3, 3]], 0.6, cplx)
        cls = _cls(gpu, cplx)
        t = cls.from_blocks(*A)
        st, ref = oracle.bs_permutedims(oracle.BlockSparse(*A), [2, 0, 1])
        p = t.permutedims([2, 0, 1])
        assert p.coords == ref.coords and p.block_sizes == ref.block_sizes
        assert np.array_equal(p.to_numpy_data(), ref.data)  # bit-exact
        dense = t.to_dense().to_numpy()
        assert np.array_equal(dense, oracle.bs_to_dense(oracle.BlockSparse(*A)))
        back = cls.from_dense(t.to_dense(), A[0], A[1])
        assert np.array_equal(back.to_numpy_data(), np.asarray(A[2]))
    with pytest.raises(ValueError):
        t.permutedims([0, 0, 1])


def test_diag_to_dense_and_contract_diag(gpu, oracle):
    rng = np.random.default_rng(10)
    for cplx in (False, True):
        dt = np.complex128 if cplx else np.float64
        sizes = [[2, 3, 4], [2, 3, 4]]
        coords = [(0, 0), (2, 2), (1, 1)]
        diag = (rng.standard_normal(9) + (1j * rng.standard_normal(9) if cplx else 0)).astype(dt)
        dcls = gpu.blocksparse.DiagBlockSparseC64 if cplx else gpu.blocksparse.DiagBlockSparseF64
        S = dcls.from_blocks(sizes, coords, diag)
        sd = S.to_dense().to_numpy()
        assert np.array_equal(sd, oracle.diag_to_dense(sizes, coords, diag))
        # fast path: A(1,2,-1) x S(-1,3) is a scaling of A's last axis
        A = random_bs(rng, [[3, 2], [1, 1], [2, 3, 4]], 0.8, cplx)
        cls = _cls(gpu, cplx)
        got = gpu.blocksparse.contract_diag(cls.from_blocks(*A), [1, 2, -1], S, [-1, 3])
        Sbs = oracle.bs_from_dense(sd, sizes, coords)
        st, ref = oracle.bs_contract(oracle.BlockSparse(*A), [1, 2, -1], Sbs, [-1, 3])
        assert st == 0 and got.coords == ref.coords
        assert rel_fro(got.to_numpy_data(), ref.data) <= RTOL
        # general path (contracted axis not last)
        A2 = random_bs(rng, [[2, 3, 4], [3, 2]], 0.8, cplx)
        got2 = gpu.blocksparse.contract_diag(cls.from_blocks(*A2), [-1, 1], S, [-1, 2])
        st, ref2 = oracle.bs_contract(oracle.BlockSparse(*A2), [-1, 1], Sbs, [-1, 2])
        assert st == 0 and got2.coords == ref2.coords
        assert rel_fro(got2.to_numpy_data(), ref2.data) <= RTOL


def test_cfg5_reduced_bond_chain_vs_oracle(gpu, oracle):
    """The c128 two-site MPS chain (A . S) . B with bond 1024 (33 sectors)."""
    A, S, B = cfg5_tensors(bond=1024)
    bs = gpu.blocksparse
    AS = bs.contract_diag(bs.BlockSparseC64.from_blocks(*A), [1, 2, -1],
                          bs.DiagBlockSparseC64.from_blocks(*S), [-1, 3])
    C = bs.contract(AS, [1, 2, -1], bs.BlockSparseC64.from_blocks(*B), [-1, 3, 4])
    Sd = oracle.diag_to_dense(*S)
    st, ASr = oracle.bs_contract(oracle.BlockSparse(*A), [1, 2, -1], oracle.bs_from_dense(Sd, S[0], S[1]), [-1, 3])
    assert st == 0
    st, Cr = oracle.bs_contract(ASr, [1, 2, -1], oracle.BlockSparse(*B), [-1, 3, 4])
    assert st == 0
    assert C.coords == Cr.coords and C.block_sizes == Cr.block_sizes
    assert rel_fro(C.to_numpy_data(), Cr.data) <= RTOL


def test_shards_with_more_ranks_than_output_blocks(gpu):
    """Eight ranks over three output blocks: five shards are empty, the rest
    hold one block each, and together they are the full result."""
    bs = gpu.blocksparse
    rng = np.random.default_rng(41)
    sizes = [[3, 4, 5], [2, 6]]
    ca = [(0, 0), (1, 1), (2, 0)]
    cb = [(0, 0), (1, 1)]
    A = bs.BlockSparseF64.from_blocks(sizes, ca, rng.standard_normal(3 * 2 + 4 * 6 + 5 * 2))
    B = bs.BlockSparseF64.from_blocks([[2, 6], [4, 3]], cb, rng.standard_normal(2 * 4 + 6 * 3))
    full = bs.contract(A, [1, -1], B, [-1, 2])
    shards = [bs.contract_shard(A, [1, -1], B, [-1, 2], r, 8) for r in range(8)]
    assert sum(s.nnzblocks for s in shards) == full.nnzblocks == 3
    assert sum(1 for s in shards if s.nnzblocks == 0) == 5
    coords, data = merge_shards(shards)
    assert coords == full.coords
    np.testing.assert_array_equal(data, full.to_numpy_data())
    blocks, flops = bs.shard_plan(A, [1, -1], B, [-1, 2], 8)
    assert blocks == [s.nnzblocks for s in shards]


@pytest.mark.parametrize("rank,nranks", [(-1, 2), (2, 2), (0, 0)])
def test_shard_rejects_bad_rank(gpu, rank, nranks):
    bs = gpu.blocksparse
    A = bs.BlockSparseF64.from_blocks([[2], [3]], [(0, 0)], np.ones(6))
    with pytest.raises(gpu.NDTensorsError):
        bs.contract_shard(A, [1, -1], A, [2, -1], rank, nranks)


def test_contract_select_from_referenced_blocks_only(gpu):
    """A share of the U(1) rank-4 contraction computed from operands that hold
    only the blocks its output blocks reference (what a rank of the literal
    8-GPU run keeps) equals those blocks of the full contraction."""
    bs = gpu.blocksparse
    (sa, ca, a), (sb, cb, b), la, lb = cfg4_tensors(scale=8)
    A = bs.BlockSparseF64.from_blocks(sa, ca, a)
    B = bs.BlockSparseF64.from_blocks(sb, cb, b)
    full = bs.contract(A, la, B, lb)
    outs = full.coords[3::4]
    want = set(outs)
    used_a = {x for x in ca for y in cb if x[2:] == y[:2] and (x[0], x[1], y[2], y[3]) in want}
    used_b = {y for x in ca for y in cb if x[2:] == y[:2] and (x[0], x[1], y[2], y[3]) in want}

    def sub(sizes, coords, data, keep):
        offs = np.cumsum([0] + [int(np.prod([sizes[ax][c] for ax, c in enumerate(cc)])) for cc in coords])
        kc = [c for c in coords if c in keep]
        kd = np.concatenate([data[offs[i]:offs[i + 1]] for i, c in enumerate(coords) if c in keep])
        return bs.BlockSparseF64.from_blocks(sizes, kc, kd)

    As, Bs = sub(sa, ca, a, used_a), sub(sb, cb, b, used_b)
    assert As.nnzblocks < A.nnzblocks
    got = bs.contract_select(As, la, Bs, lb, outs + [(0, 0, 0, 8)])  # a coordinate no pair produces: ignored
    assert got.coords == sorted(outs)
    for c in outs:
        np.testing.assert_allclose(got.block(c), full.block(c), rtol=1e-12, atol=1e-12)


def test_literal_size_selected_blocks_vs_numpy(gpu):
    """The literal U(1) rank-4 structure (sector dims [8,24,56,96,144,96,56,24,8],
    68 GB per operand): the twelve output blocks that need the fewest input
    elements, computed with contract_select from operands holding only their
    referenced blocks, against numpy (2-pair outputs included)."""
    from math import prod

    from workloads import cfg4_dims, cfg4_structure

    bs = gpu.blocksparse
    dims = cfg4_dims(1)
    sizes, coords = cfg4_structure(dims)
    el = {c: prod(dims[x] for x in c) for c in coords}
    pairs = {}
    for x in coords:
        for y in coords:
            if x[2:] == y[:2]:
                pairs.setdefault((x[0], x[1], y[2], y[3]), []).append((x, y))
    cost = {o: sum(el[c] for c in {p[0] for p in ps} | {p[1] for p in ps}) for o, ps in pairs.items()}
    outs = sorted(sorted(pairs, key=lambda o: (cost[o], o))[:12])
    need_a = [c for c in coords if any(c == p[0] for o in outs for p in pairs[o])]
    need_b = [c for c in coords if any(c == p[1] for o in outs for p in pairs[o])]
    rng = np.random.default_rng(43)
    da = {c: rng.standard_normal(el[c]) for c in need_a}
    db = {c: rng.standard_normal(el[c]) for c in need_b}
    A = bs.BlockSparseF64.from_blocks(sizes, need_a, np.concatenate([da[c] for c in need_a]))
    B = bs.BlockSparseF64.from_blocks(sizes, need_b, np.concatenate([db[c] for c in need_b]))
    got = bs.contract_select(A, [1, 2, -1, -2], B, [-1, -2, 3, 4], outs)
    assert got.coords == outs
    for o in outs:
        m, n = dims[o[0]] * dims[o[1]], dims[o[2]] * dims[o[3]]
        ref = np.zeros((m, n))
        for x, y in pairs[o]:
            k = dims[x[2]] * dims[x[3]]
            ref += da[x].reshape((m, k), order="F") @ db[y].reshape((k, n), order="F")
        blk = got.block(o).reshape((m, n), order="F")
        assert np.linalg.norm(blk - ref) <= 1e-12 * np.linalg.norm(ref)


def _through_diag_ref(oracle, A, la, S, ls, B, lb):
    """Oracle of (A . S) . B: S made dense blocks, then two contract_blocksparse."""
    P = max([x for x in list(la) + list(lb) if x > 0] + [0]) + 1
    Sbs = oracle.bs_from_dense(oracle.diag_to_dense(*S), S[0], S[1])
    st, AS = oracle.bs_contract(oracle.BlockSparse(*A), la, Sbs, [ls[0], P])
    assert st == 0
    las = sorted(x for x in la if x != ls[0]) + [ls[1]]
    st, C = oracle.bs_contract(AS, las, oracle.BlockSparse(*B), lb)
    assert st == 0
    return C


def test_through_diag_cfg5_reduced_bond(gpu, oracle):
    """(A . S) . B of the c128 two-site MPS at bond 1024 as one grouped launch
    (S's diagonal applied to A's loads) vs the oracle's two contractions, and
    vs the library's two-step path."""
    A, S, B = cfg5_tensors(bond=1024)
    bs = gpu.blocksparse
    gA, gS, gB = bs.BlockSparseC64.from_blocks(*A), bs.DiagBlockSparseC64.from_blocks(*S), bs.BlockSparseC64.from_blocks(*B)
    C = bs.contract_through_diag(gA, [1, 2, -1], gS, [-1, -2], gB, [-2, 3, 4])
    n0 = gpu.launch_count()
    bs.contract_through_diag(gA, [1, 2, -1], gS, [-1, -2], gB, [-2, 3, 4], 0, 2)
    assert gpu.launch_count() - n0 == 1  # sharded: one grouped GEMM, no scaling pass
    ref = _through_diag_ref(oracle, A, [1, 2, -1], S, [-1, -2], B, [-2, 3, 4])
    assert C.coords == ref.coords and C.block_sizes == ref.block_sizes
    assert rel_fro(C.to_numpy_data(), ref.data) <= RTOL
    two = bs.contract(bs.contract_diag(gA, [1, 2, -1], gS, [-1, 5]), [1, 2, -1], gB, [-1, 3, 4])
    assert two.coords == C.coords
    assert rel_fro(C.to_numpy_data(), two.to_numpy_data()) <= RTOL
    # sharded (fused): every rank's blocks together are the full result; the
    # same kernel arithmetic on every split, bit for bit
    first = None
    for n in (2, 3, 8):
        shards = [bs.contract_through_diag(gA, [1, 2, -1], gS, [-1, -2], gB, [-2, 3, 4], r, n) for r in range(n)]
        coords, data = merge_shards(shards)
        assert coords == C.coords
        assert rel_fro(data, ref.data) <= RTOL
        if first is None:
            first = data
        assert np.array_equal(data, first)


@pytest.mark.parametrize("cplx", [False, True])
@pytest.mark.parametrize("la,lb", [
    ([1, 2, -1], [-2, 3]),   # A MN-major, B K-major
    ([-1, 1, 2], [-2, 3]),   # A K-major
    ([1, -1], [3, -2]),      # B MN-major
    ([1, -1, 2], [3, -2, 4]),  # middle axes: both operands packed first
])
def test_through_diag_layouts_vs_oracle(gpu, oracle, cplx, la, lb):
    rng = np.random.default_rng(61)
    ksz = [2, 3, 5, 4]
    free = {1: [3, 2], 2: [1, 4], 3: [2, 5], 4: [3, 1]}
    sa = [ksz if x < 0 else free[x] for x in la]
    sb = [ksz if x < 0 else free[x] for x in lb]
    A = random_bs(rng, sa, 0.7, cplx)
    B = random_bs(rng, sb, 0.7, cplx)
    scoords = [(0, 0), (1, 1), (3, 3)]  # square diagonal blocks; coordinate 2 has none
    nd = sum(ksz[c[0]] for c in scoords)
    diag = rng.standard_normal(nd) + (1j * rng.standard_normal(nd) if cplx else 0)
    S = ([ksz, ksz], scoords, diag)
    bs = gpu.blocksparse
    cls = _cls(gpu, cplx)
    dcls = bs.DiagBlockSparseC64 if cplx else bs.DiagBlockSparseF64
    gA, gS, gB = cls.from_blocks(*A), dcls.from_blocks(*S), cls.from_blocks(*B)
    C = bs.contract_through_diag(gA, la, gS, [-1, -2], gB, lb)  # unsharded: two contractions
    ref = _through_diag_ref(oracle, A, la, S, [-1, -2], B, lb)
    assert C.coords == ref.coords and C.block_sizes == ref.block_sizes
    assert rel_fro(C.to_numpy_data(), ref.data) <= RTOL
    # sharded: the fused launch (S applied to the operand loads)
    coords, data = merge_shards([bs.contract_through_diag(gA, la, gS, [-1, -2], gB, lb, r, 2) for r in range(2)])
    assert coords == ref.coords
    assert rel_fro(data, ref.data) <= RTOL


def test_through_diag_fallbacks_and_errors(gpu, oracle):
    """Off-diagonal S blocks map A's coordinate q to B's q' (fused); a
    non-square S block or two S blocks on one coordinate take the two-step
    path; label misuse is an error."""
    rng = np.random.default_rng(62)
    bs = gpu.blocksparse
    ksz = [3, 3, 2]
    A = random_bs(rng, [[2, 4], ksz], 0.9, False)
    B = random_bs(rng, [ksz, [3, 2]], 0.9, False)
    cls, dcls = bs.BlockSparseF64, bs.DiagBlockSparseF64
    for scoords in ([(0, 1), (1, 0), (2, 2)],      # permuting square blocks: fused
                    [(0, 2), (2, 1)],              # non-square (3 vs 2): two-step
                    [(0, 0), (0, 1)]):             # one coordinate, two blocks: two-step
        nd = sum(min(ksz[c[0]], ksz[c[1]]) for c in scoords)
        S = ([ksz, ksz], scoords, rng.standard_normal(nd))
        ref = _through_diag_ref(oracle, A, [1, -1], S, [-1, -2], B, [-2, 2])
        for n in (1, 2):
            shards = [bs.contract_through_diag(cls.from_blocks(*A), [1, -1], dcls.from_blocks(*S), [-1, -2],
                                               cls.from_blocks(*B), [-2, 2], r, n) for r in range(n)]
            coords, data = merge_shards(shards)
            assert coords == ref.coords
            assert rel_fro(data, ref.data) <= RTOL
    S = dcls.from_blocks([ksz, ksz], [(0, 0)], np.ones(3))
    gA, gB = cls.from_blocks(*A), cls.from_blocks(*B)
    for la, ls, lb in (([1, -1], [-1, 2], [-2, 2]),     # S label not negative
                       ([1, -3], [-1, -2], [-2, 2]),    # A lacks S's first label
                       ([1, -1], [-1, -2], [-2, 1])):   # A and B share a label
        with pytest.raises(gpu.NDTensorsError):
            bs.contract_through_diag(gA, la, S, ls, gB, lb)


@pytest.mark.parametrize("cplx", [False, True])
def test_from_device_blocks_sorts_and_packs(gpu, cplx):
    """Blocks scattered in a device buffer (any order, gaps between them)
    become a tensor with sorted, packed blocks, in one copy launch; a block
    reaching past the buffer is rejected."""
    import torch

    rng = np.random.default_rng(71)
    sizes = [[3, 1, 4], [2, 5]]
    coords = [(2, 1), (0, 0), (1, 1), (2, 0)]
    shapes = [(sizes[0][c[0]], sizes[1][c[1]]) for c in coords]
    blocks = [rng.standard_normal(int(np.prod(sh))) + (1j * rng.standard_normal(int(np.prod(sh))) if cplx else 0)
              for sh in shapes]
    dt = np.complex128 if cplx else np.float64
    offs, buf, pos = [], [], 0
    for b in blocks:
        pos += 3  # a gap before every block
        offs.append(pos)
        buf += [np.zeros(3, dtype=dt), b.astype(dt)]
        pos += b.size
    host = np.concatenate(buf)
    width = 2 if cplx else 1
    dbuf = torch.from_numpy(host.view(np.float64).copy()).cuda()
    cls = _cls(gpu, cplx)
    n0 = gpu.launch_count()
    t = cls.from_device_blocks(sizes, coords, offs, dbuf.data_ptr(), dbuf.numel() // width)
    assert gpu.launch_count() - n0 == 1
    order = sorted(range(len(coords)), key=lambda i: coords[i])
    assert t.coords == [coords[i] for i in order]
    assert np.array_equal(t.to_numpy_data(), np.concatenate([blocks[i].astype(dt) for i in order]))
    with pytest.raises(ValueError):
        cls.from_device_blocks(sizes, coords[:1], [pos - 1], dbuf.data_ptr(), dbuf.numel() // width)


def test_cfg4_permuted_labels_many_blocks_vs_oracle(gpu, oracle):
    """U(1) rank-4 at 1/8 scale with A's labels in a non-natural order
    (-1, 1, -2, 2): the grouped GEMM reads A's 489 blocks in place through
    their index runs (rows: free axes 1, 3; contraction: axes 0, 2), so the
    contraction is that one launch; checked against the oracle."""
    (sa, ca, a), (sb, cb, b), _, lb = cfg4_tensors(scale=8)
    # A's axes relabelled: axis 0 and 2 contracted, 1 and 3 free
    la = [-1, 1, -2, 2]
    lb2 = [-1, -2, 3, 4]
    cls = gpu.blocksparse.BlockSparseF64
    At, Bt = cls.from_blocks(sa, ca, a), cls.from_blocks(sb, cb, b)
    n0 = gpu.launch_count()
    gpu.blocksparse.contract(At, la, Bt, lb2)
    assert gpu.launch_count() - n0 == 1
    _check(gpu, oracle, (sa, ca, a), la, (sb, cb, b), lb2)


# Operands and output in non-GEMM axis order, each GEMM index of every block
# in at most two strided runs: the grouped GEMM addresses the blocks in place
# (one launch, no pack of A or B, no permute of C).
STRIDED = [
    # A (contracted, free, contracted, free)
    ([[2, 3], [3, 2], [2, 4], [1, 3]], [-1, 1, -2, 2], [[2, 3], [2, 4], [4, 1], [2]], [-1, -2, 3, 4]),
    # B (free, contracted, free, contracted), its contracted axes reversed
    ([[3, 2], [1, 3], [2, 3], [2, 4]], [1, 2, -1, -2], [[4, 1], [2, 4], [2], [2, 3]], [3, -2, 4, -1]),
    # both operands interleaved, contracted axes in opposite orders
    ([[2, 2], [3, 1], [4], [2, 3]], [1, -2, 2, -1], [[2, 3], [3, 2], [3, 1], [1, 2]], [-1, 3, -2, 4]),
    # output labels descending (every output block square): C written in its
    # label-sorted axis order directly
    ([[3, 3], [4, 2]], [2, -1], [[4, 2], [3, 3]], [-1, 1]),
]


@pytest.mark.parametrize("cplx", [False, True])
@pytest.mark.parametrize("sa,la,sb,lb", STRIDED)
def test_strided_operands_one_launch_vs_oracle(gpu, oracle, sa, la, sb, lb, cplx):
    rng = np.random.default_rng(int.from_bytes(repr((sa, la, sb, lb, cplx)).encode(), "little") % (2**32))
    A = random_bs(rng, sa, 0.8, cplx)
    B = random_bs(rng, sb, 0.8, cplx)
    cls = _cls(gpu, cplx)
    At, Bt = cls.from_blocks(*A), cls.from_blocks(*B)
    n0 = gpu.launch_count()
    gpu.blocksparse.contract(At, la, Bt, lb)
    assert gpu.launch_count() - n0 == 1
    _check(gpu, oracle, A, la, B, lb)


def test_strided_pairs_vs_oracle(gpu, oracle):
    """Even block extents and A's contraction run contiguous: the strided
    f64 loads copy adjacent k pairs (16 bytes); one launch, vs the oracle."""
    rng = np.random.default_rng(2024)
    sa, la = [[2, 4], [4, 2], [2, 6], [2, 4]], [-1, 1, -2, 2]
    sb, lb = [[2, 4], [2, 6], [4, 2], [2]], [-1, -2, 3, 4]
    A = random_bs(rng, sa, 0.8, False)
    B = random_bs(rng, sb, 0.8, False)
    cls = _cls(gpu, False)
    At, Bt = cls.from_blocks(*A), cls.from_blocks(*B)
    n0 = gpu.launch_count()
    gpu.blocksparse.contract(At, la, Bt, lb)
    assert gpu.launch_count() - n0 == 1
    _check(gpu, oracle, A, la, B, lb)


def test_cfg4_quarter_scale_permuted_equals_natural(gpu):
    """U(1) rank-4 at 1/4 scale (even sector dims: pair copies): A's blocks
    permuted to (-1, 1, -2, 2) and contracted in place give the same bits as
    the natural-order contraction, in one launch."""
    (sa, ca, a), (sb, cb, b), la, lb = cfg4_tensors(scale=4)
    cls = gpu.blocksparse.BlockSparseF64
    At, Bt = cls.from_blocks(sa, ca, a), cls.from_blocks(sb, cb, b)
    ref = gpu.blocksparse.contract(At, la, Bt, lb)
    Ap = At.permutedims([2, 0, 3, 1])
    n0 = gpu.launch_count()
    got = gpu.blocksparse.contract(Ap, [-1, 1, -2, 2], Bt, [-1, -2, 3, 4])
    assert gpu.launch_count() - n0 == 1
    assert got.coords == ref.coords and got.block_sizes == ref.block_sizes
    assert np.array_equal(got.to_numpy_data(), ref.to_numpy_data())


@pytest.mark.parametrize("cplx", [False, True])
def test_three_runs_fall_back_to_packing(gpu, oracle, cplx):
    """A's free axes 1, 3, 5 lie in three separate runs: its blocks are
    packed first (more than one launch), with the same result."""
    rng = np.random.default_rng(606 + cplx)
    sa = [[2, 1], [1, 2], [2, 2], [3, 1], [1, 2], [2, 1]]
    sb = [[2, 1], [2, 2], [1, 2], [2, 3]]
    A = random_bs(rng, sa, 0.9, cplx)
    B = random_bs(rng, sb, 0.9, cplx)
    la, lb = [-1, 1, -2, 2, -3, 3], [-1, -2, -3, 4]
    cls = _cls(gpu, cplx)
    At, Bt = cls.from_blocks(*A), cls.from_blocks(*B)
    n0 = gpu.launch_count()
    gpu.blocksparse.contract(At, la, Bt, lb)
    assert gpu.launch_count() - n0 >= 2
    _check(gpu, oracle, A, la, B, lb)


def test_cfg4_permutedims_many_blocks_bit_exact(gpu, oracle):
    (sa, ca, a), _, _, _ = cfg4_tensors(scale=8)
    t = gpu.blocksparse.BlockSparseF64.from_blocks(sa, ca, a)
    for perm in ([2, 0, 3, 1], [3, 2, 1, 0]):
        st, ref = oracle.bs_permutedims(oracle.BlockSparse(sa, ca, a), perm)
        assert st == 0
        p = t.permutedims(perm)
        assert p.coords == ref.coords and p.block_sizes == ref.block_sizes
        assert np.array_equal(p.to_numpy_data(), ref.data)
