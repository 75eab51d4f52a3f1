"""Runs the reference's known-answer cases (tests/golden/known_answers.json)
against an engine: the CPU oracle or the library's C ABI on the GPU.

Both engines return C-ABI status codes (NDT_*), mapping the oracle's error
kinds the way crates/ndtensors-capi/src/lib.rs maps TensorError and panics.
"""

from __future__ import annotations

import ctypes
import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden" / "known_answers.json"

NDT_SUCCESS, NDT_INVALID_ARGUMENT, NDT_SHAPE_MISMATCH = 0, -1, -2
NDT_INDEX_OUT_OF_BOUNDS, NDT_INTERNAL_ERROR, NDT_INVALID_PERMUTATION = -3, -4, -5


def load_cases():
    return json.loads(GOLDEN.read_text())["cases"]


def arr(spec):
    """Column-major numpy array from a fixture tensor."""
    shape = tuple(spec["shape"])
    data = spec["data"]
    if spec.get("dtype") == "c64":
        flat = np.array([complex(re, im) for re, im in data], dtype=np.complex128)
    else:
        flat = np.array(data, dtype=np.float64)
    n = int(np.prod(shape, dtype=np.int64))
    if n == flat.size:
        return flat.reshape(shape, order="F")
    return flat  # storage / shape mismatch cases keep the raw data


def bs_spec(spec):
    dtype = np.complex128 if spec.get("dtype") == "c64" else np.float64
    data = spec["data"]
    if dtype == np.complex128:
        flat = np.array([complex(re, im) for re, im in data], dtype=dtype)
    else:
        flat = np.array(data, dtype=dtype)
    return spec["block_sizes"], [tuple(c) for c in spec["coords"]], flat


def map_oracle_status(st, code_for_error):
    if st == 0:
        return NDT_SUCCESS
    if st == 9:  # panic
        return NDT_INTERNAL_ERROR
    return code_for_error


# ------------------------------------------------------------------ engines
class OracleEngine:
    name = "oracle"

    def __init__(self, o):
        self.o = o

    def permutedims(self, a, perm):
        st, out = self.o.permutedims(a, perm)
        return map_oracle_status(st, NDT_INVALID_PERMUTATION), out

    def contract(self, a, la, b, lb):
        st, out = self.o.contract_naive(a, la, b, lb)
        return map_oracle_status(st, NDT_SHAPE_MISMATCH), out

    def contract_gemm(self, a, la, b, lb):
        st, out = self.o.contract_gemm(a, la, b, lb)
        return map_oracle_status(st, NDT_SHAPE_MISMATCH), out

    def bs_contract(self, A, la, B, lb):
        st, out = self.o.bs_contract(self.o.BlockSparse(*A), la, self.o.BlockSparse(*B), lb)
        if out is None:
            return map_oracle_status(st, NDT_SHAPE_MISMATCH), None
        return NDT_SUCCESS, (out.block_sizes, out.coords, out.data)

    def bs_permutedims(self, A, perm):
        st, out = self.o.bs_permutedims(self.o.BlockSparse(*A), perm)
        if out is None:
            return map_oracle_status(st, NDT_INVALID_PERMUTATION), None
        return NDT_SUCCESS, (out.block_sizes, out.coords, out.data)

    def bs_to_dense(self, A):
        return self.o.bs_to_dense(self.o.BlockSparse(*A))

    def diag_to_dense(self, S):
        return self.o.diag_to_dense(*S)


class CapiEngine:
    """The library's C ABI (ctypes), computing on the GPU."""

    name = "capi"

    def __init__(self, ndt):
        self.ndt = ndt
        self.lib = ndt.get_lib()

    def _tensor(self, a):
        cls = self.ndt.TensorC64 if np.iscomplexobj(a) else self.ndt.TensorF64
        return cls.from_numpy(a)

    def permutedims(self, a, perm):
        t = self._tensor(a)
        n = len(perm)
        parr = (ctypes.c_size_t * max(n, 1))(*perm)
        status = ctypes.c_int(-999)
        ptr = t._f("permutedims")(t._ptr, parr, n, ctypes.byref(status))
        if status.value != 0:
            return status.value, None
        return 0, type(t)(ptr).to_numpy()

    def _contract(self, fname, a, la, b, lb):
        ta, tb = self._tensor(a), self._tensor(b)
        l1 = (ctypes.c_long * max(len(la), 1))(*la)
        l2 = (ctypes.c_long * max(len(lb), 1))(*lb)
        status = ctypes.c_int(-999)
        ptr = getattr(self.lib, f"ndt_tensor_{ta._prefix}_{fname}")(
            ta._ptr, l1, len(la), tb._ptr, l2, len(lb), ctypes.byref(status))
        if status.value != 0:
            return status.value, None
        return 0, type(ta)(ptr).to_numpy()

    def contract(self, a, la, b, lb):
        return self._contract("contract", a, la, b, lb)

    def contract_gemm(self, a, la, b, lb):
        return self._contract("contract_gemm", a, la, b, lb)

    def vjp(self, a, la, b, lb, g):
        try:
            ga, gb = self.ndt.contract_vjp(self._tensor(a), la, self._tensor(b), lb, self._tensor(g))
        except ValueError:
            return NDT_SHAPE_MISMATCH, None, None
        return 0, ga.to_numpy(), gb.to_numpy()

    def jvp(self, a, la, b, lb, ta, tb):
        p, t = self.ndt.contract_jvp(self._tensor(a), la, self._tensor(b), lb,
                                     self._tensor(ta) if ta is not None else None,
                                     self._tensor(tb) if tb is not None else None)
        return 0, p.to_numpy(), (t.to_numpy() if t is not None else None)

    def bs_contract(self, A, la, B, lb):
        bs = self.ndt.blocksparse
        cls = bs.BlockSparseC64 if np.iscomplexobj(A[2]) else bs.BlockSparseF64
        try:
            c = bs.contract(cls.from_blocks(*A), la, cls.from_blocks(*B), lb)
        except ValueError:
            return NDT_SHAPE_MISMATCH, None
        return 0, (c.block_sizes, c.coords, c.to_numpy_data())

    def bs_permutedims(self, A, perm):
        bs = self.ndt.blocksparse
        cls = bs.BlockSparseC64 if np.iscomplexobj(A[2]) else bs.BlockSparseF64
        try:
            c = cls.from_blocks(*A).permutedims(perm)
        except ValueError:
            return NDT_INVALID_PERMUTATION, None
        return 0, (c.block_sizes, c.coords, c.to_numpy_data())

    def bs_to_dense(self, A):
        bs = self.ndt.blocksparse
        cls = bs.BlockSparseC64 if np.iscomplexobj(A[2]) else bs.BlockSparseF64
        return cls.from_blocks(*A).to_dense().to_numpy()

    def diag_to_dense(self, S):
        bs = self.ndt.blocksparse
        cls = bs.DiagBlockSparseC64 if np.iscomplexobj(S[2]) else bs.DiagBlockSparseF64
        return cls.from_blocks(*S).to_dense().to_numpy()


# ------------------------------------------------------------------ checks
def _at(x, idx):
    v = x[tuple(idx)]
    return v


def _val(v):
    return complex(v[0], v[1]) if isinstance(v, list) else v


def _cmp_data(out, data):
    flat = np.asarray(out).ravel(order="F")
    exp = np.array([_val(v) for v in data])
    assert flat.size == exp.size, (flat.size, exp.size)
    np.testing.assert_allclose(flat, exp, rtol=1e-12, atol=1e-12)


def run_case(eng, c, oracle_engine=None):
    """Execute one case on `eng`; raises AssertionError on a mismatch."""
    op, e = c["op"], c.get("expect")
    if op == "permutedims":
        st, out = eng.permutedims(arr(c["a"]), c["perm"])
        assert st == e["status"], (st, e["status"])
        if st == 0:
            assert list(out.shape) == e["shape"]
            if "data" in e:
                # permutes are bit-exact
                flat = out.ravel(order="F")
                exp = np.array([_val(v) for v in e["data"]])
                assert np.array_equal(flat, exp), (flat, exp)
            for i, v in e.get("index", []):
                assert out.ravel(order="F")[i] == v
    elif op in ("contract", "contract_gemm"):
        a, b = arr(c["a"]), arr(c["b"])
        st, out = getattr(eng, op)(a, c["la"], b, c["lb"])
        assert st == e["status"], (st, e["status"])
        if st == 0:
            assert list(np.shape(out)) == e["shape"], (np.shape(out), e["shape"])
            if "data" in e:
                _cmp_data(out, e["data"])
            for idx, v in e.get("at", []):
                assert abs(_at(out, idx) - _val(v)) <= 1e-12 * max(1.0, abs(_val(v)))
            if e.get("equals_naive") and oracle_engine is not None:
                st2, ref = oracle_engine.contract(a, c["la"], b, c["lb"])
                assert st2 == 0
                np.testing.assert_allclose(out, ref, rtol=1e-10, atol=1e-10)
    elif op == "vjp":
        if not hasattr(eng, "vjp"):
            return "skip"
        st, ga, gb = eng.vjp(arr(c["a"]), c["la"], arr(c["b"]), c["lb"], arr(c["grad"]))
        assert st == e["status"]
        assert list(ga.shape) == e["ga_shape"] and list(gb.shape) == e["gb_shape"]
        for idx, v in e.get("ga_at", []):
            assert abs(ga[tuple(idx)] - v) < 1e-12
        for idx, v in e.get("gb_at", []):
            assert abs(gb[tuple(idx)] - v) < 1e-12
        if "ga_data" in e:
            _cmp_data(ga, e["ga_data"])
            _cmp_data(gb, e["gb_data"])
    elif op == "jvp":
        if not hasattr(eng, "jvp"):
            return "skip"
        ta = arr(c["ta"]) if c.get("ta") else None
        tb = arr(c["tb"]) if c.get("tb") else None
        st, p, t = eng.jvp(arr(c["a"]), c["la"], arr(c["b"]), c["lb"], ta, tb)
        assert st == e["status"]
        if "primal_data" in e:
            _cmp_data(p, e["primal_data"])
        if "tangent" in e and e["tangent"] is None:
            assert t is None
        if "tangent_data" in e:
            assert list(t.shape) == e["tangent_shape"]
            _cmp_data(t, e["tangent_data"])
    elif op == "bs_contract":
        A, B = bs_spec(c["a"]), bs_spec(c["b"])
        st, out = eng.bs_contract(A, c["la"], B, c["lb"])
        assert st == e["status"], (st, e["status"])
        if st == 0:
            sizes, coords, data = out
            if "coords" in e:
                assert [list(x) for x in coords] == e["coords"]
            if "dense_shape" in e:
                assert [sum(s) for s in sizes] == e["dense_shape"]
            if "data" in e:
                _cmp_data(data, e["data"])
            if "dense_data" in e or e.get("equals_dense_gemm"):
                if oracle_engine is None:
                    oracle_engine = eng
                dense = oracle_engine.bs_to_dense((sizes, coords, data))
                if "dense_data" in e:
                    _cmp_data(dense, e["dense_data"])
                if e.get("equals_dense_gemm"):
                    da = oracle_engine.bs_to_dense(A)
                    db = oracle_engine.bs_to_dense(B)
                    st2, ref = oracle_engine.contract_gemm(da, c["la"], db, c["lb"])
                    assert st2 == 0
                    np.testing.assert_allclose(dense, ref, rtol=1e-10, atol=1e-10)
    elif op == "bs_permutedims":
        A = bs_spec(c["a"])
        st, out = eng.bs_permutedims(A, c["perm"])
        assert st == e["status"], (st, e["status"])
        if st == 0:
            sizes, coords, data = out
            if "coords" in e:
                assert [list(x) for x in coords] == e["coords"]
            assert [sum(s) for s in sizes] == e["dense_shape"]
            if e.get("equals_dense_permute"):
                ref_eng = oracle_engine or eng
                dense = ref_eng.bs_to_dense((sizes, coords, data))
                st2, ref = ref_eng.permutedims(ref_eng.bs_to_dense(A), c["perm"])
                assert np.array_equal(dense, ref)
    elif op == "diag_to_dense":
        S = bs_spec(c["s"])
        d = eng.diag_to_dense(S)
        assert list(d.shape) == e["shape"]
        for idx, v in e["at"]:
            assert d[tuple(idx)] == _val(v)
    else:
        return "skip"
    return "ok"
