"""Writes tests/golden/known_answers.json.

Every case restates a known-answer test of the reference (ndtensors-rs): its
inputs and asserted outputs, with the file:line of the test it comes from.
The reference itself cannot be built or imported in this environment (Rust
crate; no toolchain), so these asserted values are the pins of the oracle
and of the CUDA path.  Run:  python tests/golden/make_known_answers.py
"""

from __future__ import annotations

import json
from pathlib import Path

OUT = Path(__file__).resolve().parent / "known_answers.json"


def t(shape, data=None, fill=None, dtype="f64"):
    """A dense tensor: column-major data (complex as [re, im] pairs)."""
    n = 1
    for s in shape:
        n *= s
    n = max(n, 1)
    if data is None:
        data = [fill] * n
    return {"shape": list(shape), "data": data, "dtype": dtype}


def seq(lo, hi, mul=1.0, add=0.0):
    return [float(x) * mul + add for x in range(lo, hi)]


cases = []


def case(cid, source, op, **kw):
    c = {"id": cid, "source": source, "op": op}
    c.update(kw)
    cases.append(c)


# ------------------------------------------------------------- strides.rs
case("strides_3d", "crates/ndtensors/src/strides.rs:79-82", "strides", shape=[3, 4, 5], expect=[1, 3, 12])
case("strides_2d", "crates/ndtensors/src/strides.rs:84-87", "strides", shape=[2, 3], expect=[1, 2])
case("strides_1d", "crates/ndtensors/src/strides.rs:89-92", "strides", shape=[5], expect=[1])
case("strides_empty", "crates/ndtensors/src/strides.rs:94-97", "strides", shape=[], expect=[])
case("cart_to_lin", "crates/ndtensors/src/strides.rs:99-112", "cart_to_lin", shape=[3, 4, 5],
     pairs=[[[0, 0, 0], 0], [[1, 0, 0], 1], [[0, 1, 0], 3], [[0, 0, 1], 12], [[2, 3, 4], 2 + 9 + 48]])
case("lin_to_cart", "crates/ndtensors/src/strides.rs:114-121", "lin_to_cart", shape=[3, 4, 5],
     pairs=[[0, [0, 0, 0]], [1, [1, 0, 0]], [3, [0, 1, 0]], [12, [0, 0, 1]]])

# ------------------------------------------------- permutedims.rs / generic.rs
i3 = [float(i * 100 + j * 10 + k) for k in range(4) for j in range(3) for i in range(2)]  # column-major of [2,3,4]
case("permute_transpose_f64", "crates/ndtensors/src/operations/permutedims.rs:231-248", "permutedims",
     a=t([2, 3], seq(1, 7)), perm=[1, 0], expect={"status": 0, "shape": [3, 2], "data": [1.0, 3.0, 5.0, 2.0, 4.0, 6.0]})
case("permute_transpose_c64", "crates/ndtensors/src/operations/permutedims.rs:250-253", "permutedims",
     a=t([2, 3], [[float(x), 0.0] for x in range(1, 7)], dtype="c64"), perm=[1, 0],
     expect={"status": 0, "shape": [3, 2], "data": [[1.0, 0.0], [3.0, 0.0], [5.0, 0.0], [2.0, 0.0], [4.0, 0.0], [6.0, 0.0]]})
# dest[k,i,j] = src[i,j,k]
p3 = [0.0] * 24
for i in range(2):
    for j in range(3):
        for k in range(4):
            p3[k + 4 * i + 8 * j] = float(i * 100 + j * 10 + k)
case("permute_3d_201", "crates/ndtensors/src/operations/permutedims.rs:255-277 (backend/generic.rs:65-89)",
     "permutedims", a=t([2, 3, 4], i3), perm=[2, 0, 1], expect={"status": 0, "shape": [4, 2, 3], "data": p3})
case("permute_identity", "crates/ndtensors/src/operations/permutedims.rs:279-286", "permutedims",
     a=t([2, 3], seq(1, 7)), perm=[0, 1], expect={"status": 0, "shape": [2, 3], "data": seq(1, 7)})
for k, perm in enumerate([[0], [0, 1, 2], [0, 2], [0, 0]]):
    case(f"permute_invalid_{k}", "crates/ndtensors/src/operations/permutedims.rs:288-301", "permutedims",
         a=t([2, 3], fill=0.0), perm=perm, expect={"status": -5})
case("capi_permutedims", "crates/ndtensors-capi/src/lib.rs:988-1022", "permutedims",
     a=t([2, 3], seq(1, 7)), perm=[1, 0], expect={"status": 0, "shape": [3, 2], "index": [[1, 3.0]]})
case("py_permutedims_transpose", "python/ndtensors_rs/tests/test_tensor.py:173-186", "permutedims",
     a=t([2, 3], [1.0, 2.0, 3.0, 4.0, 5.0, 6.0]), perm=[1, 0],
     expect={"status": 0, "shape": [3, 2], "data": [1.0, 3.0, 5.0, 2.0, 4.0, 6.0]})

# ---------------------------------------------------------------- naive.rs
A23 = t([2, 3], seq(1, 7))
B34 = t([3, 4], seq(1, 13))
case("naive_matrix_multiply", "crates/ndtensors/src/contract/naive.rs:590-610", "contract",
     a=A23, la=[1, -1], b=B34, lb=[-1, 2], expect={"status": 0, "shape": [2, 4], "at": [[[0, 0], 22.0]]})
case("naive_inner_product", "crates/ndtensors/src/contract/naive.rs:612-623", "contract",
     a=t([3], [1.0, 2.0, 3.0]), la=[-1], b=t([3], [4.0, 5.0, 6.0]), lb=[-1],
     expect={"status": 0, "shape": [1], "data": [32.0]})
case("naive_outer_product", "crates/ndtensors/src/contract/naive.rs:625-640", "contract",
     a=t([2], [1.0, 2.0]), la=[1], b=t([3], [3.0, 4.0, 5.0]), lb=[2],
     expect={"status": 0, "shape": [2, 3], "at": [[[0, 0], 3.0], [[1, 0], 6.0], [[0, 1], 4.0], [[1, 2], 10.0]]})
case("naive_3d", "crates/ndtensors/src/contract/naive.rs:642-653", "contract",
     a=t([2, 3, 4], fill=1.0), la=[1, 2, -1], b=t([4, 5], fill=1.0), lb=[-1, 3],
     expect={"status": 0, "shape": [2, 3, 5], "at": [[[0, 0, 0], 4.0]]})
case("naive_dimension_mismatch", "crates/ndtensors/src/contract/naive.rs:655-663", "contract",
     a=t([2, 3], fill=1.0), la=[1, -1], b=t([4, 5], fill=1.0), lb=[-1, 2], expect={"status": -2})
case("capi_contract_ones", "crates/ndtensors-capi/src/lib.rs:1024-1070", "contract",
     a=t([2, 3], fill=1.0), la=[1, -1], b=t([3, 4], fill=1.0), lb=[-1, 2],
     expect={"status": 0, "shape": [2, 4], "data": [3.0] * 8})
# python/ndtensors_rs/tests/test_contract.py
case("py_matrix_multiply_values", "python/ndtensors_rs/tests/test_contract.py:23-33", "contract",
     a=t([2, 2], [1.0, 3.0, 2.0, 4.0]), la=[1, -1], b=t([2, 2], [5.0, 7.0, 6.0, 8.0]), lb=[-1, 2],
     expect={"status": 0, "shape": [2, 2], "data": [19.0, 43.0, 22.0, 50.0]})
case("py_trace_pinned", "python/ndtensors_rs/tests/test_contract.py:56-65", "contract",
     a=t([2, 2], [1.0, 3.0, 2.0, 4.0]), la=[-1, -1], b=t([], [1.0]), lb=[],
     expect={"status": 0, "shape": [1], "data": [1.0]})
case("py_multiple_contractions", "python/ndtensors_rs/tests/test_contract.py:211-221", "contract",
     a=t([2, 3, 4], fill=1.0), la=[1, -1, -2], b=t([3, 4, 5], fill=1.0), lb=[-1, -2, 2],
     expect={"status": 0, "shape": [2, 5], "data": [12.0] * 10})
case("py_contract_1d_1d", "python/ndtensors_rs/tests/test_contract.py:194-199", "contract",
     a=t([5], fill=1.0), la=[-1], b=t([5], fill=1.0), lb=[-1], expect={"status": 0, "shape": [1], "data": [5.0]})
case("py_no_contraction", "python/ndtensors_rs/tests/test_contract.py:201-209", "contract",
     a=t([2], [1.0, 2.0]), la=[1], b=t([2], [3.0, 4.0]), lb=[2],
     expect={"status": 0, "shape": [2, 2], "data": [3.0, 6.0, 4.0, 8.0]})

# VJP / JVP (naive.rs:665-862; capi/lib.rs:1071-1320)
case("vjp_matrix_multiply", "crates/ndtensors/src/contract/naive.rs:665-709", "vjp",
     a=A23, la=[1, -1], b=B34, lb=[-1, 2], grad=t([2, 4], fill=1.0),
     expect={"status": 0, "ga_shape": [2, 3], "gb_shape": [3, 4],
             "ga_at": [[[0, 0], 22.0], [[0, 1], 26.0], [[0, 2], 30.0], [[1, 0], 22.0], [[1, 1], 26.0], [[1, 2], 30.0]],
             "gb_at": [[[0, 0], 3.0], [[1, 0], 7.0], [[2, 0], 11.0]]})
case("vjp_inner_product", "crates/ndtensors/src/contract/naive.rs:711-733", "vjp",
     a=t([3], [1.0, 2.0, 3.0]), la=[-1], b=t([3], [4.0, 5.0, 6.0]), lb=[-1], grad=t([1], [1.0]),
     expect={"status": 0, "ga_shape": [3], "gb_shape": [3], "ga_data": [4.0, 5.0, 6.0], "gb_data": [1.0, 2.0, 3.0]})
case("vjp_outer_product", "crates/ndtensors/src/contract/naive.rs:735-756", "vjp",
     a=t([2], [1.0, 2.0]), la=[1], b=t([3], [3.0, 4.0, 5.0]), lb=[2], grad=t([2, 3], fill=1.0),
     expect={"status": 0, "ga_shape": [2], "gb_shape": [3], "ga_data": [12.0, 12.0], "gb_data": [3.0, 3.0, 3.0]})
case("capi_vjp_ones", "crates/ndtensors-capi/src/lib.rs:1071-1140", "vjp",
     a=t([2, 3], fill=1.0), la=[1, -1], b=t([3, 4], fill=1.0), lb=[-1, 2], grad=t([2, 4], fill=1.0),
     expect={"status": 0, "ga_shape": [2, 3], "gb_shape": [3, 4], "ga_at": [[[0, 0], 4.0]], "gb_at": [[[0, 0], 2.0]]})
case("jvp_no_tangents", "crates/ndtensors/src/contract/naive.rs:758-765", "jvp",
     a=t([2, 3], fill=1.0), la=[1, -1], b=t([3, 4], fill=1.0), lb=[-1, 2], ta=None, tb=None,
     expect={"status": 0, "primal_data": [3.0] * 8, "tangent": None})
case("jvp_tangent_a", "crates/ndtensors/src/contract/naive.rs:767-781", "jvp",
     a=t([2, 3], fill=1.0), la=[1, -1], b=t([3, 4], fill=1.0), lb=[-1, 2], ta=t([2, 3], fill=1.0), tb=None,
     expect={"status": 0, "tangent_shape": [2, 4], "tangent_data": [3.0] * 8})
case("jvp_tangent_b", "crates/ndtensors/src/contract/naive.rs:783-796", "jvp",
     a=t([2, 3], fill=1.0), la=[1, -1], b=t([3, 4], fill=1.0), lb=[-1, 2], ta=None, tb=t([3, 4], fill=1.0),
     expect={"status": 0, "tangent_shape": [2, 4], "tangent_data": [3.0] * 8})
case("jvp_both", "crates/ndtensors/src/contract/naive.rs:798-811", "jvp",
     a=t([2, 3], fill=1.0), la=[1, -1], b=t([3, 4], fill=1.0), lb=[-1, 2], ta=t([2, 3], fill=1.0),
     tb=t([3, 4], fill=1.0), expect={"status": 0, "tangent_shape": [2, 4], "tangent_data": [6.0] * 8})
case("jvp_inner", "crates/ndtensors/src/contract/naive.rs:813-826", "jvp",
     a=t([3], [1.0, 2.0, 3.0]), la=[-1], b=t([3], [4.0, 5.0, 6.0]), lb=[-1], ta=t([3], [1.0, 0.0, 0.0]), tb=None,
     expect={"status": 0, "tangent_shape": [1], "tangent_data": [4.0]})

# ------------------------------------------------------------------ gemm.rs
case("gemm_matrix_multiply", "crates/ndtensors/src/contract/gemm.rs:244-269", "contract_gemm",
     a=A23, la=[1, -1], b=B34, lb=[-1, 2],
     expect={"status": 0, "shape": [2, 4], "equals_naive": True, "at": [[[0, 0], 22.0]]})
case("gemm_inner_product", "crates/ndtensors/src/contract/gemm.rs:271-285", "contract_gemm",
     a=t([3], [1.0, 2.0, 3.0]), la=[-1], b=t([3], [4.0, 5.0, 6.0]), lb=[-1],
     expect={"status": 0, "shape": [1], "data": [32.0]})
case("gemm_outer_product", "crates/ndtensors/src/contract/gemm.rs:287-305", "contract_gemm",
     a=t([2], [1.0, 2.0]), la=[1], b=t([3], [3.0, 4.0, 5.0]), lb=[2],
     expect={"status": 0, "shape": [2, 3], "equals_naive": True})
case("gemm_3d", "crates/ndtensors/src/contract/gemm.rs:307-325", "contract_gemm",
     a=t([2, 3, 4], fill=1.0), la=[1, 2, -1], b=t([4, 5], fill=1.0), lb=[-1, 3],
     expect={"status": 0, "shape": [2, 3, 5], "equals_naive": True, "data": [4.0] * 30})
case("gemm_dimension_mismatch", "crates/ndtensors/src/contract/gemm.rs:327-334", "contract_gemm",
     a=t([2, 3], fill=1.0), la=[1, -1], b=t([4, 5], fill=1.0), lb=[-1, 2], expect={"status": -2})
case("gemm_complex", "crates/ndtensors/src/contract/gemm.rs:336-373", "contract_gemm",
     a=t([2, 2], [[1.0, 0.0], [2.0, 0.0], [3.0, 0.0], [4.0, 0.0]], dtype="c64"), la=[1, -1],
     b=t([2, 2], [[1.0, 0.0], [0.0, 1.0], [0.0, -1.0], [1.0, 0.0]], dtype="c64"), lb=[-1, 2],
     expect={"status": 0, "shape": [2, 2], "equals_naive": True,
             # C = A B: A=[[1,3],[2,4]], B=[[1,-i],[i,1]] -> [[1+3i, 3-i],[2+4i, 4-2i]]
             "data": [[1.0, 3.0], [2.0, 4.0], [3.0, -1.0], [4.0, -2.0]]})

# ------------------------------------------------------------ properties.rs
case("props_matrix_multiply", "crates/ndtensors/src/contract/properties.rs:230-246", "properties",
     la=[1, -1], sa=[2, 3], lb=[-1, 2], sb=[3, 4],
     expect={"contracted_pairs": [[1, 0]], "uncontracted_a": [0], "uncontracted_b": [1], "dleft": 2, "dmid": 3,
             "dright": 4, "permute_a": False, "permute_b": False, "permute_c": False})
case("props_inner_product", "crates/ndtensors/src/contract/properties.rs:248-261", "properties",
     la=[-1], sa=[5], lb=[-1], sb=[5],
     expect={"contracted_pairs": [[0, 0]], "uncontracted_a": [], "uncontracted_b": [], "dleft": 1, "dmid": 5,
             "dright": 1})
case("props_outer_product", "crates/ndtensors/src/contract/properties.rs:263-276", "properties",
     la=[1], sa=[3], lb=[2], sb=[4],
     expect={"contracted_pairs": [], "uncontracted_a": [0], "uncontracted_b": [0], "dleft": 3, "dmid": 1,
             "dright": 4})
case("props_with_permutation", "crates/ndtensors/src/contract/properties.rs:278-303", "properties",
     la=[1, -1, -2], sa=[2, 3, 4], lb=[-2, -1, 2], sb=[4, 3, 5],
     expect={"uncontracted_a": [0], "uncontracted_b": [2], "dleft": 2, "dmid": 12, "dright": 5,
             "permute_a": False, "permute_b": True, "perm_b": [1, 0, 2]})
case("props_permutation_needed", "crates/ndtensors/src/contract/properties.rs:305-319", "properties",
     la=[2, -1], sa=[3, 4], lb=[-1, 1], sb=[4, 5],
     expect={"dleft": 3, "dmid": 4, "dright": 5, "output_labels": [2, 1], "permute_c": True})
case("props_3d", "crates/ndtensors/src/contract/properties.rs:321-333", "properties",
     la=[1, 2, -1], sa=[2, 3, 4], lb=[-1, 3], sb=[4, 5],
     expect={"contracted_pairs": [[2, 0]], "uncontracted_a": [0, 1], "uncontracted_b": [1], "dleft": 6, "dmid": 4,
             "dright": 5})


# ------------------------------------------------- contract/blocksparse.rs
def bs(sizes, coords, blocks, dtype="f64"):
    data = []
    for b in blocks:
        data.extend(b)
    return {"block_sizes": sizes, "coords": coords, "data": data, "dtype": dtype}


eye2 = [1.0, 0.0, 0.0, 1.0]
ones4 = [1.0] * 4
case("bs_simple_matmul", "crates/ndtensors/src/contract/blocksparse.rs:294-340", "bs_contract",
     a=bs([[2, 2], [2, 2]], [[0, 0], [1, 1]], [eye2, eye2]), la=[1, -1],
     b=bs([[2, 2], [2, 2]], [[0, 0], [1, 1]], [ones4, ones4]), lb=[-1, 2],
     expect={"status": 0, "dense_shape": [4, 4], "coords": [[0, 0], [1, 1]], "data": ones4 + ones4})
case("bs_multiple_contributions", "crates/ndtensors/src/contract/blocksparse.rs:342-389", "bs_contract",
     a=bs([[2, 2], [2, 2, 2]], [[0, 0], [0, 1], [0, 2]], [ones4] * 3), la=[1, -1],
     b=bs([[2, 2, 2], [2, 2]], [[0, 0], [1, 0], [2, 0]], [ones4] * 3), lb=[-1, 2],
     expect={"status": 0, "dense_shape": [4, 4], "coords": [[0, 0]], "data": [6.0] * 4})
case("bs_matches_dense", "crates/ndtensors/src/contract/blocksparse.rs:391-437", "bs_contract",
     a=bs([[2, 3], [4, 2]], [[0, 0], [1, 1]], [seq(1, 9), seq(1, 7, 2.0)]), la=[1, -1],
     b=bs([[4, 2], [3, 4]], [[0, 1], [1, 0]], [seq(1, 17, 1.0, 10.0), seq(1, 7, 3.0)]), lb=[-1, 2],
     expect={"status": 0, "equals_dense_gemm": True})
case("bs_inner_product", "crates/ndtensors/src/contract/blocksparse.rs:439-466", "bs_contract",
     a=bs([[3, 2]], [[0], [1]], [[1.0, 2.0, 3.0], [4.0, 5.0]]), la=[-1],
     b=bs([[3, 2]], [[0], [1]], [[1.0, 1.0, 1.0], [1.0, 1.0]]), lb=[-1],
     expect={"status": 0, "dense_data": [15.0]})
cA = [[float(x), 0.0] for x in range(1, 5)]
cB = [[0.0, float(x)] for x in range(1, 5)]
case("bs_complex", "crates/ndtensors/src/contract/blocksparse.rs:468-509", "bs_contract",
     a=bs([[2, 2], [2, 2]], [[0, 0], [1, 1]], [cA, cA], dtype="c64"), la=[1, -1],
     b=bs([[2, 2], [2, 2]], [[0, 0], [1, 1]], [cB, cB], dtype="c64"), lb=[-1, 2],
     expect={"status": 0, "equals_dense_gemm": True})
case("bs_dimension_mismatch", "crates/ndtensors/src/contract/blocksparse.rs:511-525", "bs_contract",
     a=bs([[2, 3], [4, 2]], [[0, 0]], [[0.0] * 8]), la=[1, -1],
     b=bs([[3, 3], [2, 2]], [[0, 0]], [[0.0] * 6]), lb=[-1, 2], expect={"status": -2})
case("bs_3d", "crates/ndtensors/src/contract/blocksparse.rs:527-574", "bs_contract",
     a=bs([[2, 2], [3], [2, 2]], [[0, 0, 0], [1, 0, 1]], [[1.0] * 12, [1.0] * 12]), la=[1, 2, -1],
     b=bs([[2, 2], [2, 3]], [[0, 0], [1, 1]], [[1.0] * 4, [1.0] * 6]), lb=[-1, 3],
     expect={"status": 0, "equals_dense_gemm": True})

# ------------------------------------------------- operations/blocksparse.rs
case("bs_permute_transpose", "crates/ndtensors/src/operations/blocksparse.rs:406-445", "bs_permutedims",
     a=bs([[2, 3], [4, 5]], [[0, 0], [1, 1]], [seq(1, 9), seq(10, 25)]), perm=[1, 0],
     expect={"status": 0, "dense_shape": [9, 5], "coords": [[0, 0], [1, 1]], "equals_dense_permute": True})
case("bs_permute_3d", "crates/ndtensors/src/operations/blocksparse.rs:447-478", "bs_permutedims",
     a=bs([[2], [3], [4]], [[0, 0, 0]], [seq(1, 25)]), perm=[2, 0, 1],
     expect={"status": 0, "dense_shape": [4, 2, 3], "equals_dense_permute": True})
for k, perm in enumerate([[0], [0, 1, 2], [0, 2], [0, 0]]):
    case(f"bs_permute_invalid_{k}", "crates/ndtensors/src/operations/blocksparse.rs:480-495", "bs_permutedims",
         a=bs([[2, 3], [4, 5]], [[0, 0]], [[0.0] * 8]), perm=perm, expect={"status": -5})

# ------------------------------------------------------- test_diagblocksparse.rs
case("diag_to_dense", "crates/ndtensors/tests/test_diagblocksparse.rs:113-133", "diag_to_dense",
     s=bs([[2, 2], [2, 2]], [[0, 0], [1, 1]], [[1.0, 2.0], [3.0, 4.0]]),
     expect={"shape": [4, 4], "at": [[[0, 0], 1.0], [[1, 1], 2.0], [[2, 2], 3.0], [[3, 3], 4.0], [[0, 1], 0.0],
                                     [[1, 0], 0.0], [[0, 2], 0.0], [[2, 0], 0.0]]})
case("diag_to_dense_rect_block", "crates/ndtensors/tests/test_diagblocksparse.rs:135-146", "diag_to_dense",
     s=bs([[2], [1, 1]], [[0, 0]], [[1.0]]),
     expect={"shape": [2, 2], "at": [[[0, 0], 1.0], [[0, 1], 0.0], [[1, 0], 0.0], [[1, 1], 0.0]]})
case("diag_complex", "crates/ndtensors/tests/test_diagblocksparse.rs:148-168", "diag_to_dense",
     s=bs([[2, 2], [2, 2]], [[0, 0], [1, 1]], [[[1.0, 2.0], [3.0, 4.0]], [[5.0, 6.0], [7.0, 8.0]]], dtype="c64"),
     expect={"shape": [4, 4], "at": [[[0, 0], [1.0, 2.0]], [[1, 1], [3.0, 4.0]], [[2, 2], [5.0, 6.0]],
                                     [[3, 3], [7.0, 8.0]], [[0, 1], [0.0, 0.0]]]})
case("diag_rectangular_blocks", "crates/ndtensors/tests/test_diagblocksparse.rs:236-264", "diag_to_dense",
     s=bs([[2, 4], [3, 5]], [[0, 0], [1, 1]], [[1.0] * 2, [1.0] * 4]),
     expect={"shape": [6, 8], "nnz": 6, "at": [[[0, 0], 1.0], [[1, 1], 1.0], [[2, 2], 0.0], [[2, 3], 1.0]]})

# ---------------------------------------------------------------- capi tests
case("capi_from_data_get_linear", "crates/ndtensors-capi/src/lib.rs:931-950", "from_data",
     a=t([2, 3], seq(1, 7)), expect={"status": 0, "index": [[0, 1.0], [5, 6.0]]})
case("capi_from_data_len_mismatch", "crates/ndtensors-capi/src/lib.rs:307-340", "from_data",
     a={"shape": [2, 3], "data": [1.0, 2.0], "dtype": "f64"}, expect={"status": -2})
case("capi_ones_scalar", "crates/ndtensors-capi/src/lib.rs:1345-1359", "ones", shape=[],
     expect={"status": 0, "ndim": 0, "len": 1, "index": [[0, 1.0]]})

OUT.write_text(json.dumps({"generated_by": "tests/golden/make_known_answers.py", "cases": cases}, indent=1))
print(f"wrote {len(cases)} cases to {OUT}")
