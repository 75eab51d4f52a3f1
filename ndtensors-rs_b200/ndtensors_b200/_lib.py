"""Loading of libndtensors_capi.so and ctypes declarations of its C ABI.

The shared library is built in-tree (``make -C ndtensors-rs_b200``) into
``ndtensors-rs_b200/lib/``.  There is no fallback: if the library is missing
the import fails loudly.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Optional

_lib: Optional[ctypes.CDLL] = None

LIB_NAME = "libndtensors_capi.so"


def lib_path() -> Path:
    env = os.environ.get("NDT_B200_LIB")
    if env:
        return Path(env)
    return Path(__file__).resolve().parent.parent / "lib" / LIB_NAME


c_size_p = ctypes.POINTER(ctypes.c_size_t)
c_int_p = ctypes.POINTER(ctypes.c_int)
c_long_p = ctypes.POINTER(ctypes.c_long)
c_double_p = ctypes.POINTER(ctypes.c_double)
vp = ctypes.c_void_p

# (name, restype, argtypes) for every exported symbol
SIGNATURES = [
    # ---- the reference's 19 f64 symbols (crates/ndtensors-capi/src/lib.rs)
    ("ndt_tensor_f64_zeros", vp, [c_size_p, ctypes.c_size_t, c_int_p]),
    ("ndt_tensor_f64_ones", vp, [c_size_p, ctypes.c_size_t, c_int_p]),
    ("ndt_tensor_f64_rand", vp, [c_size_p, ctypes.c_size_t, c_int_p]),
    ("ndt_tensor_f64_randn", vp, [c_size_p, ctypes.c_size_t, c_int_p]),
    ("ndt_tensor_f64_from_data", vp, [c_double_p, ctypes.c_size_t, c_size_p, ctypes.c_size_t, c_int_p]),
    ("ndt_tensor_f64_release", None, [vp]),
    ("ndt_tensor_f64_clone", vp, [vp]),
    ("ndt_tensor_f64_ndim", ctypes.c_size_t, [vp]),
    ("ndt_tensor_f64_len", ctypes.c_size_t, [vp]),
    ("ndt_tensor_f64_shape", ctypes.c_int, [vp, c_size_p]),
    ("ndt_tensor_f64_data", c_double_p, [vp]),
    ("ndt_tensor_f64_data_mut", c_double_p, [vp]),
    ("ndt_tensor_f64_get_linear", ctypes.c_int, [vp, ctypes.c_size_t, c_double_p]),
    ("ndt_tensor_f64_set_linear", ctypes.c_int, [vp, ctypes.c_size_t, ctypes.c_double]),
    ("ndt_tensor_f64_fill", ctypes.c_int, [vp, ctypes.c_double]),
    ("ndt_tensor_f64_permutedims", vp, [vp, c_size_p, ctypes.c_size_t, c_int_p]),
    ("ndt_tensor_f64_contract", vp, [vp, c_long_p, ctypes.c_size_t, vp, c_long_p, ctypes.c_size_t, c_int_p]),
    (
        "ndt_tensor_f64_contract_vjp",
        None,
        [vp, c_long_p, ctypes.c_size_t, vp, c_long_p, ctypes.c_size_t, vp, ctypes.POINTER(vp), ctypes.POINTER(vp), c_int_p],
    ),
    (
        "ndt_tensor_f64_contract_jvp",
        None,
        [vp, c_long_p, ctypes.c_size_t, vp, c_long_p, ctypes.c_size_t, vp, vp, ctypes.POINTER(vp), ctypes.POINTER(vp), c_int_p],
    ),
    # ---- additive
    ("ndt_tensor_f64_contract_gemm", vp, [vp, c_long_p, ctypes.c_size_t, vp, c_long_p, ctypes.c_size_t, c_int_p]),
    ("ndt_tensor_c64_zeros", vp, [c_size_p, ctypes.c_size_t, c_int_p]),
    ("ndt_tensor_c64_ones", vp, [c_size_p, ctypes.c_size_t, c_int_p]),
    ("ndt_tensor_c64_from_data", vp, [c_double_p, ctypes.c_size_t, c_size_p, ctypes.c_size_t, c_int_p]),
    ("ndt_tensor_c64_release", None, [vp]),
    ("ndt_tensor_c64_clone", vp, [vp]),
    ("ndt_tensor_c64_ndim", ctypes.c_size_t, [vp]),
    ("ndt_tensor_c64_len", ctypes.c_size_t, [vp]),
    ("ndt_tensor_c64_shape", ctypes.c_int, [vp, c_size_p]),
    ("ndt_tensor_c64_data", c_double_p, [vp]),
    ("ndt_tensor_c64_data_mut", c_double_p, [vp]),
    ("ndt_tensor_c64_get_linear", ctypes.c_int, [vp, ctypes.c_size_t, c_double_p, c_double_p]),
    ("ndt_tensor_c64_set_linear", ctypes.c_int, [vp, ctypes.c_size_t, ctypes.c_double, ctypes.c_double]),
    ("ndt_tensor_c64_fill", ctypes.c_int, [vp, ctypes.c_double, ctypes.c_double]),
    ("ndt_tensor_c64_permutedims", vp, [vp, c_size_p, ctypes.c_size_t, c_int_p]),
    ("ndt_tensor_c64_contract", vp, [vp, c_long_p, ctypes.c_size_t, vp, c_long_p, ctypes.c_size_t, c_int_p]),
    ("ndt_tensor_c64_contract_gemm", vp, [vp, c_long_p, ctypes.c_size_t, vp, c_long_p, ctypes.c_size_t, c_int_p]),
    ("ndt_tensor_f64_from_device_ptr", vp, [vp, ctypes.c_size_t, c_size_p, ctypes.c_size_t, c_int_p]),
    ("ndt_tensor_f64_device_ptr", vp, [vp]),
    ("ndt_tensor_f64_device_ptr_mut", vp, [vp]),
    ("ndt_tensor_c64_from_device_ptr", vp, [vp, ctypes.c_size_t, c_size_p, ctypes.c_size_t, c_int_p]),
    ("ndt_tensor_c64_device_ptr", vp, [vp]),
    ("ndt_tensor_c64_device_ptr_mut", vp, [vp]),
    (
        "ndt_b200_permutedims_dev",
        ctypes.c_int,
        [ctypes.c_int, vp, vp, c_size_p, ctypes.c_size_t, c_size_p, ctypes.c_size_t, vp],
    ),
    (
        "ndt_b200_gemm_dev",
        ctypes.c_int,
        [ctypes.c_int, ctypes.c_long, ctypes.c_long, ctypes.c_long, vp, ctypes.c_long, ctypes.c_int, vp,
         ctypes.c_long, ctypes.c_int, vp, ctypes.c_long, ctypes.c_int, vp],
    ),
    *[
        sig
        for dt in ("f64", "c64")
        for sig in [
            (f"ndt_blocksparse_{dt}_zeros", vp, [ctypes.c_size_t, c_size_p, c_size_p, ctypes.c_size_t, c_size_p, c_int_p]),
            (f"ndt_blocksparse_{dt}_from_data", vp,
             [ctypes.c_size_t, c_size_p, c_size_p, ctypes.c_size_t, c_size_p, c_double_p, ctypes.c_size_t, c_int_p]),
            (f"ndt_blocksparse_{dt}_from_device_ptr", vp,
             [ctypes.c_size_t, c_size_p, c_size_p, ctypes.c_size_t, c_size_p, vp, ctypes.c_size_t, c_int_p]),
            (f"ndt_blocksparse_{dt}_release", None, [vp]),
            (f"ndt_blocksparse_{dt}_ndim", ctypes.c_size_t, [vp]),
            (f"ndt_blocksparse_{dt}_nnzblocks", ctypes.c_size_t, [vp]),
            (f"ndt_blocksparse_{dt}_nnz", ctypes.c_size_t, [vp]),
            (f"ndt_blocksparse_{dt}_nblocks_total", ctypes.c_size_t, [vp]),
            (f"ndt_blocksparse_{dt}_structure", ctypes.c_int, [vp, c_size_p, c_size_p, c_size_p, c_size_p]),
            (f"ndt_blocksparse_{dt}_insert_block", ctypes.c_int, [vp, c_size_p, c_double_p, ctypes.c_size_t]),
            (f"ndt_blocksparse_{dt}_get_block", ctypes.c_int, [vp, c_size_p, c_double_p, ctypes.c_size_t]),
            (f"ndt_blocksparse_{dt}_data", c_double_p, [vp]),
            (f"ndt_blocksparse_{dt}_device_ptr", vp, [vp]),
            (f"ndt_blocksparse_{dt}_device_ptr_mut", vp, [vp]),
            (f"ndt_blocksparse_{dt}_shard_layout", ctypes.c_int,
             [vp, c_int_p, c_size_p, c_size_p, c_int_p]),
            (f"ndt_blocksparse_{dt}_from_device_blocks", vp,
             [ctypes.c_size_t, c_size_p, c_size_p, ctypes.c_size_t, c_size_p, c_size_p, vp, ctypes.c_size_t, c_int_p]),
            (f"ndt_blocksparse_{dt}_contract", vp,
             [vp, c_long_p, ctypes.c_size_t, vp, c_long_p, ctypes.c_size_t, c_int_p]),
            (f"ndt_blocksparse_{dt}_contract_shard", vp,
             [vp, c_long_p, ctypes.c_size_t, vp, c_long_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int, c_int_p]),
            (f"ndt_blocksparse_{dt}_contract_select", vp,
             [vp, c_long_p, ctypes.c_size_t, vp, c_long_p, ctypes.c_size_t, c_size_p, ctypes.c_size_t, c_int_p]),
            (f"ndt_blocksparse_{dt}_shard_plan", ctypes.c_int,
             [vp, c_long_p, ctypes.c_size_t, vp, c_long_p, ctypes.c_size_t, ctypes.c_int, c_size_p,
              ctypes.POINTER(ctypes.c_double)]),
            (f"ndt_blocksparse_{dt}_permutedims", vp, [vp, c_size_p, ctypes.c_size_t, c_int_p]),
            (f"ndt_blocksparse_{dt}_to_dense", vp, [vp, c_int_p]),
            (f"ndt_blocksparse_{dt}_from_dense", vp,
             [vp, ctypes.c_size_t, c_size_p, c_size_p, ctypes.c_size_t, c_size_p, c_int_p]),
            (f"ndt_diagblocksparse_{dt}_from_data", vp,
             [ctypes.c_size_t, c_size_p, c_size_p, ctypes.c_size_t, c_size_p, c_double_p, ctypes.c_size_t, c_int_p]),
            (f"ndt_diagblocksparse_{dt}_release", None, [vp]),
            (f"ndt_diagblocksparse_{dt}_nnz", ctypes.c_size_t, [vp]),
            (f"ndt_diagblocksparse_{dt}_to_dense", vp, [vp, c_int_p]),
            (f"ndt_diagblocksparse_{dt}_to_blocksparse", vp, [vp, c_int_p]),
            (f"ndt_blocksparse_{dt}_contract_diag", vp,
             [vp, c_long_p, ctypes.c_size_t, vp, c_long_p, ctypes.c_size_t, c_int_p]),
            (f"ndt_blocksparse_{dt}_contract_through_diag", vp,
             [vp, c_long_p, ctypes.c_size_t, vp, c_long_p, ctypes.c_size_t, vp, c_long_p, ctypes.c_size_t,
              ctypes.c_int, ctypes.c_int, c_int_p]),
            (f"ndt_blocksparse_{dt}_contract_gathered", vp,
             [vp, c_long_p, ctypes.c_size_t, vp, c_long_p, ctypes.c_size_t, vp, c_int_p]),
            (f"ndt_blocksparse_{dt}_contract_through_diag_gathered", vp,
             [vp, c_long_p, ctypes.c_size_t, vp, c_long_p, ctypes.c_size_t, vp, c_long_p, ctypes.c_size_t, vp,
              c_int_p]),
            (f"ndt_blocksparse_{dt}_allgather", vp, [vp, vp, c_int_p]),
        ]
    ],
    *[(f"ndt_tensor_{dt}_contract_gemm_shard", vp,
       [vp, c_long_p, ctypes.c_size_t, vp, c_long_p, ctypes.c_size_t, ctypes.c_long, ctypes.c_int, ctypes.c_int,
        c_int_p]) for dt in ("f64", "c64")],
    ("ndt_b200_comm_unique_id", ctypes.c_int, [ctypes.c_char_p]),
    ("ndt_b200_comm_init", vp, [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, c_int_p]),
    ("ndt_b200_comm_from_nccl", vp, [vp, c_int_p]),
    ("ndt_b200_comm_rank", ctypes.c_int, [vp]),
    ("ndt_b200_comm_size", ctypes.c_int, [vp]),
    ("ndt_b200_comm_release", None, [vp]),
    (
        "ndt_b200_contract_f64_noalloc",
        ctypes.c_int,
        [vp, c_size_p, ctypes.c_size_t, c_long_p, vp, c_size_p, ctypes.c_size_t, c_long_p, vp, ctypes.c_size_t,
         c_size_p, c_size_p, vp],
    ),
    ("ndt_b200_device_available", ctypes.c_int, []),
    ("ndt_b200_set_stream", ctypes.c_int, [vp]),
    ("ndt_b200_get_stream", vp, []),
    ("ndt_b200_synchronize", ctypes.c_int, []),
    ("ndt_b200_last_error", ctypes.c_char_p, []),
    ("ndt_b200_launch_count", ctypes.c_ulonglong, []),
    ("ndt_b200_empty_cache", None, []),
]


def _declare(lib: ctypes.CDLL) -> None:
    for name, res, args in SIGNATURES:
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args


def get_lib() -> ctypes.CDLL:
    """Load (once) and return the library; raises if it has not been built."""
    global _lib
    if _lib is None:
        p = lib_path()
        if not p.exists():
            raise FileNotFoundError(
                f"{p} not found: build it with `make -C ndtensors-rs_b200` (nvcc, sm_100a)"
            )
        lib = ctypes.CDLL(str(p))
        _declare(lib)
        _lib = lib
    return _lib


def last_error() -> str:
    msg = get_lib().ndt_b200_last_error()
    return msg.decode() if msg else ""
