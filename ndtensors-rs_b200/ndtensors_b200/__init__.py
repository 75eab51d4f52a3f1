"""B200 implementation of ndtensors' contraction hot path (Python host side).

The compute lives in libndtensors_capi.so (C++ / CUDA for sm_100a); this
package binds its C ABI with ctypes and mirrors the reference's Python API
(TensorF64, contract, contract_vjp, contract_jvp) plus complex128,
block-sparse tensors and whole-network contraction (contract_network).
"""

from . import blocksparse
from ._lib import get_lib, last_error, lib_path
from .network import contract_network
from .ops import contract, contract_gemm, contract_gemm_shard, contract_jvp, contract_vjp
from .tensor import NDTensorsError, StatusCode, TensorC64, TensorF64, check_status


def device_available() -> bool:
    return bool(get_lib().ndt_b200_device_available())


def synchronize() -> None:
    check_status(get_lib().ndt_b200_synchronize(), "synchronize")


def launch_count() -> int:
    """Kernels launched by the library since it was loaded."""
    return int(get_lib().ndt_b200_launch_count())


def set_stream(stream_ptr) -> None:
    """Run the library's kernels on a caller CUDA stream (e.g.
    ``torch.cuda.current_stream().cuda_stream``); ``None`` restores its own."""
    import ctypes

    check_status(get_lib().ndt_b200_set_stream(ctypes.c_void_p(stream_ptr) if stream_ptr else None), "set_stream")


def __getattr__(name: str):
    """``torch_contract`` loads on first use, as in the reference binding
    (python/ndtensors_rs/src/ndtensors_rs/__init__.py)."""
    if name == "torch_contract":
        from .torch_ops import torch_contract

        return torch_contract
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")


__all__ = [
    "TensorF64",
    "TensorC64",
    "contract",
    "contract_gemm",
    "contract_gemm_shard",
    "contract_vjp",
    "contract_jvp",
    "contract_network",
    "NDTensorsError",
    "StatusCode",
    "check_status",
    "get_lib",
    "lib_path",
    "last_error",
    "device_available",
    "synchronize",
    "launch_count",
    "set_stream",
]
