"""PyTorch autograd integration: ``torch_contract``.

Mirrors the reference binding's ``ndtensors_rs.torch_ops``
(python/ndtensors_rs/src/ndtensors_rs/torch_ops.py:31-160): the same name,
arguments, label semantics (negative labels contracted, positive labels kept,
output axes A's positive labels then B's, a scalar result of shape (1,)), a
float64 result, and a backward pass through ``contract_vjp``.

What differs is where the data goes.  The reference copies every operand to
host numpy and every result back (torch_ops.py:60-76 forward, :96-116
backward).  Here CUDA tensors never leave device memory: operands enter the
library by a device-to-device copy (``TensorF64.from_torch``), the
contraction and its VJP run on the GPU, and results come back to torch by one
device-to-device copy.  CPU tensors are uploaded, contracted on the GPU and
returned as CPU float64 tensors, the devices the reference returns them on.
There is no CPU compute path: without a GPU the library raises.
"""

from __future__ import annotations

from typing import Any, Optional, Sequence, Tuple

import numpy as np

try:
    import torch
    from torch.autograd import Function

    TORCH_AVAILABLE = True
except ImportError:  # pragma: no cover - torch is part of this package's runtime
    TORCH_AVAILABLE = False

from ._lib import get_lib
from .blocksparse import _DeviceSpan
from .ops import contract, contract_vjp
from .tensor import NDTensorsError, TensorF64, check_status


def _check_torch_available() -> None:
    if not TORCH_AVAILABLE:
        raise ImportError("torch_contract requires torch")


def _to_library(x) -> TensorF64:
    """A library tensor holding x's values (float64): device-to-device for a
    CUDA tensor, one host upload for a CPU tensor."""
    x = x.detach()
    if x.is_cuda:
        return TensorF64.from_torch(x)
    return TensorF64.from_numpy(x.numpy().astype(np.float64))


def _to_torch(t: TensorF64, like):
    """t's values as a float64 torch tensor on like's device."""
    if not like.is_cuda:
        return torch.from_numpy(t.to_numpy().copy())
    shape = t.shape
    n = int(np.prod(shape, dtype=np.int64))
    ptr = t.device_ptr()
    # the library's stream has finished writing t before torch reads it
    check_status(get_lib().ndt_b200_synchronize(), "synchronize")
    with torch.cuda.device(like.device):
        span = torch.as_tensor(_DeviceSpan(ptr, max(n, 1)), device=like.device)[:n]
        # column-major storage of `shape` = row-major storage of its reverse;
        # clone always copies (contiguous() would return the library's own
        # buffer for 1-D results, which is freed with t)
        out = span.view(tuple(reversed(shape))).permute(tuple(reversed(range(len(shape))))).clone(
            memory_format=torch.contiguous_format)
        # the copy has read t's buffer before t (and its memory) is released
        torch.cuda.current_stream().synchronize()
    return out


if TORCH_AVAILABLE:

    class _TorchContractFunction(Function):
        """Autograd Function of a two-tensor contraction (forward: contract;
        backward: contract_vjp, both on the GPU)."""

        @staticmethod
        def forward(ctx: Any, a, b, labels_a: Tuple[int, ...], labels_b: Tuple[int, ...]):
            ctx.save_for_backward(a, b)
            ctx.labels_a = tuple(labels_a)
            ctx.labels_b = tuple(labels_b)
            c = contract(_to_library(a), ctx.labels_a, _to_library(b), ctx.labels_b)
            return _to_torch(c, a)

        @staticmethod
        def backward(ctx: Any, grad_output) -> Tuple[Optional[Any], Optional[Any], None, None]:
            a, b = ctx.saved_tensors
            ga, gb = contract_vjp(_to_library(a), ctx.labels_a, _to_library(b), ctx.labels_b,
                                  _to_library(grad_output))
            return _to_torch(ga, a), _to_torch(gb, b), None, None

    def torch_contract(a, labels_a: Sequence[int], b, labels_b: Sequence[int]):
        """Contract two torch tensors by labels, with autograd support.

        Negative labels are contracted (matched between the tensors), positive
        labels are kept; the output axes are a's positive labels then b's, in
        their order (shape (1,) when nothing is kept).  The result is float64
        on a's device.  CUDA tensors stay in device memory throughout (forward
        and backward).

        >>> a = torch.ones((2, 3), requires_grad=True, device="cuda")
        >>> b = torch.ones((3, 4), requires_grad=True, device="cuda")
        >>> c = torch_contract(a, (1, -1), b, (-1, 2))   # shape (2, 4)
        >>> c.sum().backward()                           # a.grad, b.grad on the GPU
        """
        if a.is_cuda != b.is_cuda:
            raise NDTensorsError("torch_contract: operands must both be CUDA tensors or both CPU tensors")
        return _TorchContractFunction.apply(a, b, tuple(labels_a), tuple(labels_b))

else:  # pragma: no cover

    def torch_contract(*args, **kwargs):
        """torch_contract (torch is not installed)."""
        _check_torch_available()


__all__ = ["torch_contract", "TORCH_AVAILABLE"]
