"""Dense tensor handles over the C ABI.

``TensorF64`` keeps the method names, argument meaning and exceptions of the
reference's Python binding (python/ndtensors_rs/src/ndtensors_rs/tensor.py),
so code written against it runs unchanged; ``TensorC64`` is the complex128
counterpart.  Data is column-major; ``from_numpy`` converts to Fortran order.
Extra: ``from_torch`` / ``to_torch`` move CUDA tensors in and out without a
host round trip.
"""

from __future__ import annotations

import ctypes
from enum import IntEnum
from typing import Sequence, Tuple

import numpy as np

from ._lib import c_double_p, c_size_p, get_lib, last_error


class StatusCode(IntEnum):
    """Status codes of the C ABI (crates/ndtensors-capi/src/lib.rs:17-25)."""

    SUCCESS = 0
    INVALID_ARGUMENT = -1
    SHAPE_MISMATCH = -2
    INDEX_OUT_OF_BOUNDS = -3
    INTERNAL_ERROR = -4
    INVALID_PERMUTATION = -5


class NDTensorsError(Exception):
    """Raised for a non-success status (python/.../_status.py)."""


def check_status(status: int, context: str = "") -> None:
    if status != StatusCode.SUCCESS:
        name = StatusCode(status).name if status in StatusCode._value2member_map_ else str(status)
        detail = last_error()
        msg = f"{context}: {name}" if context else name
        if detail:
            msg += f" ({detail})"
        raise NDTensorsError(msg)


def _shape_arr(shape: Sequence[int]):
    n = len(shape)
    return (ctypes.c_size_t * n)(*shape) if n else None


class _DenseBase:
    __slots__ = ("_ptr", "_lib", "_shape")
    _prefix = ""
    _np_dtype = np.float64
    _width = 1  # doubles per element

    def __init__(self, ptr: int) -> None:
        self._lib = get_lib()
        self._ptr = ptr
        self._shape = None  # a handle's shape never changes: cached on first query

    def __del__(self) -> None:
        if getattr(self, "_ptr", None):
            getattr(self._lib, f"ndt_tensor_{self._prefix}_release")(self._ptr)
            self._ptr = None

    def _f(self, name):
        return getattr(self._lib, f"ndt_tensor_{self._prefix}_{name}")

    @classmethod
    def _create(cls, fname: str, shape: Sequence[int]):
        lib = get_lib()
        status = ctypes.c_int(-999)
        ptr = getattr(lib, f"ndt_tensor_{cls._prefix}_{fname}")(_shape_arr(shape), len(shape), ctypes.byref(status))
        check_status(status.value, fname)
        return cls(ptr)

    @classmethod
    def zeros(cls, shape: Tuple[int, ...]):
        return cls._create("zeros", tuple(shape))

    @classmethod
    def ones(cls, shape: Tuple[int, ...]):
        return cls._create("ones", tuple(shape))

    @classmethod
    def from_numpy(cls, arr: np.ndarray):
        arr = np.asarray(arr, dtype=cls._np_dtype)
        shape = arr.shape  # before asfortranarray, which turns 0-d into shape (1,)
        flat = np.asfortranarray(arr).ravel(order="F")
        if flat.size == 0:
            flat = np.zeros(1, dtype=cls._np_dtype)  # storage holds max(1, prod) elements
        buf = np.ascontiguousarray(flat).view(np.float64)
        status = ctypes.c_int(-999)
        ptr = getattr(get_lib(), f"ndt_tensor_{cls._prefix}_from_data")(
            buf.ctypes.data_as(c_double_p), flat.size, _shape_arr(shape), len(shape), ctypes.byref(status)
        )
        check_status(status.value, "from_numpy")
        return cls(ptr)

    @classmethod
    def from_torch(cls, t):
        """Copy a CUDA torch tensor (device to device; column-major order of
        the tensor's logical shape, i.e. ``t.permute(reversed).contiguous()``)."""
        import torch

        if not t.is_cuda:
            return cls.from_numpy(t.detach().numpy())
        want = torch.complex128 if cls._width == 2 else torch.float64
        tt = t.to(want).permute(tuple(reversed(range(t.dim())))).contiguous()
        shape = tuple(t.shape)
        n = max(1, tt.numel())
        if tt.numel() == 0:
            tt = torch.zeros(1, dtype=want, device=t.device)  # storage holds max(1, prod) elements
        # torch wrote tt on its own stream; the library copies it on another
        torch.cuda.current_stream(tt.device).synchronize()
        status = ctypes.c_int(-999)
        ptr = getattr(get_lib(), f"ndt_tensor_{cls._prefix}_from_device_ptr")(
            ctypes.c_void_p(tt.data_ptr()), n, _shape_arr(shape), len(shape), ctypes.byref(status)
        )
        check_status(status.value, "from_torch")
        get_lib().ndt_b200_synchronize()
        return cls(ptr)

    def device_ptr(self) -> int:
        p = self._f("device_ptr")(self._ptr)
        if not p:
            raise NDTensorsError(f"device_ptr: {last_error()}")
        return p

    def device_ptr_mut(self) -> int:
        """Device buffer for writing from outside the library (torch, another
        kernel): copy on write if the storage is shared; the device copy
        then holds the tensor's values."""
        p = self._f("device_ptr_mut")(self._ptr)
        if not p:
            raise NDTensorsError(f"device_ptr_mut: {last_error()}")
        return p

    @property
    def ndim(self) -> int:
        if self._shape is not None:
            return len(self._shape)
        return int(self._f("ndim")(self._ptr))

    @property
    def shape(self) -> Tuple[int, ...]:
        if self._shape is None:
            n = self.ndim
            out = (ctypes.c_size_t * max(n, 1))()
            st = self._f("shape")(self._ptr, out)
            check_status(st, "shape")
            self._shape = tuple(int(out[i]) for i in range(n))
        return self._shape

    def __len__(self) -> int:
        return int(self._f("len")(self._ptr))

    def _host_view(self) -> np.ndarray:
        n = len(self) * self._width
        p = self._f("data")(self._ptr)
        if not p:
            raise NDTensorsError(f"data: {last_error()}")
        return np.ctypeslib.as_array(p, shape=(n,))

    def to_numpy(self) -> np.ndarray:
        flat = self._host_view().copy()
        if self._width == 2:
            flat = flat.view(np.complex128)
        shape = self.shape
        if int(np.prod(shape, dtype=np.int64)) != flat.size:
            return flat[: int(np.prod(shape, dtype=np.int64))].reshape(shape, order="F")
        return flat.reshape(shape, order="F")

    def fill(self, value):
        if self._width == 2:
            v = complex(value)
            st = self._f("fill")(self._ptr, v.real, v.imag)
        else:
            st = self._f("fill")(self._ptr, float(value))
        check_status(st, "fill")
        return self

    def copy(self):
        p = self._f("clone")(self._ptr)
        if not p:
            raise NDTensorsError("Failed to clone tensor")
        return type(self)(p)

    def permutedims(self, perm: Sequence[int]):
        n = len(perm)
        arr = (ctypes.c_size_t * max(n, 1))(*perm)
        status = ctypes.c_int(-999)
        ptr = self._f("permutedims")(self._ptr, arr, n, ctypes.byref(status))
        if status.value == StatusCode.INVALID_PERMUTATION:
            raise ValueError(f"Invalid permutation: {perm}")
        check_status(status.value, "permutedims")
        return type(self)(ptr)

    def __repr__(self) -> str:
        return f"{type(self).__name__}(shape={self.shape})"


class TensorF64(_DenseBase):
    """Dense float64 tensor; interface of the reference's ``TensorF64``."""

    __slots__ = ()
    _prefix = "f64"
    _np_dtype = np.float64
    _width = 1

    @classmethod
    def rand(cls, shape: Tuple[int, ...]):
        return cls._create("rand", tuple(shape))

    @classmethod
    def randn(cls, shape: Tuple[int, ...]):
        return cls._create("randn", tuple(shape))

    def __getitem__(self, idx: int) -> float:
        out = ctypes.c_double()
        st = self._f("get_linear")(self._ptr, idx, ctypes.byref(out))
        if st == StatusCode.INDEX_OUT_OF_BOUNDS:
            raise IndexError(f"index {idx} out of bounds for tensor of length {len(self)}")
        check_status(st, "getitem")
        return out.value

    def __setitem__(self, idx: int, value: float) -> None:
        st = self._f("set_linear")(self._ptr, idx, float(value))
        if st == StatusCode.INDEX_OUT_OF_BOUNDS:
            raise IndexError(f"index {idx} out of bounds for tensor of length {len(self)}")
        check_status(st, "setitem")


class TensorC64(_DenseBase):
    """Dense complex128 tensor (additive to the reference's ABI)."""

    __slots__ = ()
    _prefix = "c64"
    _np_dtype = np.complex128
    _width = 2

    def __getitem__(self, idx: int) -> complex:
        re, im = ctypes.c_double(), ctypes.c_double()
        st = self._f("get_linear")(self._ptr, idx, ctypes.byref(re), ctypes.byref(im))
        if st == StatusCode.INDEX_OUT_OF_BOUNDS:
            raise IndexError(f"index {idx} out of bounds for tensor of length {len(self)}")
        check_status(st, "getitem")
        return complex(re.value, im.value)

    def __setitem__(self, idx: int, value: complex) -> None:
        v = complex(value)
        st = self._f("set_linear")(self._ptr, idx, v.real, v.imag)
        if st == StatusCode.INDEX_OUT_OF_BOUNDS:
            raise IndexError(f"index {idx} out of bounds for tensor of length {len(self)}")
        check_status(st, "setitem")
