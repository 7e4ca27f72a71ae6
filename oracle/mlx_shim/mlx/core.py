"""Torch-CPU stand-in for the subset of ``mlx.core`` that the RFSN reference uses.

TEST INFRASTRUCTURE ONLY.  This package exists so that the reference's own
``quantization.py``, ``attention.py``, ``cache.py`` and ``storage.py`` can be
imported and executed unmodified on a machine without Apple MLX, in order to
generate golden fixtures that pin ``oracle/restate.py``.  Nothing in the
product (``apple_b200``) imports it.

The surface implemented is exactly what ``grep mx\\.`` finds in those files:
``array``, dtypes, ``zeros/zeros_like/ones_like/full/arange``, reductions,
elementwise math, ``take/argmin/where/concatenate/swapaxes/transpose/
broadcast_to``, ``random.normal/randint/seed``, ``eval`` and
``default_device``.  ``quantize``/``dequantize`` are deliberately absent, so
``hasattr(mx, "quantize")`` is False and the reference's optional affine
codebook path (quantization.py:41-42) is disabled.

Numerics: every op runs in torch on the CPU in the array's dtype; float16
arithmetic therefore rounds like MLX's float16 (IEEE binary16, round to
nearest even).  Reduction and matmul summation orders are torch's, not MLX's.
"""
from __future__ import annotations

import numpy as _np
import torch as _torch


class Dtype:
    def __init__(self, name: str, torch_dtype: _torch.dtype, np_dtype):
        self.name = name
        self.torch = torch_dtype
        self.np = _np.dtype(np_dtype)

    def __repr__(self) -> str:
        return f"mlx.core.{self.name}"

    def __eq__(self, other) -> bool:
        return isinstance(other, Dtype) and other.name == self.name

    def __hash__(self) -> int:
        return hash(self.name)


# uint16 has poor operator coverage in torch, so it is stored as int32 and only
# its logical dtype (for np.asarray / astype round trips) is uint16.
float16 = Dtype("float16", _torch.float16, _np.float16)
float32 = Dtype("float32", _torch.float32, _np.float32)
int32 = Dtype("int32", _torch.int32, _np.int32)
int64 = Dtype("int64", _torch.int64, _np.int64)
uint8 = Dtype("uint8", _torch.uint8, _np.uint8)
uint16 = Dtype("uint16", _torch.int32, _np.uint16)
uint32 = Dtype("uint32", _torch.int64, _np.uint32)
bool_ = Dtype("bool", _torch.bool, _np.bool_)

_BY_TORCH = {
    _torch.float16: float16,
    _torch.float32: float32,
    _torch.int32: int32,
    _torch.int64: int64,
    _torch.uint8: uint8,
    _torch.bool: bool_,
}
_BY_NP = {
    _np.dtype(_np.float16): float16,
    _np.dtype(_np.float32): float32,
    _np.dtype(_np.float64): float32,
    _np.dtype(_np.int32): int32,
    _np.dtype(_np.int64): int32,
    _np.dtype(_np.uint8): uint8,
    _np.dtype(_np.uint16): uint16,
    _np.dtype(_np.uint32): uint32,
    _np.dtype(_np.bool_): bool_,
}


def _wrap(t: _torch.Tensor, dtype: Dtype | None = None) -> "array":
    out = array.__new__(array)
    out._t = t
    out._dtype = dtype if dtype is not None else _BY_TORCH[t.dtype]
    return out


def _unwrap(x):
    if isinstance(x, array):
        return x._t
    return x


def _to_tensor(value, dtype: Dtype | None):
    if isinstance(value, array):
        t = value._t
        if dtype is not None and dtype.torch != t.dtype:
            t = t.to(dtype.torch)
        return t, dtype or value._dtype
    if isinstance(value, _torch.Tensor):
        t = value
        if dtype is not None:
            t = t.to(dtype.torch)
        return t, dtype or _BY_TORCH[t.dtype]
    if isinstance(value, _np.ndarray):
        np_dtype = value.dtype
        logical = dtype or _BY_NP[_np.dtype(np_dtype)]
        arr = _np.ascontiguousarray(value)
        if arr.dtype == _np.uint16 or arr.dtype == _np.uint32 or arr.dtype == _np.float64:
            arr = arr.astype(logical.np if logical.np != _np.uint16 else _np.int32)
            if logical == uint32:
                arr = arr.astype(_np.int64)
        t = _torch.from_numpy(arr.copy())
        if t.dtype != logical.torch:
            t = t.to(logical.torch)
        return t, logical
    # python scalars / nested lists
    arr = _np.asarray(value)
    if dtype is None:
        if arr.dtype == _np.float64:
            dtype = float32
        elif arr.dtype == _np.int64:
            dtype = int32
        else:
            dtype = _BY_NP[_np.dtype(arr.dtype)]
    return _torch.as_tensor(arr).to(dtype.torch), dtype


def _result_dtype(t: _torch.Tensor, *operands) -> Dtype:
    # Keep the uint16 logical tag when the computation stayed in int32 storage.
    for op in operands:
        if isinstance(op, array) and op._dtype == uint16 and t.dtype == _torch.int32:
            return uint16
    return _BY_TORCH[t.dtype]


class array:
    def __init__(self, value, dtype: Dtype | None = None):
        self._t, self._dtype = _to_tensor(value, dtype)

    # --- properties -----------------------------------------------------
    @property
    def shape(self):
        return tuple(int(d) for d in self._t.shape)

    @property
    def dtype(self) -> Dtype:
        return self._dtype

    @property
    def size(self) -> int:
        return int(self._t.numel())

    @property
    def ndim(self) -> int:
        return self._t.dim()

    @property
    def T(self) -> "array":
        return _wrap(self._t.permute(*reversed(range(self._t.dim()))), self._dtype)

    # --- conversions ----------------------------------------------------
    def astype(self, dtype: Dtype) -> "array":
        return _wrap(self._t.to(dtype.torch), dtype)

    def reshape(self, *shape) -> "array":
        if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
            shape = tuple(shape[0])
        return _wrap(self._t.reshape(*shape), self._dtype)

    def __array__(self, dtype=None, copy=None):
        out = self._t.detach().cpu().numpy()
        if self._dtype == uint16:
            out = out.astype(_np.uint16)
        elif self._dtype == uint32:
            out = out.astype(_np.uint32)
        if dtype is not None:
            out = out.astype(dtype)
        return out

    def item(self):
        return self._t.item()

    def tolist(self):
        return _np.asarray(self).tolist()

    def __float__(self) -> float:
        return float(self._t.item())

    def __int__(self) -> int:
        return int(self._t.item())

    def __bool__(self) -> bool:
        return bool(self._t.item())

    def __len__(self) -> int:
        return int(self._t.shape[0])

    def __repr__(self) -> str:
        return f"array({_np.asarray(self)!r}, dtype={self._dtype.name})"

    # --- indexing -------------------------------------------------------
    @staticmethod
    def _index(key):
        if isinstance(key, tuple):
            return tuple(_unwrap(k) if not isinstance(k, array) else k._t.long() if k._t.dtype != _torch.bool else k._t for k in key)
        if isinstance(key, array):
            return key._t.long() if key._t.dtype != _torch.bool else key._t
        return key

    def __getitem__(self, key) -> "array":
        return _wrap(self._t[self._index(key)], self._dtype)

    def __setitem__(self, key, value) -> None:
        v = _unwrap(value)
        if isinstance(v, _torch.Tensor):
            v = v.to(self._t.dtype)
        self._t[self._index(key)] = v

    # --- arithmetic -----------------------------------------------------
    def _binary(self, other, fn, reverse=False):
        o = _unwrap(other)
        a, b = (o, self._t) if reverse else (self._t, o)
        t = fn(a, b) if isinstance(a, _torch.Tensor) else fn(_torch.as_tensor(a), b) if reverse else fn(a, b)
        return _wrap(t, _result_dtype(t, self, other))

    def __add__(self, o):
        return self._binary(o, _torch.add)

    def __radd__(self, o):
        return self._binary(o, _torch.add, True)

    def __sub__(self, o):
        return self._binary(o, _torch.sub)

    def __rsub__(self, o):
        return _wrap(o - self._t) if not isinstance(o, array) else o.__sub__(self)

    def __mul__(self, o):
        return self._binary(o, _torch.mul)

    def __rmul__(self, o):
        return self._binary(o, _torch.mul, True)

    def __truediv__(self, o):
        return self._binary(o, _torch.div)

    def __rtruediv__(self, o):
        return _wrap(o / self._t)

    def __pow__(self, o):
        return _wrap(self._t ** _unwrap(o), self._dtype)

    def __neg__(self):
        return _wrap(-self._t, self._dtype)

    def __matmul__(self, o):
        return _wrap(self._t @ _unwrap(o))

    def __lt__(self, o):
        return _wrap(self._t < _unwrap(o))

    def __le__(self, o):
        return _wrap(self._t <= _unwrap(o))

    def __gt__(self, o):
        return _wrap(self._t > _unwrap(o))

    def __ge__(self, o):
        return _wrap(self._t >= _unwrap(o))

    def __eq__(self, o):  # type: ignore[override]
        return _wrap(self._t == _unwrap(o))

    def __ne__(self, o):  # type: ignore[override]
        return _wrap(self._t != _unwrap(o))

    def __and__(self, o):
        return _wrap(self._t & _unwrap(o))

    def __or__(self, o):
        return _wrap(self._t | _unwrap(o))

    def __invert__(self):
        return _wrap(~self._t)

    __hash__ = object.__hash__


# --- constructors -----------------------------------------------------------

def _shape(shape):
    if isinstance(shape, int):
        return (shape,)
    return tuple(int(s) for s in shape)


def zeros(shape, dtype: Dtype = float32) -> array:
    return _wrap(_torch.zeros(_shape(shape), dtype=dtype.torch), dtype)


def ones(shape, dtype: Dtype = float32) -> array:
    return _wrap(_torch.ones(_shape(shape), dtype=dtype.torch), dtype)


def zeros_like(x: array) -> array:
    return _wrap(_torch.zeros_like(x._t), x._dtype)


def ones_like(x: array) -> array:
    return _wrap(_torch.ones_like(x._t), x._dtype)


def full(shape, value, dtype: Dtype | None = None) -> array:
    if dtype is None:
        dtype = float32 if isinstance(value, float) else int32
    return _wrap(_torch.full(_shape(shape), _unwrap(value), dtype=dtype.torch), dtype)


def arange(start, stop=None, step=1, dtype: Dtype = int32) -> array:
    if stop is None:
        start, stop = 0, start
    return _wrap(_torch.arange(start, stop, step, dtype=dtype.torch), dtype)


# --- reductions -------------------------------------------------------------

def _axis_kw(axis, keepdims):
    return {} if axis is None else {"dim": axis, "keepdim": keepdims}


def sum(x: array, axis=None, keepdims: bool = False) -> array:  # noqa: A001
    t = x._t.sum(**_axis_kw(axis, keepdims)) if axis is not None else x._t.sum()
    return _wrap(t.to(x._t.dtype) if x._t.is_floating_point() else t)


def mean(x: array, axis=None, keepdims: bool = False) -> array:
    t = x._t.float() if not x._t.is_floating_point() else x._t
    return _wrap(t.mean(**_axis_kw(axis, keepdims)) if axis is not None else t.mean())


def max(x: array, axis=None, keepdims: bool = False) -> array:  # noqa: A001
    if axis is None:
        return _wrap(x._t.max(), x._dtype)
    return _wrap(x._t.amax(dim=axis, keepdim=keepdims), x._dtype)


def min(x: array, axis=None, keepdims: bool = False) -> array:  # noqa: A001
    if axis is None:
        return _wrap(x._t.min(), x._dtype)
    return _wrap(x._t.amin(dim=axis, keepdim=keepdims), x._dtype)


def argmin(x: array, axis=None) -> array:
    # torch.argmin returns the first minimal index, like MLX and numpy.
    return _wrap(_torch.argmin(x._t, dim=axis).to(_torch.int32), uint32 if False else int32)


# --- elementwise ------------------------------------------------------------

def maximum(a, b) -> array:
    ta, tb = _unwrap(a), _unwrap(b)
    if not isinstance(ta, _torch.Tensor):
        ta = _torch.as_tensor(ta, dtype=tb.dtype)
    if not isinstance(tb, _torch.Tensor):
        tb = _torch.as_tensor(tb, dtype=ta.dtype)
    return _wrap(_torch.maximum(ta, tb))


def abs(x: array) -> array:  # noqa: A001
    return _wrap(x._t.abs(), x._dtype)


def sqrt(x: array) -> array:
    return _wrap(x._t.sqrt(), x._dtype)


def exp(x: array) -> array:
    return _wrap(x._t.exp(), x._dtype)


def tanh(x: array) -> array:
    return _wrap(x._t.tanh(), x._dtype)


def sigmoid(x: array) -> array:
    return _wrap(x._t.sigmoid(), x._dtype)


def softmax(x: array, axis=-1) -> array:
    return _wrap(_torch.softmax(x._t, dim=axis), x._dtype)


def matmul(a: array, b: array) -> array:
    """mx.matmul (used by the reference's Llama adapter, llama32_adapter.py:493)."""
    return _wrap(_unwrap(a) @ _unwrap(b))


def where(cond, a, b) -> array:
    tc = _unwrap(cond)
    ta, tb = _unwrap(a), _unwrap(b)
    if not isinstance(ta, _torch.Tensor):
        ta = _torch.as_tensor(ta, dtype=tb.dtype)
    if not isinstance(tb, _torch.Tensor):
        tb = _torch.as_tensor(tb, dtype=ta.dtype)
    t = _torch.where(tc, ta, tb)
    return _wrap(t, _result_dtype(t, a, b))


def take(x: array, indices, axis=None) -> array:
    idx = _unwrap(indices)
    if not isinstance(idx, _torch.Tensor):
        idx = _torch.as_tensor(idx)
    idx = idx.long()
    if axis is None:
        return _wrap(x._t.reshape(-1)[idx], x._dtype)
    return _wrap(_torch.index_select(x._t, axis, idx.reshape(-1)).reshape(
        *x._t.shape[:axis], *idx.shape, *x._t.shape[axis + 1:]), x._dtype)


def concatenate(arrays, axis: int = 0) -> array:
    dtype = arrays[0]._dtype
    return _wrap(_torch.cat([a._t for a in arrays], dim=axis), dtype)


def swapaxes(x: array, a: int, b: int) -> array:
    return _wrap(x._t.transpose(a, b), x._dtype)


def transpose(x: array, axes=None) -> array:
    if axes is None:
        axes = tuple(reversed(range(x._t.dim())))
    return _wrap(x._t.permute(*axes), x._dtype)


def broadcast_to(x: array, shape) -> array:
    return _wrap(x._t.broadcast_to(_shape(shape)), x._dtype)


def eval(*args) -> None:  # noqa: A001
    return None


def default_device() -> str:
    return "cpu(torch-shim)"


class _Random:
    def __init__(self):
        self.gen = _torch.Generator().manual_seed(0)

    def seed(self, value: int) -> None:
        self.gen.manual_seed(int(value))

    def normal(self, shape=(), dtype: Dtype = float32, loc: float = 0.0, scale: float = 1.0) -> array:
        t = _torch.randn(_shape(shape), generator=self.gen, dtype=_torch.float32) * scale + loc
        return _wrap(t.to(dtype.torch), dtype)

    def randint(self, low, high, shape=(), dtype: Dtype = int32) -> array:
        t = _torch.randint(int(low), int(high), _shape(shape), generator=self.gen)
        return _wrap(t.to(dtype.torch), dtype)


random = _Random()
