"""``mlx.core`` subset over torch CPU tensors (test infrastructure only).

Semantics follow MLX's documented behaviour for the calls the reference makes:
lazy evaluation is replaced by eager torch ops, python scalars do not promote an
array's float dtype, ``arange`` over ints yields int32, ``repeat`` repeats each
element along the axis, and ``fast.scaled_dot_product_attention`` is the plain
definition softmax(q k^T * scale + mask) v computed in float32.
"""

from __future__ import annotations

import builtins
import math
import types
from typing import Any, Iterable, Sequence

import numpy as np
import torch


class Dtype:
    def __init__(self, name: str, torch_dtype: torch.dtype, np_dtype: Any) -> None:
        self.name = name
        self.torch_dtype = torch_dtype
        self.np_dtype = np_dtype

    def __repr__(self) -> str:  # pragma: no cover - debugging aid
        return f"mlx.core.{self.name}"

    @property
    def size(self) -> int:
        return torch.empty((), dtype=self.torch_dtype).element_size()


float16 = Dtype("float16", torch.float16, np.float16)
bfloat16 = Dtype("bfloat16", torch.bfloat16, None)
float32 = Dtype("float32", torch.float32, np.float32)
int32 = Dtype("int32", torch.int32, np.int32)
int64 = Dtype("int64", torch.int64, np.int64)
uint32 = Dtype("uint32", torch.int64, np.uint32)
bool_ = Dtype("bool", torch.bool, np.bool_)

_BY_TORCH = {d.torch_dtype: d for d in (float16, bfloat16, float32, int32, int64, bool_)}


def _dt(torch_dtype: torch.dtype) -> Dtype:
    return _BY_TORCH[torch_dtype]


def _raw(x: Any) -> Any:
    if isinstance(x, array):
        return x._t
    return x


def _wrap(t: Any) -> "array":
    if isinstance(t, torch.Tensor):
        if t.dtype == torch.float64:
            t = t.to(torch.float32)
        return array(t)
    return array(torch.as_tensor(t))


def _to_tensor(x: Any, dtype: Dtype | None = None) -> torch.Tensor:
    if isinstance(x, array):
        t = x._t
    elif isinstance(x, torch.Tensor):
        t = x
    elif isinstance(x, np.ndarray):
        if x.dtype == np.float64:
            t = torch.from_numpy(x.astype(np.float32))
        elif x.dtype == np.int64:
            t = torch.from_numpy(x.astype(np.int32))
        else:
            t = torch.from_numpy(np.ascontiguousarray(x))
    else:
        if isinstance(x, bool):
            t = torch.tensor(x, dtype=torch.bool)
        elif isinstance(x, int):
            t = torch.tensor(x, dtype=torch.int32)
        elif isinstance(x, float):
            t = torch.tensor(x, dtype=torch.float32)
        else:
            arr = np.asarray(x)
            if arr.dtype == np.float64:
                arr = arr.astype(np.float32)
            elif arr.dtype == np.int64:
                arr = arr.astype(np.int32)
            t = torch.from_numpy(arr)
    if dtype is not None:
        t = t.to(dtype.torch_dtype)
    return t


def _index(key: Any) -> Any:
    if isinstance(key, tuple):
        return tuple(_index(k) for k in key)
    if isinstance(key, array):
        t = key._t
        return t.long() if t.dtype != torch.bool else t
    return key


class array:
    """Eager array wrapping a torch CPU tensor."""

    __array_priority__ = 100

    def __init__(self, value: Any, dtype: Dtype | None = None) -> None:
        self._t = _to_tensor(value, dtype)

    # --- metadata ---------------------------------------------------------
    @property
    def shape(self) -> tuple[int, ...]:
        return tuple(int(s) for s in self._t.shape)

    @property
    def dtype(self) -> Dtype:
        return _dt(self._t.dtype)

    @property
    def ndim(self) -> int:
        return self._t.dim()

    @property
    def size(self) -> int:
        return int(self._t.numel())

    @property
    def nbytes(self) -> int:
        return int(self._t.numel() * self._t.element_size())

    @property
    def T(self) -> "array":
        return array(self._t.permute(*reversed(range(self._t.dim()))))

    # --- conversion -------------------------------------------------------
    def astype(self, dtype: Dtype) -> "array":
        return array(self._t.to(dtype.torch_dtype))

    def item(self) -> Any:
        return self._t.item()

    def tolist(self) -> Any:
        return self._t.tolist()

    def __array__(self, dtype: Any = None, copy: Any = None) -> np.ndarray:
        t = self._t
        if t.dtype == torch.bfloat16:
            t = t.to(torch.float32)
        out = t.detach().contiguous().numpy()
        if dtype is not None:
            out = out.astype(dtype)
        return out

    def __len__(self) -> int:
        return int(self._t.shape[0])

    def __iter__(self):
        for i in range(len(self)):
            yield array(self._t[i])

    def __repr__(self) -> str:  # pragma: no cover - debugging aid
        return f"array({self._t!r})"

    def __bool__(self) -> bool:
        return bool(self._t)

    def __int__(self) -> int:
        return int(self._t)

    def __float__(self) -> float:
        return float(self._t)

    # --- shape ops --------------------------------------------------------
    def reshape(self, *shape: Any) -> "array":
        if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
            shape = tuple(shape[0])
        return array(self._t.reshape(*shape))

    def transpose(self, *axes: Any) -> "array":
        if len(axes) == 1 and isinstance(axes[0], (tuple, list)):
            axes = tuple(axes[0])
        if not axes:
            axes = tuple(reversed(range(self._t.dim())))
        return array(self._t.permute(*axes))

    def __getitem__(self, key: Any) -> "array":
        return array(self._t[_index(key)])

    def __setitem__(self, key: Any, value: Any) -> None:
        self._t[_index(key)] = _to_tensor(value).to(self._t.dtype)

    # --- arithmetic -------------------------------------------------------
    def _bin(self, other: Any, fn) -> "array":
        return _wrap(fn(self._t, _raw(other)))

    def _rbin(self, other: Any, fn) -> "array":
        return _wrap(fn(_raw(other), self._t))

    def __add__(self, o):
        return self._bin(o, torch.add)

    def __radd__(self, o):
        return self._rbin(o, lambda a, b: b + a if not isinstance(a, torch.Tensor) else a + b)

    def __sub__(self, o):
        return self._bin(o, torch.sub)

    def __rsub__(self, o):
        return _wrap(_raw(o) - self._t)

    def __mul__(self, o):
        return self._bin(o, torch.mul)

    def __rmul__(self, o):
        return _wrap(self._t * _raw(o))

    def __truediv__(self, o):
        return _wrap(torch.true_divide(self._t, _raw(o)))

    def __rtruediv__(self, o):
        r = _raw(o)
        if not isinstance(r, torch.Tensor):
            r = torch.tensor(r, dtype=self._t.dtype if self._t.is_floating_point() else torch.float32)
        return _wrap(torch.true_divide(r, self._t))

    def __pow__(self, o):
        return _wrap(torch.pow(self._t, _raw(o)))

    def __rpow__(self, o):
        r = _raw(o)
        if not isinstance(r, torch.Tensor):
            r = torch.tensor(r, dtype=self._t.dtype if self._t.is_floating_point() else torch.float32)
        return _wrap(torch.pow(r, self._t))

    def __neg__(self):
        return array(-self._t)

    def __matmul__(self, o):
        return matmul(self, o)

    def __rmatmul__(self, o):
        return matmul(o, self)

    def __lt__(self, o):
        return self._bin(o, torch.lt)

    def __le__(self, o):
        return self._bin(o, torch.le)

    def __gt__(self, o):
        return self._bin(o, torch.gt)

    def __ge__(self, o):
        return self._bin(o, torch.ge)

    def __eq__(self, o):  # type: ignore[override]
        return self._bin(o, torch.eq)

    def __ne__(self, o):  # type: ignore[override]
        return self._bin(o, torch.ne)

    __hash__ = object.__hash__


Dtype.__module__ = __name__


# --- creation ----------------------------------------------------------------
def _shape(shape: Any) -> tuple[int, ...]:
    if isinstance(shape, int):
        return (shape,)
    return tuple(int(s) for s in shape)


def zeros(shape: Any, dtype: Dtype = float32) -> array:
    return array(torch.zeros(_shape(shape), dtype=dtype.torch_dtype))


def ones(shape: Any, dtype: Dtype = float32) -> array:
    return array(torch.ones(_shape(shape), dtype=dtype.torch_dtype))


def full(shape: Any, vals: Any, dtype: Dtype | None = None) -> array:
    v = _to_tensor(vals)
    out = torch.broadcast_to(v, _shape(shape)).clone()
    if dtype is not None:
        out = out.to(dtype.torch_dtype)
    return array(out)


def zeros_like(a: array) -> array:
    return array(torch.zeros_like(a._t))


def arange(start: Any, stop: Any = None, step: Any = None, dtype: Dtype | None = None) -> array:
    if stop is None:
        start, stop = 0, start
    if step is None:
        step = 1
    is_int = all(isinstance(v, int) for v in (start, stop, step))
    if dtype is None:
        dtype = int32 if is_int else float32
    if dtype in (float32, float16, bfloat16):
        n = builtins.max(0, int(math.ceil((stop - start) / step)))
        t = torch.arange(n, dtype=torch.float64) * step + start
        return array(t.to(dtype.torch_dtype))
    return array(torch.arange(start, stop, step, dtype=torch.int64).to(dtype.torch_dtype))


# --- manipulation -----------------------------------------------------------
def concatenate(arrays: Sequence[array], axis: int = 0) -> array:
    ts = [_to_tensor(a) for a in arrays]
    return _wrap(torch.cat(_promote_all(ts), dim=axis))


def stack(arrays: Sequence[array], axis: int = 0) -> array:
    ts = [_to_tensor(a) for a in arrays]
    return _wrap(torch.stack(_promote_all(ts), dim=axis))


def _promote_all(ts: list[torch.Tensor]) -> list[torch.Tensor]:
    dt = ts[0].dtype
    for t in ts[1:]:
        dt = torch.promote_types(dt, t.dtype)
    return [t.to(dt) for t in ts]


def broadcast_to(a: Any, shape: Any) -> array:
    return array(torch.broadcast_to(_to_tensor(a), _shape(shape)))


def put_along_axis(a: array, indices: Any, values: Any, axis: int) -> array:
    out = a._t.clone()
    idx = _to_tensor(indices).long()
    vals = _to_tensor(values).to(out.dtype)
    vals = torch.broadcast_to(vals, idx.shape)
    out.scatter_(axis, idx, vals)
    return array(out)


def take_along_axis(a: array, indices: Any, axis: int) -> array:
    return array(torch.take_along_dim(a._t, _to_tensor(indices).long(), dim=axis))


def where(cond: Any, x: Any, y: Any) -> array:
    c = _to_tensor(cond).to(torch.bool)
    xr, yr = _raw(x), _raw(y)
    if not isinstance(xr, torch.Tensor) and not isinstance(yr, torch.Tensor):
        return array(torch.where(c, torch.tensor(float(xr)), torch.tensor(float(yr))).to(torch.float32))
    return _wrap(torch.where(c, xr, yr))


def repeat(a: array, repeats: int, axis: int | None = None) -> array:
    if axis is None:
        return array(torch.repeat_interleave(a._t.reshape(-1), repeats))
    return array(torch.repeat_interleave(a._t, repeats, dim=axis))


def transpose(a: array, axes: Any = None) -> array:
    return a.transpose(*(axes or ()))


def reshape(a: array, shape: Any) -> array:
    return a.reshape(shape)


def expand_dims(a: array, axis: int) -> array:
    return array(a._t.unsqueeze(axis))


# --- math -------------------------------------------------------------------
def matmul(a: Any, b: Any) -> array:
    ta, tb = _to_tensor(a), _to_tensor(b)
    dt = torch.promote_types(ta.dtype, tb.dtype)
    return _wrap(torch.matmul(ta.to(dt), tb.to(dt)))


def maximum(a: Any, b: Any) -> array:
    ta, tb = _raw(a), _raw(b)
    if not isinstance(ta, torch.Tensor):
        ta, tb = tb, ta
    if not isinstance(tb, torch.Tensor):
        return _wrap(torch.clamp_min(ta, tb))
    return _wrap(torch.maximum(ta, tb.to(torch.promote_types(ta.dtype, tb.dtype))))


def minimum(a: Any, b: Any) -> array:
    ta, tb = _raw(a), _raw(b)
    if not isinstance(ta, torch.Tensor):
        ta, tb = tb, ta
    if not isinstance(tb, torch.Tensor):
        return _wrap(torch.clamp_max(ta, tb))
    return _wrap(torch.minimum(ta, tb))


def _axes(axis: Any, nd: int) -> Any:
    if axis is None:
        return tuple(range(nd))
    return axis


def max(a: array, axis: Any = None, keepdims: bool = False) -> array:  # noqa: A001
    return array(torch.amax(a._t, dim=_axes(axis, a.ndim), keepdim=keepdims))


def min(a: array, axis: Any = None, keepdims: bool = False) -> array:  # noqa: A001
    return array(torch.amin(a._t, dim=_axes(axis, a.ndim), keepdim=keepdims))


def sum(a: array, axis: Any = None, keepdims: bool = False) -> array:  # noqa: A001
    return array(torch.sum(a._t, dim=_axes(axis, a.ndim), keepdim=keepdims))


def mean(a: array, axis: Any = None, keepdims: bool = False) -> array:
    return array(torch.mean(a._t, dim=_axes(axis, a.ndim), keepdim=keepdims))


def exp(a: array) -> array:
    return array(torch.exp(a._t))


def log(a: array) -> array:
    return array(torch.log(a._t))


def sqrt(a: array) -> array:
    return array(torch.sqrt(a._t))


def rsqrt(a: array) -> array:
    return array(torch.rsqrt(a._t))


def cos(a: array) -> array:
    return array(torch.cos(a._t))


def sin(a: array) -> array:
    return array(torch.sin(a._t))


def abs(a: array) -> array:  # noqa: A001
    return array(torch.abs(a._t))


def sigmoid(a: array) -> array:
    return array(torch.sigmoid(a._t))


def softmax(a: array, axis: int = -1) -> array:
    return array(torch.softmax(a._t.to(torch.float32), dim=axis).to(a._t.dtype))


def argmax(a: array, axis: Any = None, keepdims: bool = False) -> array:
    if axis is None:
        return array(torch.argmax(a._t).to(torch.int32))
    return array(torch.argmax(a._t, dim=axis, keepdim=keepdims).to(torch.int32))


def argsort(a: array, axis: int = -1) -> array:
    return array(torch.argsort(a._t, dim=axis).to(torch.int32))


def topk(a: array, k: int, axis: int = -1) -> array:
    vals = torch.topk(a._t, k, dim=axis).values
    return array(torch.flip(vals, dims=(axis,)))


def cumsum(a: array, axis: int = -1) -> array:
    return array(torch.cumsum(a._t, dim=axis))


def eval(*args: Any) -> None:  # noqa: A001
    return None


def array_equal(a: Any, b: Any) -> bool:
    return bool(torch.equal(_to_tensor(a), _to_tensor(b)))


# --- namespaces -----------------------------------------------------------------
def _sdpa(q: array, k: array, v: array, *, scale: float, mask: Any = None) -> array:
    out_dtype = torch.promote_types(torch.promote_types(q._t.dtype, k._t.dtype), v._t.dtype)
    qf, kf, vf = q._t.float(), k._t.float(), v._t.float()
    if kf.shape[1] != qf.shape[1]:
        groups = qf.shape[1] // kf.shape[1]
        kf = torch.repeat_interleave(kf, groups, dim=1)
        vf = torch.repeat_interleave(vf, groups, dim=1)
    logits = torch.matmul(qf, kf.transpose(-1, -2)) * scale
    if mask is not None:
        logits = logits + _to_tensor(mask).float()
    probs = torch.softmax(logits, dim=-1)
    return array(torch.matmul(probs, vf).to(out_dtype))


fast = types.SimpleNamespace(scaled_dot_product_attention=_sdpa)

_gen = torch.Generator().manual_seed(0)


def _seed(s: int) -> None:
    _gen.manual_seed(int(s))


def _normal(shape: Any = (), dtype: Dtype = float32, loc: float = 0.0, scale: float = 1.0, key: Any = None) -> array:
    t = torch.randn(_shape(shape), generator=_gen) * scale + loc
    return array(t.to(dtype.torch_dtype))


def _uniform(low: float = 0.0, high: float = 1.0, shape: Any = (), dtype: Dtype = float32, key: Any = None) -> array:
    t = torch.rand(_shape(shape), generator=_gen) * (high - low) + low
    return array(t.to(dtype.torch_dtype))


def _categorical(logits: array, axis: int = -1, num_samples: Any = None, key: Any = None) -> array:
    probs = torch.softmax(logits._t.float(), dim=axis)
    flat = probs.reshape(-1, probs.shape[-1])
    draws = torch.multinomial(flat, 1, generator=_gen).reshape(probs.shape[:-1])
    return array(draws.to(torch.int32))


random = types.SimpleNamespace(seed=_seed, normal=_normal, uniform=_uniform, categorical=_categorical)
