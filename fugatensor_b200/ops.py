"""Public tensor operations as Fuga primitives (reference: src/fugatensor/ops.py).

Each function records the same primitive decomposition the reference traces
(e.g. subtract = x + y * -1, square = x * x, mean = sum / count), so that the
partitions reaching the backend are the reference's partitions.
"""
from __future__ import annotations

import builtins as _bi
import math as _math

from . import dtypes as _dt
from .tensor import Tensor, _prim, _prim_on


def _pair(x, y):
    if isinstance(x, Tensor):
        return x, x._operand(y)
    if isinstance(y, Tensor):
        return y._operand(x), y
    raise TypeError("operation requires a Tensor operand")


def add(x, y):
    return x + y


def multiply(x, y):
    return x * y


def negative(x):
    return x * -1


def subtract(x, y):
    return x + y * -1


def square(x):
    return x * x


def cast(x, dtype):
    return x.astype(dtype)


def reshape(input, shape):
    if not isinstance(input, Tensor):
        raise TypeError("reshape requires a Tensor")
    if not isinstance(shape, (tuple, list)):
        raise TypeError("reshape shape must be a tuple or list of dimensions")
    return input.reshape(tuple(shape))


def _filled_like(x, value):
    if not isinstance(x, Tensor):
        raise TypeError("like operators expect a Tensor")
    return x._engine._splat(_bi.bool(value) if x.dtype is _dt.bool else value, x.dtype, x.shape)


def zeros_like(x):
    return _filled_like(x, 0)


def ones_like(x):
    return _filled_like(x, 1)


def divide(x, y):
    a, b = _pair(x, y)
    return _prim("div", (a, b))


def compare(x, y, predicate="eq"):
    a, b = _pair(x, y)
    return _prim("compare", (a, b), (predicate,))


def where(condition, x, y):
    a, b = _pair(x, y)
    if not isinstance(condition, Tensor) or condition.dtype is not _dt.bool:
        raise TypeError("where condition must be a bool Tensor")
    if condition.shape != a.shape:
        raise ValueError("where condition must match the value shape")
    return _prim("select", (condition, a, b))


def _unary(x, opcode):
    if not isinstance(x, Tensor):
        raise TypeError(f"{opcode} expects a Tensor")
    return _prim(opcode, (x,))


def _binary(x, y, opcode):
    a, b = _pair(x, y)
    return _prim(opcode, (a, b))


def exp(x):
    return _unary(x, "exp")


def log(x):
    return _unary(x, "log")


def sqrt(x):
    return _unary(x, "sqrt")


def sin(x):
    return _unary(x, "sin")


def cos(x):
    return _unary(x, "cos")


def tanh(x):
    return _unary(x, "tanh")


def erf(x):
    return _unary(x, "erf")


def abs(x):
    return _unary(x, "abs")


def floor(x):
    return _unary(x, "floor")


def ceil(x):
    return _unary(x, "ceil")


def round(x):
    return _unary(x, "round")


def bitwise_not(x):
    return _unary(x, "bitwise_not")


def pow(x, y):
    return _binary(x, y, "pow")


def floordiv(x, y):
    return _binary(x, y, "floordiv")


def mod(x, y):
    return _binary(x, y, "mod")


def maximum(x, y):
    return _binary(x, y, "maximum")


def minimum(x, y):
    return _binary(x, y, "minimum")


def clamp(x, min=None, max=None):
    if min is not None:
        x = maximum(x, min)
    if max is not None:
        x = minimum(x, max)
    return x


clip = clamp


def bitwise_and(x, y):
    return _binary(x, y, "bitwise_and")


def bitwise_or(x, y):
    return _binary(x, y, "bitwise_or")


def bitwise_xor(x, y):
    return _binary(x, y, "bitwise_xor")


def shift_left(x, y):
    return _binary(x, y, "shift_left")


def shift_right(x, y):
    return _binary(x, y, "shift_right")


def _as_bool(x):
    return x if x.dtype is _dt.bool else x.astype(_dt.bool)


def logical_not(x):
    return bitwise_not(_as_bool(x))


def _logical(x, y, opcode):
    if isinstance(x, Tensor):
        xb = _as_bool(x)
        yb = _as_bool(y) if isinstance(y, Tensor) else _bi.bool(y)
        return _binary(xb, yb, opcode)
    return _binary(_bi.bool(x), _as_bool(y), opcode)


def logical_and(x, y):
    return _logical(x, y, "bitwise_and")


def logical_or(x, y):
    return _logical(x, y, "bitwise_or")


def logical_xor(x, y):
    return _logical(x, y, "bitwise_xor")


def broadcast_in_dim(x, shape, dimensions):
    shape, dims = tuple(shape), tuple(dimensions)
    if shape == x.shape and dims == tuple(range(len(shape))):
        return x
    return _prim("broadcast_in_dim", (x,), (shape, dims))


def broadcast_to(x, shape):
    shape = tuple(shape)
    dims = tuple(range(len(shape) - len(x.shape), len(shape)))
    return broadcast_in_dim(x, shape, dims)


def transpose(x, permutation=None):
    perm = tuple(reversed(range(x.ndim))) if permutation is None else tuple(permutation)
    if perm == tuple(range(x.ndim)):
        return x
    return _prim("transpose", (x,), (perm,))


def squeeze(x, axis=None):
    if axis is None:
        return x.reshape(tuple(s for s in x.shape if s != 1))
    axes = (axis,) if type(axis) is int else tuple(axis)
    axes = tuple(a % x.ndim for a in axes)
    if any(x.shape[a] != 1 for a in axes):
        raise ValueError("squeeze axis must have size one")
    return x.reshape(tuple(s for i, s in enumerate(x.shape) if i not in axes))


def unsqueeze(x, axis):
    rank = x.ndim + 1
    axis = axis % rank
    return x.reshape(x.shape[:axis] + (1,) + x.shape[axis:])


def flatten(x):
    return x.reshape((-1,))


def _axes(axis, rank):
    axes = tuple(range(rank)) if axis is None else (axis,) if type(axis) is int else tuple(axis)
    if _bi.any(type(v) is not int or not -rank <= v < rank for v in axes):
        raise ValueError("reduction axes must be integer dimensions in range")
    axes = tuple(v % rank for v in axes)
    if len(set(axes)) != len(axes):
        raise ValueError("reduction axes must be unique")
    return tuple(sorted(axes))


def _reduce(x, opcode, axis, keepdims, dtype):
    if not isinstance(x, Tensor):
        raise TypeError(f"{opcode} expects a Tensor")
    axes = _axes(axis, x.ndim)
    if type(keepdims) is not bool:
        raise TypeError("keepdims must be bool")
    if dtype is not None:
        x = x.astype(dtype)
    result = _prim(opcode, (x,), (axes,))
    shape = tuple(1 if a in axes else s for a, s in enumerate(x.shape))
    if keepdims and result.shape != shape:
        result = result.reshape(shape)
    return result


def sum(x, axis=None, *, keepdims=False, dtype=None):
    return _reduce(x, "reduce_sum", axis, keepdims, dtype)


def amax(x, axis=None, *, keepdims=False):
    return _reduce(x, "reduce_max", axis, keepdims, None)


def amin(x, axis=None, *, keepdims=False):
    return _reduce(x, "reduce_min", axis, keepdims, None)


def prod(x, axis=None, *, keepdims=False, dtype=None):
    return _reduce(x, "reduce_prod", axis, keepdims, dtype)


def any(x, axis=None, *, keepdims=False):
    return _reduce(_as_bool(x), "reduce_any", axis, keepdims, None)


def all(x, axis=None, *, keepdims=False):
    return _reduce(_as_bool(x), "reduce_all", axis, keepdims, None)


def mean(x, axis=None, *, keepdims=False, dtype=None):
    axes = _axes(axis, x.ndim)
    count = _math.prod(x.shape[a] for a in axes)
    reduced = sum(x, axes, keepdims=keepdims, dtype=dtype)
    try:
        return reduced / count
    except (ValueError, TypeError):
        return reduced * (1.0 / count) if count else reduced


def _argreduce(x, opcode, axis, keepdims):
    if not isinstance(x, Tensor):
        raise TypeError(f"{opcode} expects a Tensor")
    if axis is None:
        if x.size == 0:
            raise ValueError(f"{opcode} requires a nonempty tensor")
        res = _prim(opcode, (x.reshape((-1,)),), (0,))
        if keepdims and x.shape:
            return res.reshape((1,) * x.ndim)
        return res
    if type(axis) is not int:
        raise TypeError(f"{opcode} axis must be an int or None")
    rank = x.ndim
    ax = axis + rank if axis < 0 else axis
    if not 0 <= ax < rank:
        raise ValueError(f"{opcode} axis out of range")
    if x.shape[ax] == 0:
        raise ValueError(f"{opcode} requires a nonempty reduction domain")
    res = _prim(opcode, (x,), (ax,))
    if keepdims:
        res = res.reshape(tuple(1 if i == ax else s for i, s in enumerate(x.shape)))
    return res


def argmax(x, axis=None, *, keepdims=False):
    return _argreduce(x, "argmax", axis, keepdims)


def argmin(x, axis=None, *, keepdims=False):
    return _argreduce(x, "argmin", axis, keepdims)


def iota(shape, dimension, dtype=_dt.int64, engine=None):
    from .engine import current_engine
    eng = engine or current_engine()
    return _prim_on(eng, "iota", (tuple(shape), dimension, _dt.normalize(dtype).ir))
