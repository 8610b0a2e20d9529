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
    if _bi.any(x.shape[a] != 1 for a in axes):
        raise ValueError("squeeze axis must have size one")
    return x.reshape(tuple(s for i, s in enumerate(x.shape) if i not in axes))


def unsqueeze(x, axis):
    rank = x.ndim + 1
    axis = axis % rank
    return x.reshape(x.shape[:axis] + (1,) + x.shape[axis:])


def flatten(x, start_dim=0, end_dim=-1):
    """Merge dimensions [start_dim, end_dim] into one (reference ops.py flatten)."""
    rank = x.ndim
    if rank == 0:
        if start_dim in (0, -1) and end_dim in (0, -1):
            return x.reshape((1,))
        raise IndexError("flatten dimension out of range for scalar")
    lo = start_dim + rank if start_dim < 0 else start_dim
    hi = end_dim + rank if end_dim < 0 else end_dim
    if not (0 <= lo < rank and 0 <= hi < rank and lo <= hi):
        raise ValueError("invalid flatten start_dim/end_dim")
    merged = 1
    for s in x.shape[lo:hi + 1]:
        merged *= s
    return x.reshape(x.shape[:lo] + (merged,) + x.shape[hi + 1:])


# ---------------------------------------------------------- index transforms
# Semantics of src/fugatensor/ops.py:481-800 and 833-920 (slice, pad,
# concatenate / stack / split / chunk, gather, scatter_add, indexing).

def _norm_slice(dim, start, stop, step):
    """Normalised (start, stop, step) of one axis; empty ranges become (0, 0, 1)."""
    if type(step) is not int or step == 0:
        raise ValueError("slice step must be a nonzero integer")
    st, sp, stp = _bi.slice(start, stop, step).indices(dim)
    if len(range(st, sp, stp)) == 0:
        return 0, 0, 1
    return st, sp, stp


def slice(x, starts, stops, steps=None):  # noqa: A001 - the reference's name
    """Strided slice along every axis of x (Python slice semantics per axis)."""
    rank = x.ndim
    steps = (1,) * rank if steps is None else tuple(steps)
    starts, stops = tuple(starts), tuple(stops)
    if not (len(starts) == len(stops) == len(steps) == rank):
        raise ValueError(f"slice expects sequences of length {rank}")
    bounds = [_norm_slice(d, a, b, c) for d, a, b, c in zip(x.shape, starts, stops, steps)]
    return _slice_norm(x, bounds)


def _slice_norm(x, bounds):
    if _bi.all(st == 0 and sp == d and stp == 1 for (st, sp, stp), d in zip(bounds, x.shape)):
        return x
    return _prim("slice", (x,), (tuple(b[0] for b in bounds), tuple(b[1] for b in bounds), tuple(b[2] for b in bounds)))


def pad(x, pad_width, constant_value=0, *, interior=None):
    """Pad x with constant_value at the edges and, with interior, between elements."""
    rank = x.ndim
    if isinstance(pad_width, int):
        if pad_width < 0:
            raise ValueError("pad_width must be nonnegative")
        low = high = (pad_width,) * rank
    else:
        pairs = tuple(pad_width)
        if len(pairs) != rank:
            raise ValueError(f"pad_width must have length {rank}")
        low = tuple(p if isinstance(p, int) else p[0] for p in pairs)
        high = tuple(p if isinstance(p, int) else p[1] for p in pairs)
    if _bi.any(v < 0 for v in low + high):
        raise ValueError("pad_width entries must be nonnegative")
    inner = (0,) * rank if interior is None else (interior,) * rank if isinstance(interior, int) else tuple(interior)
    if len(inner) != rank or _bi.any(v < 0 for v in inner):
        raise ValueError(f"interior must be length {rank} of nonnegative integers")
    if isinstance(constant_value, Tensor):
        if constant_value.shape != () or constant_value.dtype is not x.dtype:
            raise TypeError("pad constant_value must be a 0-D scalar of matching dtype")
        pv = constant_value
    else:
        if type(constant_value) not in (_bi.bool, int, float):
            raise TypeError("pad constant_value must be a scalar")
        pv = x.engine._splat(_bi.bool(constant_value) if x.dtype.ir == "bool" else constant_value, x.dtype, ())
    return _prim("pad", (x, pv), (low, high, inner))


def concatenate(tensors, axis=0):
    """Join a non-empty sequence of tensors along axis."""
    seq = tuple(tensors)
    if not seq:
        raise ValueError("concatenate requires at least one tensor")
    rank = seq[0].ndim
    if rank == 0:
        raise ValueError("zero-dimensional tensors cannot be concatenated")
    if type(axis) is not int:
        raise TypeError("concatenate axis must be an integer")
    ax = axis + rank if axis < 0 else axis
    if not 0 <= ax < rank:
        raise ValueError("concatenate axis out of range")
    if len(seq) == 1:
        return seq[0]
    return _prim("concatenate", seq, (ax,))


cat = concatenate


def stack(tensors, axis=0):
    seq = tuple(tensors)
    if not seq:
        raise ValueError("stack requires at least one tensor")
    rank = seq[0].ndim
    ax = axis + rank + 1 if axis < 0 else axis
    if not 0 <= ax <= rank:
        raise ValueError("stack axis out of range")
    return concatenate([unsqueeze(t, ax) for t in seq], axis=ax)


def split(x, split_size_or_sections, axis=0):
    rank = x.ndim
    ax = axis + rank if axis < 0 else axis
    if not 0 <= ax < rank:
        raise ValueError("split axis out of range")
    dim = x.shape[ax]
    if isinstance(split_size_or_sections, int):
        if split_size_or_sections <= 0:
            raise ValueError("split size must be positive")
        sizes = [split_size_or_sections] * (dim // split_size_or_sections)
        if dim % split_size_or_sections:
            sizes.append(dim % split_size_or_sections)
        if not sizes:
            sizes = [0]
    else:
        sizes = list(split_size_or_sections)
        if _bi.any(type(v) is not int or v < 0 for v in sizes) or _bi.sum(sizes) != dim:
            raise ValueError(f"split sections must be nonnegative integers summing to {dim}")
    out, at = [], 0
    for n in sizes:
        bounds = [(0, d, 1) for d in x.shape]
        bounds[ax] = (at, at + n, 1) if n else (0, 0, 1)
        out.append(_slice_norm(x, bounds))
        at += n
    return tuple(out)


def chunk(x, chunks, axis=0):
    if isinstance(chunks, _bi.bool) or type(chunks) is not int or chunks <= 0:
        raise ValueError("chunks must be a positive integer")
    rank = x.ndim
    ax = axis + rank if axis < 0 else axis
    if not 0 <= ax < rank:
        raise ValueError("chunk axis out of range")
    dim = x.shape[ax]
    if dim == 0:
        return split(x, [0] * chunks, axis=ax)
    return split(x, -(-dim // chunks), axis=ax)


def gather(params, indices, axis=0):
    """params[..., indices[i...], ...] along axis; indices outside [0, extent) read 0."""
    rank = params.ndim
    if rank == 0:
        raise ValueError("gather params must have rank at least one")
    if type(axis) is not int:
        raise TypeError("gather axis must be an int")
    ax = axis + rank if axis < 0 else axis
    if not 0 <= ax < rank:
        raise ValueError("gather axis out of range")
    if indices.dtype.ir not in ("i32", "i64"):
        raise TypeError("gather indices must be an int32 or int64 Tensor")
    return _prim("gather", (params, indices), (ax,))


take = gather


def scatter_add(base, indices, updates, axis=0):
    """base plus updates added at indices along axis; indices outside [0, extent) are dropped."""
    rank = base.ndim
    if rank == 0:
        raise ValueError("scatter_add base must have rank at least one")
    if type(axis) is not int:
        raise TypeError("scatter_add axis must be an int")
    ax = axis + rank if axis < 0 else axis
    if not 0 <= ax < rank:
        raise ValueError("scatter_add axis out of range")
    return _prim("scatter_add", (base, indices, updates), (ax,))


def getitem(x, key):
    """Static slices, ints, None, Ellipsis and at most one integer Tensor index."""
    items = key if isinstance(key, tuple) else (key,)
    if _bi.sum(1 for k in items if k is Ellipsis) > 1:
        raise IndexError("an index can only have a single ellipsis ('...')")
    rank = x.ndim
    used = _bi.sum(1 for k in items if k is not None and k is not Ellipsis)
    if used > rank:
        raise IndexError(f"too many indices for tensor of dimension {rank}")
    full = []
    for k in items:
        full.extend([_bi.slice(None)] * (rank - used) if k is Ellipsis else [k])
    if not _bi.any(k is Ellipsis for k in items):
        full.extend([_bi.slice(None)] * (rank - used))
    bounds, dropped, out_shape = [], [], []
    index_axis = index = None
    axis = 0      # axis of x being indexed
    kept = 0      # axis of the sliced value
    for k in full:
        if k is None:
            out_shape.append(1)
            continue
        dim = x.shape[axis]
        if isinstance(k, int) and not isinstance(k, _bi.bool):
            i = k + dim if k < 0 else k
            if not 0 <= i < dim:
                raise IndexError(f"index {k} is out of bounds for axis {axis} with size {dim}")
            bounds.append((i, i + 1, 1))
            dropped.append(kept)
        elif isinstance(k, _bi.slice):
            st, sp, stp = _norm_slice(dim, k.start, k.stop, 1 if k.step is None else k.step)
            bounds.append((st, sp, stp))
            out_shape.append(len(range(st, sp, stp)))
        elif isinstance(k, Tensor):
            if index is not None:
                raise TypeError("indexing with multiple Tensor indices is not supported")
            if k.dtype.ir not in ("i32", "i64"):
                raise TypeError("Tensor indices must have int32 or int64 dtype")
            bounds.append((0, dim, 1))
            index_axis, index = kept, k
            out_shape.extend(k.shape)
        else:
            raise TypeError(f"unsupported index type {type(k).__name__}")
        axis += 1
        kept += 1
    y = _slice_norm(x, bounds) if rank else x
    if dropped:
        if index_axis is not None:
            index_axis -= _bi.sum(1 for a in dropped if a < index_axis)
        y = y.reshape(tuple(s for i, s in enumerate(y.shape) if i not in dropped))
    if index is not None:
        y = gather(y, index, axis=index_axis)
    if tuple(out_shape) != y.shape:
        y = y.reshape(tuple(out_shape))
    return y


def one_hot(indices, num_classes, dtype=_dt.fp32):
    """1 where iota == index (indices outside [0, num_classes) give an all-zero row)."""
    shape = tuple(indices.shape) + (num_classes,)
    cls = _prim_on(indices.engine, "iota", (shape, len(shape) - 1, indices.dtype.ir))
    idx = broadcast_in_dim(indices, shape, tuple(range(indices.ndim)))
    return where(compare(cls, idx, "eq"), _filled_like_shape(indices, shape, 1, dtype),
                 _filled_like_shape(indices, shape, 0, dtype))


def _filled_like_shape(x, shape, value, dtype):
    return x.engine._splat(value, _dt.normalize(dtype), shape)


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
