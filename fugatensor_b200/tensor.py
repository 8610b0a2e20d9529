"""Lazy tensors (reference: src/fugatensor/tensor.py, src/fugatensor/tracing.py).

A Tensor is either materialised (it owns a device buffer) or pending (it
holds one Fuga primitive over other Tensors). Nothing runs until
``evaluate`` joins the requested pending tensors into one partition and
hands it to the native backend. Operator semantics follow the reference's
traced tensors (tracing.py:44-56): no implicit broadcasting, equal dtypes
required, Python scalars become a constant splatted in the tensor's dtype.
"""
from __future__ import annotations

import math

from . import dtypes as _dt
from . import ir


class Tensor:
    __slots__ = ("_engine", "_dtype", "_shape", "_data", "_expr", "__weakref__")

    def __init__(self, engine, dtype, shape, data=None, expr=None):
        self._engine = engine
        self._dtype = _dt.normalize(dtype)
        self._shape = tuple(int(s) for s in shape)
        self._data = data
        self._expr = expr

    # -- metadata ----------------------------------------------------------
    @property
    def dtype(self):
        return self._dtype

    @property
    def shape(self):
        return self._shape

    @property
    def ndim(self):
        return len(self._shape)

    @property
    def size(self):
        return math.prod(self._shape)

    @property
    def engine(self):
        return self._engine

    @property
    def device(self):
        return self._engine.device

    @property
    def is_pending(self):
        return self._expr is not None

    def __repr__(self):
        state = "pending" if self._expr is not None else "materialized"
        return f"Tensor(shape={self._shape}, dtype={self._dtype.name}, {state})"

    def __len__(self):
        if not self._shape:
            raise TypeError("len() of a 0-d tensor")
        return self._shape[0]

    # -- host access -------------------------------------------------------
    def torch(self):
        """The materialised device buffer (evaluates if pending)."""
        if self._expr is not None:
            self._engine.evaluate(self)
        return self._data

    def numpy(self):
        t = self.torch()
        if self._dtype is _dt.bf16:
            return t.view(__import__("torch").int16).cpu().numpy().view("uint16")
        return t.cpu().numpy()

    def tolist(self):
        t = self.torch()
        if self._dtype is _dt.bf16 or self._dtype is _dt.fp16:
            t = t.float()
        return t.cpu().tolist()

    def item(self):
        if self.size != 1:
            raise ValueError("item() requires a tensor with one element")
        v = self.tolist()
        while isinstance(v, list):
            v = v[0]
        return v

    def __bool__(self):
        if self._shape != ():
            raise TypeError("the truth value of a non-scalar Tensor is ambiguous")
        return bool(self.item())

    def __float__(self):
        return float(self.item())

    def __int__(self):
        return int(self.item())

    # -- operand handling (tracing.py:44-56) ------------------------------
    def _operand(self, other):
        if isinstance(other, Tensor):
            if other._engine is not self._engine:
                raise ValueError("tensors belong to different engines")
            if other._shape != self._shape:
                raise ValueError("tensor operands require equal shapes; use broadcast_to explicitly")
            if other._dtype is not self._dtype:
                raise TypeError("tensor operands require equal dtypes; use astype explicitly")
            return other
        if type(other) not in (bool, int, float):
            raise TypeError("operations accept tensors or Python scalars")
        return self._engine._splat(other, self._dtype, self._shape)

    def _binary(self, op, other, reverse=False):
        if self._dtype is _dt.bool and not isinstance(other, Tensor):
            raise TypeError("bool arithmetic is not defined; use astype to select a numeric type")
        o = self._operand(other)
        a, b = (o, self) if reverse else (self, o)
        return _prim(op, (a, b))

    def __add__(self, other):
        return self._binary("add", other)

    def __radd__(self, other):
        return self._binary("add", other, reverse=True)

    def __mul__(self, other):
        return self._binary("mul", other)

    def __rmul__(self, other):
        return self._binary("mul", other, reverse=True)

    def __neg__(self):
        return self * -1

    def __sub__(self, other):
        return self + (-other)

    def __rsub__(self, other):
        return (-self) + other

    def __truediv__(self, other):
        from .ops import divide
        return divide(self, other)

    def __rtruediv__(self, other):
        from .ops import divide
        return divide(other, self)

    def __floordiv__(self, other):
        from .ops import floordiv
        return floordiv(self, other)

    def __rfloordiv__(self, other):
        from .ops import floordiv
        return floordiv(other, self)

    def __mod__(self, other):
        from .ops import mod
        return mod(self, other)

    def __rmod__(self, other):
        from .ops import mod
        return mod(other, self)

    def __pow__(self, other):
        from .ops import pow
        return pow(self, other)

    def __rpow__(self, other):
        from .ops import pow
        return pow(other, self)

    def __abs__(self):
        from .ops import abs
        return abs(self)

    def __and__(self, other):
        from .ops import bitwise_and
        return bitwise_and(self, other)

    def __rand__(self, other):
        from .ops import bitwise_and
        return bitwise_and(other, self)

    def __or__(self, other):
        from .ops import bitwise_or
        return bitwise_or(self, other)

    def __ror__(self, other):
        from .ops import bitwise_or
        return bitwise_or(other, self)

    def __xor__(self, other):
        from .ops import bitwise_xor
        return bitwise_xor(self, other)

    def __rxor__(self, other):
        from .ops import bitwise_xor
        return bitwise_xor(other, self)

    def __invert__(self):
        from .ops import bitwise_not
        return bitwise_not(self)

    def __lshift__(self, other):
        from .ops import shift_left
        return shift_left(self, other)

    def __rshift__(self, other):
        from .ops import shift_right
        return shift_right(self, other)

    def _cmp(self, other, predicate):
        from .ops import compare
        return compare(self, other, predicate)

    def __eq__(self, other):  # noqa: D105 - elementwise, like the reference
        return self._cmp(other, "eq")

    def __ne__(self, other):
        return self._cmp(other, "ne")

    def __lt__(self, other):
        return self._cmp(other, "lt")

    def __le__(self, other):
        return self._cmp(other, "le")

    def __gt__(self, other):
        return self._cmp(other, "gt")

    def __ge__(self, other):
        return self._cmp(other, "ge")

    __hash__ = object.__hash__

    # -- methods -----------------------------------------------------------
    def astype(self, dtype):
        return _prim("cast", (self,), (_dt.normalize(dtype).ir,))

    def reshape(self, *shape):
        from ._shape import infer_reshape
        shape = infer_reshape(shape, self.size)
        if shape == self._shape:
            return self
        return _prim("reshape", (self,), (shape,))

    def detach(self):
        return _prim("stop_gradient", (self,))

    def square(self):
        return self * self

    def transpose(self, permutation=None):
        from .ops import transpose
        return transpose(self, permutation)

    def sum(self, axis=None, *, keepdims=False, dtype=None):
        from .ops import sum
        return sum(self, axis, keepdims=keepdims, dtype=dtype)

    def amax(self, axis=None, *, keepdims=False):
        from .ops import amax
        return amax(self, axis, keepdims=keepdims)

    def amin(self, axis=None, *, keepdims=False):
        from .ops import amin
        return amin(self, axis, keepdims=keepdims)

    def mean(self, axis=None, *, keepdims=False, dtype=None):
        from .ops import mean
        return mean(self, axis, keepdims=keepdims, dtype=dtype)

    def prod(self, axis=None, *, keepdims=False, dtype=None):
        from .ops import prod
        return prod(self, axis, keepdims=keepdims, dtype=dtype)

    def any(self, axis=None, *, keepdims=False):
        from .ops import any
        return any(self, axis, keepdims=keepdims)

    def all(self, axis=None, *, keepdims=False):
        from .ops import all
        return all(self, axis, keepdims=keepdims)

    def argmax(self, axis=None, *, keepdims=False):
        from .ops import argmax
        return argmax(self, axis, keepdims=keepdims)

    def argmin(self, axis=None, *, keepdims=False):
        from .ops import argmin
        return argmin(self, axis, keepdims=keepdims)

    def abs(self):
        from .ops import abs
        return abs(self)

    def clamp(self, min=None, max=None):
        from .ops import clamp
        return clamp(self, min, max)

    def exp(self):
        from .ops import exp
        return exp(self)

    def log(self):
        from .ops import log
        return log(self)

    def sqrt(self):
        from .ops import sqrt
        return sqrt(self)

    def __getitem__(self, key):
        from .ops import getitem
        return getitem(self, key)

    def split(self, split_size_or_sections, axis=0):
        from .ops import split
        return split(self, split_size_or_sections, axis)

    def chunk(self, chunks, axis=0):
        from .ops import chunk
        return chunk(self, chunks, axis)

    def flatten(self, start_dim=0, end_dim=-1):
        from .ops import flatten
        return flatten(self, start_dim, end_dim)

    def squeeze(self, axis=None):
        from .ops import squeeze
        return squeeze(self, axis)

    def unsqueeze(self, axis):
        from .ops import unsqueeze
        return unsqueeze(self, axis)


def _infer(op, args, attrs):
    """Result type of a primitive, by the same rules as the IR builder."""
    g = ir.Graph()
    vals = [g.parameter(a._dtype.ir, a._shape) for a in args]
    if op == "constant":
        v = g.constant(attrs[0], attrs[1])
    elif op == "cast":
        v = g.cast(vals[0], attrs[0])
    elif op == "reshape":
        v = g.reshape(vals[0], attrs[0])
    elif op == "broadcast_in_dim":
        v = g.broadcast_in_dim(vals[0], attrs[0], attrs[1])
    elif op == "transpose":
        v = g.transpose(vals[0], attrs[0])
    elif op == "splat":
        v = g.splat(vals[0], attrs[0])
    elif op == "iota":
        v = g.iota(attrs[0], attrs[1], attrs[2])
    elif op == "compare":
        v = g.compare(vals[0], vals[1], attrs[0])
    elif op in ir.REDUCTIONS:
        v = getattr(g, op)(vals[0], attrs[0])
    elif op in ("argmax", "argmin"):
        v = getattr(g, op)(vals[0], attrs[0])
    elif op in ("slice", "pad", "concatenate", "gather", "scatter_add"):
        v = _index_op(g, op, vals, attrs)
    else:
        v = getattr(g, op)(*vals)
    return v.dtype, v.shape


def _index_op(g, op, vals, attrs):
    """IR builder call of an index transform (shared by typing and tracing)."""
    if op == "slice":
        return g.slice(vals[0], *attrs)
    if op == "pad":
        return g.pad(vals[0], vals[1], *attrs)
    if op == "concatenate":
        return g.concatenate(list(vals), attrs[0])
    if op == "gather":
        return g.gather(vals[0], vals[1], attrs[0])
    return g.scatter_add(vals[0], vals[1], vals[2], attrs[0])


def _prim(op, args, attrs=()):
    """A pending tensor for primitive `op` over `args`."""
    engine = None
    for a in args:
        if not isinstance(a, Tensor):
            raise TypeError(f"{op} operands must be Tensors")
        if engine is None:
            engine = a._engine
        elif a._engine is not engine:
            raise ValueError("tensors belong to different engines")
    dtype, shape = _infer(op, args, attrs)
    return Tensor(engine, _dt.BY_IR[dtype], shape, expr=(op, tuple(args), tuple(attrs)))


def _prim_on(engine, op, attrs):
    dtype, shape = _infer(op, (), attrs)
    return Tensor(engine, _dt.BY_IR[dtype], shape, expr=(op, (), tuple(attrs)))
