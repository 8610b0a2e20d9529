"""Partition IR builder: Fuga primitives -> the fgt_partition_desc of include/fgt.h.

A :class:`Graph` records one partition as SSA nodes with Fuga's primitive
names and typing rules (reference: src/fugatensor/ir/tensor_rules.py,
src/fugatensor/ir/primitives.py). Result types are inferred here so that
callers (the front end, the VJP transform, tests) get early, Python-level
errors; the C library re-checks every node before planning.

Scalar constants are encoded once, round-to-nearest-even, directly from the
Python value to the target format (reference: src/fugatensor/_ask/numerics.py:28-78
``encode_float`` -- same contract, own implementation).
"""
from __future__ import annotations

import ctypes
import math
import struct
from fractions import Fraction

# dtype names follow Fuga IR; the public aliases map onto them.
DTYPES = ("bool", "i32", "i64", "f32", "f16", "bf16")
DTYPE_CODE = {name: code for code, name in enumerate(DTYPES)}
ALIASES = {"fp32": "f32", "float32": "f32", "fp16": "f16", "float16": "f16", "bfloat16": "bf16",
           "int32": "i32", "int64": "i64", "bool_": "bool"}
FLOAT_DTYPES = frozenset({"f32", "f16", "bf16"})
INT_DTYPES = frozenset({"i32", "i64"})
WIDTH = {"bool": 1, "i32": 4, "i64": 8, "f32": 4, "f16": 2, "bf16": 2}

MAX_RANK = 8
MAX_ATTRS = 24

OP = {
    "parameter": 0, "constant": 1, "splat": 2, "reshape": 3, "broadcast_in_dim": 4, "transpose": 5,
    "stop_gradient": 6, "iota": 7, "cast": 8,
    "add": 10, "mul": 11, "div": 12, "maximum": 13, "minimum": 14, "pow": 15, "floordiv": 16, "mod": 17,
    "bitwise_and": 18, "bitwise_or": 19, "bitwise_xor": 20, "shift_left": 21, "shift_right": 22,
    "exp": 30, "log": 31, "sqrt": 32, "sin": 33, "cos": 34, "tanh": 35, "erf": 36, "abs": 37,
    "floor": 38, "ceil": 39, "round": 40, "bitwise_not": 41,
    "compare": 50, "select": 51,
    "reduce_sum": 60, "reduce_max": 61, "reduce_min": 62, "reduce_prod": 63, "reduce_any": 64,
    "reduce_all": 65, "argmax": 66, "argmin": 67,
    "slice": 70, "pad": 71, "concatenate": 72, "gather": 73, "scatter_add": 74,
}
PREDICATES = {"eq": 0, "ne": 1, "lt": 2, "le": 3, "gt": 4, "ge": 5}
BINARY = ("add", "mul", "div", "maximum", "minimum", "pow", "floordiv", "mod", "bitwise_and",
          "bitwise_or", "bitwise_xor", "shift_left", "shift_right")
UNARY = ("exp", "log", "sqrt", "sin", "cos", "tanh", "erf", "abs", "floor", "ceil", "round", "bitwise_not")
REDUCTIONS = ("reduce_sum", "reduce_max", "reduce_min", "reduce_prod", "reduce_any", "reduce_all")


def dtype_name(dtype) -> str:
    name = getattr(dtype, "name", dtype)
    name = ALIASES.get(name, name)
    if name not in DTYPE_CODE:
        raise TypeError(f"unsupported dtype: {dtype!r}")
    return name


# ---------------------------------------------------------------- codecs ---
_FORMATS = {"f16": (5, 10), "bf16": (8, 7), "f32": (8, 23)}


def encode_float(value, dtype: str) -> int:
    """Bits of ``value`` rounded once (RNE, subnormals included) to dtype.

    Finite values that round beyond the format raise ValueError, as the
    reference's boundary codec does; inf/nan are accepted.
    """
    exp_bits, frac_bits = _FORMATS[dtype]
    width = 1 + exp_bits + frac_bits
    bias = (1 << (exp_bits - 1)) - 1
    emask = (1 << exp_bits) - 1
    if isinstance(value, float) and math.isnan(value):
        return (emask << frac_bits) | (1 << (frac_bits - 1))
    if isinstance(value, float) and math.isinf(value):
        return ((1 if value < 0 else 0) << (width - 1)) | (emask << frac_bits)
    sign = 1 if (value < 0 or (isinstance(value, float) and value == 0 and math.copysign(1, value) < 0)) else 0
    q = abs(Fraction(value))
    if q == 0:
        return sign << (width - 1)
    # exponent of the leading bit
    e = q.numerator.bit_length() - q.denominator.bit_length()
    if Fraction(2) ** e > q:
        e -= 1
    e = max(e, 1 - bias)  # subnormal spacing
    scaled = q / (Fraction(2) ** (e - frac_bits))
    n, rem = divmod(scaled.numerator, scaled.denominator)
    twice = 2 * rem
    if twice > scaled.denominator or (twice == scaled.denominator and n & 1):
        n += 1
    if n >= (1 << (frac_bits + 1)):
        n >>= 1
        e += 1
    if e > bias:
        raise ValueError(f"finite value is outside the {dtype} range")
    if n < (1 << frac_bits):  # subnormal (or rounded to zero)
        return (sign << (width - 1)) | n
    return (sign << (width - 1)) | ((e + bias) << frac_bits) | (n & ((1 << frac_bits) - 1))


def decode_float(bits: int, dtype: str) -> float:
    exp_bits, frac_bits = _FORMATS[dtype]
    width = 1 + exp_bits + frac_bits
    bias = (1 << (exp_bits - 1)) - 1
    sign = -1.0 if (bits >> (width - 1)) & 1 else 1.0
    e = (bits >> frac_bits) & ((1 << exp_bits) - 1)
    f = bits & ((1 << frac_bits) - 1)
    if e == (1 << exp_bits) - 1:
        return math.copysign(math.nan if f else math.inf, sign)
    if e == 0:
        return sign * math.ldexp(f, 1 - bias - frac_bits)
    return sign * math.ldexp((1 << frac_bits) | f, e - bias - frac_bits)


def round_float(value, dtype: str) -> float:
    return decode_float(encode_float(value, dtype), dtype)


def constant_bits(value, dtype: str) -> int:
    if dtype == "bool":
        return 1 if value else 0
    if dtype in INT_DTYPES:
        width = 32 if dtype == "i32" else 64
        return int(value) & ((1 << width) - 1)
    return encode_float(value, dtype)


# ------------------------------------------------------------------ graph ---
class Value:
    __slots__ = ("graph", "id", "dtype", "shape")

    def __init__(self, graph, id, dtype, shape):
        self.graph, self.id, self.dtype, self.shape = graph, id, dtype, tuple(shape)

    @property
    def rank(self):
        return len(self.shape)

    def __repr__(self):
        return f"%{self.id}:{self.dtype}{list(self.shape)}"


class Node:
    __slots__ = ("op", "dtype", "shape", "operands", "attrs", "predicate", "bits")

    def __init__(self, op, dtype, shape, operands=(), attrs=(), predicate=0, bits=0):
        self.op, self.dtype, self.shape = op, dtype, tuple(shape)
        self.operands, self.attrs, self.predicate, self.bits = tuple(operands), tuple(attrs), predicate, bits


def _numel(shape):
    return math.prod(shape)


class Graph:
    """One partition under construction (SSA, topological by construction)."""

    def __init__(self):
        self.nodes: list[Node] = []
        self.num_inputs = 0

    # -- plumbing ---------------------------------------------------------
    def _add(self, op, dtype, shape, operands=(), attrs=(), predicate=0, bits=0) -> Value:
        if len(shape) > MAX_RANK:
            raise ValueError(f"rank {len(shape)} exceeds the backend limit of {MAX_RANK}")
        for v in operands:
            if v.graph is not self:
                raise ValueError("operands must belong to this graph")
        self.nodes.append(Node(op, dtype, shape, [v.id for v in operands], attrs, predicate, bits))
        return Value(self, len(self.nodes) - 1, dtype, shape)

    def value(self, id) -> Value:
        n = self.nodes[id]
        return Value(self, id, n.dtype, n.shape)

    # -- leaves and views -------------------------------------------------
    def parameter(self, dtype, shape) -> Value:
        dtype = dtype_name(dtype)
        port = self.num_inputs
        self.num_inputs += 1
        return self._add("parameter", dtype, tuple(int(s) for s in shape), (), (port,))

    def constant(self, value, dtype) -> Value:
        dtype = dtype_name(dtype)
        return self._add("constant", dtype, (), bits=constant_bits(value, dtype))

    def splat(self, x: Value, shape) -> Value:
        if x.shape != ():
            raise TypeError("splat takes a rank-0 operand")
        return self._add("splat", x.dtype, tuple(shape), (x,))

    def filled(self, value, dtype, shape) -> Value:
        c = self.constant(value, dtype)
        return c if tuple(shape) == () else self.splat(c, shape)

    def reshape(self, x: Value, shape) -> Value:
        shape = tuple(int(s) for s in shape)
        if _numel(shape) != _numel(x.shape):
            raise ValueError("reshape must keep the element count")
        if shape == x.shape:
            return x
        return self._add("reshape", x.dtype, shape, (x,))

    def broadcast_in_dim(self, x: Value, shape, dimensions) -> Value:
        shape, dims = tuple(shape), tuple(dimensions)
        if len(dims) != x.rank or tuple(sorted(set(dims))) != dims or any(not 0 <= d < len(shape) for d in dims):
            raise ValueError("broadcast dimensions must be an increasing input-to-output axis mapping")
        if any(s != 1 and s != shape[d] for s, d in zip(x.shape, dims)):
            raise ValueError("broadcast mapped dimensions must match or have size one")
        if shape == x.shape:
            return x
        return self._add("broadcast_in_dim", x.dtype, shape, (x,), dims)

    def transpose(self, x: Value, permutation) -> Value:
        perm = tuple(permutation)
        if sorted(perm) != list(range(x.rank)):
            raise ValueError("transpose permutation must contain each axis exactly once")
        if perm == tuple(range(x.rank)):
            return x
        return self._add("transpose", x.dtype, tuple(x.shape[a] for a in perm), (x,), perm)

    def stop_gradient(self, x: Value) -> Value:
        return self._add("stop_gradient", x.dtype, x.shape, (x,))

    def iota(self, shape, dimension, dtype="i64") -> Value:
        dtype = dtype_name(dtype)
        shape = tuple(shape)
        if not shape or not 0 <= dimension < len(shape) or dtype == "bool":
            raise ValueError("iota requires rank >= 1, a dimension in range and a numeric dtype")
        return self._add("iota", dtype, shape, (), (dimension,))

    def cast(self, x: Value, dtype) -> Value:
        dtype = dtype_name(dtype)
        if dtype == x.dtype:
            return x
        return self._add("cast", dtype, x.shape, (x,))

    # -- elementwise ------------------------------------------------------
    def _binary(self, op, x: Value, y: Value) -> Value:
        if x.shape != y.shape or x.dtype != y.dtype:
            raise TypeError(f"{op} requires matching operands (no implicit broadcast)")
        if op in ("add", "mul", "pow", "floordiv", "mod") and x.dtype == "bool":
            raise TypeError("bool arithmetic is undefined")
        if op == "div" and x.dtype not in FLOAT_DTYPES:
            raise TypeError("div is floating division")
        if op.startswith("bitwise") and x.dtype in FLOAT_DTYPES:
            raise TypeError("bitwise operations take integer or bool operands")
        if op.startswith("shift") and x.dtype not in INT_DTYPES:
            raise TypeError("shifts take integer operands")
        return self._add(op, x.dtype, x.shape, (x, y))

    def _unary(self, op, x: Value) -> Value:
        if op == "abs":
            if x.dtype == "bool":
                raise TypeError("abs requires a numeric dtype")
        elif op == "bitwise_not":
            if x.dtype in FLOAT_DTYPES:
                raise TypeError("bitwise_not takes integer or bool")
        elif x.dtype not in FLOAT_DTYPES:
            raise TypeError(f"{op} requires a floating dtype")
        return self._add(op, x.dtype, x.shape, (x,))

    def compare(self, x: Value, y: Value, predicate="eq") -> Value:
        if x.shape != y.shape or x.dtype != y.dtype:
            raise TypeError("compare requires matching operand types")
        if predicate not in PREDICATES:
            raise ValueError("compare predicate must be eq/ne/lt/le/gt/ge")
        return self._add("compare", "bool", x.shape, (x, y), predicate=PREDICATES[predicate])

    def select(self, cond: Value, x: Value, y: Value) -> Value:
        if cond.dtype != "bool" or cond.shape != x.shape or x.shape != y.shape or x.dtype != y.dtype:
            raise TypeError("select requires a bool condition and matching value shapes and dtypes")
        return self._add("select", x.dtype, x.shape, (cond, x, y))

    # -- reductions -------------------------------------------------------
    def _reduce(self, op, x: Value, axes) -> Value:
        axes = tuple(axes)
        if tuple(sorted(set(axes))) != axes or any(not 0 <= a < x.rank for a in axes):
            raise ValueError("reduction axes must be sorted, unique and in range")
        boolean = op in ("reduce_any", "reduce_all")
        if boolean != (x.dtype == "bool"):
            raise TypeError("boolean reductions take bool; numeric reductions take numbers")
        if op in ("reduce_max", "reduce_min") and any(x.shape[a] == 0 for a in axes):
            raise ValueError("max/min reduction requires a nonempty reduction domain")
        shape = tuple(s for a, s in enumerate(x.shape) if a not in axes)
        return self._add(op, x.dtype, shape, (x,), axes)

    def _argreduce(self, op, x: Value, axis: int) -> Value:
        if x.rank == 0 or not 0 <= axis < x.rank:
            raise ValueError(f"{op} axis out of range")
        if x.shape[axis] == 0:
            raise ValueError(f"{op} requires a nonempty reduction domain")
        if x.dtype == "bool":
            raise TypeError(f"{op} requires a numeric operand")
        shape = tuple(s for a, s in enumerate(x.shape) if a != axis)
        return self._add(op, "i64", shape, (x,), (axis,))

    # -- index transforms (typing: ir/tensor_rules.py:124-237) -------------
    def slice(self, x: Value, starts, stops, steps) -> Value:
        """Strided slice with normalised bounds (ops.py:481-508 produces them)."""
        starts, stops, steps = tuple(starts), tuple(stops), tuple(steps)
        if not (len(starts) == len(stops) == len(steps) == x.rank):
            raise ValueError("slice starts, stops and steps must match operand rank")
        shape = []
        for dim, st, sp, step in zip(x.shape, starts, stops, steps):
            if step == 0:
                raise ValueError("slice step must be nonzero")
            if step > 0:
                if not 0 <= st <= sp <= dim:
                    raise ValueError("slice forward bounds out of range")
                shape.append(0 if sp == st else (sp - st + step - 1) // step)
            elif st == sp:
                if not 0 <= st <= dim:
                    raise ValueError("slice empty bounds out of range")
                shape.append(0)
            else:
                if not (0 <= st < dim and -1 <= sp < st):
                    raise ValueError("slice reverse bounds out of range")
                shape.append((st - sp + (-step) - 1) // (-step))
        if tuple(shape) == x.shape and all(st == 0 and step == 1 for st, step in zip(starts, steps)):
            return x
        return self._add("slice", x.dtype, tuple(shape), (x,), starts + steps)

    def pad(self, x: Value, pad_value: Value, low, high, interior) -> Value:
        low, high, interior = tuple(low), tuple(high), tuple(interior)
        if pad_value.shape != () or pad_value.dtype != x.dtype:
            raise TypeError("pad requires a 0-D scalar pad_value with the same dtype as input")
        if not (len(low) == len(high) == len(interior) == x.rank):
            raise ValueError("pad attributes must match operand rank")
        if any(v < 0 for v in low + high + interior):
            raise ValueError("pad amounts and interior dilation must be nonnegative integers")
        shape = tuple(l + (d + (d - 1) * i if d > 0 else 0) + h for d, l, h, i in zip(x.shape, low, high, interior))
        return self._add("pad", x.dtype, shape, (x, pad_value), low + interior)

    def concatenate(self, xs, axis) -> Value:
        xs = list(xs)
        if not xs:
            raise TypeError("concatenate requires at least one operand")
        first = xs[0]
        if first.rank < 1 or not 0 <= axis < first.rank:
            raise ValueError("concatenate axis out of range")
        for v in xs:
            if v.dtype != first.dtype or v.rank != first.rank:
                raise TypeError("concatenate operands must match rank and dtype")
            if any(a != axis and s != first.shape[a] for a, s in enumerate(v.shape)):
                raise ValueError("concatenate non-axis dimensions must match")
        xs = [v for v in xs if v.shape[axis] > 0] or xs[:1]
        if len(xs) == 1:
            return xs[0]
        # n-ary joins nest as binary ones (left to right)
        acc = xs[0]
        for v in xs[1:]:
            shape = tuple(s + v.shape[a] if a == axis else s for a, s in enumerate(acc.shape))
            acc = self._add("concatenate", acc.dtype, shape, (acc, v), (axis,))
        return acc

    def gather(self, params: Value, indices: Value, axis) -> Value:
        if params.rank < 1:
            raise ValueError("gather params must be a concrete tensor of rank at least one")
        if indices.dtype not in INT_DTYPES:
            raise TypeError("gather indices must have i32 or i64 dtype")
        if not 0 <= axis < params.rank:
            raise ValueError("gather axis out of range")
        shape = params.shape[:axis] + indices.shape + params.shape[axis + 1:]
        return self._add("gather", params.dtype, shape, (params, indices), (axis,))

    def scatter_add(self, base: Value, indices: Value, updates: Value, axis) -> Value:
        if base.rank < 1:
            raise ValueError("scatter_add base must be a concrete tensor of rank at least one")
        if base.dtype == "bool":
            raise TypeError("scatter_add base must have a numeric dtype")
        if indices.dtype not in INT_DTYPES:
            raise TypeError("scatter_add indices must have concrete i32 or i64 type")
        if not 0 <= axis < base.rank:
            raise ValueError("scatter_add axis out of range")
        want = base.shape[:axis] + indices.shape + base.shape[axis + 1:]
        if updates.shape != want or updates.dtype != base.dtype:
            raise TypeError("scatter_add updates shape/dtype does not match base, indices and axis")
        return self._add("scatter_add", base.dtype, base.shape, (base, indices, updates), (axis,))

    # -- descriptor -------------------------------------------------------
    def descriptor(self, outputs):
        return Descriptor(self, [o.id if isinstance(o, Value) else int(o) for o in outputs])


for _op in BINARY:
    setattr(Graph, _op, (lambda op: lambda self, x, y: self._binary(op, x, y))(_op))
for _op in UNARY:
    setattr(Graph, _op, (lambda op: lambda self, x: self._unary(op, x))(_op))
for _op in REDUCTIONS:
    setattr(Graph, _op, (lambda op: lambda self, x, axes: self._reduce(op, x, axes))(_op))
Graph.argmax = lambda self, x, axis: self._argreduce("argmax", x, axis)
Graph.argmin = lambda self, x, axis: self._argreduce("argmin", x, axis)


# ------------------------------------------------------- C ABI structures ---
class CNode(ctypes.Structure):
    _fields_ = [("opcode", ctypes.c_int32), ("dtype", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("num_operands", ctypes.c_int32), ("shape", ctypes.c_int64 * MAX_RANK),
                ("operands", ctypes.c_int32 * 3), ("num_attrs", ctypes.c_int32),
                ("attrs", ctypes.c_int64 * MAX_ATTRS), ("predicate", ctypes.c_int32),
                ("reserved", ctypes.c_int32), ("constant_bits", ctypes.c_uint64)]


class CPartition(ctypes.Structure):
    _fields_ = [("abi_version", ctypes.c_int32), ("num_nodes", ctypes.c_int32),
                ("nodes", ctypes.POINTER(CNode)), ("num_outputs", ctypes.c_int32),
                ("outputs", ctypes.POINTER(ctypes.c_int32))]


ABI_VERSION = 5


class Descriptor:
    """Keeps the ctypes arrays alive for as long as the descriptor is used."""

    def __init__(self, graph: Graph, outputs):
        self.graph = graph
        self.outputs = list(outputs)
        n = len(graph.nodes)
        self._nodes = (CNode * max(1, n))()
        for i, node in enumerate(graph.nodes):
            c = self._nodes[i]
            c.opcode = OP[node.op]
            c.dtype = DTYPE_CODE[node.dtype]
            c.rank = len(node.shape)
            for k, s in enumerate(node.shape):
                c.shape[k] = s
            c.num_operands = len(node.operands)
            for k, a in enumerate(node.operands):
                c.operands[k] = a
            c.num_attrs = len(node.attrs)
            for k, a in enumerate(node.attrs):
                c.attrs[k] = a
            c.predicate = node.predicate
            c.constant_bits = node.bits
        self._outputs = (ctypes.c_int32 * max(1, len(self.outputs)))(*self.outputs)
        self.struct = CPartition(ABI_VERSION, n, self._nodes, len(self.outputs), self._outputs)

    def input_types(self):
        ports = {}
        for node in self.graph.nodes:
            if node.op == "parameter":
                ports[node.attrs[0]] = (node.dtype, node.shape)
        return [ports[i] for i in range(len(ports))]

    def output_types(self):
        return [(self.graph.nodes[o].dtype, self.graph.nodes[o].shape) for o in self.outputs]

    def key(self):
        """Structural key: equal for structurally identical partitions."""
        parts = []
        for n in self.graph.nodes:
            parts.append((n.op, n.dtype, n.shape, n.operands, n.attrs, n.predicate, n.bits))
        return (tuple(parts), tuple(self.outputs))


def struct_pack_f32(value) -> int:
    return struct.unpack("<I", struct.pack("<f", value))[0]
