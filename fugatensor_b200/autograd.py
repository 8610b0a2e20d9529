"""Reverse-mode derivatives as lazy tensors (reference: src/fugatensor/autograd.py:204-239).

``grad`` walks the pending expression graph of the outputs, applies Fuga's
primitive VJP rules (reference: src/fugatensor/ir/tensor_rules.py:270-482,
src/fugatensor/ir/primitives.py:88-115, cotangent accumulation by ``add`` as
in src/fugatensor/ir/differentiate.py:92-160) and returns ordinary pending
tensors. Nothing executes here: the derivative graph reaches the backend as
ordinary partitions, evaluated together with the forward when requested
together.
"""
from __future__ import annotations

import builtins as _builtins
import math

from . import dtypes as _dt
from .tensor import Tensor, _prim

FLOAT = ("f32", "f16", "bf16")
_builtins_any = _builtins.any


class DifferentiationError(RuntimeError):
    pass


def _filled(like_dtype, shape, value, engine):
    return engine._splat(value, like_dtype, shape)


def _neg(v):
    return _prim("mul", (v, _filled(v.dtype, v.shape, -1, v.engine)))


def _restore(value, dtype, shape):
    if value.shape == shape:
        return value
    if value.shape == ():
        return _prim("splat", (value,), (shape,))
    return value.reshape(shape)


def _expand_reduction(value, in_shape, axes):
    if in_shape == ():
        return value
    dims = tuple(a for a in range(len(in_shape)) if a not in axes)
    if value.shape == in_shape and dims == tuple(range(len(in_shape))):
        return value
    return _prim("broadcast_in_dim", (value,), (tuple(in_shape), dims))


def _unary_factor(op, x):
    e = x.engine
    if op == "exp":
        return _prim("exp", (x,))
    if op == "log":
        return _prim("div", (_filled(x.dtype, x.shape, 1, e), x))
    if op == "sin":
        return _prim("cos", (x,))
    if op == "cos":
        return _neg(_prim("sin", (x,)))
    if op == "tanh":
        t = _prim("tanh", (x,))
        return _prim("add", (_filled(x.dtype, x.shape, 1, e), _neg(_prim("mul", (t, t)))))
    if op == "erf":
        scale = _filled(x.dtype, x.shape, 2.0 / math.sqrt(math.pi), e)
        return _prim("mul", (scale, _prim("exp", (_neg(_prim("mul", (x, x))),))))
    # sqrt
    return _prim("div", (_filled(x.dtype, x.shape, 0.5, e), _prim("sqrt", (x,))))


def _extremum_weights(x, axes, is_max):
    e = x.engine
    ext = _prim("reduce_max" if is_max else "reduce_min", (x,), (axes,))
    ext = _expand_reduction(ext, x.shape, axes)
    mask = _prim("compare", (x, ext), ("eq",))
    maskf = mask.astype(_dt.fp32)
    counts = _expand_reduction(_prim("reduce_sum", (maskf,), (axes,)), x.shape, axes)
    weight = _prim("div", (maskf, counts)).astype(x.dtype)
    isnan = _prim("compare", (ext, ext), ("ne",))
    return _prim("select", (isnan, _filled(x.dtype, x.shape, float("nan"), e), weight))


def _abs_sign(x):
    e = x.engine
    zero, one, neg_one = (_filled(x.dtype, x.shape, v, e) for v in (0, 1, -1))
    sign = _prim("select", (_prim("compare", (x, zero), ("gt",)), one,
                            _prim("select", (_prim("compare", (x, zero), ("lt",)), neg_one, zero))))
    return _prim("select", (_prim("compare", (x, x), ("ne",)), x, sign))


def _vjp(t, g, active):
    """Cotangents of t's operands given t's cotangent g (None where inactive)."""
    op, args, attrs = t._expr
    e = t.engine
    if op == "add":
        return [g if a else None for a in active]
    if op == "mul":
        return [_prim("mul", (g, args[1])) if active[0] else None, _prim("mul", (g, args[0])) if active[1] else None]
    if op == "div":
        q = _prim("div", (args[0], args[1])) if active[1] else None
        return [_prim("div", (g, args[1])) if active[0] else None,
                _neg(_prim("div", (_prim("mul", (g, q)), args[1]))) if active[1] else None]
    if op in ("exp", "log", "sqrt", "sin", "cos", "tanh", "erf"):
        return [_prim("mul", (g, _unary_factor(op, args[0])))]
    if op == "abs":
        if args[0].dtype.ir not in FLOAT:
            return [None]
        return [_prim("mul", (g, _abs_sign(args[0])))]
    if op == "cast":
        src = args[0].dtype
        if src.ir not in FLOAT or t.dtype.ir not in FLOAT:
            raise DifferentiationError("integer/bool casts on a derivative path have no floating VJP rule")
        return [g.astype(src)]
    if op == "reshape":
        return [g.reshape(args[0].shape)]
    if op == "stop_gradient":
        return [None]
    if op == "broadcast_in_dim":
        src, target = args[0].shape, g.shape
        dims = attrs[1]
        expanded = {d for s, d in zip(src, dims) if s == 1 and target[d] != 1}
        axes = tuple(a for a in range(len(target)) if a not in dims or a in expanded)
        reduced = _prim("reduce_sum", (g,), (axes,))
        return [_restore(reduced, args[0].dtype, src)]
    if op == "transpose":
        perm = attrs[0]
        inverse = tuple(perm.index(a) for a in range(len(perm)))
        return [_prim("transpose", (g,), (inverse,))]
    if op == "splat":
        return [_prim("reduce_sum", (g,), (tuple(range(g.ndim)),)) if g.ndim else g]
    if op == "reduce_sum":
        return [_expand_reduction(g, args[0].shape, attrs[0])]
    if op in ("reduce_max", "reduce_min"):
        w = _extremum_weights(args[0], attrs[0], op == "reduce_max")
        return [_prim("mul", (w, _expand_reduction(g, args[0].shape, attrs[0])))]
    if op == "select":
        zero = _filled(g.dtype, g.shape, 0, e)
        return [None, _prim("select", (args[0], g, zero)) if active[1] else None,
                _prim("select", (args[0], zero, g)) if active[2] else None]
    if op in ("maximum", "minimum"):
        x, y = args
        if x.dtype.ir not in FLOAT:
            return [None, None]
        is_max = op == "maximum"
        zero = _filled(g.dtype, g.shape, 0, e)
        half_g = _prim("mul", (g, _filled(g.dtype, g.shape, 0.5, e)))
        xnan = _prim("compare", (x, x), ("ne",))
        either_nan = _prim("bitwise_or", (xnan, _prim("compare", (y, y), ("ne",))))
        nan_val = _prim("select", (xnan, x, y))
        eq = _prim("compare", (x, y), ("eq",))
        win_x = _prim("compare", (x, y), ("gt" if is_max else "lt",))
        win_y = _prim("compare", (y, x), ("gt" if is_max else "lt",))
        dx = _prim("select", (either_nan, nan_val, _prim("select", (win_x, g, _prim("select", (eq, half_g, zero))))))
        dy = _prim("select", (either_nan, nan_val, _prim("select", (win_y, g, _prim("select", (eq, half_g, zero))))))
        return [dx if active[0] else None, dy if active[1] else None]
    if op == "pow":
        x, y = args
        if x.dtype.ir not in FLOAT:
            return [None, None]
        zero, one = _filled(x.dtype, x.shape, 0, e), _filled(x.dtype, x.shape, 1, e)
        dx = dy = None
        if active[0]:
            y_is_zero = _prim("compare", (y, zero), ("eq",))
            safe = _prim("add", (_prim("select", (y_is_zero, one, y)), _filled(y.dtype, y.shape, -1, e)))
            fx = _prim("select", (y_is_zero, zero, _prim("mul", (y, _prim("pow", (x, safe))))))
            dx = _prim("mul", (g, fx))
        if active[1]:
            x_pos = _prim("compare", (x, zero), ("gt",))
            safe_x = _prim("select", (x_pos, x, one))
            fy = _prim("select", (x_pos, _prim("mul", (_prim("pow", (x, y)), _prim("log", (safe_x,)))), zero))
            dy = _prim("mul", (g, fy))
        return [dx, dy]
    if op == "mod":
        x, y = args
        if x.dtype.ir not in FLOAT:
            return [None, None]
        return [g if active[0] else None,
                _neg(_prim("mul", (g, _prim("floordiv", (x, y))))) if active[1] else None]
    # index transforms (src/fugatensor/ir/tensor_rules.py:521-640)
    if op == "slice":
        x = args[0]
        if x.dtype.ir not in FLOAT:
            return [None]
        starts, _, steps = attrs
        out = t.shape
        if 0 in out:
            return [_filled(x.dtype, x.shape, 0, e)]
        if _builtins_any(st < 0 for st in steps):
            # reverse the cotangent along the reversed axes first
            g = _prim("slice", (g,), (tuple(n - 1 if st < 0 else 0 for n, st in zip(out, steps)),
                                     tuple(-1 if st < 0 else n for n, st in zip(out, steps)),
                                     tuple(-1 if st < 0 else 1 for st in steps)))
        low, high, inner = [], [], []
        for dim, n, st0, step in zip(x.shape, out, starts, steps):
            first = st0 if step > 0 else st0 + (n - 1) * step
            low.append(first)
            inner.append(abs(step) - 1)
            high.append(dim - 1 - (first + (n - 1) * abs(step)))
        zero = _filled(x.dtype, (), 0, e)
        return [_prim("pad", (g, zero), (tuple(low), tuple(high), tuple(inner)))]
    if op == "pad":
        x, pv = args
        if x.dtype.ir not in FLOAT:
            return [None, None]
        low, _, inner = attrs
        dx = dpv = None
        if active[0]:
            starts = tuple(l if d > 0 else 0 for d, l in zip(x.shape, low))
            stops = tuple(l + (d - 1) * (i + 1) + 1 if d > 0 else 0 for d, l, i in zip(x.shape, low, inner))
            steps = tuple(i + 1 for i in inner)
            dx = _prim("slice", (g,), (starts, stops, steps)) if x.ndim else g
        if active[1]:
            mask = _prim("pad", (_filled(x.dtype, x.shape, 0, e), _filled(x.dtype, (), 1, e)), attrs)
            dpv = _prim("reduce_sum", (_prim("mul", (g, mask)),), (tuple(range(g.ndim)),)) if g.ndim else g
        return [dx, dpv]
    if op == "concatenate":
        if args[0].dtype.ir not in FLOAT:
            return [None] * len(args)
        ax = attrs[0]
        out, at = [], 0
        for a, act in zip(args, active):
            n = a.shape[ax]
            if act:
                starts = tuple(at if k == ax else 0 for k in range(g.ndim))
                stops = tuple(at + n if k == ax else s for k, s in enumerate(g.shape))
                out.append(_prim("slice", (g,), (starts, stops, (1,) * g.ndim)) if n else _filled(a.dtype, a.shape, 0, e))
            else:
                out.append(None)
            at += n
        return out
    if op == "gather":
        p, ix = args
        if not active[0] or p.dtype.ir not in FLOAT:
            return [None, None]
        return [_prim("scatter_add", (_filled(p.dtype, p.shape, 0, e), ix, g), (attrs[0],)), None]
    if op == "scatter_add":
        if args[0].dtype.ir not in FLOAT:
            return [None, None, None]
        return [g if active[0] else None, None, _prim("gather", (g, args[1]), (attrs[0],)) if active[2] else None]
    # compare, argmax/argmin, iota, constant, floor/ceil/round, bitwise...: zero derivative
    if op in ("floor", "ceil", "round"):
        return [None]
    return [None] * len(args)


def _topo(outputs):
    order, seen = [], set()
    stack = [(o, False) for o in outputs]
    while stack:
        t, done = stack.pop()
        if done:
            order.append(t)
            continue
        if id(t) in seen:
            continue
        seen.add(id(t))
        stack.append((t, True))
        if t._expr is not None:
            for a in t._expr[1]:
                if id(a) not in seen:
                    stack.append((a, False))
    return order


_NONDIFF = ("compare", "argmax", "argmin", "iota", "constant", "stop_gradient", "floor", "ceil", "round",
            "bitwise_and", "bitwise_or", "bitwise_xor", "bitwise_not", "shift_left", "shift_right",
            "reduce_any", "reduce_all", "floordiv")


def grad(outputs, inputs, *, seed=None):
    """Lazy vector-Jacobian product of ``outputs`` w.r.t. ``inputs``.

    Scalar outputs default to unit seeds; nonscalar outputs require matching
    explicit seeds. Disconnected inputs get zeros. A Tensor input returns one
    Tensor, a tuple/list returns a tuple.
    """
    single_out = isinstance(outputs, Tensor)
    outs = [outputs] if single_out else list(outputs)
    single_in = isinstance(inputs, Tensor)
    ins = [inputs] if single_in else list(inputs)
    for v in (*outs, *ins):
        if not isinstance(v, Tensor):
            raise TypeError("grad outputs and inputs must be Tensors")
        if v.dtype.ir not in FLOAT:
            raise TypeError("grad outputs and inputs must have floating dtype")
    if seed is None:
        seeds = [None] * len(outs)
    elif isinstance(seed, Tensor):
        seeds = [seed]
    else:
        seeds = list(seed)
    if len(seeds) != len(outs):
        raise ValueError("one seed per output is required")
    resolved = []
    for o, s in zip(outs, seeds):
        if s is None:
            if o.shape != ():
                raise ValueError("nonscalar outputs require an explicit seed")
            s = o.engine._splat(1, o.dtype, ())
        if s.shape != o.shape or s.dtype is not o.dtype:
            raise ValueError("seed must match its output's shape and dtype")
        resolved.append(s)

    order = _topo(outs)
    in_ids = {id(t) for t in ins}
    # activity: depends (differentiably) on a requested input
    active = {}
    for t in order:
        if id(t) in in_ids:
            active[id(t)] = True
            continue
        if t._expr is None or t.dtype.ir not in FLOAT:
            active[id(t)] = False
            continue
        op, args, _ = t._expr
        active[id(t)] = op not in _NONDIFF and any(active.get(id(a), False) for a in args)

    adj = {}

    def contribute(t, g):
        if not active.get(id(t), False):
            return
        adj[id(t)] = _prim("add", (adj[id(t)], g)) if id(t) in adj else g

    for o, s in zip(outs, resolved):
        contribute(o, s)
    for t in reversed(order):
        g = adj.get(id(t))
        if g is None or t._expr is None or id(t) in in_ids and t._expr is None:
            continue
        op, args, _ = t._expr
        if op in _NONDIFF:
            continue
        flags = [active.get(id(a), False) for a in args]
        if not any(flags):
            continue
        for a, ga in zip(args, _vjp(t, g, flags)):
            if ga is not None:
                contribute(a, ga)
    from .ops import zeros_like
    result = tuple(adj[id(t)] if id(t) in adj else zeros_like(t) for t in ins)
    return result[0] if single_in else result


def stop_gradient(tensor):
    if not isinstance(tensor, Tensor):
        raise TypeError("stop_gradient expects a Tensor")
    return tensor.detach()
