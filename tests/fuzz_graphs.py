"""Seeded random partitions for the planner and the kernels.

Each graph draws one to three leaf tensors (f32 or i32; bf16 instead of f32 for
seeds from 1000 on, a range of its own so earlier seeds keep their graphs), then
a random mix of continuous
elementwise chains, broadcasts and transposes, slices / pads / concatenations,
selects on comparisons of leaf values, and row, column, whole-tensor and arg
reductions. Its outputs mix element, row and scalar results. Values stay in
ranges where the f32 results are well conditioned: no discontinuous function
(floor, mod, comparisons) is applied to a computed float, so last-ulp
differences of the transcendentals cannot flip a result.
"""
from __future__ import annotations

import numpy as np

import fugatensor_b200 as ft
from fugatensor_b200 import ir
from fugatensor_b200 import workloads as W


def _leaf_shapes(rng):
    rank = int(rng.integers(1, 4))
    dims = [int(rng.choice([1, 3, 7, 16, 33, 64, 129, 256, 1000])) for _ in range(rank)]
    if np.prod(dims) > 300_000:
        dims[-1] = 64
    return tuple(dims)


def build(seed):
    """(graph, outputs, input arrays) for one seeded random partition."""
    rng = np.random.default_rng(seed)
    g = ir.Graph()
    shape = _leaf_shapes(rng)
    arrays, vals = [], []
    kind = "i32" if rng.random() < 0.2 else "f32"
    if kind == "f32" and seed >= 1000:
        kind = "bf16"
    fl = kind in ("f32", "bf16")
    for _ in range(int(rng.integers(1, 4))):
        if kind == "i32":
            a = rng.integers(-50, 50, shape, dtype=np.int32)
        else:
            a = (rng.standard_normal(shape) * rng.choice([0.5, 1.0, 3.0])).astype(np.float32)
            if kind == "bf16":
                a = W.f32_to_bf16_bits(a)
        arrays.append(a)
        vals.append(g.parameter(kind, shape))
    leaves = list(vals)
    pool = list(vals)

    def pick():
        return pool[int(rng.integers(len(pool)))]

    def same_shape(v, w):
        return v.shape == w.shape

    for _ in range(int(rng.integers(3, 12))):
        x = pick()
        op = rng.choice(["add", "mul", "max", "min", "unary", "select", "bcast", "transpose", "slice", "pad",
                         "concat"])
        y = pick()
        if op in ("add", "mul", "max", "min") and same_shape(x, y) and x.dtype == y.dtype:
            name = {"add": "add", "mul": "mul", "max": "maximum", "min": "minimum"}[op]
            if op == "mul" and fl:
                # keep products bounded
                y = g.tanh(y)
            pool.append(getattr(g, name)(x, y))
        elif op == "unary" and x.dtype in ("f32", "bf16"):
            u = rng.choice(["tanh", "exp_tanh", "abs", "square", "sqrt_abs", "neg"])
            if u == "tanh":
                pool.append(g.tanh(x))
            elif u == "exp_tanh":
                pool.append(g.exp(g.tanh(x)))
            elif u == "abs":
                pool.append(g.abs(x))
            elif u == "square":
                t = g.tanh(x)
                pool.append(g.mul(t, t))
            elif u == "sqrt_abs":
                pool.append(g.sqrt(g.add(g.abs(x), g.filled(1.0, x.dtype, x.shape))))
            else:
                pool.append(g.mul(x, g.filled(-1.0, x.dtype, x.shape)))
        elif op == "select" and len(leaves) >= 2 and same_shape(x, leaves[0]) and x.dtype == leaves[0].dtype:
            c = g.compare(leaves[0], leaves[-1], rng.choice(["gt", "le", "eq"]))
            y2 = y if same_shape(y, x) and y.dtype == x.dtype else x
            pool.append(g.select(c, x, y2))
        elif op == "bcast" and x.rank < 3:
            pos = int(rng.integers(0, x.rank + 1))
            ext = int(rng.choice([2, 5, 32]))
            new_shape = x.shape[:pos] + (ext,) + x.shape[pos:]
            dims = tuple(d if d < pos else d + 1 for d in range(x.rank))
            if np.prod(new_shape) <= 400_000:
                pool.append(g.broadcast_in_dim(x, new_shape, dims))
        elif op == "transpose" and x.rank >= 2:
            perm = tuple(int(p) for p in rng.permutation(x.rank))
            pool.append(g.transpose(x, perm))
        elif op == "slice" and x.rank >= 1:
            starts, stops, steps = [], [], []
            for d in x.shape:
                step = int(rng.choice([1, 1, 2, -1]))
                if step > 0:
                    st = int(rng.integers(0, max(1, d // 3) + 1))
                    starts.append(min(st, d - 1) if d > 0 else 0)
                    stops.append(d)
                else:
                    starts.append(d - 1)
                    stops.append(-1)
                steps.append(step)
            pool.append(g.slice(x, starts, stops, steps))
        elif op == "pad" and x.rank >= 1 and np.prod(x.shape) < 200_000:
            lo = tuple(int(rng.integers(0, 3)) for _ in x.shape)
            hi = tuple(int(rng.integers(0, 3)) for _ in x.shape)
            inner = tuple(int(rng.integers(0, 2)) if d < 100 else 0 for d in x.shape)
            pv = g.constant(0.5 if x.dtype in ("f32", "bf16") else 7, x.dtype)
            pool.append(g.pad(x, pv, lo, hi, inner))
        elif op == "concat" and x.rank >= 1:
            ax = int(rng.integers(0, x.rank))
            parts = [p for p in pool if p.dtype == x.dtype and p.rank == x.rank
                     and all(a == ax or p.shape[a] == x.shape[a] for a in range(x.rank))]
            if len(parts) >= 2:
                chosen = [parts[int(i)] for i in rng.choice(len(parts), size=2, replace=False)]
                if sum(np.prod(p.shape) for p in chosen) <= 400_000:
                    pool.append(g.concatenate(chosen, ax))
    outs = []
    last = pool[-1]
    outs.append(last)
    for v in rng.permutation(len(pool))[:3]:
        x = pool[int(v)]
        if x.rank == 0:
            continue
        r = rng.choice(["sum_last", "sum_first", "max_last", "argmax", "full_sum", "mean_last", "min_mid"])
        if r == "sum_last":
            outs.append(g.reduce_sum(x, (x.rank - 1,)))
        elif r == "sum_first":
            outs.append(g.reduce_sum(x, (0,)))
        elif r == "max_last" and all(s > 0 for s in x.shape):
            outs.append(g.reduce_max(x, (x.rank - 1,)))
        elif r == "argmax" and all(s > 0 for s in x.shape):
            outs.append(g.argmax(x, int(rng.integers(0, x.rank))))
        elif r == "full_sum":
            outs.append(g.reduce_sum(x, tuple(range(x.rank))))
        elif r == "mean_last" and x.dtype in ("f32", "bf16") and x.shape[-1] > 0:
            s = g.reduce_sum(x, (x.rank - 1,))
            outs.append(g.div(s, g.filled(float(x.shape[-1]), x.dtype, s.shape)))
        elif r == "min_mid" and x.rank >= 2 and all(s > 0 for s in x.shape):
            outs.append(g.reduce_min(x, (x.rank // 2,)))
    return g, outs, arrays
