"""GPU parity of the index-transform partitions against the CPU oracle at mid sizes:
slices with every step sign, pads with interior dilation, concatenation, gather with
out-of-range indices, scatter_add with duplicates, and fusions of them with row
reductions (a softmax over a padded row, a gather feeding a row sum)."""
import numpy as np
import pytest

import fugatensor_b200 as ft
import fugatensor_b200.nn.functional as F
import oracle as O
from tests._util import assert_matches

pytestmark = pytest.mark.gpu


def _check(outs, arrays, dtype="f32"):
    eng = outs[0].engine
    desc, leaves, roots = eng.trace(*outs)
    ref = O.evaluate(desc, [arrays[id(l)] for l in leaves])
    ft.evaluate(*outs)
    for o, r in zip(outs, ref):
        got = o.numpy()
        if o.dtype.ir in ("i32", "i64", "bool"):
            assert np.array_equal(got, r)
        else:
            assert_matches(got, r, o.dtype.ir, what=o._expr[0] if o._expr else "output")


def _inputs(rng, rows, cols):
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    return x, ft.tensor(x)


@pytest.mark.parametrize("rows,cols", [(7, 33), (256, 1024), (1000, 4096)])
def test_slices_pads_concat(rows, cols):
    rng = np.random.default_rng(rows)
    x, X = _inputs(rng, rows, cols)
    y, Y = _inputs(rng, rows, cols)
    outs = [X[::-1, 1::3], X[1:-1:2, ::-2] * 2.0, ft.pad(X, ((2, 1), (0, 3)), constant_value=0.5),
            ft.pad(X[:, :cols // 2], ((0, 0), (1, 1)), interior=(0, 2)), ft.cat([X, Y, X[:, :5]], axis=1),
            ft.cat([X[: rows // 2], Y], axis=0), ft.stack([X[:, 0], Y[:, -1]], axis=0)]
    _check(outs, {id(X): x, id(Y): y})


@pytest.mark.parametrize("rows,cols", [(64, 100), (4096, 512)])
def test_gather_rows_and_columns(rows, cols):
    rng = np.random.default_rng(7)
    x, X = _inputs(rng, rows, cols)
    ri = rng.integers(-3, rows + 3, 333).astype(np.int64)
    ci = rng.integers(-2, cols + 2, (5, 7)).astype(np.int32)
    RI, CI = ft.tensor(ri, dtype=ft.int64), ft.tensor(ci, dtype=ft.int32)
    outs = [ft.gather(X, RI, axis=0), ft.gather(X, CI, axis=1), X[RI, 2:9] + 1.0, ft.gather(X.exp(), RI, 0).sum(axis=1)]
    _check(outs, {id(X): x, id(RI): ri, id(CI): ci})


@pytest.mark.parametrize("rows,cols,n", [(512, 96, 4000), (1021, 33, 3000), (70001, 8, 50000), (65536, 64, 131072)])
@pytest.mark.parametrize("dtype", ["f32", "bf16", "i32", "i64"])
def test_scatter_add_random(dtype, rows, cols, n):
    """Row scatter_add (the bucket-list form) against the oracle: duplicate and
    out-of-range indices, odd row counts, more rows than one scan step, and
    more vector chunks than the grid has threads (each thread walks several
    rows' lists in its grid-stride loop, with the next list head read ahead)."""
    rng = np.random.default_rng(11 + rows)
    idx = rng.integers(-5, rows + 5, n).astype(np.int32)
    if dtype in ("i32", "i64"):
        base = rng.integers(-1000, 1000, (rows, cols)).astype(np.int32 if dtype == "i32" else np.int64)
        upd = rng.integers(-1000, 1000, (n, cols)).astype(base.dtype)
        B, U = ft.tensor(base, dtype=getattr(ft, {"i32": "int32", "i64": "int64"}[dtype])), None
        U = ft.tensor(upd, dtype=B.dtype)
        arrays = {id(B): base, id(U): upd}
    else:
        base = rng.standard_normal((rows, cols)).astype(np.float32)
        upd = rng.standard_normal((n, cols)).astype(np.float32)
        if dtype == "bf16":
            base, upd = O.f32_to_bf16_bits(base), O.f32_to_bf16_bits(upd)
        B = ft.tensor(base, dtype=ft.bf16 if dtype == "bf16" else ft.fp32)
        U = ft.tensor(upd, dtype=B.dtype)
        arrays = {id(B): base, id(U): upd}
    I = ft.tensor(idx, dtype=ft.int32)
    arrays[id(I)] = idx
    out = ft.scatter_add(B, I, U, axis=0)
    eng = out.engine
    desc, leaves, roots = eng.trace(out)
    (ref,) = O.evaluate(desc, [arrays[id(l)] for l in leaves])
    ft.evaluate(out)
    got = out.numpy()
    if dtype in ("i32", "i64"):
        assert np.array_equal(got, ref)
    else:
        if dtype == "bf16":
            got, ref = O.bf16_bits_to_f32(got), O.bf16_bits_to_f32(ref)
        assert_matches(got, ref, dtype)


def test_index_ops_fuse_with_row_reductions():
    """A softmax over a padded / concatenated row and a row sum of gathered columns."""
    rng = np.random.default_rng(5)
    rows, cols = 300, 2000
    x, X = _inputs(rng, rows, cols)
    ci = rng.integers(0, cols, 1500).astype(np.int64)
    CI = ft.tensor(ci, dtype=ft.int64)
    padded = ft.pad(X, ((0, 0), (3, 5)), constant_value=-1e30)
    outs = [F.softmax(padded, axis=-1), F.softmax(ft.cat([X, X[:, ::-1]], axis=1), axis=-1),
            ft.gather(X, CI, axis=1).sum(axis=1)]
    _check(outs, {id(X): x, id(CI): ci})


def test_index_op_gradients_match_oracle():
    rng = np.random.default_rng(9)
    x, X = _inputs(rng, 64, 256)
    ri = rng.integers(0, 64, 100).astype(np.int64)
    RI = ft.tensor(ri, dtype=ft.int64)
    loss = (ft.pad(X[::2, 1::3], ((1, 1), (2, 0)), constant_value=0.25) ** 2).sum() + ft.gather(X, RI, 0).sum()
    (gx,) = ft.grad(loss, (X,))
    _check([gx], {id(X): x, id(RI): ri})
