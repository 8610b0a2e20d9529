"""The reference's own known-answer tests for this path, through the public API.

Each case restates an assertion of the reference test suite (file:line in the
test's docstring) and runs on two backends: the CPU oracle (pins the oracle
to the reference's goldens; runs everywhere) and the GPU backend (marked
gpu; the parity check proper).
"""
import math
import struct

import numpy as np
import pytest

import fugatensor_b200 as ft
import fugatensor_b200.nn.functional as F
import oracle as O

BACKENDS = [pytest.param("oracle", id="oracle"), pytest.param("gpu", id="gpu", marks=pytest.mark.gpu)]
FLOATS = ("fp32", "fp16", "bf16")


@pytest.fixture(params=BACKENDS)
def backend(request):
    return request.param


def _host(t):
    data = t._data
    if t.dtype is ft.bf16:
        return data.view(__import__("torch").int16).cpu().numpy().view(np.uint16)
    return data.cpu().numpy()


def run(backend, *outs, accumulation="wide"):
    """Evaluate outputs; numeric numpy results (bf16 decoded to float)."""
    eng = outs[0].engine
    if backend == "oracle":
        desc, leaves, roots = eng.trace(*outs)
        mode = O.LITERAL if accumulation == "storage" else O.ACCURATE
        res = O.evaluate(desc, [_host(l) for l in leaves], mode)
        return [O.bf16_bits_to_f32(r) if o.dtype is ft.bf16 else r for r, o in zip(res, outs)]
    eng.accumulation = accumulation
    try:
        eng.clear_cache()
        ft.evaluate(*outs)
    finally:
        eng.accumulation = "wide"
        eng.clear_cache()
    return [O.bf16_bits_to_f32(o.numpy()) if o.dtype is ft.bf16 else o.numpy() for o in outs]


def T(data, dtype=ft.fp32):
    return ft.tensor(data, dtype=getattr(ft, dtype) if isinstance(dtype, str) else dtype)


def close(got, want, tol):
    got = np.asarray(got, dtype=np.float64).reshape(-1)
    want = np.asarray(want, dtype=np.float64).reshape(-1)
    assert got.shape == want.shape
    for g, w in zip(got, want):
        if math.isnan(w):
            assert math.isnan(g)
        elif math.isinf(w):
            assert g == w
        else:
            assert abs(g - w) <= tol + tol * abs(w), (g, w)


def test_storage_dtype_sum_rounding(backend):
    """tests/test_tensor_primitives.py:184-192: [L, 1, -L] sums to 0 in storage dtype; fp32 accumulation gives 1."""
    large = {"fp32": 2**24, "fp16": 2**11, "bf16": 2**8}
    for name in FLOATS:
        x = T([large[name], 1, -large[name]], name)
        (s,) = run(backend, x.sum(), accumulation="storage")
        assert float(s) == 0.0
        if name != "fp32":
            (s32,) = run(backend, x.sum(dtype=ft.fp32), accumulation="storage")
            assert float(s32) == 1.0
    if backend == "gpu":
        # default (wide) policy: a whole-tensor f32 sum folds per-thread
        # partials in f64, so it is exact here (documented deviation)
        (s,) = run(backend, T([2**24, 1, -2**24]).sum())
        assert float(s) == 1.0


def test_wide_accumulation_is_exact_for_narrow_sums(backend):
    """Default policy: f16/bf16 sums accumulate in f32 and round once (documented deviation)."""
    for name, big in (("fp16", 2**11), ("bf16", 2**8)):
        (s,) = run(backend, T([big, 1, -big], name).sum())
        assert float(s) == 1.0


def test_nan_max_and_tie_averaged_gradient(backend):
    """tests/test_tensor_primitives.py:193-197."""
    for name in FLOATS:
        x = T([[1, float("nan"), 3], [2, 2, 0]], name)
        m = x.amax(axis=1)
        g = ft.grad(m, x, seed=ft.ones_like(m))
        mv, gv = run(backend, m, g)
        close(mv, [float("nan"), 2], 0)
        close(gv, [float("nan")] * 3 + [0.5, 0.5, 0], 0)


def test_log_sqrt_exceptional_values(backend):
    """tests/test_tensor_primitives.py:198-200."""
    for name in FLOATS:
        x = T([0, -1, float("inf")], name)
        lv, sv = run(backend, ft.log(x), ft.sqrt(x))
        close(lv, [-math.inf, math.nan, math.inf], 0)
        close(sv, [0, math.nan, math.inf], 0)


def test_integer_sums_wrap(backend):
    """tests/test_tensor_primitives.py:201-204."""
    for dt, width in ((ft.int32, 32), (ft.int64, 64)):
        x = ft.tensor([2 ** (width - 1) - 1, 1], dtype=dt)
        (s,) = run(backend, x.sum())
        assert int(s) == -2 ** (width - 1)


def test_f32_division_rounds_once(backend):
    """tests/test_tensor_primitives.py:205-207."""
    (q,) = run(backend, T([7]) / T([3]))
    assert float(q[0]) == struct.unpack("<f", struct.pack("<f", 7 / 3))[0]


def test_softmax_probabilities(backend):
    """tests/test_tensor_primitives.py:208-217 (explicit max-shift composition)."""
    x = T([[1, 2, 3], [2, 3, 4]])
    shifted = x - ft.broadcast_to(x.amax(axis=1, keepdims=True), x.shape)
    num = ft.exp(shifted)
    p = num / ft.broadcast_to(num.sum(axis=1, keepdims=True), x.shape)
    (pv,) = run(backend, p)
    expected = [math.exp(v) / sum(math.exp(u) for u in (1, 2, 3)) for v in (1, 2, 3)] * 2
    close(pv, expected, 2e-6)


def test_elementary_values_and_gradients(backend):
    """tests/test_tensor_primitives.py:126-146: exp/log/sqrt/div values, first and second derivatives."""
    cases = (
        (ft.exp, math.exp, math.exp, math.exp),
        (ft.log, math.log, lambda x: 1 / x, lambda x: -1 / (x * x)),
        (ft.sqrt, math.sqrt, lambda x: 0.5 / math.sqrt(x), lambda x: -0.25 / x ** 1.5),
        (lambda x: x / (x + 1), lambda x: x / (x + 1), lambda x: 1 / (x + 1) ** 2, lambda x: -2 / (x + 1) ** 3),
    )
    data = [0.5, 1, 2]
    for name in FLOATS:
        tol = {"fp32": 2e-5, "fp16": 0.003, "bf16": 0.015}[name]
        for fn, ref, d1, d2 in cases:
            x = T(data, name)
            y = fn(x)
            dx = ft.grad(y, x, seed=ft.ones_like(y))
            ddx = ft.grad(dx, x, seed=ft.ones_like(dx))
            yv, dv, ddv = run(backend, y, dx, ddx)
            for got, oracle_fn in ((yv, ref), (dv, d1), (ddv, d2)):
                want = [oracle_fn(v) for v in data]
                for g, w in zip(np.asarray(got, dtype=np.float64), want):
                    assert abs(g - w) <= tol * max(1.0, abs(w)), (name, g, w)


def test_composed_views(backend):
    """tests/test_tensor_primitives.py:160-163: transpose of a broadcast, log(exp), where."""
    x = T([[0.25, 0.5, 1]])
    mapped = ft.transpose(ft.broadcast_in_dim(x, (2, 1, 3), (1, 2)), (2, 0, 1))
    y = ft.where(mapped > 0, ft.log(ft.exp(mapped)) / ft.sqrt(mapped + 1), mapped)
    (yv,) = run(backend, y)
    assert yv.shape == (3, 2, 1)
    close(yv, [v / math.sqrt(v + 1) for v in (0.25, 0.25, 0.5, 0.5, 1, 1)], 2e-6)


def test_broadcast_reduction_max_gradients(backend):
    """tests/test_tensor_primitives.py:165-176."""
    for name in FLOATS:
        x = T([[1, 2, 2], [3, 3, 0]], name)
        m = x.amax(axis=1)
        g = ft.grad(m, x, seed=ft.ones_like(m))
        total = ft.broadcast_in_dim(x, (4, 2, 3), (1, 2)).transpose((2, 0, 1)).sum()
        gt = ft.grad(total, x)
        gv, gtv = run(backend, g, gt)
        close(gv, [0, 0.5, 0.5, 0.5, 0.5, 0], 0)
        close(gtv, [4] * 6, 0)


def test_reductions_at_warp_boundaries(backend):
    """tests/test_stage2_ops.py:122-134: widths 1, 10, 32, 65, 300."""
    for cols in (1, 10, 32, 65, 300):
        data = [[float(((r * 17 + c * 7) % 19) - 9) * 0.25 for c in range(cols)] for r in range(3)]
        t = T(data)
        mn, mx, am, an = run(backend, t.amin(axis=1), t.amax(axis=1), t.argmax(axis=1), t.argmin(axis=1))
        close(mn, [min(r) for r in data], 0)
        close(mx, [max(r) for r in data], 0)
        assert list(am) == [r.index(max(r)) for r in data]
        assert list(an) == [r.index(min(r)) for r in data]
        flags_any = [[c == cols - 1 if r == 0 else False for c in range(cols)] for r in range(2)]
        flags_all = [[True] * cols, [c != 0 for c in range(cols)]]
        a1, a2 = run(backend, ft.tensor(flags_any, dtype=ft.bool).any(axis=1),
                     ft.tensor(flags_all, dtype=ft.bool).all(axis=1))
        assert list(a1) == [True, False] and list(a2) == [True, False]


def test_argmax_ties_nan_and_global(backend):
    """tests/test_stage2_ops.py:148-157."""
    tie = T([[2.0, 5.0, 5.0, 1.0], [3.0, 1.0, 1.0, 3.0]])
    a, b, c, d = run(backend, tie.argmax(axis=1, keepdims=True), tie.argmin(axis=1), tie.argmax(),
                     tie.argmin(keepdims=True))
    assert a.tolist() == [[1], [0]] and b.tolist() == [3, 1] and int(c) == 1 and d.tolist() == [[3]]
    nan_row = T([1.0, float("nan"), 9.0, float("nan")])
    e, f = run(backend, nan_row.argmax(axis=0), nan_row.argmin(axis=0))
    assert int(e) == 1 and int(f) == 1


def test_products_and_empty_reductions(backend):
    """tests/test_stage2_ops.py:136-146."""
    p = T([[1.5, -2.0, 3.0], [0.5, 4.0, -1.0]])
    pr, pa = run(backend, p.prod(axis=1), p.prod())
    close(pr, [-9.0, -2.0], 1e-6)
    close([pa], [18.0], 1e-6)


def test_nn_functional_small(backend):
    """tests/test_stage2_ops.py:326-360 (2x4 case) vs the reference's pure-Python refs: the
    row graphs on this path (the case's pointwise activations are not part of it)."""
    rows = [[-2.0, -0.5, 0.0, 1.5], [1.0, -3.0, 2.0, 0.5]]
    x = T(rows)
    w = T([1.0, 2.0, 0.5, 1.5])
    b = T([0.1, -0.2, 0.3, 0.0])
    outs = run(backend, F.softmax(x, axis=1), F.log_softmax(x, axis=1), F.layer_norm(x, weight=w, bias=b),
               F.rms_norm(x, weight=w))

    def sm(r):
        m = max(r)
        e = [math.exp(v - m) for v in r]
        return [v / sum(e) for v in e]

    def lsm(r):
        m = max(r)
        lse = math.log(sum(math.exp(v - m) for v in r))
        return [v - m - lse for v in r]

    def ln(r):
        mu = sum(r) / len(r)
        var = sum((v - mu) ** 2 for v in r) / len(r)
        inv = 1 / math.sqrt(var + 1e-5)
        return [(v - mu) * inv * wi + bi for v, wi, bi in zip(r, [1, 2, 0.5, 1.5], [0.1, -0.2, 0.3, 0])]

    def rn(r):
        inv = 1 / math.sqrt(sum(v * v for v in r) / len(r) + 1e-6)
        return [v * inv * wi for v, wi in zip(r, [1, 2, 0.5, 1.5])]

    refs = ([sm(r) for r in rows], [lsm(r) for r in rows], [ln(r) for r in rows], [rn(r) for r in rows])
    tols = (1e-5, 1e-5, 1e-4, 1e-4)
    for got, want, tol in zip(outs, refs, tols):
        close(got, [v for r in want for v in r], tol)


def test_ieee_maximum_matrix(backend):
    """tests/support/reduction_max.py:25-70, tests/test_cuda_reduction_max.py:45-67: IEEE max
    over every axis set of a [7,2,W] tensor in two layouts, including NaN / signed-zero / inf rows."""
    from itertools import combinations

    def values(shape):
        out = []
        for g in range(shape[0]):
            for r in range(shape[1]):
                for c in range(shape[2]):
                    pos, count = r * shape[2] + c, shape[1] * shape[2]
                    pats = (pos % 7 - 3, math.nan if pos == 0 else -2, math.nan if pos == count - 1 else 2,
                            -0.0 if pos % 2 else 0.0, -0.0, math.inf if pos == count - 1 else 1, -math.inf)
                    out.append(float(pats[g]))
        return out

    def ieee_max(vals):
        if any(v != v for v in vals):
            return math.nan
        m = max(vals)
        if m == 0:
            return 0.0 if any(v == 0 and math.copysign(1, v) > 0 for v in vals) else -0.0
        return m

    axes_sets = [a for n in range(1, 4) for a in combinations(range(3), n)]
    for width in (1, 31, 33, 65):
        shape = (7, 2, width)
        data = values(shape)
        arr = np.array(data, dtype=np.float32).reshape(shape)
        for layout in ((0, 1, 2), (2, 0, 1)):
            phys = np.ascontiguousarray(np.transpose(arr, layout))
            stored = ft.tensor(phys)
            inverse = tuple(layout.index(a) for a in range(3))
            x = stored if layout == (0, 1, 2) else ft.transpose(stored, inverse)
            outs = [ft.amax(x, axis=a) for a in axes_sets]
            res = run(backend, *outs)
            for a, got in zip(axes_sets, res):
                rem = [d for d in range(3) if d not in a]
                want = np.empty([shape[d] for d in rem] or [1], dtype=np.float64).reshape(-1)
                moved = np.moveaxis(arr.astype(np.float64), rem + list(a), list(range(3)))
                flat = moved.reshape(int(np.prod([shape[d] for d in rem])), -1)
                for i in range(flat.shape[0]):
                    want[i] = ieee_max(list(flat[i]))
                g = np.asarray(got, dtype=np.float64).reshape(-1)
                for gi, wi in zip(g, want):
                    if math.isnan(wi):
                        assert math.isnan(gi)
                    else:
                        assert gi == wi and math.copysign(1, gi) == math.copysign(1, wi), (width, layout, a, gi, wi)


def test_saturating_casts_and_bool(backend):
    """tests/backend/test_numerics.py:49-60 (cast_reference): NaN->0, +-inf saturate, NaN->bool True, -0->False."""
    x = T([math.nan, math.inf, -math.inf, -0.0, 2.75, -2.75])
    i32, i64, bl = run(backend, x.astype(ft.int32), x.astype(ft.int64), x.astype(ft.bool))
    assert i32.tolist() == [0, 2**31 - 1, -2**31, 0, 2, -2]
    assert i64.tolist() == [0, 2**63 - 1, -2**63, 0, 2, -2]
    assert bl.tolist() == [True, True, True, False, True, True]


def test_no_fma_contraction(backend):
    """tests/backend/test_host_compiler.py:127-138: (1 + 2^-23) * (1 - 2^-23) - 1 == 0 without FMA."""
    x = T([1.0 + 2**-23])
    y = x * (1.0 - 2**-23) + (-1.0)
    (v,) = run(backend, y)
    assert float(v[0]) == 0.0


def test_argmax_rows_of_identity_values(backend):
    """First-occurrence argmax/argmin where every element equals the scan identity (+-inf) or ties."""
    x = T([[-math.inf] * 5, [math.inf] * 5, [2.0] * 5, [-math.inf, -math.inf, 3.0, -math.inf, 3.0]])
    a, b, c = run(backend, x.argmax(axis=1), x.argmin(axis=1), x.argmax())
    assert a.tolist() == [0, 0, 0, 2] and b.tolist() == [0, 0, 0, 0] and int(c) == 5
    big = T([[-math.inf] * 3000])
    (d,) = run(backend, big.argmax())
    assert int(d) == 0


# ------------------------------------------------------ index transforms ---
def _grid():
    return T([[float(r * 5 + c) for c in range(5)] for r in range(4)])


def test_slicing_and_tensor_indexing(backend):
    """tests/test_stage2_ops.py:180-191: strided / reversed slices, None, Ellipsis, empty slices,
    and an integer-tensor row index whose -1 entry reads a zero row."""
    x = _grid()
    a, b, c = x[::-1, 1:5:2], x[-1, None, ::2], x[..., 0]
    got = run(backend, a, b, c)
    assert got[0].tolist() == [[16.0, 18.0], [11.0, 13.0], [6.0, 8.0], [1.0, 3.0]]
    assert got[1].tolist() == [[15.0, 17.0, 19.0]]
    assert got[2].tolist() == [0.0, 5.0, 10.0, 15.0]
    assert x[2:1].shape == (0, 5) and x[1:3:-1].shape == (0, 5)
    tidx = T([3, 0, 3, -1], "int64")
    (g,) = run(backend, x[tidx, 1:4])
    assert g.tolist() == [[16.0, 17.0, 18.0], [1.0, 2.0, 3.0], [16.0, 17.0, 18.0], [0.0, 0.0, 0.0]]


def test_pad_interior_and_concatenate(backend):
    """tests/test_stage2_ops.py:193-212: interior pad with an empty edge; cat with an empty
    operand; stack; split and chunk of the concatenation."""
    small = T([[1.0, 2.0], [3.0, 4.0]])
    padded = ft.pad(small, ((1, 0), (0, 1)), constant_value=-1.0, interior=(1, 1))
    assert padded.shape == (4, 4)
    a = T([[1.0, 2.0]])
    b = T([[3.0, 4.0], [5.0, 6.0]])
    empty = ft.tensor(np.zeros((0, 2), np.float32))
    cat = ft.cat([a, empty, b], axis=0)
    stk = ft.stack([a.squeeze(0), a.squeeze(0)], axis=1)
    p0, p1, p2 = cat.split([1, 0, 2], axis=0)
    ch0, ch1 = cat.chunk(2, axis=0)
    got = run(backend, padded, cat, stk, p0, p2, ch0, ch1)
    assert got[0].tolist() == [[-1.0, -1.0, -1.0, -1.0], [1.0, -1.0, 2.0, -1.0], [-1.0, -1.0, -1.0, -1.0],
                               [3.0, -1.0, 4.0, -1.0]]
    assert got[1].tolist() == [[1.0, 2.0], [3.0, 4.0], [5.0, 6.0]]
    assert got[2].tolist() == [[1.0, 1.0], [2.0, 2.0]]
    assert got[3].tolist() == [[1.0, 2.0]] and p1.shape == (0, 2) and got[4].tolist() == [[3.0, 4.0], [5.0, 6.0]]
    assert ch0.shape == (2, 2) and ch1.shape == (1, 2)
    assert got[5].tolist() == [[1.0, 2.0], [3.0, 4.0]] and got[6].tolist() == [[5.0, 6.0]]


def test_one_hot_and_triangles(backend):
    """tests/test_stage2_ops.py:219-224: one_hot with an out-of-range class gives a zero row."""
    oh = ft.one_hot(T([2, 0, -1], "int32"), 4, dtype=ft.fp32)
    (got,) = run(backend, oh)
    assert got.tolist() == [[0.0, 0.0, 1.0, 0.0], [1.0, 0.0, 0.0, 0.0], [0.0, 0.0, 0.0, 0.0]]


@pytest.mark.parametrize("dtype", FLOATS)
def test_scatter_add_duplicates_and_out_of_range(backend, dtype):
    """tests/test_stage2_ops.py:230-238: duplicate indices accumulate, -1 and 4 are dropped."""
    base = ft.tensor(np.zeros((4, 2), np.float32), dtype=getattr(ft, dtype))
    idx = T([1, 3, 1, -1, 4, 1], "int32")
    upd = T([[1.0, 2.0], [3.0, 4.0], [5.0, 6.0], [10.0, 10.0], [20.0, 20.0], [0.5, -1.0]], dtype)
    (got,) = run(backend, ft.scatter_add(base, idx, upd, axis=0))
    close(got, [[0.0, 0.0], [6.5, 7.0], [0.0, 0.0], [3.0, 4.0]], 1e-5 if dtype == "fp32" else 1e-2)


def test_scatter_add_axis1_and_empty_updates(backend):
    """tests/test_stage2_ops.py:240-260: scatter along axis 1 with repeats (then abs); empty
    updates keep the base."""
    for scale in (1.0, 2.0, -3.0):
        b = T([[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]])
        i = T([2, 0, 2], "int64")
        u = T([[scale, scale, scale], [-scale, scale, 0.0]])
        (got,) = run(backend, ft.scatter_add(b, i, u, axis=1).abs())
        close(got, [[abs(1.0 + scale), 2.0, abs(3.0 + 2.0 * scale)], [abs(4.0 + scale), 5.0, abs(6.0 - scale)]], 1e-6)
    keep = T([[1.0, 2.0], [3.0, 4.0]])
    e_idx = ft.tensor(np.zeros((0,), np.int32), dtype=ft.int32)
    e_upd = ft.tensor(np.zeros((0, 2), np.float32))
    (got,) = run(backend, ft.scatter_add(keep, e_idx, e_upd, axis=0))
    assert got.tolist() == [[1.0, 2.0], [3.0, 4.0]]


def test_index_transform_gradients(backend):
    """tests/test_stage2_ops.py:291-322: gradients through a reversed strided slice, a pad
    whose pad value is differentiated, gather and scatter_add, against central differences."""
    w0 = [1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0, 8.0]

    def geom(wf, pv):
        rows = [[pv, pv, pv], [wf[3], wf[1], pv], [pv, pv, pv], [wf[7], wf[5], pv]]
        res = [[1.0, 1.0], [1.0, 1.0]]
        for ii in (1, 0, 1):
            res[ii][0] += rows[ii][0]
            res[ii][1] += rows[ii][1]
        return res[0][0] * 1 + res[0][1] * 2 + res[1][0] * 3 + res[1][1] * 4

    def cdiff(f, xs, eps=1e-3):
        out = []
        for k in range(len(xs)):
            hi, lo = list(xs), list(xs)
            hi[k] += eps
            lo[k] -= eps
            out.append((f(hi) - f(lo)) / (2 * eps))
        return out

    w = T([w0[:4], w0[4:]])
    pv = ft.tensor(0.5)
    idx = T([1, 0, 1], "int32")
    sl = w[:, ::-2]
    pd = ft.pad(sl, ((1, 0), (0, 1)), constant_value=pv, interior=(1, 0))
    gth = ft.gather(pd, idx, axis=0)
    sc2 = ft.scatter_add(ft.tensor(np.ones((2, 2), np.float32)), idx, gth[:, :2], axis=0)
    loss = (sc2 * T([[1.0, 2.0], [3.0, 4.0]])).sum()
    gw, gpv = ft.grad(loss, (w, pv))
    got_w, got_pv = run(backend, gw, gpv)
    close(got_w, cdiff(lambda wf: geom(wf, 0.5), w0), 1e-3)
    close([float(got_pv)], cdiff(lambda p: geom(w0, p[0]), [0.5]), 1e-3)
