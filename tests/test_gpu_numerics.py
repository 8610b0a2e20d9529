"""Bit-level GPU checks of the kernel arithmetic against the oracle's IEEE arithmetic."""
import numpy as np
import pytest

import fugatensor_b200 as ft
import oracle as O

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def _random_floats(rng, n, lo_exp, hi_exp):
    mant = rng.integers(0, 1 << 23, n, dtype=np.uint32)
    exp = rng.integers(lo_exp, hi_exp, n, dtype=np.uint32)
    sign = rng.integers(0, 2, n, dtype=np.uint32) << 31
    return (sign | (exp << 23) | mant).view(np.float32)


@pytest.mark.parametrize("lo,hi", [(1, 254), (100, 156), (1, 30), (225, 254)])
def test_division_by_row_constant_is_ieee(lo, hi):
    """x / broadcast(d[row]) uses a per-row reciprocal + correction: must equal x / d bitwise."""
    rng = np.random.default_rng(lo * 1000 + hi)
    rows, cols = 257, 1024
    x = _random_floats(rng, rows * cols, lo, hi).reshape(rows, cols)
    d = _random_floats(rng, rows, lo, hi).reshape(rows, 1)
    x[0, :8] = [0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, -1e-45, 3.4e38]
    d[1, 0], d[2, 0], d[3, 0], d[4, 0] = 0.0, np.inf, np.nan, 1e-40
    X, D = ft.tensor(x), ft.tensor(d)
    q = X / ft.broadcast_to(D, X.shape)
    desc, leaves, roots = q.engine.trace(q)
    (ref,) = O.evaluate(desc, [x, d])
    got = q.numpy()
    both_nan = np.isnan(got) & np.isnan(ref)
    mism = (_bits(got) != _bits(ref)) & ~both_nan
    assert not mism.any(), f"{mism.sum()} mismatches, e.g. x={x[mism][:3]} d={np.broadcast_to(d, x.shape)[mism][:3]}"


def test_division_by_kernel_constant_is_ieee():
    rng = np.random.default_rng(7)
    x = _random_floats(rng, 1 << 20, 1, 254)
    X = ft.tensor(x)
    got = (X / 3.0).numpy()
    ref = x / np.float32(3.0)
    both_nan = np.isnan(got) & np.isnan(ref)
    assert not ((_bits(got) != _bits(ref)) & ~both_nan).any()


def test_softmax_rows_match_oracle_bitwise_except_exp():
    """Row softmax: max, shift and division are exact; only expf may differ in the last ulp."""
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((64, 8192)) * 2).astype(np.float32)
    X = ft.tensor(x)
    y = ft.nn.functional.softmax(X, axis=-1)
    desc, leaves, roots = y.engine.trace(y)
    (ref,) = O.evaluate(desc, [x])
    got = y.numpy()
    rel = np.abs(got.astype(np.float64) - ref) / np.abs(ref)
    assert rel.max() < 2e-6


def _special_floats():
    sp = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, -1e-45, 3.4028235e38, -3.4028235e38, 65504.0, 65520.0,
                   6.1e-5, 5.96e-8, 2.98e-8, 1.0 + 2.0**-8, 1.0 + 3 * 2.0**-8, 1.0 + 2.0**-11, 1.0 + 3 * 2.0**-11],
                  dtype=np.float32)
    # bf16 ties (low 16 bits exactly 0x8000) with even and odd kept bits, both signs
    ties = (np.arange(64, dtype=np.uint32) << 16 | 0x3f808000).view(np.float32)
    return np.concatenate([sp, ties, -ties])


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_narrowing_casts_are_rne_bitwise(dtype):
    """f32 -> bf16/f16 casts (packed conversions with a zero partner) against the oracle's RNE codec,
    over random patterns of every exponent, ties, overflow, subnormals, signed zeros and NaN."""
    rng = np.random.default_rng(5 if dtype == "bf16" else 6)
    x = np.concatenate([_special_floats(), _random_floats(rng, 1 << 20, 0, 256)]).astype(np.float32)
    X = ft.tensor(x)
    y = X.astype(dtype)
    desc, leaves, roots = y.engine.trace(y)
    (ref,) = O.evaluate(desc, [x])
    got = y.numpy()
    gb = got.view(np.uint16)
    rb = np.ascontiguousarray(ref).view(np.uint16)
    if dtype == "bf16":
        nan = np.isnan(O.bf16_bits_to_f32(gb)) & np.isnan(O.bf16_bits_to_f32(rb))
    else:
        nan = np.isnan(got) & np.isnan(ref)
    mism = (gb != rb) & ~nan
    assert not mism.any(), f"{mism.sum()} mismatches, e.g. x={x[mism][:4]} got={gb[mism][:4]} ref={rb[mism][:4]}"


def test_phase_redo_on_out_of_range_quotients():
    """Row phases check their quotients once per thread; threads whose quotients leave the
    exact range (zero, signed zero, subnormal, huge, inf, NaN, subnormal divisor) redo the
    phase with IEEE division. Quotients stay bitwise IEEE, the phase's row sums and maxima
    are rebuilt from scratch, and benign rows beside them are unaffected."""
    from tests._util import assert_matches
    rng = np.random.default_rng(3)
    rows, cols = 600, 4096
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    d = (rng.random((rows, 1)) + 0.5).astype(np.float32)
    x[3, 7] = -0.0
    x[5, :] = 0.0
    x[9, 100] = np.inf
    x[11, 5] = 1e-38
    x[13, 9] = np.nan
    x[17, 1] = 3e38
    d[19, 0] = 1e-39
    d[21, 0] = 0.0
    x[300:310, 4000] = -1e-40
    X, D = ft.tensor(x), ft.tensor(d)
    q = X / ft.broadcast_to(D, X.shape)
    s = ft.sum(q, axis=1)
    m = ft.amax(q, axis=1)
    desc, leaves, roots = q.engine.trace(q, s, m)
    ref_q, ref_s, ref_m = O.evaluate(desc, [x, d])
    ft.evaluate(q, s, m)
    got_q, got_s, got_m = q.numpy(), s.numpy(), m.numpy()
    nan = np.isnan(got_q) & np.isnan(ref_q)
    assert not ((_bits(got_q) != _bits(ref_q)) & ~nan).any()
    nan = np.isnan(got_m) & np.isnan(ref_m)
    assert not ((_bits(got_m) != _bits(ref_m)) & ~nan).any()
    fin = np.isfinite(ref_s)
    assert np.array_equal(np.isnan(got_s), np.isnan(ref_s)) and np.array_equal(got_s[~fin & ~np.isnan(ref_s)], ref_s[~fin & ~np.isnan(ref_s)])
    assert_matches(got_s[fin], ref_s[fin], "f32", what="row sums of quotients")


def test_bf16_row_max_min_packed_ieee():
    """Row max/min of widened bf16 rows run on packed bf16x2 words; they keep the IEEE
    maximum/minimum of the reference (NaN wins, +0 above -0) bit for bit."""
    rng = np.random.default_rng(21)
    rows, cols = 16, 4096
    x = (rng.standard_normal((rows, cols)) * 4).astype(np.float32)
    x[0, :] = -0.0
    x[1, :] = -0.0
    x[1, 1234] = 0.0
    x[2, :] = 0.0
    x[2, 77] = -0.0
    x[3, 999] = np.nan
    x[4, :] = -np.inf
    x[5, :] = np.inf
    x[6, 4095] = np.nan
    x[7, :] = -1e-40  # subnormal f32 -> bf16 subnormal
    bits = O.f32_to_bf16_bits(x)
    X = ft.tensor(bits, dtype=ft.bf16)
    w = X.astype(ft.fp32)
    mx, mn = ft.amax(w, axis=1), ft.amin(w, axis=1)
    desc, leaves, roots = X.engine.trace(mx, mn)
    ref = O.evaluate(desc, [bits])
    ft.evaluate(mx, mn)
    for got, want in zip((mx.numpy(), mn.numpy()), ref):
        nan = np.isnan(got) & np.isnan(want)
        assert not ((_bits(got) != _bits(want)) & ~nan).any(), (got[:8], want[:8])


def _run_spec(desc, arrays, pairs):
    import os
    import torch
    from fugatensor_b200 import _fgt
    old = os.environ.get("FGT_LANE_PAIRS")
    os.environ["FGT_LANE_PAIRS"] = "1" if pairs else "0"
    try:
        spec = _fgt.Spec(desc)
    finally:
        if old is None:
            del os.environ["FGT_LANE_PAIRS"]
        else:
            os.environ["FGT_LANE_PAIRS"] = old
    src = "".join(spec.kernel_source(i) for i in range(spec.kernel_count))
    assert ("v += 2" in src) == pairs
    dev = torch.device("cuda", 0)
    ins = [torch.from_numpy(a.view(np.int16)).view(torch.bfloat16) if a.dtype == np.uint16 else torch.from_numpy(a)
           for a in arrays]
    outs = _fgt.run(spec, *[t.to(dev) for t in ins])
    torch.cuda.synchronize()
    return [(o.view(torch.int16) if o.dtype == torch.bfloat16 else o).cpu().numpy() for o in outs]


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_lane_pairs_change_no_bit(dtype):
    """Element loops run two lanes per f32x2 instruction (adds, multiplies, tracked
    divisions, row and column sums). Every output equals the one-lane kernel's bit
    for bit, and the elementwise results equal IEEE f32 (subnormals included)."""
    from fugatensor_b200 import ir
    rng = np.random.default_rng(11)
    rows, cols = 64, 4096
    a = _random_floats(rng, rows * cols, 1, 254).reshape(rows, cols)
    b = _random_floats(rng, rows * cols, 1, 254).reshape(rows, cols)
    a[0], b[0] = _random_floats(rng, cols, 0, 3), _random_floats(rng, cols, 0, 3)          # subnormal sums
    a[1], b[1] = _random_floats(rng, cols, 1, 40), _random_floats(rng, cols, 60, 110)      # subnormal products
    a[2, :6] = [0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45]
    g = ir.Graph()
    x, y = g.parameter(dtype, (rows, cols)), g.parameter(dtype, (rows, cols))
    s, p = g.add(x, y), g.mul(x, y)
    t = g.tanh(g.mul(x, g.filled(1e-30, dtype, (rows, cols))))
    rs = g.reduce_sum(g.mul(t, t), (1,))
    q = g.div(t, g.broadcast_in_dim(g.add(rs, g.filled(1.0, dtype, (rows,))), (rows, cols), (0,)))
    cs = g.reduce_sum(g.add(q, t), (0,))
    desc = g.descriptor([s, p, q, cs, rs])
    arrays = [a, b] if dtype == "f32" else [O.f32_to_bf16_bits(a), O.f32_to_bf16_bits(b)]
    paired, single = _run_spec(desc, arrays, True), _run_spec(desc, arrays, False)
    for k, (u, w) in enumerate(zip(paired, single)):
        assert np.array_equal(u.view(np.uint8), w.view(np.uint8)), f"output {k} differs between lane pairs and one lane"
    if dtype == "f32":
        with np.errstate(all="ignore"):
            for got, ref in ((paired[0], a + b), (paired[1], a * b)):
                both_nan = np.isnan(got) & np.isnan(ref)
                assert not ((_bits(got) != _bits(ref)) & ~both_nan).any()


def test_row_phase_exp_within_two_ulp():
    """exp inside a redoable row phase runs as fgt_exp_q (2^f by ex2.approx,
    2^n in the exponent field) and falls back to expf for the rows whose
    arguments leave |x| <= 86 or hold NaN / inf: every normal result is within
    2 ulp of e^x and the special values match."""
    from fugatensor_b200 import ir
    rng = np.random.default_rng(21)
    rows, cols = 96, 4096
    x = rng.uniform(-86, 86, (rows, cols)).astype(np.float32)
    x[1] = rng.uniform(-1e-3, 1e-3, cols)
    x[2] = np.linspace(-1, 1, cols, dtype=np.float32)
    x[3, :8] = [np.nan, np.inf, -np.inf, 88.5, 89.0, -87.5, -100.0, -200.0]
    x[4, :2] = [86.5, -86.5]
    g = ir.Graph()
    xv = g.parameter("f32", (rows, cols))
    e = g.exp(xv)
    desc = g.descriptor([e, g.reduce_sum(e, (1,))])
    got = _run_spec(desc, [x], True)[0].astype(np.float64)
    with np.errstate(all="ignore"):
        ref = np.exp(x.astype(np.float64))
    ref32 = ref.astype(np.float32)
    normal = np.isfinite(ref32) & (np.abs(ref32) >= np.finfo(np.float32).tiny)
    ulp = np.abs(got[normal] - ref[normal]) / np.spacing(ref32[normal]).astype(np.float64)
    assert ulp.max() <= 2.0, f"max {ulp.max():.2f} ulp"
    assert np.array_equal(np.isnan(got), np.isnan(ref32))
    assert np.array_equal(np.isinf(got), np.isinf(ref32))
    tiny = np.isfinite(ref32) & ~normal  # zero and subnormal results
    assert np.all(np.abs(got[tiny] - ref[tiny]) <= 2 * 2.0 ** -149)


@pytest.mark.parametrize("cols", [1024, 64])
def test_row_max_min_signed_zeros_and_nan(cols):
    """Row max / min combine warps with redux.sync (rows of 32-lane groups) or
    shuffles (narrower groups): +0 beats -0 for max, -0 beats +0 for min, and a
    NaN anywhere in the row gives NaN, bit for bit as the oracle."""
    from fugatensor_b200 import ir
    rng = np.random.default_rng(cols)
    rows = 256
    x = np.where(rng.random((rows, cols)) < 0.5, np.float32(0.0), np.float32(-0.0)).astype(np.float32)
    x[: rows // 4] = -0.0                      # all -0: max is -0
    x[rows // 4: rows // 2] = 0.0              # all +0: min is +0
    one = rng.integers(0, cols, rows)
    x[np.arange(rows // 2, 3 * rows // 4), one[rows // 2: 3 * rows // 4]] = np.nan
    x[3 * rows // 4:, :] = rng.standard_normal((rows // 4, cols)).astype(np.float32)
    g = ir.Graph()
    xv = g.parameter("f32", (rows, cols))
    desc = g.descriptor([g.reduce_max(xv, (1,)), g.reduce_min(xv, (1,))])
    got = _run_spec(desc, [x], True)
    ref = O.evaluate(desc, [x])
    for u, r in zip(got, ref):
        both_nan = np.isnan(u) & np.isnan(r)
        assert not ((_bits(u) != _bits(r)) & ~both_nan).any()
        assert np.array_equal(np.isnan(u), np.isnan(r))


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_shared_memory_column_accumulators_change_no_bit(dtype):
    """Column reductions with their accumulators in shared memory (row flag 4)
    add the same values in the same order as in registers: every output of a
    LayerNorm VJP equals the register kernel's bit for bit. (With fewer rows
    than resident CTAs each CTA sums one row in both kernels; with more, the
    kernels' different occupancy groups the rows differently and the column
    sums may differ in the last bits, as between any two geometries.)"""
    import torch
    import fugatensor_b200.nn.functional as F
    from fugatensor_b200 import _fgt
    rng = np.random.default_rng(5)
    rows, cols = 128, 4096
    eng = ft.Engine("cuda:0", tune=False)
    tdt = ft.fp32 if dtype == "f32" else ft.bf16
    host = {"x": rng.standard_normal((rows, cols)), "dy": rng.standard_normal((rows, cols)),
            "w": rng.uniform(0.5, 1.5, cols), "b": rng.standard_normal(cols) * 0.1}
    host = {k: (v.astype(np.float32) if dtype == "f32" else O.f32_to_bf16_bits(v.astype(np.float32))) for k, v in host.items()}
    T = {k: eng.tensor(v, dtype=tdt) for k, v in host.items()}
    y = F.layer_norm(T["x"], (cols,), T["w"], T["b"])
    outs = ft.grad(y, [T["x"], T["w"], T["b"]], seed=T["dy"])
    desc, leaves, roots = eng.trace(*outs)
    ins = [l._data for l in leaves]
    res = []
    for flags in (0, 4):
        spec = _fgt.Spec(desc, row_elems=32, ring_kb=32, row_flags=flags)
        src = "".join(spec.kernel_source(i) for i in range(spec.kernel_count))
        assert ("* const cacc" in src) == (flags == 4)
        out = _fgt.run(spec, *ins)
        torch.cuda.synchronize()
        res.append([(o.view(torch.int16) if o.dtype == torch.bfloat16 else o).cpu().numpy() for o in out])
    for k, (u, w) in enumerate(zip(*res)):
        assert np.array_equal(u.view(np.uint8), w.view(np.uint8)), f"output {k}"


def test_narrow_division_within_one_bf16_ulp_of_exact():
    """Row flag 256 (narrow division) computes a bf16 softmax VJP's element
    divisions as x * RN(1/s): every output equals the exact-division kernel's
    or is one bf16 ulp from it (a rounding tie moved by the product's f32
    error), few outputs move at all, and both match the oracle. Rows whose
    statistics are not finite take IEEE division in both kernels."""
    import torch
    import fugatensor_b200.nn.functional as F
    from fugatensor_b200 import _fgt
    from tests._util import assert_matches
    rng = np.random.default_rng(17)
    rows, cols = 96, 8192
    x = rng.standard_normal((rows, cols)).astype(np.float32) * 3
    dy = rng.standard_normal((rows, cols)).astype(np.float32)
    x[1, :5] = -np.inf           # exp underflows to 0 there
    x[2, :] = 0.5                # a flat row
    x[3, 7] = np.inf             # the row's statistics are NaN: the IEEE form runs
    x[4, :100] = -80.0           # a wide spread: tiny quotients
    eng = ft.Engine("cuda:0", tune=False)
    X = eng.tensor(O.f32_to_bf16_bits(x), dtype=ft.bf16)
    DY = eng.tensor(O.f32_to_bf16_bits(dy), dtype=ft.bf16)
    y = F.softmax(X, axis=-1)
    (dx,) = ft.grad(y, [X], seed=DY)
    desc, leaves, roots = eng.trace(dx)
    ins = [l._data for l in leaves]
    res = []
    for flags in (0, 256):
        spec = _fgt.Spec(desc, row_elems=32, ring_kb=24, row_flags=flags)
        src = "".join(spec.kernel_source(i) for i in range(spec.kernel_count))
        assert ("fgt_div_note" in src) == (flags == 0)
        (out,) = _fgt.run(spec, *ins)
        torch.cuda.synchronize()
        res.append(out.view(torch.int16).cpu().numpy().view(np.uint16))
    exact, narrow = res
    host = {id(X): O.f32_to_bf16_bits(x), id(DY): O.f32_to_bf16_bits(dy)}
    ref = O.evaluate(desc, [host[id(l)] for l in leaves], O.ACCURATE)[0]
    rn = np.isnan(O.bf16_bits_to_f32(ref))
    for name, got in (("exact", exact), ("narrow", narrow)):
        bad = np.flatnonzero((np.isnan(O.bf16_bits_to_f32(got)) != rn).any(axis=1))
        assert bad.size == 0, f"{name}: NaN positions differ from the oracle in rows {bad[:8]}"
    assert_matches(narrow, ref, "bf16", what="narrow division")
    assert_matches(exact, ref, "bf16", what="exact division")
    ev = O.bf16_bits_to_f32(exact).astype(np.float64)
    nv = O.bf16_bits_to_f32(narrow).astype(np.float64)
    fin = np.isfinite(ev)
    assert np.array_equal(exact[~fin], narrow[~fin])
    assert np.array_equal(exact[3], narrow[3])   # IEEE form in both
    # one bf16 ulp is at most 2^-7 of the larger magnitude (plus a sliver of
    # the output's scale where the exact result cancels to zero)
    gap = np.abs(ev - nv)[fin]
    scale = np.abs(ev[fin]).max()
    assert np.all(gap <= np.maximum(np.abs(ev), np.abs(nv))[fin] * 2.0 ** -7 + scale * 2.0 ** -20), gap.max()
    assert (gap > 0).mean() < 0.01
