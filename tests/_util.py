"""Shared test helpers: run a workload through the backend and through the oracle."""
from __future__ import annotations

import numpy as np

import oracle as O
from fugatensor_b200 import workloads as W

RTOL = {"f32": 1e-5, "f16": 1e-2, "bf16": 1e-2}


def to_numeric(a, dtype):
    if dtype == "bf16":
        return O.bf16_bits_to_f32(a).astype(np.float64)
    if dtype in ("f16", "f32"):
        return np.asarray(a).astype(np.float64)
    return np.asarray(a)


def assert_matches(got, ref, dtype, rtol=None, what=""):
    """Integer/bool/index outputs bit-exact; floats within rtol of the output's scale.

    |got - ref| <= rtol * (|ref| + max|ref|) elementwise: relative for
    well-conditioned values, relative to the output's magnitude where the
    graph cancels (VJPs). NaN and inf positions must agree exactly.
    """
    got, ref = np.asarray(got), np.asarray(ref)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    if dtype not in RTOL:
        mism = np.flatnonzero(got.reshape(-1) != ref.reshape(-1))
        assert mism.size == 0, f"{what}: {mism.size} mismatches, first at {mism[:5]}: {got.reshape(-1)[mism[:5]]} vs {ref.reshape(-1)[mism[:5]]}"
        return
    rtol = RTOL[dtype] if rtol is None else rtol
    g, r = to_numeric(got, dtype), to_numeric(ref, dtype)
    assert np.array_equal(np.isnan(g), np.isnan(r)), f"{what}: NaN positions differ"
    fin = np.isfinite(r)
    assert np.array_equal(np.isinf(g), np.isinf(r)) and np.array_equal(g[~fin & ~np.isnan(r)], r[~fin & ~np.isnan(r)]), \
        f"{what}: inf positions differ"
    if not fin.any():
        return
    scale = np.max(np.abs(r[fin])) if r[fin].size else 0.0
    err = np.abs(g[fin] - r[fin])
    bound = rtol * (np.abs(r[fin]) + scale) + 1e-30
    worst = np.argmax(err / bound)
    assert np.all(err <= bound), (f"{what}: max err {err[worst]:.3e} at ref {r[fin][worst]:.6e} "
                                  f"(got {g[fin][worst]:.6e}), bound {bound[worst]:.3e}")


def trace_workload(engine, cfg, variant, rows, cols, dtype=None):
    inp = W.make_inputs(cfg, rows, cols, dtype)
    dts = W.input_dtypes(cfg, dtype)
    tensors = {k: engine.tensor(v, dtype=dts[k]) for k, v in inp.items()}
    outs = W.build(cfg, variant, tensors)
    return inp, tensors, outs


def oracle_outputs(engine, outs, tensors, inp, mode=O.ACCURATE):
    desc, leaves, roots = engine.trace(*outs)
    name_of = {id(v): k for k, v in tensors.items()}
    arrays = [inp[name_of[id(l)]] for l in leaves]
    return O.evaluate(desc, arrays, mode), desc
