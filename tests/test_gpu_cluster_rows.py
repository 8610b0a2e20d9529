"""Rows split over a thread-block cluster (two CTAs per row, reductions combined
through distributed shared memory): parity with the oracle for every kind of
row work the split touches. That covers multi-phase rows (softmax and its VJP),
column partials across rows (norm VJPs), single-phase rows (broadcast-select
count), arg-reduction index exchange, boolean and integer exchanges, and the
per-phase division redo."""
import numpy as np
import pytest
import torch

import fugatensor_b200 as ft
import fugatensor_b200.nn.functional as F
import oracle as O
from fugatensor_b200 import _fgt
from fugatensor_b200 import workloads as W
from tests._util import assert_matches, oracle_outputs, trace_workload

pytestmark = pytest.mark.gpu

CASES = [("c2", "softmax_fwd", "f32"), ("c2", "softmax_vjp", "f32"), ("c2", "softmax_vjp", "bf16"),
         ("c3", "layernorm_vjp", "bf16"), ("c3", "rmsnorm_vjp", "bf16"), ("c3", "layernorm_fwd", "bf16"),
         ("c5", "broadcast_select", "mixed")]


def _run_spec(spec, arrays):
    dev = torch.device("cuda", 0)
    ins = []
    for a, (dt, shape) in zip(arrays, spec.input_types):
        t = torch.from_numpy(np.ascontiguousarray(a))
        if dt == "bf16":
            t = t.view(torch.int16).view(torch.bfloat16)
        ins.append(t.to(dev))
    outs = _fgt.run(spec, *ins)
    torch.cuda.synchronize()
    res = []
    for o, (dt, _) in zip(outs, spec.output_types):
        if dt == "bf16":
            res.append(o.view(torch.int16).cpu().numpy().view(np.uint16))
        else:
            res.append(o.cpu().numpy())
    return res


@pytest.mark.parametrize("elems", [16, 32])
@pytest.mark.parametrize("cfg,variant,dtype", CASES)
def test_cluster_rows_match_oracle(cfg, variant, dtype, elems):
    rows, cols = (300, 8192) if cfg != "c5" else (300, 8192)
    eng = ft.Engine("cuda:0", tune=False)
    inp, tensors, outs = trace_workload(eng, cfg, variant, rows, cols, dtype)
    ref, desc = oracle_outputs(eng, outs, tensors, inp)
    spec = _fgt.Spec(desc, row_elems=elems, ring_kb=32, row_cluster=2)
    main = spec.execution_plan["cuda_lowering"]["kernels"][0]
    assert main["cluster"] == 2, main
    desc2, leaves, roots = eng.trace(*outs)
    arrays = [inp[next(k for k, v in tensors.items() if v is l)] for l in leaves]
    got = _run_spec(spec, arrays)
    for k, (g, r) in enumerate(zip(got, ref)):
        assert_matches(g, r, spec.output_types[k][0], what=f"{cfg}/{variant}/{dtype} E{elems} output {k}")


def test_cluster_rows_arg_bool_int_and_redo():
    rng = np.random.default_rng(12)
    rows, cols = 130, 8192
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    x[5, 100] = np.nan
    x[7, :] = 0.0
    d = (rng.random((rows, 1)) + 0.5).astype(np.float32)
    d[9, 0] = 1e-39
    a = rng.integers(-2**31, 2**31 - 1, (rows, cols), dtype=np.int64).astype(np.int32)
    g = ft.ir.Graph()
    X, D, A = g.parameter("f32", (rows, cols)), g.parameter("f32", (rows, 1)), g.parameter("i32", (rows, cols))
    q = g.div(X, g.broadcast_in_dim(D, (rows, cols), (0, 1)))
    outs = [g.argmax(X, 1), g.argmin(X, 1), g.reduce_sum(q, (1,)), g.reduce_max(q, (1,)), g.reduce_sum(A, (1,)),
            g.reduce_any(g.compare(A, g.filled(0, "i32", (rows, cols)), "gt"), (1,)), q]
    desc = g.descriptor(outs)
    ref = O.evaluate(desc, [x, d, a])
    spec = _fgt.Spec(desc, row_elems=16, ring_kb=32, row_cluster=2)
    assert spec.execution_plan["cuda_lowering"]["kernels"][0]["cluster"] == 2
    got = _run_spec(spec, [x, d, a])
    for k, (gv, r) in enumerate(zip(got, ref)):
        dt = spec.output_types[k][0]
        if dt in ("i32", "i64", "bool"):
            assert np.array_equal(gv, r), k
        else:
            assert_matches(gv, r, dt, what=f"output {k}")
