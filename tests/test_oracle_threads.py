"""The oracle's multi-threaded evaluation gives the single-threaded results bit for bit.

Large parity checks (the benchmark configurations at full size) run the oracle
on many host threads; these cases pin that the thread count changes no bit,
including whole-tensor reductions split into chunks and a cancelling sum that
crosses chunk boundaries.
"""
import numpy as np
import pytest
import torch

import oracle as O
import fugatensor_b200 as ft
from fugatensor_b200 import workloads as W


def _same(a, b):
    return all(np.array_equal(np.atleast_1d(x).view(np.uint8), np.atleast_1d(y).view(np.uint8)) for x, y in zip(a, b))


@pytest.mark.parametrize("cfg,variant,dtype,rows,cols", [
    ("c1", "chain_rowsum", "f32", 64, 4096),
    ("c2", "softmax_vjp", "bf16", 48, 8192),
    ("c3", "layernorm_vjp", "bf16", 64, 1024),
    ("c3", "rmsnorm_vjp", "bf16", 40, 2048),
    ("c4", "global_reductions", "f32", 48, 65536),
    ("c5", "broadcast_select", None, 32, 4096),
])
@pytest.mark.parametrize("mode", [O.ACCURATE, O.LITERAL])
def test_thread_count_changes_no_bit(cfg, variant, dtype, rows, cols, mode):
    eng = ft.Engine("cuda:0", tune=False)
    inp = W.make_inputs(cfg, rows, cols, dtype)
    dts = W.input_dtypes(cfg, dtype)
    tens = {k: ft.Tensor(eng, dts[k], v.shape, data=torch.empty(0)) for k, v in inp.items()}
    desc, leaves, _ = eng.trace(*W.build(cfg, variant, tens))
    name_of = {id(v): k for k, v in tens.items()}
    arrays = [inp[name_of[id(l)]] for l in leaves]
    one = O.evaluate(desc, arrays, mode)
    for threads in (2, 7):
        assert _same(one, O.evaluate(desc, arrays, mode, threads=threads)), threads


def test_cancelling_sum_across_chunks():
    """2^24 + 1 - 2^24 spread over three 2^20-element chunks sums to exactly 1."""
    from fugatensor_b200 import ir
    n = 3 << 20
    x = np.zeros(n, dtype=np.float32)
    x[5], x[(1 << 20) + 7], x[(2 << 20) + 9] = 2.0 ** 24, 1.0, -(2.0 ** 24)
    g = ir.Graph()
    p = g.parameter("f32", (n,))
    desc = g.descriptor([g.reduce_sum(p, (0,)), g.argmax(p, 0), g.reduce_max(p, (0,))])
    for threads in (1, 4):
        s, a, m = O.evaluate(desc, [x], O.ACCURATE, threads=threads)
        assert float(s) == 1.0 and int(a) == 5 and float(m) == 2.0 ** 24
