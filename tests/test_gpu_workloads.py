"""GPU parity of the five benchmark workloads against the CPU oracle (small and mid sizes)."""
import numpy as np
import pytest
import torch

import fugatensor_b200 as ft
from fugatensor_b200 import workloads as W
from tests._util import assert_matches, oracle_outputs, trace_workload

pytestmark = pytest.mark.gpu

CASES = []
for cfg, variants in W.VARIANTS.items():
    for var in variants:
        dtypes = W.LABELS[cfg]
        for dt in dtypes:
            for rows, cols in ((3, 5), (7, 33), (64, 1000), (40, 8192), (256, 256)):
                CASES.append((cfg, var, dt, rows, cols))


def _host(t):
    return t.numpy()


@pytest.mark.parametrize("cfg,variant,dtype,rows,cols", CASES)
def test_workload_matches_oracle(cfg, variant, dtype, rows, cols):
    eng = ft.current_engine()
    inp, tensors, outs = trace_workload(eng, cfg, variant, rows, cols, dtype)
    ref, desc = oracle_outputs(eng, outs, tensors, inp)
    ft.evaluate(*outs)
    for k, (o, r) in enumerate(zip(outs, ref)):
        assert_matches(_host(o), r, o.dtype.ir, what=f"{cfg}/{variant}/{dtype} output {k}")
