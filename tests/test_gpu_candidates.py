"""Every row geometry the tuner may choose computes the oracle's results.

The engine measures the row geometry of large partitions
(fugatensor_b200/tuning.py: elements per thread, shared-memory ring size, row
flags 1 = occupancy step, 2 = CUDA expf, 8 = shuffle butterfly, 32 = phase-local
operand copies, 64 = packed column operands) and keeps the fastest, so any candidate can end up being the benchmarked kernel. Each
benchmark row partition runs here in every candidate geometry at a medium
size (several rows per CTA, so the prefetch ring wraps and column partials
span many rows), against one oracle evaluation per partition. The geometries
kept out of the candidate list (tuning.PARITY_EXTRA: ring-resident rows,
column accumulators in shared or tensor memory) run here too.
"""
import os

import numpy as np
import pytest
import torch

import oracle as O
import fugatensor_b200 as ft
from fugatensor_b200 import _fgt, tuning
from fugatensor_b200 import workloads as W
from tests._util import assert_matches

pytestmark = pytest.mark.gpu

THREADS = max(1, min(64, os.cpu_count() or 1))
ROWS = W.PARITY_ROWS  # ~3-14 rows per CTA at 1-4 CTAs per SM on 148 SMs

PARTITIONS = [(cfg, variant, dtype) for cfg, variants in W.VARIANTS.items() if cfg != "c4"
              for dtype in W.LABELS[cfg] for variant in variants]


def to_host(t, dt):
    t = t.cpu()
    if dt == "bf16":
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


@pytest.mark.parametrize("cfg,variant,dtype", PARTITIONS, ids=[f"{c}-{v}-{d}" for c, v, d in PARTITIONS])
def test_every_candidate_geometry_matches_oracle(cfg, variant, dtype):
    cols = W.FULL[cfg][1]
    eng = ft.Engine("cuda:0", tune=False)
    device = torch.device("cuda:0")
    dt_arg = None if dtype == "mixed" else dtype
    dts = W.input_dtypes(cfg, dt_arg)
    dev_in = W.device_inputs(cfg, ROWS, cols, dt_arg, device, seed=5)
    tens = {k: ft.Tensor(eng, dts[k], tuple(v.shape), data=v) for k, v in dev_in.items()}
    desc, leaves, _ = eng.trace(*W.build(cfg, variant, tens))
    name_of = {id(v): k for k, v in tens.items()}
    order = [name_of[id(l)] for l in leaves]
    ref = O.evaluate(desc, [to_host(dev_in[k], dts[k]) for k in order], O.ACCURATE, threads=THREADS)
    inputs = [dev_in[k] for k in order]
    seen, checked, failures = set(), [], []
    for e, r, c, f in tuning.CANDIDATES + tuning.PARITY_EXTRA:
        spec = _fgt.Spec(desc, row_elems=e, ring_kb=r, row_cluster=c, row_flags=f)
        src = tuple(spec.kernel_source(i).replace(k["name"], "K")
                    for i, k in enumerate(spec.execution_plan["cuda_lowering"]["kernels"]))
        if src in seen:
            continue
        seen.add(src)
        outs = _fgt.run(spec, *inputs)
        torch.cuda.synchronize()
        checked.append((e, r, c, f))
        for k, (o, rr) in enumerate(zip(outs, ref)):
            odt = desc.output_types()[k][0]
            try:
                assert_matches(to_host(o, odt), rr, odt, what=f"geometry {(e, r, c, f)} output {k}")
            except AssertionError as err:
                failures.append(str(err))
    assert not failures, "\n".join(failures)
    assert checked
    print(f"{cfg}/{variant}/{dtype}: {len(checked)} distinct candidates checked: {checked}")
