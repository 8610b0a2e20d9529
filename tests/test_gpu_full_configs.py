"""GPU parity of every benchmark configuration at its configured size.

Each case builds the workload exactly as ``bench.py`` does: seeded device
inputs with the workload's distributions, the public API graph, and an
``ft.Engine`` with measured geometry (``tune=True``), so the spec checked
here is the one the benchmark times (geometry and row flags included). The
outputs are compared with the CPU oracle in ACCURATE mode (reductions
accumulated in f64 and rounded once) on the same inputs, evaluated on many
host threads (the oracle's results do not depend on the thread count).

Sizes: c1 [4096, 4096], c2 [16384, 8192] fp32 and bf16, c3 [32768, 8192]
bf16 (including the bf16 dgamma / dbeta column sums over 32768 rows),
c4 2^31 elements, c5 [8192, 8192]. Tolerances are the suite's: integer,
bool and index outputs bit-exact; floats within 1e-5 (f32) or 1e-2
(f16 / bf16) of the output's scale (tests/_util.py).
"""
import os

import numpy as np
import pytest
import torch

import oracle as O
import fugatensor_b200 as ft
from fugatensor_b200 import workloads as W
from tests._util import assert_matches

pytestmark = pytest.mark.gpu

THREADS = max(1, min(64, os.cpu_count() or 1))

CASES = [(cfg, variant, dtype) for cfg, variants in W.VARIANTS.items() for dtype in W.LABELS[cfg]
         for variant in variants]


def to_host(t, dt):
    """Oracle-side numpy view of a device tensor (bf16 as uint16 bits)."""
    t = t.cpu()
    if dt == "bf16":
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


@pytest.fixture(scope="module")
def engine():
    # one tuned engine for the module, as the benchmark keeps one per device
    return ft.Engine("cuda:0")


@pytest.mark.parametrize("cfg,variant,dtype", CASES, ids=[f"{c}-{v}-{d}" for c, v, d in CASES])
def test_full_size_matches_oracle(engine, cfg, variant, dtype):
    rows, cols = W.FULL[cfg]
    torch.cuda.empty_cache()
    device = torch.device("cuda:0")
    dts = W.input_dtypes(cfg, None if dtype == "mixed" else dtype)
    dev_in = W.device_inputs(cfg, rows, cols, None if dtype == "mixed" else dtype, device, seed=11)
    tens = {k: ft.Tensor(engine, dts[k], tuple(v.shape), data=v) for k, v in dev_in.items()}
    outs = W.build(cfg, variant, tens)
    desc, leaves, roots = engine.trace(*outs)
    ft.evaluate(*outs)
    spec = engine.last_spec
    got = [to_host(o._data, o.dtype.ir) for o in outs]
    name_of = {id(v): k for k, v in tens.items()}
    host_in = [to_host(dev_in[name_of[id(l)]], dts[name_of[id(l)]]) for l in leaves]
    del dev_in, tens, outs
    torch.cuda.empty_cache()
    ref = O.evaluate(desc, host_in, O.ACCURATE, threads=THREADS)
    del host_in
    geometry = list(spec.geometry)
    for k, (g, r) in enumerate(zip(got, ref)):
        odt = desc.output_types()[k][0]
        assert_matches(g, r, odt, what=f"{cfg}/{variant}/{dtype} output {k} (geometry {geometry})")
    print(f"{cfg}/{variant}/{dtype} [{rows}, {cols}]: geometry {geometry}, kernels {spec.kernel_count}")
