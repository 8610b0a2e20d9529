"""evaluate_host: row-streamed evaluation from pinned host memory equals device evaluation bit for bit."""
import numpy as np
import pytest
import torch

import fugatensor_b200 as ft
from fugatensor_b200 import streaming
from fugatensor_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint8)


def _both(cfg, variants, rows, cols, dtype=None):
    inp = W.make_inputs(cfg, rows, cols, dtype)
    dts = W.input_dtypes(cfg, dtype)
    eng = ft.Engine("cuda:0")
    dev = {k: eng.tensor(v, dtype=dts[k]) for k, v in inp.items()}
    host = {k: eng.tensor(v, dtype=dts[k], host=True) for k, v in inp.items()}
    assert all(not t._data.is_cuda and t._data.is_pinned() for t in host.values())
    want = [o for v in variants for o in W.build(cfg, v, dev)]
    got = [o for v in variants for o in W.build(cfg, v, host)]
    eng.evaluate(*want)
    eng.evaluate_host(*got)
    return eng, want, got


@pytest.mark.parametrize("chunk_bytes", [streaming.CHUNK_BYTES, 1 << 20])
@pytest.mark.parametrize("cfg,variants,rows,cols,dtype", [
    ("c2", ("softmax_fwd", "softmax_vjp"), 1024, 8192, "f32"),
    ("c2", ("softmax_fwd", "softmax_vjp"), 512, 8192, "bf16"),
    ("c3", ("layernorm_fwd",), 256, 8192, "bf16"),
    ("c1", ("chain_rowsum",), 2048, 4096, "f32"),
    ("c5", ("broadcast_select",), 1024, 8192, "mixed"),
])
def test_streamed_rows_match_device_evaluate(monkeypatch, cfg, variants, rows, cols, dtype, chunk_bytes):
    monkeypatch.setattr(streaming, "CHUNK_BYTES", chunk_bytes)
    eng, want, got = _both(cfg, variants, rows, cols, dtype)
    assert eng.last_report["row_chunks"] >= 2
    for w, g in zip(want, got):
        assert not g._data.is_cuda and g._data.is_pinned()
        assert np.array_equal(_bits(w.numpy()), _bits(g.numpy()))


@pytest.mark.parametrize("cfg,variant", [("c4", "global_reductions"), ("c3", "layernorm_vjp")])
def test_cross_row_partitions_run_whole(cfg, variant):
    """Reductions over the rows need every row: evaluated whole, results downloaded to pinned memory."""
    eng, want, got = _both(cfg, (variant,), 256, 1024)
    assert "row_chunks" not in eng.last_report
    for w, g in zip(want, got):
        assert not g._data.is_cuda
        assert np.array_equal(_bits(w.numpy()), _bits(g.numpy()))
