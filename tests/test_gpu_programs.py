"""Cache-hit dispatch through prepared programs: multi-kernel plans replay as one CUDA graph.

The engine prepares every compiled partition once (fgt_program through the
_native extension) and runs it on each evaluate; a plan of two or more
kernels (the norm VJPs: row kernel + column finaliser) replays as one CUDA
graph whose kernel nodes get the new buffers each time. The replayed results
must equal an eager launch of the same spec bit for bit, on new inputs, and
the cache accounting must not change (one compilation, then hits).
"""
import numpy as np
import pytest
import torch

import fugatensor_b200 as ft
from fugatensor_b200 import _fgt
from fugatensor_b200 import workloads as W
from tests._util import assert_matches, oracle_outputs

pytestmark = pytest.mark.gpu


def _bits(t):
    t = t.detach().cpu().contiguous()
    return t.view(torch.uint8).numpy() if t.dim() else t.reshape(1).view(torch.uint8).numpy()


def test_layer_norm_vjp_replays_as_one_graph_on_cache_hits():
    eng = ft.Engine("cuda:0", tune=False)
    rows, cols = 512, 8192
    results = []
    for seed in (0, 1, 2):
        dev = W.device_inputs("c3", rows, cols, "bf16", torch.device("cuda:0"), seed=seed)
        t = {k: ft.Tensor(eng, W.input_dtypes("c3", "bf16")[k], tuple(v.shape), data=v) for k, v in dev.items()}
        outs = W.build("c3", "layernorm_vjp", t)
        desc, leaves, _ = eng.trace(*outs)
        ft.evaluate(*outs)
        spec = eng.last_spec
        assert spec.kernel_count == 2
        # eager launch of the same spec on the same inputs
        name_of = {id(v): k for k, v in t.items()}
        eager = _fgt.run(spec, *[dev[name_of[id(l)]] for l in leaves])
        torch.cuda.synchronize()
        for o, e in zip(outs, eager):
            assert np.array_equal(_bits(o._data), _bits(e))
        results.append([o._data.clone() for o in outs])
    assert eng.cache_info() == {"compilations": 1, "cache_hits": 2, "specializations": 1}
    assert eng.stats["graph_replays"] == 3 and eng.stats["launches"] == 6
    assert not torch.equal(results[0][0], results[1][0])  # new inputs, new results


def test_graph_and_eager_programs_agree_and_match_the_oracle():
    eng = ft.Engine("cuda:0", tune=False)
    rng = np.random.default_rng(7)
    x = rng.standard_normal((300, 1000)).astype(np.float32)
    X = eng.tensor(x)
    outs = [ft.sum(X, axis=0), ft.amax(X, axis=1), ft.argmax(X), ft.mean(X)]
    ref, desc = oracle_outputs(eng, outs, {"x": X}, {"x": x})
    spec = _fgt.Spec(desc)
    assert spec.kernel_count >= 2
    got = {}
    for graph in (True, False):
        prog = _fgt.Program(spec, graph=graph)
        for _ in range(3):  # the first graph run instantiates, later runs replay
            o = _fgt.run(spec, X._data, program=prog)
        torch.cuda.synchronize()
        got[graph] = o
    for a, b, r, (dt, _) in zip(got[True], got[False], ref, desc.output_types()):
        assert np.array_equal(_bits(a), _bits(b))
        assert_matches(a.cpu().numpy(), r, dt)


def test_program_replay_inside_stream_capture():
    """On a capturing stream a program adds its kernels to the captured graph."""
    g_in = torch.randn(256, 4096, device="cuda")
    eng = ft.Engine("cuda:0", tune=False)
    X = ft.Tensor(eng, "f32", (256, 4096), data=g_in)
    outs = [ft.sum(X, axis=0), ft.sum(X, axis=1)]
    desc, leaves, _ = eng.trace(*outs)
    spec = _fgt.Spec(desc)
    prog = _fgt.Program(spec, graph=True)
    out = [torch.empty(s, dtype=torch.float32, device="cuda") for _, s in spec.output_types]
    ws = torch.empty(max(1, spec.workspace_bytes), dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        _fgt.run(spec, g_in, outputs=out, workspace=ws, stream=s, program=prog)  # instantiate outside capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        _fgt.run(spec, g_in, outputs=out, workspace=ws, stream=s, program=prog)
    g_in.copy_(torch.randn_like(g_in))
    graph.replay()
    torch.cuda.synchronize()
    ref = _fgt.run(spec, g_in)
    torch.cuda.synchronize()
    for a, b in zip(out, ref):
        assert torch.equal(a, b)
    del graph
