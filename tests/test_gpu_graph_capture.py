"""fgt_spec_launch inside a CUDA graph, the reference's default replay
(src/fugatensor/engine.py:420). The launch allocates nothing and is stream
ordered, so after one warm-up launch (which loads the module) it can be
captured on torch's capture stream and replayed with new input contents."""
import numpy as np
import pytest
import torch

import fugatensor_b200 as ft
import fugatensor_b200.nn.functional as F
import oracle as O
from fugatensor_b200 import _fgt
from tests._util import assert_matches

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cfg", ["softmax_vjp", "global_reductions"])
def test_captured_launch_replays_with_new_inputs(cfg):
    eng = ft.Engine("cuda:0", tune=False)
    rng = np.random.default_rng(17)
    rows, cols = 256, 2048
    shapes = [(rows, cols), (rows, cols)] if cfg == "softmax_vjp" else [(rows, cols)]
    host = [rng.standard_normal(s).astype(np.float32) for s in shapes]
    leaves = [eng.tensor(h) for h in host]
    if cfg == "softmax_vjp":
        y = F.softmax(leaves[0], axis=-1)
        outs = [y, ft.grad(y, leaves[0], seed=leaves[1])]
    else:
        outs = [ft.sum(leaves[0]), ft.amax(leaves[0]), ft.argmax(leaves[0]), ft.mean(leaves[0])]
    spec, desc, lv, roots = eng.compile(*outs)
    order = [next(i for i, l in enumerate(leaves) if l is x) for x in lv]
    dev = torch.device("cuda", 0)
    ins = [torch.from_numpy(host[i]).to(dev) for i in order]
    res = [torch.empty(s, dtype=_fgt.torch_dtype(d), device=dev) for d, s in spec.output_types]
    ws = torch.empty(max(1, spec.workspace_bytes), dtype=torch.uint8, device=dev)

    def launch():
        spec.launch([t.data_ptr() for t in ins], [t.data_ptr() for t in res], ws.data_ptr(), spec.workspace_bytes,
                    torch.cuda.current_stream(dev).cuda_stream)

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        launch()  # warm-up: loads the module outside the capture
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        launch()
    for trial in range(3):
        new = [rng.standard_normal(s).astype(np.float32) * (trial + 1) for s in shapes]
        for t, i in zip(ins, order):
            t.copy_(torch.from_numpy(new[i]))
        graph.replay()
        torch.cuda.synchronize()
        ref = O.evaluate(desc, [new[i] for i in order])
        for got, want, (dt, _) in zip(res, ref, spec.output_types):
            g = got.cpu().numpy()
            if dt in ("i64", "i32", "bool"):
                assert np.array_equal(g, want)
            else:
                assert_matches(g, want, dt, what=f"{cfg} replay {trial}")
    del graph
