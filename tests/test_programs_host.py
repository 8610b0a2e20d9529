"""Prepared programs (fgt_program_*) on the host: creation rules and pre-launch validation."""
import ctypes

import pytest

from fugatensor_b200 import _fgt, ir


def _ln_like_spec():
    g = ir.Graph()
    x = g.parameter("f32", (64, 256))
    s = g.reduce_sum(x, (1,))
    return _fgt.Spec(g.descriptor([s, g.reduce_sum(x, (0,))]))


def test_program_of_a_local_spec_is_created_and_counts_kernels():
    spec = _ln_like_spec()
    for graph in (True, False):
        prog = _fgt.Program(spec, graph=graph)
        assert prog.kernel_count == spec.kernel_count
        assert prog.graph is graph


def test_sharded_spec_with_collectives_is_rejected():
    g = ir.Graph()
    x = g.parameter("f32", (64, 256))
    spec = _fgt.Spec(g.descriptor([g.reduce_sum(x, (0, 1))]), world=2, rank=0, shard_inputs=(0,))
    assert spec.collective_count == 1
    with pytest.raises(RuntimeError, match="fgt_spec_launch_sharded"):
        _fgt.Program(spec)


@pytest.mark.parametrize("graph", [True, False])
def test_buffers_are_validated_before_anything_is_enqueued(graph):
    spec = _ln_like_spec()
    prog = _fgt.Program(spec, graph=graph)
    ws, wsb = 0x100000, spec.workspace_bytes  # addresses only: nothing is dereferenced on the host
    with pytest.raises(_fgt.FgtError, match="16-byte aligned") as e:
        prog.launch([0x1008], [0x2000, 0x3000], ws, wsb, 0)
    assert e.value.status == 1
    with pytest.raises(_fgt.FgtError, match="input 0 is NULL"):
        prog.launch([0], [0x2000, 0x3000], ws, wsb, 0)
    assert spec.workspace_bytes > 0
    with pytest.raises(_fgt.FgtError, match="workspace") as e:
        prog.launch([0x1000], [0x2000, 0x3000], 0, 0, 0)
    assert e.value.status == 6
