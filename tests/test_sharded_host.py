"""Host-side sharding logic on CPU with two gloo ranks (no GPU needed).

Each rank plans its rank-local specs of the benchmark partitions (planning
and sm_100a specialisation run without a GPU); the ranks then compare what
they planned: the same kernels, collectives and workspace on every rank,
local slabs for split inputs and row-local outputs, global shapes for the
outputs that are combined across ranks.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

CASES = (("c4", "global_reductions", 64, 1024), ("c3", "layernorm_vjp", 64, 512), ("c2", "softmax_vjp", 16, 256),
         ("c1", "chain_rowsum", 8, 64), ("c5", "broadcast_select", 32, 128))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _plan(rank, world):
    import fugatensor_b200 as ft
    from fugatensor_b200 import sharded
    from fugatensor_b200 import workloads as W
    eng = ft.Engine("cuda:0")
    out = {}
    for cfg, var, rows, cols in CASES:
        dts = W.input_dtypes(cfg)
        shapes = {"x": (rows, cols), "y": (rows, cols), "X": (rows, cols), "dY": (rows, cols), "gamma": (cols,),
                  "beta": (cols,), "A": (rows, cols), "B": (rows, 1), "C": (1, cols)}
        t = {k: ft.Tensor(eng, dts[k], shapes[k], data=torch.empty(0)) for k in dts}
        desc, leaves, _ = eng.trace(*W.build(cfg, var, t))
        names = [next(k for k, v in t.items() if v is l) for l in leaves]
        split = [i for i, k in enumerate(names) if k in ("x", "y", "X", "dY", "A", "B")]
        spec = sharded.shard_spec(desc, world, rank, split)
        out[(cfg, var)] = {
            # family and index; the trailing partition hash differs per rank (rank offsets)
            "kernels": [k["name"].rsplit("_", 1)[0] for k in spec.execution_plan["cuda_lowering"]["kernels"]],
            "collectives": spec.collective_count, "workspace": spec.workspace_bytes,
            "inputs": spec.input_types, "outputs": spec.output_types,
            "global_inputs": desc.input_types(), "global_outputs": desc.output_types(), "split": split,
        }
    return out


def _worker(rank, world, port, errors):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = _plan(rank, world)
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        for key, p in mine.items():
            for other in gathered:
                q = other[key]
                assert (q["kernels"], q["collectives"], q["workspace"]) == (p["kernels"], p["collectives"], p["workspace"])
            for i, ((dt, shape), (gdt, gshape)) in enumerate(zip(p["inputs"], p["global_inputs"])):
                want = (gshape[0] // world,) + tuple(gshape[1:]) if i in p["split"] else tuple(gshape)
                assert dt == gdt and tuple(shape) == want, (key, i, shape, want)
            for (dt, shape), (gdt, gshape) in zip(p["outputs"], p["global_outputs"]):
                assert dt == gdt
                combined = tuple(shape) == tuple(gshape)
                assert combined or tuple(shape) == (gshape[0] // world,) + tuple(gshape[1:])
            needs_combine = key[0] in ("c4",) or key[1].endswith("norm_vjp")
            assert (p["collectives"] == 1) == needs_combine, key
        dist.barrier()
    except Exception as exc:  # surfaced to the parent
        errors.put(f"rank {rank}: {exc!r}")
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_ranks_plan_consistent_sharded_specs(world):
    ctx = mp.get_context("spawn")
    errors = ctx.SimpleQueue()
    mp.start_processes(_worker, args=(world, _free_port(), errors), nprocs=world, join=True, start_method="spawn")
    assert errors.empty()


def test_unshardable_inputs_are_rejected():
    import fugatensor_b200 as ft
    from fugatensor_b200 import _fgt, ir, sharded
    g = ir.Graph()
    x = g.parameter("f32", (7, 16))  # 7 rows do not split over 2 ranks
    desc = g.descriptor([g.reduce_sum(x, (1,))])
    with pytest.raises(_fgt.FgtError, match="divisible"):
        sharded.shard_spec(desc, 2, 0, [0])
    with pytest.raises(ValueError):
        sharded.local_rows(7, 2, 0)
    g = ir.Graph()
    x = g.parameter("f32", (8, 16))
    w = g.parameter("f32", (8, 16))  # an unsplit input combined elementwise with a split one
    desc = g.descriptor([g.add(x, w)])
    with pytest.raises(_fgt.FgtError, match="unsharded input"):
        sharded.shard_spec(desc, 2, 0, [0])
