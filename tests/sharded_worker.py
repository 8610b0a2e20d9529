"""One rank of the 2-GPU sharded parity check (launched by tests/test_gpu_sharded.py).

Every rank builds the global partition, keeps its dim-0 slab of the sharded
inputs, runs the rank-local spec (reductions over the sharded dimension
exchange per-rank records through the peer mailboxes, or with an NCCL
all-gather when FGT_PEER_EXCHANGE=0) and checks its outputs against the CPU
oracle of the whole (unsharded) problem, three launches in a row. Replicated
outputs must be bit-identical on every rank.

With the peer mailboxes, a last check makes an exchange time out on
purpose, with the failure made on the host: rank 1 skips one launch, rank
0's finalising kernel waits FGT_EXCHANGE_WAIT_MS for the missing record,
marks the communicator and returns; rank 0's next launch must then fail with
an NCCL error before launching anything.
"""
import datetime
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import fugatensor_b200 as ft  # noqa: E402
import oracle as O  # noqa: E402
from fugatensor_b200 import _fgt, sharded  # noqa: E402
from fugatensor_b200 import workloads as W  # noqa: E402
from tests._util import assert_matches  # noqa: E402


def main():
    world = int(os.environ["WORLD_SIZE"])
    rank = int(os.environ["RANK"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    group = sharded.ShardGroup(world, rank)
    path = "peer" if group.comm.peer_exchange else "nccl"
    print(f"rank {rank}: exchange path {path}", flush=True)
    eng = ft.Engine(f"cuda:{local}")
    keep = None
    cases = [("c4", "global_reductions", 64, 1024), ("c3", "layernorm_vjp", 64, 512), ("c3", "rmsnorm_vjp", 32, 256),
             ("c2", "softmax_vjp", 16, 256), ("c5", "broadcast_select", 32, 128)]
    for cfg, var, rows, cols in cases:
        inp = W.make_inputs(cfg, rows, cols)
        dts = W.input_dtypes(cfg)
        t = {k: ft.Tensor(eng, dts[k], v.shape, data=torch.empty(0)) for k, v in inp.items()}
        outs = W.build(cfg, var, t)
        desc, leaves, roots = eng.trace(*outs)
        names = [next(k for k, v in t.items() if v is l) for l in leaves]
        split = [k in ("x", "y", "X", "dY", "A", "B") for k in names]
        ref = O.evaluate(desc, [inp[k] for k in names])
        spec = sharded.shard_spec(desc, world, rank, [i for i, s in enumerate(split) if s])
        lo, hi = sharded.local_rows(rows, world, rank)
        ins = []
        for k, s in zip(names, split):
            a = inp[k][lo:hi] if s else inp[k]
            tt = torch.from_numpy(np.ascontiguousarray(a).view(np.int16) if dts[k] == "bf16" else np.ascontiguousarray(a))
            ins.append((tt.view(torch.bfloat16) if dts[k] == "bf16" else tt).to(f"cuda:{local}"))
        first = None
        for it in range(3):  # successive launches: epochs advance, record slots alternate
            dist.barrier()
            got = sharded.run_sharded(spec, group, *ins)
            torch.cuda.synchronize()
            bits = [g.cpu().view(torch.uint8).numpy().tobytes() if g.dim() else g.cpu().reshape(1).view(torch.uint8).numpy().tobytes()
                    for g in got]
            if first is None:
                first = bits
            assert bits == first, f"rank {rank} {cfg}/{var}: launch {it} differs from the first"
        for k, (g, r, (dt, gshape)) in enumerate(zip(got, ref, desc.output_types())):
            host = g.view(torch.int16).cpu().numpy().view(np.uint16) if dt == "bf16" else g.cpu().numpy()
            local_out = tuple(host.shape) != tuple(gshape)
            want = r[lo:hi] if local_out else r
            assert_matches(host, want, dt, what=f"rank {rank} {cfg}/{var} output {k}")
            if not local_out:  # replicated: identical bits on every rank
                gathered = [None] * world
                dist.all_gather_object(gathered, host.tobytes())
                assert all(b == gathered[0] for b in gathered), f"{cfg}/{var} output {k} differs across ranks"
        if cfg == "c4":
            keep = (spec, ins)
        print(f"rank {rank}: {cfg}/{var} ok (collectives={spec.collective_count}, path={path})", flush=True)
    if group.comm.peer_exchange and os.environ.get("FGT_TEST_EXCHANGE_TIMEOUT") == "1":
        spec, ins = keep
        dist.barrier()
        if rank == 0:
            sharded.run_sharded(spec, group, *ins)  # rank 1 does not launch: the wait runs out
            torch.cuda.synchronize()
            try:
                sharded.run_sharded(spec, group, *ins)
                detected = False
            except _fgt.NCCLError as e:
                detected = "timed out" in str(e)
            assert detected, "rank 0: the timed-out exchange was not reported"
            print("rank 0: exchange timeout reported", flush=True)
        dist.barrier()
    group.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
