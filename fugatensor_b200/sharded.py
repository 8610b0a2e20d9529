"""Leading-dimension sharding of partitions across GPUs (one process per GPU).

The reference binds an Engine to one device (src/fugatensor/engine.py:145,
237-239); this module adds the multi-GPU layer for this path. Every rank
traces the same global partition; inputs flagged as sharded hold that
rank's contiguous dim-0 slab. The native library plans the rank-local
kernels (fgt_spec_create with shard options): row-local work runs with no
communication; reductions over the sharded dimension (whole-tensor
sum/max/argmax/mean, column sums such as LayerNorm's dgamma/dbeta) write a
per-rank partial record that one NCCL all-gather exchanges, after which
every rank combines the records in rank order on the device -- the same
result on every rank, bit for bit.

Process-group plumbing (the NCCL unique id) goes through torch.distributed;
the collective itself is issued by libfgt on the launch stream.
"""
from __future__ import annotations

import ctypes

from . import _fgt, ir


class ShardGroup:
    """The communicator of one rank; created collectively by all ranks."""

    def __init__(self, world: int, rank: int, group=None):
        import torch.distributed as dist
        self.world, self.rank = world, rank
        obj = [_fgt.Comm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=group)
        self.comm = _fgt.Comm(obj[0], world, rank)

    def close(self):
        self.comm.close()


def shard_spec(descriptor: ir.Descriptor, world: int, rank: int, shard_inputs, accumulation="wide", geometry=None):
    """Rank-local spec of a global partition; shard_inputs lists the dim-0-split input ports.
    geometry: row geometry (elements, ring KB, cluster, flags) of the rank-local kernels, e.g.
    the one tuning.select_geometry measured for the unsharded partition of the local shapes."""
    e, r, c, f = tuple(geometry) if geometry else (0, 0, 0, 0)
    return _fgt.Spec(descriptor, accumulation=accumulation, world=world, rank=rank, shard_inputs=tuple(shard_inputs),
                     row_elems=e, ring_kb=r, row_cluster=c, row_flags=f)


def local_rows(global_rows: int, world: int, rank: int):
    if global_rows % world:
        raise ValueError(f"{global_rows} rows do not split evenly over {world} ranks")
    n = global_rows // world
    return rank * n, (rank + 1) * n


def run_sharded(spec, group: ShardGroup, *local_inputs, outputs=None, workspace=None, stream=None):
    """Launch a sharded spec on this rank's slabs (torch CUDA tensors)."""
    comm = group.comm if spec.collective_count else None
    return _fgt.run(spec, *local_inputs, outputs=outputs, workspace=workspace, stream=stream, comm=comm)
