"""Row-streamed evaluation of partitions whose inputs live in host memory.

The reference evaluates on device-resident tensors; a caller holding its
data on the host uploads it (``ft.tensor``), evaluates, and downloads the
results, each step waiting for the previous one (src/fugatensor/engine.py
441-446 for evaluate; the session copies in src/fugatensor/runtime.py).
For a partition whose every output is row-local -- each output row depends
only on the same rows of the dim-0-split inputs (softmax and its VJP,
RMSNorm/LayerNorm forward, row reductions, broadcast-select) -- the rows can
be cut into chunks that flow through three CUDA streams: host-to-device
copies of chunk k+1, the fused kernels of chunk k, and the device-to-host
copies of chunk k-1 run at the same time. PCIe then carries both directions
at once and the kernels hide behind the copies.

Chunks are planned with the same leading-dimension split as multi-GPU
sharding (fgt_spec_create with shard options): a chunk is a "rank" of the
split, so results are the partition's own results, row for row. Partitions
that reduce across rows (whole-tensor reductions, column sums) need a
combine over all rows and are evaluated whole: upload, run, download.
"""
from __future__ import annotations

from . import _fgt, ir

# Chunk size target: inputs plus outputs of one chunk.
CHUNK_BYTES = 64 << 20
BUFFERS = 3  # device buffer sets in rotation
WHOLE_LIMIT = 16 << 30  # partitions above this are not specialised whole (no device-size tuning run)


def _moved_bytes(desc):
    n = 0
    for dt, shape in list(desc.input_types()) + list(desc.output_types()):
        n += ir.WIDTH[dt] * _numel(shape)
    return n


def _width(dt):
    return ir.WIDTH[dt]


def _row_split(desc, leaves, roots):
    """(rows, split ports) when every output is row-local over dim 0, else None."""
    out_types = desc.output_types()
    if not out_types or any(len(s) == 0 for _, s in out_types):
        return None
    R = out_types[0][1][0]
    if R < 2 or any(s[0] != R for _, s in out_types):
        return None
    in_types = desc.input_types()
    cands = [i for i, (_, s) in enumerate(in_types) if len(s) >= 1 and s[0] == R]
    if not cands:
        return None
    # Prefer splitting only inputs of rank >= 2: a rank-1 input of length R
    # may be a column vector (gamma on a square problem) rather than per-row.
    tries = [tuple(i for i in cands if len(in_types[i][1]) >= 2), tuple(cands)]
    for split in tries:
        if not split:
            continue
        try:
            probe = _fgt.Spec(desc, world=2, rank=1, shard_inputs=split)
        except _fgt.FgtError:
            continue
        if probe.collective_count == 0:
            return R, split
    return None


def _chunk_count(R, row_bytes, chunk_bytes):
    best = None
    for c in range(2, R + 1):
        if R % c:
            continue
        best = c
        if (R // c) * row_bytes <= chunk_bytes:
            return c
    return best


class RowStream:
    """Chunk specs of one partition (cached per engine)."""

    def __init__(self, desc, rows, split, chunks, accumulation, geometry=(0, 0, 0, 0)):
        self.rows, self.split, self.chunks = rows, split, chunks
        e, r, c, o = tuple(geometry) + (0,) * (4 - len(geometry))
        mk = lambda k: _fgt.Spec(desc, accumulation=accumulation, world=chunks, rank=k, shard_inputs=split,
                                 row_elems=e, ring_kb=r, row_cluster=c, row_flags=o)
        first, second = mk(0), mk(1)
        names = lambda s: [k["name"] for k in s.execution_plan["cuda_lowering"]["kernels"]]
        if names(first) == names(second):
            self.specs = [first] * chunks  # no rank offsets: one spec serves every chunk
        else:
            self.specs = [first, second] + [mk(k) for k in range(2, chunks)]
        self.spec = first


def plan(engine, desc, leaves, roots):
    key = ("rows", desc.key())
    rs = engine._stream_cache.get(key)
    if rs is None and key not in engine._stream_cache:
        found = _row_split(desc, leaves, roots)
        if found is not None:
            R, split = found
            in_types, out_types = desc.input_types(), desc.output_types()
            row_bytes = sum(_width(dt) * _numel(s[1:]) for i, (dt, s) in enumerate(in_types) if i in split)
            row_bytes += sum(_width(dt) * _numel(s[1:]) for dt, s in out_types)
            chunks = _chunk_count(R, row_bytes, CHUNK_BYTES)
            # The chunks run the row geometry the engine chose for the whole
            # partition, so streamed results equal evaluate()'s bit for bit
            # (the geometry fixes each row's summation order). Partitions too
            # large to measure on the device keep the default geometry.
            geometry = (0, 0, 0, 0)
            if _moved_bytes(desc) <= WHOLE_LIMIT:
                geometry = engine._spec(desc).geometry
            rs = RowStream(desc, R, split, chunks, engine.accumulation, geometry) if chunks else None
        engine._stream_cache[key] = rs
    return rs


def _numel(shape):
    n = 1
    for s in shape:
        n *= s
    return n


def run(engine, rs, leaves, out_types, device):
    """Stream the chunks of ``rs`` over host (or device) leaves; returns pinned host outputs."""
    import torch
    cur = torch.cuda.current_stream(device)
    s_in, s_run, s_out = (torch.cuda.Stream(device) for _ in range(3))
    for s in (s_in, s_run, s_out):
        s.wait_stream(cur)
    C, R = rs.chunks, rs.rows
    rc = R // C
    host_out = [torch.empty(s, dtype=_fgt.torch_dtype(dt), pin_memory=True) for dt, s in out_types]
    # inputs that are not split: on the device once
    with torch.cuda.stream(s_in):
        whole = {i: (t._data if t._data.device == device else t._data.to(device, non_blocking=True))
                 for i, t in enumerate(leaves) if i not in rs.split}
    spec = rs.spec
    din = [[torch.empty((rc,) + tuple(leaves[i]._shape[1:]), dtype=leaves[i]._data.dtype, device=device)
            for i in rs.split] for _ in range(min(BUFFERS, C))]
    dout = [[torch.empty((rc,) + tuple(s[1:]), dtype=_fgt.torch_dtype(dt), device=device) for dt, s in out_types]
            for _ in range(min(BUFFERS, C))]
    ws = torch.empty(spec.workspace_bytes, dtype=torch.uint8, device=device) if spec.workspace_bytes else None
    ev_run, ev_out = [], []
    for k in range(C):
        b = k % len(din)
        lo, hi = k * rc, (k + 1) * rc
        with torch.cuda.stream(s_in):
            if k >= len(din):
                s_in.wait_event(ev_run[k - len(din)])  # the kernels of chunk k-B no longer read buffer b
            for j, i in enumerate(rs.split):
                din[b][j].copy_(leaves[i]._data[lo:hi], non_blocking=True)
            ev_in = torch.cuda.Event()
            ev_in.record(s_in)
        s_run.wait_event(ev_in)
        if k >= len(din):
            s_run.wait_event(ev_out[k - len(din)])  # chunk k-B's results have left buffer b
        inputs, j = [], 0
        for i in range(len(leaves)):
            if i in rs.split:
                inputs.append(din[b][j])
                j += 1
            else:
                inputs.append(whole[i])
        rs.specs[k].launch([t.data_ptr() for t in inputs], [t.data_ptr() for t in dout[b]],
                           ws.data_ptr() if ws is not None else 0, spec.workspace_bytes, s_run.cuda_stream)
        e = torch.cuda.Event()
        e.record(s_run)
        ev_run.append(e)
        s_out.wait_event(e)
        with torch.cuda.stream(s_out):
            for h, d in zip(host_out, dout[b]):
                h[lo:hi].copy_(d, non_blocking=True)
            e = torch.cuda.Event()
            e.record(s_out)
            ev_out.append(e)
    for s in (s_in, s_run, s_out):
        cur.wait_stream(s)
    return host_out
