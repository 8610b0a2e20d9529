"""Measured choice of row-kernel geometry per partition.

Block-per-row kernels trade per-row work (barriers, reductions, ring
management) against occupancy: more elements per thread amortise the
per-row instructions but hold more registers, and a smaller shared-memory
ring lets more CTAs share an SM. Which point is fastest depends on the
partition (measured on B200: LayerNorm forward is fastest at 32 elements per
thread with a 24 KB ring, the bf16 softmax VJP at 16 with a 32 KB ring), so
the engine measures instead of guessing. The first compile of a large
partition on a GPU builds the candidate geometries, times each on synthetic
inputs of the partition's own types and shapes (CUDA events, L2 flushed
between launches), and keeps the fastest. The choice is stored in
``tuning.json`` in the kernel cache directory, keyed by the partition's
structure, the GPU, and the library build, so later processes skip the
measurement. Every geometry must compute the partition's results within its
tolerances: before a candidate is kept, its outputs on the tuning inputs are
compared with the default geometry's (integer, bool and index outputs bit for
bit; floats within 1e-5 for f32 and 1e-2 for f16/bf16 of the output's scale),
and a candidate that disagrees is rejected and recorded. Floating-point sums
may still differ in the last bits between geometries (a row's summation
order follows how its elements are spread over threads), and the persisted
choice keeps one geometry per partition.
"""
from __future__ import annotations

import hashlib
import json
import os
import threading
from pathlib import Path

from . import _fgt, ir

# (elements per thread per row operand, shared-memory ring KB, CTAs per row, row flags);
# (0, 0, 0, 0) is the library default. Rows split over a cluster (third field 2) measured slower on
# every benchmark partition (half-size CTAs give no more warps per SM, and each phase adds a
# cluster barrier), so they are not candidates; the option stays available through the spec
# options. Row flags (fgt_row_flag): 1 bounds a kernel's registers to fit one more CTA per SM
# when it is close; 2 computes exp with CUDA's expf instead of the library's exp, whose extra
# independent work can cost a CTA per SM (the bf16 softmax forward: 58 -> 79 registers); 8 folds
# the warp partials of a row reduction with a shuffle butterfly instead of a tree read from shared
# memory (faster for the LayerNorm forward, 0.93 -> 0.97 of peak, slower for the VJPs).
# Flag 4 (column accumulators in shared memory) measured no faster on any benchmark partition (the
# LayerNorm VJP keeps one CTA per SM at 169 registers, and two with the occupancy step spill), so it
# is not a candidate. Candidates a flag leaves unchanged compile to the same source (kernel names
# aside) and are timed once. Four and eight elements per thread (1024 / 512 threads per 4096-wide
# f32 row) suit short single-phase rows: the c1 chain + row sum ran at 0.84 of peak at 4 elements
# against 0.77 at 16. Flag 32 (phase-local operand copies) with 64 (packed column operands) is
# tried where it measured ahead: the bf16 softmax forward with expf (0.86 against 0.84) and the
# RMSNorm VJP at 32 elements (0.92, level with the default).
_GEOMETRIES = ((0, 0, 0), (16, 32, 0), (16, 24, 0), (32, 96, 0), (32, 32, 0), (32, 24, 0), (32, 64, 0), (8, 16, 0),
               (4, 16, 0))
CANDIDATES = tuple(g + (f,) for f in (0, 1, 2, 8) for g in _GEOMETRIES) + ((32, 24, 0, 34), (32, 32, 0, 96))
# Narrow division (flag 256) changes only partitions whose floating outputs are all f16 / bf16, where
# the outputs' rounding hides its one-ulp f32 error; the agreement check above bounds it too.
CANDIDATES += tuple(g + (f,) for f in (256, 258) for g in ((32, 24, 0), (32, 32, 0), (16, 32, 0), (32, 64, 0)))
# Geometries outside the candidate list that stay available through the spec options and are
# parity-checked with the candidates: ring-resident rows (row flag 16) measured slower on every
# benchmark partition (re-reading the row from shared memory in every phase); column accumulators
# in shared memory with phase-local copies (4 + 32 + 64: two CTAs per SM for the LayerNorm VJP, but
# 0.58 of peak against 0.74) and in tensor memory (128: the driver then places one CTA per SM, and
# each chunk's tcgen05.ld / wait / st round trip cost the RMSNorm VJP 0.92 -> 0.73) measured slower.
PARITY_EXTRA = ((32, 64, 0, 16), (16, 64, 0, 16), (32, 32, 0, 100), (32, 32, 0, 224), (16, 32, 0, 224))
MIN_BYTES = 64 << 20  # partitions moving less than this keep the default geometry
RTOL = {"f32": 1e-5, "f16": 1e-2, "bf16": 1e-2}  # agreement with the default geometry
_lock = threading.Lock()


def _lib_tag():
    st = os.stat(_fgt.LIB_PATH)
    return f"{st.st_size}-{int(st.st_mtime)}"


def _db_path(cache_dir):
    return Path(cache_dir or _fgt.KERNEL_CACHE) / "tuning.json"


def _load(path):
    try:
        return json.loads(path.read_text())
    except (OSError, ValueError):
        return {}


def _store(path, key, value):
    with _lock:
        db = _load(path)
        db[key] = value
        path.parent.mkdir(parents=True, exist_ok=True)
        tmp = path.with_suffix(f".tmp.{os.getpid()}")
        tmp.write_text(json.dumps(db, indent=0, sort_keys=True))
        os.replace(tmp, path)


def _moved_bytes(desc):
    n = 0
    for dt, shape in list(desc.input_types()) + list(desc.output_types()):
        k = ir.WIDTH[dt]
        for s in shape:
            k *= s
        n += k
    return n


def _block_rows(spec):
    return any(k["name"].startswith("fgt_row") and k["threads_per_row"] >= 256
               for k in spec.execution_plan["cuda_lowering"]["kernels"])


def _synthetic(dt, shape, device, gen):
    import torch
    tdt = _fgt.torch_dtype(dt)
    if dt in ("f32", "f16", "bf16"):
        return torch.randn(shape, device=device, generator=gen).to(tdt)
    if dt == "bool":
        return torch.rand(shape, device=device, generator=gen) < 0.5
    return torch.randint(-1000, 1001, shape, device=device, generator=gen).to(tdt)


def _time_all(specs, inputs, device, flush, rounds=9):
    """Median launch time of each spec, timed round-robin (one launch of every
    spec per round, L2 flushed before each) so that clock drift during the
    measurement affects all candidates alike."""
    import torch
    stream = torch.cuda.current_stream(device)
    ptrs_in = [t.data_ptr() for t in inputs]
    bound = []
    for spec in specs:
        outs = [torch.empty(s, dtype=_fgt.torch_dtype(dt), device=device) for dt, s in spec.output_types]
        ws = torch.empty(max(spec.workspace_bytes, 1), dtype=torch.uint8, device=device)
        bound.append((spec, [t.data_ptr() for t in outs], ws, outs))
    times = [[] for _ in specs]
    for rnd in range(rounds + 2):
        for k, (spec, ptrs_out, ws, _) in enumerate(bound):
            # the benchmark's flush: writing 256 MiB evicts L2, reading another
            # 256 MiB then writes those dirty lines back before the timed launch
            flush[0].add_(1)
            flush[1].sum()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            spec.launch(ptrs_in, ptrs_out, ws.data_ptr(), spec.workspace_bytes, stream.cuda_stream)
            b.record(stream)
            b.synchronize()
            if rnd >= 2:
                times[k].append(a.elapsed_time(b))
    return [sorted(t)[len(t) // 2] for t in times]


def _outputs(spec, inputs, device):
    import torch
    outs = [torch.empty(s, dtype=_fgt.torch_dtype(dt), device=device) for dt, s in spec.output_types]
    ws = torch.empty(max(spec.workspace_bytes, 1), dtype=torch.uint8, device=device)
    spec.launch([t.data_ptr() for t in inputs], [t.data_ptr() for t in outs], ws.data_ptr(), spec.workspace_bytes,
                torch.cuda.current_stream(device).cuda_stream)
    torch.cuda.current_stream(device).synchronize()
    return outs


def agrees(outs, ref, types):
    """Outputs `outs` agree with `ref`: non-float outputs bit for bit; floats with
    the same NaN and inf positions and |a - b| <= rtol * (|b| + max|b|)."""
    import torch
    for (dt, _), a, b in zip(types, outs, ref):
        if dt not in RTOL:
            if not torch.equal(a, b):
                return False
            continue
        a, b = a.double().reshape(-1), b.double().reshape(-1)
        if not torch.equal(torch.isnan(a), torch.isnan(b)):
            return False
        inf = torch.isinf(b)
        if not torch.equal(torch.isinf(a), inf) or not torch.equal(a[inf], b[inf]):
            return False
        fin = torch.isfinite(b)
        if not bool(fin.any()):
            continue
        bf, af = b[fin], a[fin]
        scale = bf.abs().max()
        if bool(((af - bf).abs() > RTOL[dt] * (bf.abs() + scale) + 1e-30).any()):
            return False
    return True


def select(desc, *, accumulation="wide", device="cuda:0", cache_dir=None):
    """The spec of `desc` with the fastest measured row geometry (default geometry without a GPU)."""
    return select_geometry(desc, accumulation=accumulation, device=device, cache_dir=cache_dir)[1]


def select_geometry(desc, *, accumulation="wide", device="cuda:0", cache_dir=None):
    """(geometry, spec): the measured row geometry of `desc` as (elements, ring KB,
    cluster, flags) and its spec. A sharded partition's rank-local kernels take
    the geometry measured for the unsharded partition of the local shapes."""
    import torch
    default = _fgt.Spec(desc, accumulation=accumulation, cache_dir=cache_dir)
    if not torch.cuda.is_available() or not _block_rows(default) or _moved_bytes(desc) < MIN_BYTES:
        return (0, 0, 0, 0), default
    dev = torch.device(device)
    name = torch.cuda.get_device_name(dev)
    key = hashlib.sha256(f"{desc.key()}|{accumulation}|{name}|{_lib_tag()}".encode()).hexdigest()[:32]
    path = _db_path(cache_dir)
    hit = _load(path).get(key)
    if hit is not None:
        geom = tuple(hit["geometry"]) + (0,) * (4 - len(hit["geometry"]))
        if geom == (0, 0, 0, 0):
            return geom, default
        e, r, c, o = geom
        return geom, _fgt.Spec(desc, accumulation=accumulation, cache_dir=cache_dir, row_elems=e, ring_kb=r, row_cluster=c,
                               row_flags=o)
    specs, seen = [], {}
    for e, r, c, o in CANDIDATES:
        s = default if (e, r, c, o) == (0, 0, 0, 0) else _fgt.Spec(desc, accumulation=accumulation, cache_dir=cache_dir,
                                                                   row_elems=e, ring_kb=r, row_cluster=c, row_flags=o)
        src = tuple(s.kernel_source(i).replace(k["name"], "K")
                    for i, k in enumerate(s.execution_plan["cuda_lowering"]["kernels"]))
        if src in seen:
            continue
        seen[src] = True
        specs.append(((e, r, c, o), s))
    if len(specs) == 1:
        _store(path, key, {"geometry": [0, 0, 0, 0], "ms": None})
        return (0, 0, 0, 0), default
    gen = torch.Generator(device=dev).manual_seed(0)
    with torch.cuda.device(dev):
        inputs = [_synthetic(dt, s, dev, gen) for dt, s in default.input_types]
        flush = torch.zeros((2, 256 << 20), dtype=torch.uint8, device=dev)
        ms_all = _time_all([s for _, s in specs], inputs, dev, flush)
        timed = sorted(((ms, g, s) for ms, (g, s) in zip(ms_all, specs)), key=lambda t: t[0])
        del flush
        # the fastest candidate whose outputs agree with the default geometry's
        ref = _outputs(default, inputs, dev)
        rejected = []
        for ms, geom, best in timed:
            if geom == (0, 0, 0, 0) or agrees(_outputs(best, inputs, dev), ref, default.output_types):
                break
            rejected.append("x".join(map(str, geom)))
        del inputs, ref
    _store(path, key, {"geometry": list(geom), "ms": round(ms, 5), "rejected": rejected,
                       "candidates": {"x".join(map(str, g)): round(t, 5) for t, g, _ in timed}})
    return tuple(geom), best
