"""Engine: evaluate pending tensors through the native backend.

Mirrors the reference's Engine surface for this path
(src/fugatensor/engine.py:128-446): ``tensor``, ``evaluate``,
``cache_info`` -> {compilations, cache_hits, specializations},
``clear_cache``, ``last_execution_plan`` (Execution Plan v1, validated shape
of src/fugatensor/_ask/plan.py:21-86), ``last_report['cuda_lowering']`` and
session ``stats`` (launches, program_submissions).

``evaluate`` joins the requested pending tensors into ONE partition (as
_lazy.materialize does, src/fugatensor/_lazy.py:200-221), keys it
structurally, and on a cache hit goes straight to the partition's prepared
program (the role of materialize_cached -> ProgramPorts::runFastCore,
cpp/lazy.cpp:871-1008, 946-948): the native extension runs it with the GIL
released, and a plan of two or more kernels replays as one CUDA graph (the
reference prepares every program with graph=True, engine.py:416-423). There
is no CPU path and no fallback: a device without the native library raises.
"""
from __future__ import annotations

import threading

from . import dtypes as _dt
from . import ir
from .tensor import Tensor

_ENGINES = {}
_DEFAULT = ["cuda:0"]
_LOCK = threading.RLock()


def _normalize_device(device):
    if device is None:
        device = _DEFAULT[0]
    device = str(device)
    if device == "cuda":
        device = "cuda:0"
    if not device.startswith("cuda"):
        raise ValueError(f"fugatensor_b200 executes on CUDA devices only, not {device!r}")
    return device


class Engine:
    """One engine per CUDA device."""

    def __init__(self, device="cuda:0", *, accumulation="wide", tune=True):
        self.device = _normalize_device(device)
        self.accumulation = accumulation
        # tune: measure the row-kernel geometry of large partitions on first
        # compile (fugatensor_b200/tuning.py); False keeps the default geometry.
        self.tune = tune
        self._lock = threading.RLock()
        self._cache = {}
        self._programs = {}
        self._stream_cache = {}
        self._stats = {"compilations": 0, "cache_hits": 0}
        self.stats = {"launches": 0, "program_submissions": 0, "graph_replays": 0}
        self.last_execution_plan = None
        self.last_report = None
        self.last_spec = None

    # -- tensors -----------------------------------------------------------
    def tensor(self, values, *, dtype=_dt.fp32, shape=None, host=False):
        """A leaf tensor. host=True keeps the values in pinned host memory until a
        computation needs them (``evaluate`` uploads them; ``evaluate_host``
        streams them row block by row block)."""
        import numpy as np
        import torch
        dtype = _dt.normalize(dtype)
        from . import _fgt
        tdt = _fgt.torch_dtype(dtype.ir)
        if isinstance(values, torch.Tensor):
            data = values.detach().to(tdt)
        elif isinstance(values, np.ndarray) and dtype is _dt.bf16 and values.dtype == np.uint16:
            data = torch.from_numpy(values.astype(np.int16)).view(torch.bfloat16)
        elif isinstance(values, np.ndarray):
            data = torch.from_numpy(np.ascontiguousarray(values)).to(tdt)
        else:
            data = _from_python(values, dtype, tdt)
        if shape is not None:
            data = data.reshape(tuple(shape))
        data = data.contiguous()
        if host:
            data = data.cpu()
            if torch.cuda.is_available():
                data = data.pin_memory()
        elif torch.cuda.is_available():
            data = data.to(self.device)
        return Tensor(self, dtype, tuple(data.shape), data=data)

    def _splat(self, value, dtype, shape):
        from .tensor import _prim, _prim_on
        dtype = _dt.normalize(dtype)
        c = _prim_on(self, "constant", (value, dtype.ir))
        return c if tuple(shape) == () else _prim("splat", (c,), (tuple(shape),))

    # -- compilation -------------------------------------------------------
    def trace(self, *tensors):
        """Join pending tensors into one partition: (descriptor, leaves, roots)."""
        roots, seen_roots = [], set()
        for t in tensors:
            if not isinstance(t, Tensor):
                raise TypeError("evaluate expects Tensors")
            if t._engine is not self:
                raise ValueError("tensor belongs to a different engine")
            if t._expr is not None and id(t) not in seen_roots:
                seen_roots.add(id(t))
                roots.append(t)
        g = ir.Graph()
        value_of, memo, leaves = {}, {}, []
        order = []
        seen = set()
        stack = [(r, False) for r in reversed(roots)]
        while stack:
            t, done = stack.pop()
            if done:
                order.append(t)
                continue
            if id(t) in seen:
                continue
            seen.add(id(t))
            stack.append((t, True))
            if t._expr is not None:
                for a in reversed(t._expr[1]):
                    if id(a) not in seen:
                        stack.append((a, False))
        for t in order:
            if t._expr is None:
                v = g.parameter(t.dtype.ir, t.shape)
                leaves.append(t)
            else:
                op, args, attrs = t._expr
                argv = [value_of[id(a)] for a in args]
                key = (op, tuple(a.id for a in argv), _hashable(attrs))
                v = memo.get(key)
                if v is None:
                    v = _build(g, op, argv, attrs)
                    memo[key] = v
            value_of[id(t)] = v
        desc = g.descriptor([value_of[id(r)] for r in roots])
        return desc, leaves, roots

    def compile(self, *tensors):
        """Plan + compile the partition of `tensors` without running it."""
        from . import _fgt
        desc, leaves, roots = self.trace(*tensors)
        return self._spec(desc), desc, leaves, roots

    def _spec(self, desc):
        from . import _fgt
        key = desc.key()
        spec = self._cache.get(key)
        if spec is None:
            if self.tune:
                from . import tuning
                spec = tuning.select(desc, accumulation=self.accumulation, device=self.device)
            else:
                spec = _fgt.Spec(desc, accumulation=self.accumulation)
            self._cache[key] = spec
            self._stats["compilations"] += 1
        else:
            self._stats["cache_hits"] += 1
        return spec

    def _program(self, key, spec):
        """The prepared program of a cached spec (graph replay for multi-kernel plans)."""
        from . import _fgt
        prog = self._programs.get(key)
        if prog is None or prog.spec is not spec:
            prog = self._programs[key] = _fgt.Program(spec, graph=spec.kernel_count > 1)
        return prog

    def evaluate(self, *tensors):
        """Compile and materialise the requested tensors together."""
        import torch
        from . import _fgt
        with self._lock:
            desc, leaves, roots = self.trace(*tensors)
            if not roots:
                return tensors[0] if len(tensors) == 1 else tensors
            if not torch.cuda.is_available():
                raise _fgt.CUDAError(4, "no CUDA device: fugatensor_b200 has no CPU execution path")
            spec = self._spec(desc)
            prog = self._program(desc.key(), spec)
            device = torch.device(self.device)
            inputs = [t._data if t._data.device == device else t._data.to(device) for t in leaves]
            with torch.cuda.device(device):
                outs = _fgt.run(spec, *inputs, program=prog)
            for r, o in zip(roots, outs):
                r._data = o
                r._expr = None
            plan = dict(spec.execution_plan)
            lowering = plan.pop("cuda_lowering")
            self.last_execution_plan = plan
            self.last_report = {"cuda_lowering": lowering}
            self.last_spec = spec
            self.stats["launches"] += spec.kernel_count
            self.stats["program_submissions"] += 1
            self.stats["graph_replays"] += 1 if prog.graph else 0
            return tensors[0] if len(tensors) == 1 else tensors

    def evaluate_host(self, *tensors):
        """Materialise `tensors` jointly into pinned host memory.

        Row-local partitions (every output row depends only on the same rows of
        the inputs split along dim 0) stream row blocks through three CUDA
        streams, so uploads, kernels and downloads overlap; other partitions
        are uploaded, run and downloaded whole. Returns when the host values
        are ready."""
        import torch
        from . import _fgt, streaming
        with self._lock:
            desc, leaves, roots = self.trace(*tensors)
            if not torch.cuda.is_available():
                raise _fgt.CUDAError(4, "no CUDA device: fugatensor_b200 has no CPU execution path")
            device = torch.device(self.device)
            rs = streaming.plan(self, desc, leaves, roots) if roots else None
            with torch.cuda.device(device):
                if rs is None:
                    if roots:
                        self.evaluate(*tensors)
                    for t in tensors:
                        if t._data.is_cuda:
                            h = torch.empty(t._data.shape, dtype=t._data.dtype, pin_memory=True)
                            h.copy_(t._data, non_blocking=True)
                            t._data = h
                else:
                    outs = streaming.run(self, rs, leaves, desc.output_types(), device)
                    for r, o in zip(roots, outs):
                        r._data = o
                        r._expr = None
                    plan = dict(rs.spec.execution_plan)
                    lowering = plan.pop("cuda_lowering")
                    self.last_execution_plan = plan
                    self.last_report = {"cuda_lowering": lowering, "row_chunks": rs.chunks}
                    self.last_spec = rs.spec
                    self.stats["launches"] += rs.spec.kernel_count * rs.chunks
                    self.stats["program_submissions"] += rs.chunks
                torch.cuda.current_stream(device).synchronize()
            return tensors[0] if len(tensors) == 1 else tensors

    def cache_info(self):
        with self._lock:
            return {"compilations": self._stats["compilations"], "cache_hits": self._stats["cache_hits"],
                    "specializations": len(self._cache)}

    def clear_cache(self):
        with self._lock:
            self._cache.clear()
            self._programs.clear()
            self._stream_cache.clear()
            self.last_execution_plan = self.last_report = self.last_spec = None


def _hashable(attrs):
    out = []
    for a in attrs:
        if isinstance(a, list):
            a = tuple(a)
        if isinstance(a, float) and a != a:
            a = ("nan",)
        out.append(a)
    return tuple(out)


def _build(g, op, argv, attrs):
    if op == "constant":
        return g.constant(attrs[0], attrs[1])
    if op == "cast":
        return g.cast(argv[0], attrs[0])
    if op == "reshape":
        return g.reshape(argv[0], attrs[0])
    if op == "broadcast_in_dim":
        return g.broadcast_in_dim(argv[0], attrs[0], attrs[1])
    if op == "transpose":
        return g.transpose(argv[0], attrs[0])
    if op == "splat":
        return g.splat(argv[0], attrs[0])
    if op == "iota":
        return g.iota(attrs[0], attrs[1], attrs[2])
    if op == "compare":
        return g.compare(argv[0], argv[1], attrs[0])
    if op == "stop_gradient":
        return g.stop_gradient(argv[0])
    if op in ir.REDUCTIONS or op in ("argmax", "argmin"):
        return getattr(g, op)(argv[0], attrs[0])
    if op in ("slice", "pad", "concatenate", "gather", "scatter_add"):
        from .tensor import _index_op
        return _index_op(g, op, argv, attrs)
    return getattr(g, op)(*argv)


def _from_python(values, dtype, tdt):
    import torch
    flat, shape = _flatten(values)
    if dtype.ir in ("f16", "bf16", "f32"):
        bits = [ir.constant_bits(float(v), dtype.ir) for v in flat]
        if dtype.ir == "f32":
            raw = torch.tensor(bits, dtype=torch.int64).to(torch.int32) if bits else torch.empty(0, dtype=torch.int32)
            return raw.view(torch.float32).reshape(shape)
        raw = torch.tensor([b if b < 32768 else b - 65536 for b in bits], dtype=torch.int16)
        return raw.view(tdt).reshape(shape)
    if dtype.ir == "bool":
        return torch.tensor([bool(v) for v in flat], dtype=torch.bool).reshape(shape)
    width = 32 if dtype.ir == "i32" else 64
    vals = []
    for v in flat:
        v = int(v) & ((1 << width) - 1)
        vals.append(v - (1 << width) if v >= 1 << (width - 1) else v)
    return torch.tensor(vals, dtype=tdt).reshape(shape)


def _flatten(values):
    if isinstance(values, (list, tuple)):
        if not values:
            return [], (0,)
        parts = [_flatten(v) for v in values]
        shape = parts[0][1]
        if any(p[1] != shape for p in parts):
            raise ValueError("ragged nested sequence")
        return [x for p in parts for x in p[0]], (len(values),) + shape
    return [values], ()


def current_engine(device=None) -> Engine:
    device = _normalize_device(device)
    with _LOCK:
        eng = _ENGINES.get(device)
        if eng is None:
            eng = _ENGINES[device] = Engine(device)
        return eng


def set_default_device(device):
    _DEFAULT[0] = _normalize_device(device)


def get_default_device():
    return _DEFAULT[0]


def tensor(data, *, dtype=_dt.fp32, engine=None, device=None, host=False):
    return (engine or current_engine(device)).tensor(data, dtype=dtype, host=host)


def evaluate(*tensors):
    if not tensors:
        return None
    return tensors[0].engine.evaluate(*tensors)


def evaluate_host(*tensors):
    """Engine.evaluate_host on the tensors' engine."""
    if not tensors:
        return None
    return tensors[0].engine.evaluate_host(*tensors)


def synchronize():
    import torch
    if torch.cuda.is_available():
        torch.cuda.synchronize()
