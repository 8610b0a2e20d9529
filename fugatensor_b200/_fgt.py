"""ctypes binding of libfgt.so (include/fgt.h).

This is the Python caller of the C ABI -- the same calls a cgo / JNI caller
would make. Device memory and streams come from torch (plumbing only); no
torch type crosses the ABI. There is no fallback: if the native library is
missing, importing this module raises.
"""
from __future__ import annotations

import ctypes
import json
import os
from pathlib import Path

from . import ir

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libfgt.so"
KERNEL_CACHE = Path(os.environ.get("FGT_CACHE_DIR", str(_PKG / "_kernel_cache")))

FGT_OK = 0
STATUS_NAMES = {1: "invalid", 2: "unsupported", 3: "compile", 4: "cuda", 5: "nccl", 6: "workspace"}
ACCUMULATION = {"wide": 0, "storage": 1}


class FgtError(RuntimeError):
    """A failed C-ABI call; ``status`` is the fgt_status code."""

    def __init__(self, status, message):
        super().__init__(f"fgt {STATUS_NAMES.get(status, status)} error: {message}")
        self.status = status


class CompileError(FgtError):
    pass


class CUDAError(FgtError):
    pass


class NCCLError(FgtError):
    """A collective or communicator failed or passed its deadline (FGT_COMM_TIMEOUT_MS)."""


if not LIB_PATH.exists():
    raise ImportError(f"native backend {LIB_PATH} is not built; run `python -m fugatensor_b200.build`")

lib = ctypes.CDLL(str(LIB_PATH))


class SpecOptions(ctypes.Structure):
    _fields_ = [("accumulation", ctypes.c_int32), ("shard_world", ctypes.c_int32), ("shard_rank", ctypes.c_int32),
                ("row_elems", ctypes.c_int32), ("shard_inputs", ctypes.c_uint64), ("cache_dir", ctypes.c_char_p),
                ("ring_kb", ctypes.c_int32), ("row_cluster", ctypes.c_int32), ("row_flags", ctypes.c_int32)]


class SpecInfo(ctypes.Structure):
    _fields_ = [("num_inputs", ctypes.c_int32), ("num_outputs", ctypes.c_int32), ("kernel_count", ctypes.c_int32),
                ("collective_count", ctypes.c_int32), ("workspace_bytes", ctypes.c_size_t)]


_vp = ctypes.c_void_p
lib.fgt_last_error.restype = ctypes.c_char_p
lib.fgt_abi_version.restype = ctypes.c_int32
lib.fgt_spec_create.argtypes = [ctypes.POINTER(ir.CPartition), ctypes.POINTER(SpecOptions), ctypes.POINTER(_vp)]
lib.fgt_spec_destroy.argtypes = [_vp]
lib.fgt_spec_destroy.restype = None
lib.fgt_spec_get_info.argtypes = [_vp, ctypes.POINTER(SpecInfo)]
lib.fgt_spec_port.argtypes = [_vp, ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(ctypes.c_int32),
                              ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int64)]
lib.fgt_spec_plan_json.argtypes = [_vp, ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]
lib.fgt_spec_kernel_source.argtypes = [_vp, ctypes.c_int32, ctypes.c_char_p, ctypes.c_size_t,
                                       ctypes.POINTER(ctypes.c_size_t)]
lib.fgt_spec_launch.argtypes = [_vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp), _vp, ctypes.c_size_t, _vp]
lib.fgt_comm_unique_id.argtypes = [ctypes.POINTER(ctypes.c_uint8)]
lib.fgt_comm_create.argtypes = [ctypes.POINTER(ctypes.c_uint8), ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(_vp)]
lib.fgt_comm_destroy.argtypes = [_vp]
lib.fgt_comm_destroy.restype = None
lib.fgt_comm_peer_exchange.argtypes = [_vp]
lib.fgt_comm_peer_exchange.restype = ctypes.c_int32
lib.fgt_spec_launch_sharded.argtypes = [_vp, _vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp), _vp, ctypes.c_size_t, _vp]
lib.fgt_program_create.argtypes = [_vp, ctypes.c_int32, ctypes.POINTER(_vp)]
lib.fgt_program_run.argtypes = [_vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp), _vp, ctypes.c_size_t, _vp]
lib.fgt_program_kernel_count.argtypes = [_vp]
lib.fgt_program_kernel_count.restype = ctypes.c_int32
lib.fgt_program_destroy.argtypes = [_vp]
lib.fgt_program_destroy.restype = None

EXPORTED = ("fgt_last_error", "fgt_abi_version", "fgt_spec_create", "fgt_spec_destroy", "fgt_spec_get_info",
            "fgt_spec_port", "fgt_spec_plan_json", "fgt_spec_kernel_source", "fgt_spec_launch",
            "fgt_comm_unique_id", "fgt_comm_create", "fgt_comm_peer_exchange", "fgt_comm_destroy",
            "fgt_spec_launch_sharded",
            "fgt_program_create", "fgt_program_run", "fgt_program_kernel_count", "fgt_program_destroy",
            "fgt_reduce_f32_noalloc")


def check(status):
    if status != FGT_OK:
        msg = lib.fgt_last_error().decode(errors="replace")
        cls = CompileError if status == 3 else CUDAError if status == 4 else NCCLError if status == 5 else FgtError
        raise cls(status, msg)


def _copy_string(fn, *args):
    needed = ctypes.c_size_t(0)
    check(fn(*args, None, 0, ctypes.byref(needed)))
    buf = ctypes.create_string_buffer(needed.value)
    check(fn(*args, buf, needed.value, ctypes.byref(needed)))
    return buf.value.decode()


class Spec:
    """A planned, compiled partition (owns an fgt_spec*)."""

    def __init__(self, descriptor: ir.Descriptor, *, accumulation="wide", world=1, rank=0, shard_inputs=(),
                 cache_dir=None, row_elems=0, ring_kb=0, row_cluster=0, row_flags=0):
        self.descriptor = descriptor
        self.geometry = (row_elems, ring_kb, row_cluster, row_flags)
        opts = SpecOptions()
        opts.accumulation = ACCUMULATION[accumulation]
        opts.shard_world = world
        opts.shard_rank = rank
        opts.row_elems = row_elems
        opts.ring_kb = ring_kb
        opts.row_cluster = row_cluster
        opts.row_flags = row_flags
        mask = 0
        for i in shard_inputs:
            mask |= 1 << i
        opts.shard_inputs = mask
        self._cache = str(cache_dir or KERNEL_CACHE).encode()
        opts.cache_dir = self._cache
        handle = _vp()
        check(lib.fgt_spec_create(ctypes.byref(descriptor.struct), ctypes.byref(opts), ctypes.byref(handle)))
        self._h = handle
        info = SpecInfo()
        check(lib.fgt_spec_get_info(self._h, ctypes.byref(info)))
        self.num_inputs = info.num_inputs
        self.num_outputs = info.num_outputs
        self.kernel_count = info.kernel_count
        self.collective_count = info.collective_count
        self.workspace_bytes = info.workspace_bytes
        self.world, self.rank = world, rank
        self.input_types = [self._port(0, i) for i in range(self.num_inputs)]
        self.output_types = [self._port(1, i) for i in range(self.num_outputs)]
        self.execution_plan = json.loads(_copy_string(lib.fgt_spec_plan_json, self._h))

    def _port(self, is_output, index):
        dt, rank = ctypes.c_int32(), ctypes.c_int32()
        shape = (ctypes.c_int64 * ir.MAX_RANK)()
        check(lib.fgt_spec_port(self._h, is_output, index, ctypes.byref(dt), ctypes.byref(rank), shape))
        return ir.DTYPES[dt.value], tuple(shape[k] for k in range(rank.value))

    def kernel_source(self, index):
        return _copy_string(lib.fgt_spec_kernel_source, self._h, index)

    def launch(self, inputs, outputs, workspace=0, workspace_bytes=0, stream=0, comm=None):
        """Launch with raw device addresses (ints) on a raw stream handle."""
        ins = (_vp * max(1, len(inputs)))(*[_vp(int(p)) for p in inputs])
        outs = (_vp * max(1, len(outputs)))(*[_vp(int(p)) for p in outputs])
        if comm is None:
            check(lib.fgt_spec_launch(self._h, ins, outs, _vp(int(workspace)), workspace_bytes, _vp(int(stream))))
        else:
            check(lib.fgt_spec_launch_sharded(self._h, comm._h, ins, outs, _vp(int(workspace)), workspace_bytes,
                                              _vp(int(stream))))

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and lib is not None:
            lib.fgt_spec_destroy(h)
            self._h = None


class Program:
    """A spec prepared for repeated runs (fgt_program, through the _native extension).

    graph=True: the first run on a CUDA context instantiates the spec's
    kernels as one CUDA graph, and every later run replays it with that run's
    buffers (the reference prepares its programs the same way,
    src/fugatensor/engine.py:416-423). graph=False launches kernel by kernel.
    """

    def __init__(self, spec: Spec, graph: bool = True):
        from . import _native
        self.spec = spec  # the program borrows the spec: keep it alive
        self._p = _native.prepare_program(spec._h.value, bool(graph))
        self.graph = bool(graph)
        self.kernel_count = self._p.kernel_count

    def launch(self, inputs, outputs, workspace=0, workspace_bytes=0, stream=0):
        """Run with raw device addresses (ints) on a raw stream handle."""
        check(self._p.run([int(p) for p in inputs], [int(p) for p in outputs], int(workspace), int(workspace_bytes),
                          int(stream)))


class Comm:
    """One rank of an NCCL communicator owned by libfgt."""

    def __init__(self, unique_id: bytes, world: int, rank: int):
        if len(unique_id) != 128:
            raise ValueError("NCCL unique id must be 128 bytes")
        buf = (ctypes.c_uint8 * 128)(*unique_id)
        handle = _vp()
        check(lib.fgt_comm_create(buf, world, rank, ctypes.byref(handle)))
        self._h = handle
        self.world, self.rank = world, rank
        # records of reductions over the sharded dimension: peer mailboxes (NVLink) or NCCL
        self.peer_exchange = bool(lib.fgt_comm_peer_exchange(handle))

    @staticmethod
    def unique_id() -> bytes:
        buf = (ctypes.c_uint8 * 128)()
        check(lib.fgt_comm_unique_id(buf))
        return bytes(buf)

    def close(self):
        if getattr(self, "_h", None) and lib is not None:
            lib.fgt_comm_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()


# ------------------------------------------------------------ torch glue ---
def torch_dtype(name):
    import torch
    return {"bool": torch.bool, "i32": torch.int32, "i64": torch.int64, "f32": torch.float32,
            "f16": torch.float16, "bf16": torch.bfloat16}[name]


def run(spec: Spec, *inputs, outputs=None, workspace=None, stream=None, comm=None, program=None):
    """Launch ``spec`` on torch CUDA tensors; allocates outputs/workspace if not given.
    With ``program`` (a Program of this spec) the run goes through it."""
    import torch
    if len(inputs) != spec.num_inputs:
        raise ValueError(f"partition takes {spec.num_inputs} inputs, got {len(inputs)}")
    device = None
    for t, (dt, shape) in zip(inputs, spec.input_types):
        if not t.is_cuda or tuple(t.shape) != shape or t.dtype != torch_dtype(dt) or not t.is_contiguous():
            raise ValueError(f"input must be a contiguous CUDA tensor {dt}{list(shape)}, got {t.dtype}{list(t.shape)}")
        device = t.device
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    if outputs is None:
        outputs = [torch.empty(shape, dtype=torch_dtype(dt), device=device) for dt, shape in spec.output_types]
    if workspace is None and spec.workspace_bytes:
        workspace = torch.empty(spec.workspace_bytes, dtype=torch.uint8, device=device)
    if stream is None:
        stream = torch.cuda.current_stream(device)
    ins, outs = [t.data_ptr() for t in inputs], [t.data_ptr() for t in outputs]
    ws = workspace.data_ptr() if workspace is not None else 0
    if program is not None:
        if program.spec is not spec:
            raise ValueError("program was prepared for another spec")
        program.launch(ins, outs, ws, spec.workspace_bytes, stream.cuda_stream)
    else:
        spec.launch(ins, outs, ws, spec.workspace_bytes, stream.cuda_stream, comm=comm)
    return outputs
