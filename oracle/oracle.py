"""TEST INFRASTRUCTURE ONLY: Python entry to the CPU oracle (fgt_oracle.c).

Used by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg as
the checker. The product (fugatensor_b200) never imports this module.

Arrays cross as numpy: bool/int32/int64/float32/float16 as themselves, bf16
as uint16 bit patterns (helpers below convert).
"""
from __future__ import annotations

import ctypes
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"

LITERAL = 0
ACCURATE = 1

NP_DTYPE = {"bool": np.bool_, "i32": np.int32, "i64": np.int64, "f32": np.float32, "f16": np.float16,
            "bf16": np.uint16}


def build():
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def _load():
    if not LIB.exists() or LIB.stat().st_mtime < (HERE / "fgt_oracle.c").stat().st_mtime:
        build()
    lib = ctypes.CDLL(str(LIB))
    lib.fgt_oracle_eval.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_void_p),
                                    ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p, ctypes.c_size_t]
    lib.fgt_oracle_eval.restype = ctypes.c_int
    lib.fgt_oracle_eval_mt.argtypes = lib.fgt_oracle_eval.argtypes + [ctypes.c_int]
    lib.fgt_oracle_eval_mt.restype = ctypes.c_int
    return lib


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = _load()
    return _lib


# ---------------------------------------------------------------- bf16 ---
def f32_to_bf16_bits(x):
    """Round-to-nearest-even f32 -> bf16 bit patterns (NaN kept quiet)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    quiet = ((u >> 16) | 0x40).astype(np.uint16)
    return np.where(nan, quiet, rounded)


def bf16_bits_to_f32(b):
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def as_float(array, dtype):
    """Numeric float32 view of an array of dtype (bf16 given as bits)."""
    if dtype == "bf16":
        return bf16_bits_to_f32(array)
    return np.asarray(array).astype(np.float32) if dtype in ("f16", "f32") else np.asarray(array)


# ---------------------------------------------------------------- eval ---
def evaluate(descriptor, inputs, mode=ACCURATE, threads=1):
    """Evaluate a partition descriptor on numpy inputs; returns output arrays.

    threads > 1 runs the oracle's loops on that many OpenMP threads; every
    result is the same for any thread count (whole-tensor sums fold fixed
    chunks of 2^20 elements in order)."""
    in_types = descriptor.input_types()
    if len(inputs) != len(in_types):
        raise ValueError("input count mismatch")
    ins = []
    for arr, (dt, shape) in zip(inputs, in_types):
        a = np.ascontiguousarray(arr, dtype=NP_DTYPE[dt])
        if a.shape != tuple(shape):
            a = a.reshape(shape)
        ins.append(a)
    outs = [np.empty(shape, dtype=NP_DTYPE[dt]) for dt, shape in descriptor.output_types()]
    in_ptrs = (ctypes.c_void_p * max(1, len(ins)))(*[a.ctypes.data for a in ins])
    out_ptrs = (ctypes.c_void_p * max(1, len(outs)))(*[o.ctypes.data for o in outs])
    err = ctypes.create_string_buffer(512)
    if threads > 1:
        rc = lib().fgt_oracle_eval_mt(ctypes.addressof(descriptor.struct), mode, in_ptrs, out_ptrs, err, 512, threads)
    else:
        rc = lib().fgt_oracle_eval(ctypes.addressof(descriptor.struct), mode, in_ptrs, out_ptrs, err, 512)
    if rc:
        raise RuntimeError("oracle failed: " + err.value.decode())
    return outs


def evaluate_rows(make_descriptor, inputs, row_split, mode=ACCURATE, threads=1):
    """Evaluate a row-local partition in row blocks on `threads` host threads.

    make_descriptor(rows) builds the partition for a block of `rows` rows;
    row_split[i] says whether input i is split along dim 0. ctypes releases
    the GIL during the call, so blocks run in parallel.
    """
    n = next(a.shape[0] for a, s in zip(inputs, row_split) if s)
    blocks = [(lo, min(n, lo + max(1, n // threads))) for lo in range(0, n, max(1, n // threads))]
    descs = {}

    def one(block):
        lo, hi = block
        rows = hi - lo
        if rows not in descs:
            descs[rows] = make_descriptor(rows)
        sub = [a[lo:hi] if s else a for a, s in zip(inputs, row_split)]
        return evaluate(descs[rows], sub, mode)

    for lo, hi in blocks:
        if hi - lo not in descs:
            descs[hi - lo] = make_descriptor(hi - lo)
    with ThreadPoolExecutor(max_workers=threads) as ex:
        parts = list(ex.map(one, blocks))
    return [np.concatenate([p[k] for p in parts]) if parts[0][k].ndim else parts[0][k] for k in range(len(parts[0]))]
