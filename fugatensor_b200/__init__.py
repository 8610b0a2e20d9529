"""fugatensor_b200 — B200-native (sm_100a) backend for FugaTensor's fused
elementwise / broadcast / reduction partitions, behind the reference's
tensor API (``tensor``, ``evaluate``, ``grad``, ``Engine.cache_info``,
``Engine.last_execution_plan``).

The native library (libfgt.so, C ABI in include/fgt.h) is loaded lazily on
first compile/evaluate; ``import fugatensor_b200`` itself needs no GPU.
"""
from .dtypes import DType, bool, int32, int64, fp32, fp16, bf16  # noqa: A004
from .engine import Engine, current_engine, evaluate, evaluate_host, get_default_device, set_default_device, synchronize, tensor
from .tensor import Tensor
from .autograd import grad, stop_gradient
from .ops import (add, multiply, subtract, negative, square, abs, floor, ceil, round, cast, reshape,  # noqa: A004
                  zeros_like, ones_like, divide, floordiv, mod, pow, maximum, minimum, clamp, clip, compare, where,
                  exp, log, sqrt, sin, cos, tanh, erf, logical_and, logical_or, logical_xor, logical_not,
                  bitwise_and, bitwise_or, bitwise_xor, bitwise_not, shift_left, shift_right, broadcast_in_dim,
                  broadcast_to, transpose, squeeze, unsqueeze, flatten, sum, amax, amin, prod, mean, any, all,
                  argmax, argmin, iota, slice, pad, concatenate, cat, stack, split, chunk, gather, take,
                  scatter_add, getitem, one_hot)
from . import nn, ir  # noqa: F401

__all__ = ["DType", "bool", "int32", "int64", "fp32", "fp16", "bf16", "Engine", "Tensor", "tensor", "evaluate", "evaluate_host",
           "grad", "stop_gradient", "current_engine", "set_default_device", "get_default_device", "synchronize",
           "nn", "ir"]
