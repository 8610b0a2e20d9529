"""Reshape inference (reference: src/fugatensor/_shape.py)."""
from __future__ import annotations

import math


def infer_reshape(shape, count):
    if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
        shape = tuple(shape[0])
    shape = tuple(shape)
    if any(type(s) is not int for s in shape):
        raise TypeError("reshape dimensions must be integers")
    if shape.count(-1) > 1:
        raise ValueError("reshape can infer at most one dimension")
    if any(s < -1 for s in shape):
        raise ValueError("reshape dimensions must be nonnegative or -1")
    if -1 in shape:
        known = math.prod(s for s in shape if s != -1)
        if known == 0 or count % known:
            raise ValueError(f"cannot reshape {count} elements into {shape}")
        shape = tuple(count // known if s == -1 else s for s in shape)
    if math.prod(shape) != count:
        raise ValueError(f"cannot reshape {count} elements into {shape}")
    return shape
