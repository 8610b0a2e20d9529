"""Row graphs written in primitives (reference: src/fugatensor/nn/functional.py:82-198).

The decompositions are the reference's, op for op: f16/bf16 inputs are
upcast to f32 for statistics and cast back, the affine ``* weight`` and
``+ bias`` run after the cast back in the input dtype, softmax's max is under
stop_gradient, mean is sum / count. The backend fuses each of these (and
their VJPs) into one row kernel.
"""
from __future__ import annotations

from .. import dtypes as _dt
from .. import ops as _ops
from ..autograd import stop_gradient


def _norm_axes(x, normalized_shape, axis):
    rank = x.ndim
    if normalized_shape is not None and axis is not None:
        raise ValueError("specify either normalized_shape or axis, not both")
    if axis is not None:
        axes = _ops._axes(axis, rank)
        return axes, tuple(x.shape[a] for a in axes)
    if normalized_shape is None:
        if rank == 0:
            raise ValueError("normalization requires at least 1D input when normalized_shape is omitted")
        norm_shape = (x.shape[-1],)
    elif isinstance(normalized_shape, int):
        norm_shape = (normalized_shape,)
    else:
        norm_shape = tuple(normalized_shape)
    if not norm_shape or len(norm_shape) > rank or x.shape[-len(norm_shape):] != norm_shape:
        raise ValueError(f"normalized_shape {norm_shape} does not match trailing shape {x.shape}")
    return tuple(range(rank - len(norm_shape), rank)), norm_shape


def _apply_affine(x, normalized_shape, weight=None, bias=None):
    target = x.shape
    if weight is not None:
        w = weight.astype(x.dtype) if weight.dtype is not x.dtype else weight
        x = x * _ops.broadcast_to(w, target)
    if bias is not None:
        b = bias.astype(x.dtype) if bias.dtype is not x.dtype else bias
        x = x + _ops.broadcast_to(b, target)
    return x


def _work(x):
    return x.astype(_dt.fp32) if x.dtype in (_dt.fp16, _dt.bf16) else x


def softmax(x, axis=-1):
    """Numerically stable softmax along ``axis`` (f16/bf16 statistics in f32)."""
    work = _work(x)
    m = stop_gradient(_ops.amax(work, axis=axis, keepdims=True))
    shifted = work - _ops.broadcast_to(m, work.shape)
    ex = _ops.exp(shifted)
    denom = _ops.broadcast_to(_ops.sum(ex, axis=axis, keepdims=True), work.shape)
    out = ex / denom
    return out.astype(x.dtype) if work is not x else out


def log_softmax(x, axis=-1):
    work = _work(x)
    m = stop_gradient(_ops.amax(work, axis=axis, keepdims=True))
    shifted = work - _ops.broadcast_to(m, work.shape)
    lse = _ops.log(_ops.sum(_ops.exp(shifted), axis=axis, keepdims=True))
    out = shifted - _ops.broadcast_to(lse, work.shape)
    return out.astype(x.dtype) if work is not x else out


def layer_norm(x, normalized_shape=None, weight=None, bias=None, *, eps=1e-5, axis=None):
    axes, norm_shape = _norm_axes(x, normalized_shape, axis)
    work = _work(x)
    mean = _ops.broadcast_to(_ops.mean(work, axis=axes, keepdims=True), work.shape)
    diff = work - mean
    var = _ops.mean(diff * diff, axis=axes, keepdims=True)
    inv_std = _ops.broadcast_to(1 / _ops.sqrt(var + eps), work.shape)
    normed = diff * inv_std
    out = normed.astype(x.dtype) if work is not x else normed
    return _apply_affine(out, norm_shape, weight=weight, bias=bias)


def rms_norm(x, normalized_shape=None, weight=None, *, eps=1e-6, axis=None):
    axes, norm_shape = _norm_axes(x, normalized_shape, axis)
    work = _work(x)
    ms = _ops.mean(work * work, axis=axes, keepdims=True)
    inv_rms = _ops.broadcast_to(1 / _ops.sqrt(ms + eps), work.shape)
    out = work * inv_rms
    out = out.astype(x.dtype) if work is not x else out
    return _apply_affine(out, norm_shape, weight=weight, bias=None)
