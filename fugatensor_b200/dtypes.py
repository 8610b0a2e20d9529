"""Public dtypes (reference: src/fugatensor/dtypes.py) mapped onto Fuga IR names."""
from __future__ import annotations


class DType:
    __slots__ = ("name", "ir", "itemsize")

    def __init__(self, name, ir, itemsize):
        self.name, self.ir, self.itemsize = name, ir, itemsize

    def __repr__(self):
        return f"fugatensor_b200.{self.name}"

    def __str__(self):
        return self.ir

    @property
    def is_floating(self):
        return self.ir in ("f32", "f16", "bf16")


bool = DType("bool", "bool", 1)  # noqa: A001 - mirrors the reference's public name
int32 = DType("int32", "i32", 4)
int64 = DType("int64", "i64", 8)
fp32 = DType("fp32", "f32", 4)
fp16 = DType("fp16", "f16", 2)
bf16 = DType("bf16", "bf16", 2)

ALL = (bool, int32, int64, fp32, fp16, bf16)
BY_IR = {d.ir: d for d in ALL}
_BY_NAME = {d.name: d for d in ALL}
_BY_NAME.update({"float32": fp32, "float16": fp16, "bfloat16": bf16, "f32": fp32, "f16": fp16, "i32": int32,
                 "i64": int64})


def normalize(dtype) -> DType:
    if isinstance(dtype, DType):
        return dtype
    if isinstance(dtype, str) and dtype in _BY_NAME:
        return _BY_NAME[dtype]
    if isinstance(dtype, str) and dtype in BY_IR:
        return BY_IR[dtype]
    try:
        import torch
        m = {torch.bool: bool, torch.int32: int32, torch.int64: int64, torch.float32: fp32, torch.float16: fp16,
             torch.bfloat16: bf16}
        if dtype in m:
            return m[dtype]
    except ImportError:  # pragma: no cover
        pass
    raise TypeError(f"unsupported dtype: {dtype!r}")
