"""The five partition workloads of the benchmark, written in the public API.

Each workload is a row-major problem of R rows x H columns; the benchmark's
full sizes are in FULL. Inputs are seeded synthetic arrays with the
distributions of the benchmark definition (there is no public dataset for
this path): numpy ``default_rng(seed)``, generated in the order listed,
bf16/f16 rounded to nearest-even from f32.

    c1  x, y f32 ~U(-1,1), seed 0:  sum(square((x + y) * 2) + 3 * x, axis=1)
    c2  X ~N(0, sd 2) f32 or bf16, seed 1; dY ~N(0,1): softmax(X) and its VJP
    c3  X bf16 ~N(0,1), gamma ~U(0.5,1.5), beta ~N(0,0.1), seed 2; dY ~N(0,1):
        rms_norm / layer_norm (eps 1e-6) and VJPs w.r.t. X, gamma (and beta)
    c4  x f32 ~N(0,1), seed 3: sum, amax, argmax (flat, i64), mean
    c5  A i32 ~U[-1000,1000], B i32 [R,1] same, C f16 [1,H] ~N(0,1), seed 4:
        out = where(A > B, C*2 + 1, exp(C) - A.astype(f16)), cnt = sum(A > B, axis=1)
"""
from __future__ import annotations

import numpy as np

FULL = {
    "c1": (4096, 4096),
    "c2": (16384, 8192),
    "c3": (32768, 8192),
    "c4": (32768, 65536),
    "c5": (8192, 8192),
}

# rows of the medium-size check that runs every row partition in every
# candidate geometry of the tuner (several rows per CTA on 148 SMs)
PARITY_ROWS = 2048

VARIANTS = {
    "c1": ("chain_rowsum",),
    "c2": ("softmax_fwd", "softmax_vjp"),
    "c3": ("rmsnorm_fwd", "rmsnorm_vjp", "layernorm_fwd", "layernorm_vjp"),
    "c4": ("global_reductions",),
    "c5": ("broadcast_select",),
}


def f32_to_bf16_bits(x):
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def make_inputs(cfg, rows, cols, dtype=None):
    """Seeded host inputs (numpy; bf16 as uint16 bits) for a workload."""
    if cfg == "c1":
        rng = np.random.default_rng(0)
        x = rng.uniform(-1, 1, (rows, cols)).astype(np.float32)
        y = rng.uniform(-1, 1, (rows, cols)).astype(np.float32)
        return {"x": x, "y": y}
    if cfg == "c2":
        rng = np.random.default_rng(1)
        X = rng.normal(0.0, 2.0, (rows, cols)).astype(np.float32)
        dY = rng.normal(0.0, 1.0, (rows, cols)).astype(np.float32)
        if dtype == "bf16":
            return {"X": f32_to_bf16_bits(X), "dY": f32_to_bf16_bits(dY)}
        return {"X": X, "dY": dY}
    if cfg == "c3":
        rng = np.random.default_rng(2)
        X = rng.normal(0.0, 1.0, (rows, cols)).astype(np.float32)
        gamma = rng.uniform(0.5, 1.5, (cols,)).astype(np.float32)
        beta = rng.normal(0.0, 0.1, (cols,)).astype(np.float32)
        dY = rng.normal(0.0, 1.0, (rows, cols)).astype(np.float32)
        return {k: f32_to_bf16_bits(v) for k, v in (("X", X), ("gamma", gamma), ("beta", beta), ("dY", dY))}
    if cfg == "c4":
        rng = np.random.default_rng(3)
        return {"x": rng.standard_normal((rows, cols), dtype=np.float32)}
    if cfg == "c5":
        rng = np.random.default_rng(4)
        A = rng.integers(-1000, 1001, (rows, cols), dtype=np.int32)
        B = rng.integers(-1000, 1001, (rows, 1), dtype=np.int32)
        C = rng.normal(0.0, 1.0, (1, cols)).astype(np.float32).astype(np.float16)
        return {"A": A, "B": B, "C": C}
    raise KeyError(cfg)


INPUT_DTYPES = {
    "c1": {"x": "f32", "y": "f32"},
    "c2": {"X": "f32", "dY": "f32"},
    "c3": {"X": "bf16", "gamma": "bf16", "beta": "bf16", "dY": "bf16"},
    "c4": {"x": "f32"},
    "c5": {"A": "i32", "B": "i32", "C": "f16"},
}


# the dtype labels each workload runs at (c3 is bf16 throughout; c5 mixes i32 and f16)
LABELS = {"c1": ("f32",), "c2": ("f32", "bf16"), "c3": ("bf16",), "c4": ("f32",), "c5": ("mixed",)}


def input_dtypes(cfg, dtype=None):
    dtype = dtype or LABELS[cfg][0]
    if dtype not in LABELS[cfg]:
        raise ValueError(f"workload {cfg} runs at {LABELS[cfg]}, not {dtype}")
    d = dict(INPUT_DTYPES[cfg])
    if cfg == "c2" and dtype == "bf16":
        d = {"X": "bf16", "dY": "bf16"}
    return d


SHAPES = lambda rows, cols: {"x": (rows, cols), "y": (rows, cols), "X": (rows, cols), "dY": (rows, cols),
                              "gamma": (cols,), "beta": (cols,), "A": (rows, cols), "B": (rows, 1), "C": (1, cols)}


def device_inputs(cfg, rows, cols, dtype, device, seed=0):
    """Seeded inputs generated on the device (torch) with the workload's
    distributions; the benchmark and the full-size parity checks use these
    (the numpy generator of make_inputs is too slow for 2^31 elements)."""
    import torch
    from . import _fgt
    g = torch.Generator(device=device).manual_seed(seed)
    out = {}
    for k, dt in input_dtypes(cfg, dtype).items():
        shape = SHAPES(rows, cols)[k]
        if dt == "i32":
            v = torch.randint(-1000, 1001, shape, device=device, dtype=torch.int32, generator=g)
        elif cfg == "c1":
            v = torch.rand(shape, device=device, generator=g) * 2 - 1
        elif cfg == "c2" and k == "X":
            v = torch.randn(shape, device=device, generator=g) * 2
        elif cfg == "c3" and k == "gamma":
            v = torch.rand(shape, device=device, generator=g) + 0.5
        elif cfg == "c3" and k == "beta":
            v = torch.randn(shape, device=device, generator=g) * 0.1
        else:
            v = torch.randn(shape, device=device, generator=g)
        out[k] = v.to(_fgt.torch_dtype(dt)).contiguous()
    return out


def build(cfg, variant, t, eps=1e-6):
    """Output tensors of a workload variant over input tensors `t` (dict)."""
    import fugatensor_b200 as ft
    from fugatensor_b200.nn import functional as F
    if cfg == "c1":
        x, y = t["x"], t["y"]
        z = ft.square((x + y) * 2) + 3 * x
        return [ft.sum(z, axis=1)]
    if cfg == "c2":
        X = t["X"]
        y = F.softmax(X, axis=-1)
        if variant == "softmax_fwd":
            return [y]
        return [ft.grad(y, X, seed=t["dY"])]
    if cfg == "c3":
        X, gamma, beta, dY = t["X"], t["gamma"], t["beta"], t["dY"]
        if variant.startswith("rmsnorm"):
            y = F.rms_norm(X, weight=gamma, eps=eps)
            if variant == "rmsnorm_fwd":
                return [y]
            return list(ft.grad(y, (X, gamma), seed=dY))
        y = F.layer_norm(X, weight=gamma, bias=beta, eps=eps)
        if variant == "layernorm_fwd":
            return [y]
        return list(ft.grad(y, (X, gamma, beta), seed=dY))
    if cfg == "c4":
        x = t["x"]
        return [ft.sum(x), ft.amax(x), ft.argmax(x), ft.mean(x)]
    if cfg == "c5":
        A, B, C = t["A"], t["B"], t["C"]
        shape = A.shape
        cond = A > ft.broadcast_to(B, shape)
        out = ft.where(cond, ft.broadcast_to(C * 2 + 1, shape), ft.broadcast_to(ft.exp(C), shape) - A.astype(ft.fp16))
        cnt = ft.sum(cond.astype(ft.int32), axis=1)
        return [out, cnt]
    raise KeyError(cfg)


def algorithmic_bytes(cfg, variant, rows, cols, dtype="f32"):
    """Unique HBM bytes of one evaluation: inputs read once, outputs written once."""
    n = rows * cols
    if cfg == "c1":
        return 2 * n * 4 + rows * 4
    if cfg == "c2":
        w = 2 if dtype == "bf16" else 4
        return 2 * n * w if variant == "softmax_fwd" else 3 * n * w
    if cfg == "c3":
        w = 2
        params = cols * w
        if variant == "rmsnorm_fwd":
            return 2 * n * w + params
        if variant == "layernorm_fwd":
            return 2 * n * w + 2 * params
        if variant == "rmsnorm_vjp":
            return 3 * n * w + 2 * params
        return 3 * n * w + 3 * params
    if cfg == "c4":
        return n * 4
    if cfg == "c5":
        return n * 4 + rows * 4 + cols * 2 + n * 2 + rows * 4
    raise KeyError(cfg)


# ------------------------------------------------------- index transforms ---
# Synthetic index-transform partitions (no BASELINE config names them): an
# embedding-style row gather, a row scatter_add with repeated indices, and a
# pad / reversed-slice / concatenate row rewrite. Shapes exceed L2.
INDEX_WORKLOADS = ("gather_rows", "scatter_add_rows", "pad_concat")


def index_inputs(name, device, seed=6):
    """Device inputs (torch) of an index-transform workload."""
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    if name == "gather_rows":
        return {"T": torch.randn((262144, 512), device=device, generator=g),
                "I": torch.randint(0, 262144, (131072,), device=device, generator=g)}
    if name == "scatter_add_rows":
        return {"B": torch.randn((65536, 512), device=device, generator=g),
                "I": torch.randint(0, 65536, (131072,), device=device, generator=g, dtype=torch.int32),
                "U": torch.randn((131072, 512), device=device, generator=g)}
    if name == "pad_concat":
        return {"X": torch.randn((16384, 8192), device=device, generator=g)}
    raise KeyError(name)


INDEX_DTYPES = {"gather_rows": {"T": "f32", "I": "i64"}, "scatter_add_rows": {"B": "f32", "I": "i32", "U": "f32"},
                "pad_concat": {"X": "f32"}}


def index_build(name, t):
    import fugatensor_b200 as ft
    if name == "gather_rows":
        return [ft.gather(t["T"], t["I"], axis=0)]
    if name == "scatter_add_rows":
        return [ft.scatter_add(t["B"], t["I"], t["U"], axis=0)]
    X = t["X"]
    return [ft.cat([ft.pad(X[:, 1:], ((0, 0), (0, 1))), X[:, ::-1]], axis=1)]


def index_bytes(name):
    """Algorithmic HBM bytes: rows read or written once each, indices once (scratch excluded)."""
    if name == "gather_rows":
        return 131072 * 512 * 4 * 2 + 131072 * 8
    if name == "scatter_add_rows":
        return 65536 * 512 * 4 * 2 + 131072 * 512 * 4 + 131072 * 4
    return 16384 * 8192 * 4 + 16384 * 16384 * 4
