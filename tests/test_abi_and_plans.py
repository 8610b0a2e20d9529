"""Host-side tests (no GPU): the C ABI library, descriptor validation, planning,
kernel specialisation (NVRTC runs without a GPU) and the Execution Plan v1 shape."""
import ctypes
import math
import re
from fractions import Fraction
from pathlib import Path

import pytest

import fugatensor_b200 as ft
from fugatensor_b200 import _fgt, ir
from fugatensor_b200 import workloads as W
import fugatensor_b200.nn.functional as F

ROOT = Path(__file__).resolve().parent.parent


def test_library_exports_every_declared_symbol():
    header = (ROOT / "include" / "fgt.h").read_text()
    declared = set(re.findall(r"^\s*(?:fgt_status|void|const char\*|int32_t)\s+(fgt_\w+)\s*\(", header, re.M))
    assert declared == set(_fgt.EXPORTED)
    lib = ctypes.CDLL(str(_fgt.LIB_PATH))
    for name in declared:
        assert hasattr(lib, name), name
    assert _fgt.lib.fgt_abi_version() == ir.ABI_VERSION


def _spec(outputs, **kw):
    return _fgt.Spec(outputs[0].graph.descriptor(outputs), **kw)


def test_type_errors_are_reported_before_any_launch():
    g = ir.Graph()
    x = g.parameter("f32", (4, 4))
    y = g.parameter("f32", (4, 4))
    out = g.add(x, y)
    desc = g.descriptor([out])
    # corrupt the declared type: the library re-infers and rejects it
    desc._nodes[2].shape[1] = 5
    with pytest.raises(_fgt.FgtError, match="result type must match"):
        _fgt.Spec(desc)
    desc = g.descriptor([out])
    desc._nodes[2].operands[1] = 7
    with pytest.raises(_fgt.FgtError, match="earlier nodes"):
        _fgt.Spec(desc)


def test_python_builder_enforces_fuga_typing():
    g = ir.Graph()
    x = g.parameter("f32", (2, 3))
    with pytest.raises(TypeError):
        g.add(x, g.parameter("f32", (3, 2)))
    with pytest.raises(TypeError):
        g.div(g.parameter("i32", (2,)), g.parameter("i32", (2,)))
    with pytest.raises(ValueError):
        g.reduce_max(g.parameter("f32", (2, 0)), (1,))
    with pytest.raises(ValueError):
        g.broadcast_in_dim(x, (2, 4), (0, 1))


def test_launch_without_driver_or_with_bad_arguments_fails_loudly():
    g = ir.Graph()
    x = g.parameter("f32", (8,))
    spec = _spec([g.exp(x)])
    with pytest.raises(_fgt.FgtError):
        spec.launch([0], [0])  # NULL buffers (or no driver): rejected, nothing runs


def test_workspace_too_small_is_rejected():
    g = ir.Graph()
    x = g.parameter("f32", (1000,))
    spec = _spec([g.reduce_sum(x, (0,))])
    assert spec.workspace_bytes > 0
    with pytest.raises(_fgt.FgtError, match="workspace"):
        spec.launch([16], [16], workspace=256, workspace_bytes=spec.workspace_bytes - 1)


def _validate_plan_v1(plan):
    """The structural checks of the reference's validate_plan (src/fugatensor/_ask/plan.py:21-86)."""
    assert set(plan) == {"schema_version", "kind", "inputs", "outputs", "buffers", "steps", "scheduling"}
    assert plan["schema_version"] == 1 and plan["kind"] == "ask.cuda.execution_plan"
    assert plan["scheduling"] == {"policy": "sequential", "stream": "session"}
    buffers = {b["id"]: b for b in plan["buffers"]}
    for b in plan["buffers"]:
        assert set(b) == {"id", "shape", "element_type"} and b["element_type"] in ir.WIDTH
    producers = dict.fromkeys(plan["inputs"])
    for step in plan["steps"]:
        assert set(step) == {"id", "kind", "function", "inputs", "outputs", "depends_on"}
        assert step["kind"] == "owned"
        assert all(n in producers for n in step["inputs"])
        producers.update(dict.fromkeys(step["outputs"], step["id"]))
    assert all(n in producers for n in plan["outputs"])
    assert set(plan["inputs"]) | set(plan["outputs"]) <= set(buffers)


EXPECTED_KERNELS = {
    ("c1", "chain_rowsum"): ["row"],
    ("c2", "softmax_fwd"): ["row"],
    ("c2", "softmax_vjp"): ["row"],
    ("c3", "rmsnorm_fwd"): ["row"],
    ("c3", "rmsnorm_vjp"): ["row", "colfin"],
    ("c3", "layernorm_fwd"): ["row"],
    ("c3", "layernorm_vjp"): ["row", "colfin"],
    ("c4", "global_reductions"): ["elem", "fullfin"],
    ("c5", "broadcast_select"): ["row"],
}


@pytest.mark.parametrize("cfg,variant", sorted(EXPECTED_KERNELS))
def test_workloads_fuse_into_one_pass(cfg, variant):
    """Each workload is one HBM pass: one main kernel (+ a partial-combine kernel for
    reductions across rows). The reference needs >= 3 owned steps for softmax."""
    eng = ft.Engine("cuda:0")
    inp = W.make_inputs(cfg, 16, 256)
    dts = W.input_dtypes(cfg)
    t = {k: eng.tensor(v, dtype=dts[k]) for k, v in inp.items()}
    outs = W.build(cfg, variant, t)
    spec, desc, leaves, roots = eng.compile(*outs)
    kinds = [k["name"].split("_")[1] for k in spec.execution_plan["cuda_lowering"]["kernels"]]
    assert kinds == EXPECTED_KERNELS[(cfg, variant)]
    plan = dict(spec.execution_plan)
    plan.pop("cuda_lowering")
    _validate_plan_v1(plan)
    # compiled once; a structurally equal partition hits the cache
    t2 = {k: eng.tensor(v, dtype=dts[k]) for k, v in inp.items()}
    eng.compile(*W.build(cfg, variant, t2))
    assert eng.cache_info() == {"compilations": 1, "cache_hits": 1, "specializations": 1}


@pytest.mark.parametrize("cfg,variant", sorted(EXPECTED_KERNELS))
@pytest.mark.parametrize("n", [64, 8192])
def test_square_shapes_keep_column_reductions_in_one_pass(cfg, variant, n):
    """With rows == columns a column reduction also matches the row extents
    transposed; orientation must follow the reduced axes, so square shapes plan
    the same kernels as rectangular ones (no second, strided row kernel)."""
    import torch
    eng = ft.Engine("cuda:0")
    dts = W.input_dtypes(cfg)
    shapes = {"x": (n, n), "y": (n, n), "X": (n, n), "dY": (n, n), "gamma": (n,), "beta": (n,), "A": (n, n),
              "B": (n, 1), "C": (1, n)}
    t = {k: ft.Tensor(eng, dts[k], shapes[k], data=torch.empty(0)) for k in dts}
    spec, *_ = eng.compile(*W.build(cfg, variant, t))
    kinds = [k["name"].split("_")[1] for k in spec.execution_plan["cuda_lowering"]["kernels"]]
    assert kinds == EXPECTED_KERNELS[(cfg, variant)]


def test_full_size_workloads_specialise():
    """Planning + sm_100a compilation of every benchmark workload at its full size."""
    eng = ft.Engine("cuda:0")
    for cfg, variants in W.VARIANTS.items():
        rows, cols = W.FULL[cfg]
        for variant in variants:
            g = ir.Graph()
            # build via the public API on tiny placeholders, then re-trace at full size
            dts = W.input_dtypes(cfg)
            import torch
            shapes = {"x": (rows, cols), "y": (rows, cols), "X": (rows, cols), "dY": (rows, cols), "gamma": (cols,),
                      "beta": (cols,), "A": (rows, cols), "B": (rows, 1), "C": (1, cols)}
            t = {k: ft.Tensor(eng, dts[k], shapes[k], data=torch.empty(0)) for k in dts}
            outs = W.build(cfg, variant, t)
            spec, *_ = eng.compile(*outs)
            lw = spec.execution_plan["cuda_lowering"]
            main = lw["kernels"][0]
            if main["name"].startswith("fgt_row"):
                assert main["streaming"] is False  # the row stays in registers
            for k in lw["kernels"]:  # the sm_100a compile report travels with the plan
                assert 0 < k["registers"] <= 255 and k["spill_bytes"] == 0, k
            assert spec.kernel_count == len(EXPECTED_KERNELS[(cfg, variant)])


def test_layer_norm_vjp_materialises_no_row_temporaries():
    eng = ft.Engine("cuda:0")
    inp = W.make_inputs("c3", 8, 512)
    t = {k: eng.tensor(v, dtype="bf16") for k, v in inp.items()}
    outs = W.build("c3", "layernorm_vjp", t)
    spec, *_ = eng.compile(*outs)
    assert spec.execution_plan["cuda_lowering"]["temporary_buffer_count"] == 0


# ------------------------------------------------------------ codec KATs ---
def test_encode_float_rne_subnormals_overflow():
    """tests/backend/test_numerics.py:27-46 restated against the builder's codec."""
    for dtype, step, smallest in (("f16", 2.0**-10, 2.0**-24), ("bf16", 2.0**-7, 2.0**-133), ("f32", 2.0**-23, 2.0**-149)):
        assert ir.round_float(1 + step / 2, dtype) == 1
        assert ir.round_float(1 + 3 * step / 2, dtype) == 1 + 2 * step
        assert ir.round_float(smallest, dtype) == smallest
        assert ir.round_float(smallest / 2, dtype) == 0
        assert ir.round_float(3 * smallest / 2, dtype) == 2 * smallest
        assert math.copysign(1, ir.round_float(-smallest / 2, dtype)) == -1
    assert ir.round_float(2**100 + 2**76 + 1, "f32") == float(2**100 + 2**77)
    assert ir.round_float(Fraction(1) + Fraction(1, 2**24) + Fraction(1, 2**80), "f32") == 1 + 2**-23
    assert ir.round_float(65504, "f16") == 65504
    with pytest.raises(ValueError):
        ir.encode_float(65520, "f16")


def test_empty_rows_keep_the_bound_check():
    """A row reduction over empty rows ([R, 0]) must keep the per-chunk bound check:
    every chunk is out of range, so the kernel reads nothing and writes identities."""
    import torch
    eng = ft.Engine("cuda:0", tune=False)
    x = ft.Tensor(eng, ft.fp32, (6, 10), data=torch.empty(0))
    s = x[:, 7:3].sum(axis=1)
    spec, *_ = eng.compile(s)
    src = spec.kernel_source(0)
    assert "if (e0 < NI)" in src and "if (true)" not in src


def test_column_reductions_over_long_rows_plan_as_tiles():
    """Rows past the register-resident limit: a column-only group splits the row
    into column tiles; a group with row reductions too keeps the seed's role and
    leaves the other role to a later group."""
    from fugatensor_b200 import _fgt
    g = ir.Graph()
    x = g.parameter("f32", (8, 100001))
    s = _fgt.Spec(g.descriptor([g.reduce_sum(x, (0,)), g.argmax(x, 0)]))
    ks = s.execution_plan["cuda_lowering"]["kernels"]
    row = [k for k in ks if k["name"].startswith("fgt_row")]
    assert len(row) == 1 and row[0]["col_tiles"] == 25 and not row[0]["streaming"]
    assert "blockIdx.y * 4096LL" in s.kernel_source(0) and "if (e0 < NI)" in s.kernel_source(0)
    for first_row in (True, False):
        g = ir.Graph()
        x = g.parameter("f32", (64, 100000))
        rs, cs = g.reduce_sum(x, (1,)), g.reduce_sum(g.mul(x, x), (0,))
        s = _fgt.Spec(g.descriptor([rs, cs] if first_row else [cs, rs]))
        row = [k for k in s.execution_plan["cuda_lowering"]["kernels"] if k["name"].startswith("fgt_row")]
        assert sorted((k["streaming"], k["col_tiles"]) for k in row) == [(False, 25), (True, 1)]
    # a row just past 256 threads x 16 chunks takes more threads instead of streaming
    g = ir.Graph()
    x = g.parameter("f32", (64, 129, 33))
    s = _fgt.Spec(g.descriptor([g.reduce_sum(x, (0,))]))
    k0 = s.execution_plan["cuda_lowering"]["kernels"][0]
    assert k0["threads_per_row"] == 512 and not k0["streaming"] and k0["col_tiles"] == 1


def test_row_scatter_plans_as_bucket_lists():
    """scatter_add along axis 0 with 1-D indices and materialised updates takes
    the bucket-list form (clear the list heads, link every in-range update into
    its row's list, walk each row's list once); other scatters keep the atomic
    accumulator form."""
    from fugatensor_b200 import _fgt
    g = ir.Graph()
    b, i, u = g.parameter("f32", (1000, 64)), g.parameter("i32", (300,)), g.parameter("f32", (300, 64))
    s = _fgt.Spec(g.descriptor([g.scatter_add(b, i, u, 0)]))
    ks = s.execution_plan["cuda_lowering"]["kernels"]
    assert len(ks) == 3 and "] = -1;" in s.kernel_source(0) and "atomicExch(" in s.kernel_source(1)
    assert "atomic" not in s.kernel_source(2) and "fgt_vload_keep(ua_" in s.kernel_source(2)
    # along axis 1: the accumulator form
    g = ir.Graph()
    b, i, u = g.parameter("f32", (64, 1000)), g.parameter("i32", (300,)), g.parameter("f32", (64, 300))
    s = _fgt.Spec(g.descriptor([g.scatter_add(b, i, u, 1)]))
    assert s.kernel_count == 3 and "atomicAdd" in s.kernel_source(1)
    # computed updates (not materialised): the accumulator form
    g = ir.Graph()
    b, i, u = g.parameter("f32", (1000, 64)), g.parameter("i32", (300,)), g.parameter("f32", (300, 64))
    s = _fgt.Spec(g.descriptor([g.scatter_add(b, i, g.mul(u, u), 0)]))
    assert s.kernel_count == 3


def test_every_kernel_waits_for_its_predecessor_first():
    """Kernels are launched with programmatic stream serialization, so each may
    be scheduled before the kernel ahead of it on the stream has finished: the
    first statement of every generated kernel (row, element, whole-tensor and
    column finaliser kinds) lets its own dependents be scheduled and waits for its predecessor
    (griddepcontrol) before anything is read."""
    from fugatensor_b200 import _fgt
    g = ir.Graph()
    b, i, u = g.parameter("f32", (1000, 64)), g.parameter("i32", (300,)), g.parameter("f32", (300, 64))
    x = g.parameter("f32", (64, 512))
    specs = [_fgt.Spec(g.descriptor([g.scatter_add(b, i, u, 0)])),
             _fgt.Spec(g.descriptor([g.reduce_sum(g.exp(x), (1,)), g.reduce_sum(x, (0, 1))])),
             _fgt.Spec(g.descriptor([g.reduce_sum(g.exp(x), (1,)), g.reduce_sum(x, (0,))]))]
    for s in specs:
        for k in range(s.kernel_count):
            src = s.kernel_source(k)
            body = src[src.index("(const FgtArgs p) {") + len("(const FgtArgs p) {"):].lstrip()
            assert body.startswith("fgt_pdl_enter();"), src[:400]


def test_vector_width_ignores_per_row_and_guarded_loads():
    """The vector width follows the loads that can be vector loads: a row gather
    of f32 rows with i64 indices (one index per row, guarded element reads)
    runs at 4 elements per chunk, not the 2 an 8-byte load would allow."""
    from fugatensor_b200 import _fgt
    g = ir.Graph()
    t, i = g.parameter("f32", (1000, 512)), g.parameter("i64", (300,))
    s = _fgt.Spec(g.descriptor([g.gather(t, i, 0)]))
    assert [k["vector"] for k in s.execution_plan["cuda_lowering"]["kernels"]] == [4]
    # a contiguous i64 operand still limits the width to two 8-byte elements
    g = ir.Graph()
    a, b = g.parameter("i64", (1000, 512)), g.parameter("f32", (1000, 512))
    s = _fgt.Spec(g.descriptor([g.add(g.cast(a, "f32"), b)]))
    assert [k["vector"] for k in s.execution_plan["cuda_lowering"]["kernels"]] == [2]


def test_digits_taken_once_per_chunk():
    """When the innermost extent is a whole number of vector chunks the element
    digits come from the chunk's first element; otherwise each element divides."""
    from fugatensor_b200 import _fgt
    def src(cols):
        g = ir.Graph()
        x = g.parameter("f32", (64, cols))
        r = g.slice(x, (0, cols - 1), (64, -1), (1, -1))
        return _fgt.Spec(g.descriptor([g.concatenate([x, r], 1)])).kernel_source(0)
    assert "(unsigned long long)e0" in src(256)
    assert "(unsigned long long)e0" not in src(255)
    # extents below 2^30: the digits are 32-bit values
    assert "const int i0 = (int)(((unsigned long long)e0" in src(256)


def test_chunk_digit_rule_matches_per_element_digits():
    """The per-chunk digit rule the generator uses: with the innermost extent a
    whole number of vector chunks (innermost weight 1), the digits of element
    e0 + v equal e0's outer digits and e0's innermost digit plus v."""
    import numpy as np
    rng = np.random.default_rng(3)
    for _ in range(200):
        vec = int(rng.choice([2, 4, 8]))
        dims = [int(rng.integers(1, 7)) for _ in range(int(rng.integers(1, 4)))]
        dims.append(vec * int(rng.integers(1, 9)))
        weights = [int(np.prod(dims[k + 1:])) for k in range(len(dims))]
        n = int(np.prod(dims))
        for e0 in range(0, n, vec):
            for v in range(vec):
                full = [((e0 + v) // w) % m for w, m in zip(weights, dims)]
                chunk = [(e0 // w) % m for w, m in zip(weights, dims)]
                chunk[-1] += v
                assert full == chunk
