"""fgt_reduce_f32_noalloc: the allocation-free variant of the whole-tensor reduction.

Some callers cannot allocate device memory at all -- code running inside an
allocator or memory-manager callback, services that must not touch the
device allocator once started, hosts that own every device buffer -- so they
cannot provide the workspace the regular entry point (fgt_spec_launch) asks
for. The variant keeps its partials in a static device array instead. These
tests call it through the C ABI and check it against the regular entry point
on the same data, twice in a row (the array keeps the previous call's
contents, which must not leak into the next result).
"""
import ctypes

import numpy as np
import pytest
import torch

from fugatensor_b200 import _fgt, ir

pytestmark = pytest.mark.gpu

lib = _fgt.lib
lib.fgt_reduce_f32_noalloc.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
lib.fgt_reduce_f32_noalloc.restype = ctypes.c_int32

RTOL = 1e-5  # the f32 tolerance of every other parity test


def regular(x):
    """sum, amax, argmax, mean through a partition launched with fgt_spec_launch (workspace scratch)."""
    n = x.numel()
    g = ir.Graph()
    p = g.parameter("f32", (n,))
    s = g.reduce_sum(p, (0,))
    mean = g.div(s, g.constant(n, "f32"))
    spec = _fgt.Spec(g.descriptor([s, g.reduce_max(p, (0,)), g.argmax(p, 0), mean]))
    outs = _fgt.run(spec, x)
    torch.cuda.synchronize()
    return [o.item() for o in outs]


def no_alloc(x):
    dev = x.device
    s, m, mean = (torch.empty((), dtype=torch.float32, device=dev) for _ in range(3))
    a = torch.empty((), dtype=torch.int64, device=dev)
    st = lib.fgt_reduce_f32_noalloc(x.data_ptr(), x.numel(), s.data_ptr(), m.data_ptr(), a.data_ptr(),
                                    mean.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    assert st == 0, lib.fgt_last_error().decode()
    torch.cuda.synchronize()
    return [s.item(), m.item(), a.item(), mean.item()]


def check_same(got, ref):
    gs, gm, ga, gmean = got
    rs, rm, ra, rmean = ref
    assert ga == ra
    assert (gm == rm) or (np.isnan(gm) and np.isnan(rm))
    for g, r in ((gs, rs), (gmean, rmean)):
        if np.isnan(r):
            assert np.isnan(g)
        elif np.isinf(r):
            assert g == r
        else:
            assert abs(g - r) <= RTOL * abs(r) + 1e-30, (g, r)


@pytest.mark.parametrize("n", [1, 3, 1000003, 1 << 20, 2 << 20, (1 << 22) + 1])
def test_matches_regular_entry_point_on_two_calls(n):
    gen = torch.Generator(device="cuda").manual_seed(n)
    x1 = torch.rand(n, device="cuda", generator=gen) + 0.25
    x2 = torch.randn(n, device="cuda", generator=gen)
    if n > 10:
        x2[n // 3] = float("inf")
        x2[n // 2] = float("inf")  # tie: the first occurrence wins
    for x in (x1, x2):
        check_same(no_alloc(x), regular(x))


def test_nan_counts_as_maximum():
    x = torch.randn(300001, device="cuda")
    x[12345] = float("nan")
    x[200000] = float("nan")
    got, ref = no_alloc(x), regular(x)
    assert got[2] == ref[2] == 12345 and np.isnan(got[1]) and np.isnan(got[0])


def test_cancelling_terms_match_bit_for_bit():
    """Chunks of [2^24, 1, -2^24, 0]: an f32 running sum loses every 1 (2^24 + 1
    rounds to 2^24); adding each element in f64, as both entry points do, keeps
    them. Also a cancelling triple spread over three scratch slots."""
    n = 1 << 20
    chunk = torch.tensor([2.0 ** 24, 1.0, -(2.0 ** 24), 0.0], device="cuda")
    x1 = chunk.repeat(n // 4)
    x2 = torch.zeros(3 << 20, device="cuda")
    x2[5], x2[(1 << 20) + 7], x2[(2 << 20) + 9] = 2.0 ** 24, 1.0, -(2.0 ** 24)
    for x, total in ((x1, n // 4), (x2, 1)):
        for _ in range(2):
            got, ref = no_alloc(x), regular(x)
            assert got[0] == ref[0] == float(total)
            assert got == ref  # every output bit for bit (sum, max, argmax, mean)


def test_exact_size_limit():
    """n = 2^31 (FGT_NOALLOC_SLOTS x FGT_NOALLOC_ELEMS_PER_SLOT, 8 GiB of f32) is
    accepted and matches the regular entry point; one more element is rejected
    before anything is launched."""
    limit = 2048 * (1 << 20)
    torch.cuda.empty_cache()
    gen = torch.Generator(device="cuda").manual_seed(31)
    x = torch.randn(limit, device="cuda", generator=gen)
    x[limit - 1] = 1e30  # the maximum sits in the last element of the last slot
    for _ in range(2):
        got, ref = no_alloc(x), regular(x)
        check_same(got, ref)
        assert got[2] == limit - 1
    out = torch.zeros(4, device="cuda")
    st = lib.fgt_reduce_f32_noalloc(x.data_ptr(), limit + 1, out.data_ptr(), out.data_ptr(), out.data_ptr(),
                                    out.data_ptr(), 0)
    assert st == 1 and b"exceeds the static scratch limit" in lib.fgt_last_error()
    del x
    torch.cuda.empty_cache()


def test_sizes_beyond_the_static_scratch_are_rejected():
    x = torch.zeros(16, device="cuda")
    out = torch.zeros(4, device="cuda")
    for n in (2048 * (1 << 20) + 1, 1 << 40):
        st = lib.fgt_reduce_f32_noalloc(x.data_ptr(), n, out.data_ptr(), out.data_ptr(), out.data_ptr(),
                                        out.data_ptr(), 0)
        assert st == 1 and b"exceeds the static scratch limit" in lib.fgt_last_error()
    for n in (0, -1):
        st = lib.fgt_reduce_f32_noalloc(x.data_ptr(), n, out.data_ptr(), out.data_ptr(), out.data_ptr(),
                                        out.data_ptr(), 0)
        assert st == 1 and b"n must be positive" in lib.fgt_last_error()
