"""Host logic of the tuner's parity gate (tuning.agrees), on CPU tensors."""
import torch

from fugatensor_b200 import tuning


def test_integer_outputs_must_match_bit_for_bit():
    a = torch.tensor([1, 2, 3], dtype=torch.int64)
    assert tuning.agrees([a], [a.clone()], [("i64", (3,))])
    assert not tuning.agrees([a], [a + torch.tensor([0, 0, 1])], [("i64", (3,))])


def test_float_tolerance_is_relative_to_output_scale():
    ref = torch.tensor([1000.0, 1.0, -2.0])
    ok = ref + torch.tensor([0.0, 1000.0 * 0.9e-5, 0.0])  # within rtol * (|r| + max|r|)
    bad = ref + torch.tensor([0.0, 1000.0 * 1.2e-5 + 1e-5, 0.0])
    assert tuning.agrees([ok], [ref], [("f32", (3,))])
    assert not tuning.agrees([bad], [ref], [("f32", (3,))])
    # bf16: 1e-2
    rb = ref.to(torch.bfloat16)
    assert tuning.agrees([rb], [rb], [("bf16", (3,))])


def test_nan_and_inf_positions_must_agree():
    ref = torch.tensor([float("nan"), float("inf"), 1.0])
    assert tuning.agrees([ref.clone()], [ref], [("f32", (3,))])
    assert not tuning.agrees([torch.tensor([0.0, float("inf"), 1.0])], [ref], [("f32", (3,))])
    assert not tuning.agrees([torch.tensor([float("nan"), float("-inf"), 1.0])], [ref], [("f32", (3,))])
