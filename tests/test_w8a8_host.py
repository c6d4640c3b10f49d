"""Host logic of the W8A8 activation plans (no GPU): the calibration-range
resolution of AexisOps.SetInt8ActivationQuantization(QuantizedActivationPlan)
(AexisOps.cs:763-785) and ActivationCalibrationRange.SymmetricScale
(Core/AexisPrecisionContracts.cs:30-37), and the oracle's fake-quantisation
(HLSL Pack4Matmul:792-800)."""
import numpy as np
import pytest

from aiimage_b200 import errors
from aiimage_b200.ops import resolve_int8_activation_plan


def test_unsigned_plan_scale_and_zero_point():
    scale, zp, uns = resolve_int8_activation_plan(-1.0, 3.0, True)
    assert uns and scale == float(np.float32(4.0) / np.float32(255.0))
    assert zp == 64                                # RoundToInt(63.75)
    assert resolve_int8_activation_plan(2.0, 2.0, True) == (1.0, 0, True)     # empty range -> scale 1
    assert resolve_int8_activation_plan(1.0, 5.0, True)[1] == 0               # clamp to [0, 255]
    assert resolve_int8_activation_plan(-10.0, -5.0, True)[1] == 255


def test_symmetric_plan_scale():
    scale, zp, uns = resolve_int8_activation_plan(-2.0, 1.0, False)
    assert (zp, uns) == (0, False) and scale == float(np.float32(2.0) / np.float32(127.0))
    assert resolve_int8_activation_plan(0.0, 0.0, False) == (1.0, 0, False)


@pytest.mark.parametrize("lo,hi", [(1.0, -1.0), (float("nan"), 1.0), (0.0, float("inf"))])
def test_plan_bounds_must_be_finite_and_ordered(lo, hi):
    with pytest.raises(errors.InvalidOperationError):
        resolve_int8_activation_plan(lo, hi, True)


def test_oracle_fake_quant_rounds_half_to_even_and_clamps(oracle):
    x = np.array([0.25, 0.75, -0.25, 100.0, -100.0, 1.1], dtype=np.float32)
    got = oracle.quantize_activation_int8(x, 0.5)
    assert list(got) == [0.0, 1.0, -0.0, 63.5, -64.0, 1.0]
    got_u = oracle.quantize_activation_int8(x, 0.5, zp=128, unsigned=True)
    assert list(got_u) == [0.0, 1.0, -0.0, 63.5, -64.0, 1.0]
    assert list(oracle.quantize_activation_int8(np.array([-1.0, 300.0], np.float32), 1.0, zp=0, unsigned=True)) == [0.0, 255.0]
