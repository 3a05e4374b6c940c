"""The division of the fused requant epilogue (trba_gemm_int8_requant): an
FMA-based division against a host-rounded reciprocal (Markstein's method)
must equal the IEEE division bit for bit for every s32 accumulator value.
trba_requant_division_check runs all 2^32 values on the device for one
divisor; divisors outside the method's range (|div| < 2^-90 or > 2^90, or
not finite) are reported as -1 and divided with the IEEE division by the
epilogue itself."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

DIVISORS = [127.0, 50.0, 1.0, 3.0, 0.5, 1e-3, 7.77, -127.0, 2.0 ** -90, 2.0 ** 90, 6.0221e23, 1.0000001,
            0.99999994, 16777215.0]


@pytest.mark.parametrize("div", DIVISORS)
def test_epilogue_division_equals_ieee_division(div, lib, cuda):
    assert lib.trba_requant_division_check(float(np.float32(div)), None) == 0
    assert lib.trba_last_error() == 0, lib.trba_last_error_string()


def test_random_divisors(lib, cuda):
    rng = np.random.default_rng(11)
    for e in rng.uniform(-89, 89, 6):
        d = float(np.float32(rng.uniform(1, 2) * 2.0 ** e))
        assert lib.trba_requant_division_check(d, None) == 0, d


@pytest.mark.parametrize("div", [2.0 ** -100, 2.0 ** 100, float("inf")])
def test_divisors_outside_the_range_take_the_ieee_division(div, lib, cuda):
    assert lib.trba_requant_division_check(div, None) == -1
