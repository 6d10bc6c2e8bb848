"""The reciprocal inside every device sigmoid (rcp.approx + one
Newton-Raphson step, no branch) equals IEEE round-to-nearest division for
every float in [1, 2^126) -- all 1,056,964,608 of them, the whole range of
the sigmoid's denominator 1 + e^t, t in [-17, 87] -- so the device sigmoid
and its host twin (which divides) agree bit for bit.  The packed form (two
sigmoids per call with paired FP32 operations, used by the stage-0/1 scans
and the stage-2/3 GEMM epilogue) equals two scalar calls for every float."""
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def test_device_reciprocal_is_correctly_rounded():
    from ssla_rt_b200.engine import selftest_reciprocal
    bad, first = selftest_reciprocal(0)
    assert bad == 0, f"{bad} mismatches, first at bits {first:#010x}"
    assert first == 0xFFFFFFFF


def test_packed_sigmoid_equals_scalar_for_every_float():
    from ssla_rt_b200.engine import selftest_sigmoid_pair
    bad, first = selftest_sigmoid_pair(0)
    assert bad == 0, f"{bad} mismatches, first at bits {first:#010x}"
    assert first == 0xFFFFFFFF
