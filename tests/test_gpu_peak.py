"""The tcgen05 dense-throughput probe (aeisu_tensor_peak) behind the bench's E4M3 roofline
denominator."""
import pytest

pytestmark = pytest.mark.gpu


def test_tensor_peak_probe():
    """aeisu_tensor_peak: dense tcgen05 rates of this GPU for the roofline denominators.  The
    bounds only exclude a probe that did not run the MMAs (B200 dense f16 is 2.25 PFLOP/s
    nominal, E4M3 twice that)."""
    import ctypes as C
    from aeisu_b200 import _lib
    lib = _lib.lib()
    rates = {}
    for kind in (0, 1):
        v = C.c_double()
        _lib.check(lib.aeisu_tensor_peak(0, kind, 2, 1024, 2, C.byref(v)))
        rates[kind] = v.value
    assert 800.0 < rates[0] < 2600.0, rates
    assert 1.6 < rates[1] / rates[0] < 2.4, rates
    v = C.c_double()
    assert lib.aeisu_tensor_peak(0, 2, 2, 1024, 2, C.byref(v)) == _lib.INVALID_ARG
    assert lib.aeisu_tensor_peak(0, 0, 3, 1024, 2, C.byref(v)) == _lib.INVALID_ARG
