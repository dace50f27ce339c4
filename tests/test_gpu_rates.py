"""atlb_measure_unit_rates: the execution-unit rates behind the pair kernels' compute roofline come out
positive and within the range a B200-class device can reach (whole-device operations per second)."""
import pytest

pytestmark = pytest.mark.gpu


def test_unit_rates_plausible():
    from x_b200 import _lib
    r = _lib.unit_rates()
    # FP32 lanes: 148 SMs x 128 lanes x ~2 GHz = 3.7e13 FMA/s; packed f32x2 at most twice that
    assert 5e12 < r["fp32_lane_ops"] < 1e14
    assert 5e12 < r["fp32x2_lane_ops"] < 2e14
    # SFU: 16 lanes per SM and clock = 4.6e12/s at 1.965 GHz
    assert 5e11 < r["ex2"] < 2e13
    for k in ("red_f32", "red_v4", "smem_atomic"):
        assert 1e9 < r[k] < 1e14, (k, r[k])


def test_unit_rates_rejects_small_scratch():
    import ctypes
    import torch
    from x_b200 import _lib
    L = _lib.lib()
    out = _lib.UnitRates()
    buf = torch.empty(1024, dtype=torch.uint8, device="cuda")
    st = L.atlb_measure_unit_rates(ctypes.byref(out), _lib.ptr(buf), 1024, _lib.stream())
    assert st == _lib.ATLB_ERR_WORKSPACE
