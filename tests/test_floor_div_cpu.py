"""The plan's cell index floor(RN(a / c)) is computed on the device as floor(RN(a * RN(1/c))) unless that
product lies within 2^-21 |q| of an integer (then by the division itself) -- plan_math.cuh floor_div.  This
restates the rule in numpy float32 (IEEE-rounded like the device's __fmul_rn / div_rn) and checks it
against the division on random and adversarial (near-integer quotient) inputs."""
import numpy as np

f32 = np.float32


def floor_div(a, c):
    with np.errstate(invalid="ignore"):  # inf - inf for infinite quotients: NaN takes the division path
        return _floor_div(a, c)


def _floor_div(a, c):
    rc = (f32(1.0) / c).astype(f32)
    q = (a * rc).astype(f32)
    f = np.floor(q).astype(f32)
    fr = (q - f).astype(f32)
    d = (np.abs(q) * f32(2.0 ** -21)).astype(f32)
    fast = (fr > d) & (fr < (f32(1.0) - d).astype(f32))
    return np.where(fast, f, np.floor((a / c).astype(f32))), fast


def test_floor_div_matches_division():
    rng = np.random.default_rng(0)
    n = 400_000
    for kind in range(3):
        c = rng.uniform(1.0, 40.0, n).astype(f32)
        if kind == 0:  # quotients within a few ulps of an integer
            a = (rng.integers(-300, 3000, n).astype(f32) * c).astype(f32)
            a = (a + rng.integers(-3, 4, n) * np.spacing(a)).astype(f32)
        elif kind == 1:
            a = rng.uniform(-50, 12000, n).astype(f32)
        else:
            a = (rng.standard_normal(n) * 10.0 ** rng.uniform(-30, 4, n)).astype(f32)
        got, fast = floor_div(a, c)
        np.testing.assert_array_equal(got, np.floor((a / c).astype(f32)))
        if kind == 1:
            assert fast.mean() > 0.999  # the division is the rare path on ordinary coordinates


def test_floor_div_special_values():
    a = np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, -1e-38, 1e-38, 3.0], dtype=f32)
    c = np.full_like(a, f32(3.0))
    got, _ = floor_div(a, c)
    np.testing.assert_array_equal(got, np.floor((a / c).astype(f32)))
