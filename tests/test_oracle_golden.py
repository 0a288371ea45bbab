"""Pin the NumPy oracle against the reference's own outputs and known answers.

The golden fixtures were written by ``tests/golden/make_golden.py`` running the
reference trnfft on its ``"pytorch"`` backend.  The oracle restates the same
float32 arithmetic, so agreement is at the level of a few float32 ulps
(rel-L2 <= 1e-6 for power-of-2 paths).
"""

import math

import numpy as np
import pytest

from oracle import trnfft_oracle as O

POW2 = [2, 4, 8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096]


@pytest.mark.parametrize("n", POW2)
def test_pow2_c2c(golden, n):
    g = golden("pow2_c2c")
    xr, xi = g[f"x_re_{n}"], g[f"x_im_{n}"]
    yr, yi = O.fft(xr, xi)
    zr, zi = O.ifft(xr, xi)
    assert O.rel_l2(yr + 1j * yi, g[f"fft_re_{n}"] + 1j * g[f"fft_im_{n}"]) < 1e-6
    assert O.rel_l2(zr + 1j * zi, g[f"ifft_re_{n}"] + 1j * g[f"ifft_im_{n}"]) < 1e-6


@pytest.mark.parametrize("n", [8192, 16384])
def test_pow2_large(golden, n):
    g = golden("pow2_large")
    yr, yi = O.fft(g[f"x_re_{n}"], g[f"x_im_{n}"])
    assert O.rel_l2(yr + 1j * yi, g[f"fft_re_{n}"] + 1j * g[f"fft_im_{n}"]) < 1e-6


@pytest.mark.parametrize("n", [3, 5, 7, 11, 100, 127, 997, 1000, 4093, 6000])
@pytest.mark.parametrize("prec", ["fast", "double"])
def test_bluestein(golden, n, prec):
    g = golden("bluestein")
    xr, xi = g[f"x_re_{n}"], g[f"x_im_{n}"]
    yr, yi = O.fft(xr, xi, precision=prec)
    zr, zi = O.ifft(xr, xi, precision=prec)
    tol = 1e-6 if prec == "double" else 2e-6
    assert O.rel_l2(yr + 1j * yi, g[f"fft_{prec}_re_{n}"] + 1j * g[f"fft_{prec}_im_{n}"]) < tol
    assert O.rel_l2(zr + 1j * zi, g[f"ifft_{prec}_re_{n}"] + 1j * g[f"ifft_{prec}_im_{n}"]) < tol


@pytest.mark.parametrize("n", [4093, 6000])
def test_bluestein_fast_mode_error_is_the_chirp(golden, n):
    """The reference's "fast" Bluestein is ~1e-4 off the exact DFT (float32 chirp angle,
    trnfft/fft_core.py:1316-1320); "double" is ~1e-8.  This pins the discrepancy
    the CUDA Bluestein is measured against."""
    g = golden("bluestein")
    x = g[f"x_re_{n}"].astype(np.float64) + 1j * g[f"x_im_{n}"]
    exact = np.fft.fft(x)
    fast = g[f"fft_fast_re_{n}"] + 1j * g[f"fft_fast_im_{n}"]
    dbl = g[f"fft_double_re_{n}"] + 1j * g[f"fft_double_im_{n}"]
    assert O.rel_l2(fast, exact) > 2e-5
    assert O.rel_l2(dbl, exact) < 1e-7


@pytest.mark.parametrize("n", [16, 128, 1024, 100, 4093])
def test_real(golden, n):
    g = golden("real")
    x = g[f"x_{n}"]
    for prec, tol in [("fast", 2e-6), ("double", 1e-6)]:
        r, i = O.rfft(x, precision=prec)
        ref = g[f"rfft_{prec}_re_{n}"] + 1j * g[f"rfft_{prec}_im_{n}"]
        assert O.rel_l2(r + 1j * i, ref) < tol
        back = O.irfft(g[f"rfft_{prec}_re_{n}"], g[f"rfft_{prec}_im_{n}"], n=n, precision=prec)
        assert O.rel_l2(back, g[f"irfft_{prec}_{n}"]) < tol
        spec = O.irfft(g[f"spec_re_{n}"], g[f"spec_im_{n}"], n=n, precision=prec)
        assert O.rel_l2(spec, g[f"irfft_spec_{prec}_{n}"]) < tol


def test_nd(golden):
    g = golden("nd")
    for key in ["16x32", "64x64", "8x256"]:
        yr, yi = O.fft2(g[f"x_re_{key}"], g[f"x_im_{key}"])
        assert O.rel_l2(yr + 1j * yi, g[f"fft2_re_{key}"] + 1j * g[f"fft2_im_{key}"]) < 1e-6
        zr, zi = O.ifft2(g[f"x_re_{key}"], g[f"x_im_{key}"])
        assert O.rel_l2(zr + 1j * zi, g[f"ifft2_re_{key}"] + 1j * g[f"ifft2_im_{key}"]) < 1e-6
    yr, yi = O.fftn(g["x3"])
    assert O.rel_l2(yr + 1j * yi, g["fftn3_re"] + 1j * g["fftn3_im"]) < 1e-6
    yr, yi = O.fftn(g["x3"], dim=(0, 2))
    assert O.rel_l2(yr + 1j * yi, g["fftn3_d02_re"] + 1j * g["fftn3_d02_im"]) < 1e-6


@pytest.mark.parametrize("name,kw", [
    ("c512", dict(n_fft=512, hop_length=256)),
    ("c256_64", dict(n_fft=256, hop_length=64)),
    ("c128_nocenter", dict(n_fft=128, hop_length=32, center=False)),
    ("c512_norm_two", dict(n_fft=512, hop_length=128, normalized=True, onesided=False)),
    ("c256_win200", dict(n_fft=256, hop_length=100, win_length=200)),
    ("c64_const", dict(n_fft=64, hop_length=16, pad_mode="constant")),
])
def test_stft(golden, name, kw):
    g = golden("stft")
    r, i = O.stft(g["wave"], **kw)
    ref = g[f"stft_re_{name}"] + 1j * g[f"stft_im_{name}"]
    assert r.shape == ref.shape
    assert O.rel_l2(r + 1j * i, ref) < 1e-6


def test_istft(golden):
    g = golden("stft")
    r, i = O.stft(g["wave"], n_fft=256, hop_length=64)
    back = O.istft(r, i, n_fft=256, hop_length=64, length=4000)
    assert O.rel_l2(back, g["istft_256_64"]) < 1e-6
    np.testing.assert_allclose(back, g["wave"], atol=1e-3)


@pytest.mark.parametrize("n", [64, 4096, 65536])
def test_four_step(golden, n):
    g = golden("four_step")
    yr, yi = O.stage_parallel_fft(g[f"x_re_{n}"], g[f"x_im_{n}"], False)
    zr, zi = O.stage_parallel_fft(g[f"x_re_{n}"], g[f"x_im_{n}"], True)
    assert O.rel_l2(yr + 1j * yi, g[f"sp_re_{n}"] + 1j * g[f"sp_im_{n}"]) < 1e-6
    assert O.rel_l2(zr + 1j * zi, g[f"spi_re_{n}"] + 1j * g[f"spi_im_{n}"]) < 1e-6


def test_linear(golden):
    g = golden("linear")
    yr, yi = O.complex_linear(g["x_re"], g["x_im"], g["w_re"], g["w_im"], g["b_re"], g["b_im"])
    assert O.rel_l2(yr + 1j * yi, g["y_re"] + 1j * g["y_im"]) < 1e-6
    cr, ci = O.complex_matmul(g["a_re"], g["a_im"], g["b2_re"], g["b2_im"])
    assert O.rel_l2(cr + 1j * ci, g["c_re"] + 1j * g["c_im"]) < 1e-6


# --- the reference's known-answer tests (tests/test_fft.py:12-69, test_complex.py:35-55)

def test_known_answers():
    x = np.zeros(16, np.float32)
    x[0] = 1
    r, i = O.fft(x)
    np.testing.assert_allclose(r, np.ones(16), atol=1e-6)
    np.testing.assert_allclose(i, np.zeros(16), atol=1e-6)
    r, i = O.fft(np.ones(16, np.float32))
    assert abs(r[0] - 16) < 1e-5 and np.abs(np.hypot(r[1:], i[1:])).max() < 1e-5
    t = np.arange(64, dtype=np.float32)
    r, i = O.fft(np.cos(2 * np.pi * 5 * t / 64).astype(np.float32))
    mag = np.hypot(r, i)
    assert mag[5] > 31 and mag[59] > 31
    r, i = O.fft(np.array([1, 2, 3, 4], np.float32), n=8)
    e = np.fft.fft([1, 2, 3, 4, 0, 0, 0, 0])
    np.testing.assert_allclose(r, e.real, atol=1e-5)
    np.testing.assert_allclose(i, e.imag, atol=1e-5)
    cr, ci = O.complex_matmul(np.array([[1.0]]), np.array([[2.0]]), np.array([[3.0]]), np.array([[4.0]]))
    assert abs(cr[0, 0] + 5) < 1e-6 and abs(ci[0, 0] - 10) < 1e-6


def test_oracle_vs_fp64_numpy(rng):
    """The oracle (like the reference) is an accurate float32 FFT: ~1e-7 vs fp64."""
    for n in [64, 1024, 4096]:
        x = rng.standard_normal((4, n)) + 1j * rng.standard_normal((4, n))
        r, i = O.fft(x.real.astype(np.float32), x.imag.astype(np.float32))
        assert O.rel_l2(r + 1j * i, np.fft.fft(x.astype(np.complex64).astype(np.complex128))) < 1e-6
    assert O.factorize(1 << 30) == (32768, 32768)
    assert O.padded_length(4093) == 8192 and O.padded_length(6000) == 16384
    assert math.isclose(O.hann_window_periodic(4)[2], 1.0)
