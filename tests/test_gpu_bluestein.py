"""GPU parity of the fused Bluestein kernel (any n <= 8192, padded length <= 16384).

Parity gate: the reference run with precision="double" (its accurate mode,
trnfft/fft_core.py:1306-1309) and the fp64 NumPy FFT, rel-L2 <= 1e-5.  The
reference's default "fast" mode is itself ~1e-4 off the exact DFT for
n ~ 4000 (float32 chirp angle, fft_core.py:1316-1320); the kernel tabulates an
exactly reduced chirp, so it is compared with "fast" only at small n.
"""

import numpy as np
import pytest
import torch

import trnfft_b200 as trnfft
from trnfft_b200 import ComplexTensor
from oracle import trnfft_oracle as O
from tests.helpers import TOL, cplx, cuda, host, rel_l2

pytestmark = pytest.mark.gpu

GOLDEN_N = [3, 5, 7, 11, 100, 127, 997, 1000, 4093, 6000]


@pytest.mark.parametrize("n", GOLDEN_N)
def test_vs_reference_double_golden(golden, n):
    g = golden("bluestein")
    x = ComplexTensor(cuda(g[f"x_re_{n}"]), cuda(g[f"x_im_{n}"]))
    y = trnfft.fft(x)
    z = trnfft.ifft(x)
    assert rel_l2(cplx(y), g[f"fft_double_re_{n}"] + 1j * g[f"fft_double_im_{n}"]) < TOL
    assert rel_l2(cplx(z), g[f"ifft_double_re_{n}"] + 1j * g[f"ifft_double_im_{n}"]) < TOL
    if n <= 11:  # the reference's float32 chirp is still exact enough only for tiny n
        assert rel_l2(cplx(y), g[f"fft_fast_re_{n}"] + 1j * g[f"fft_fast_im_{n}"]) < TOL


@pytest.mark.parametrize("n", [6, 12, 17, 31, 33, 100, 255, 257, 1000, 2047, 4093, 6000, 8190, 8191])
@pytest.mark.parametrize("batch", [1, 4])
def test_vs_fp64(n, batch):
    rng = np.random.default_rng(n + 17 * batch)
    x = rng.standard_normal((batch, n)) + 1j * rng.standard_normal((batch, n))
    x = x.astype(np.complex64)
    y = trnfft.fft(ComplexTensor(cuda(x.real), cuda(x.imag)))
    ref = np.fft.fft(x.astype(np.complex128))
    assert rel_l2(cplx(y), ref) < 2e-6
    z = trnfft.ifft(ComplexTensor(cuda(x.real), cuda(x.imag)))
    assert rel_l2(cplx(z), np.fft.ifft(x.astype(np.complex128))) < 2e-6


def test_roundtrip_config4_shape():
    """Config 4 shape: batch 4096 of n = 4093; ifft(fft(x)) == x."""
    torch.manual_seed(4)
    xr = torch.randn(4096, 4093, device="cuda")
    xi = torch.randn(4096, 4093, device="cuda")
    X = trnfft.fft(ComplexTensor(xr, xi))
    back = trnfft.ifft(X)
    assert rel_l2(cplx(back), host(xr) + 1j * host(xi)) < 2e-6
    sel = [0, 1, 2047, 4095]
    ref = np.fft.fft(host(xr)[sel].astype(np.float64) + 1j * host(xi)[sel])
    assert rel_l2(cplx(X)[sel], ref) < 2e-6


@pytest.mark.parametrize("n", [100, 4093])
def test_real_vs_reference_double_golden(golden, n):
    g = golden("real")
    X = trnfft.rfft(cuda(g[f"x_{n}"]))
    assert X.shape[-1] == n // 2 + 1
    assert rel_l2(cplx(X), g[f"rfft_double_re_{n}"] + 1j * g[f"rfft_double_im_{n}"]) < TOL
    y = trnfft.irfft(ComplexTensor(cuda(g[f"spec_re_{n}"]), cuda(g[f"spec_im_{n}"])), n=n)
    assert rel_l2(host(y), g[f"irfft_spec_double_{n}"]) < TOL


@pytest.mark.parametrize("n", [7, 100, 1000, 4093, 6000])
def test_real_roundtrip_and_fp64(n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal((5, n)).astype(np.float32)
    X = trnfft.rfft(cuda(x))
    assert rel_l2(cplx(X), np.fft.rfft(x.astype(np.float64))) < 2e-6
    back = trnfft.irfft(X, n=n)
    assert rel_l2(host(back), x) < 2e-6
    sr = rng.standard_normal((5, n // 2 + 1)).astype(np.float32)
    si = rng.standard_normal((5, n // 2 + 1)).astype(np.float32)
    y = trnfft.irfft(ComplexTensor(cuda(sr), cuda(si)), n=n)
    assert rel_l2(host(y), O.irfft(sr, si, n=n, precision="double")) < TOL


@pytest.mark.parametrize("n,batch", [(8193, 3), (10007, 2), (100003, 1), (1 << 20 | 1, 1)])
def test_multipass_bluestein_vs_fp64(n, batch):
    """Lengths beyond the fused kernel (padded m > 16384): multi-pass Bluestein."""
    rng = np.random.default_rng(n)
    x = (rng.standard_normal((batch, n)) + 1j * rng.standard_normal((batch, n))).astype(np.complex64)
    X = trnfft.fft(ComplexTensor(cuda(x.real), cuda(x.imag)))
    assert rel_l2(cplx(X), np.fft.fft(x.astype(np.complex128))) < 5e-6
    Z = trnfft.ifft(ComplexTensor(cuda(x.real), cuda(x.imag)))
    assert rel_l2(cplx(Z), np.fft.ifft(x.astype(np.complex128))) < 5e-6
    r = trnfft.rfft(cuda(x.real))
    assert rel_l2(cplx(r), np.fft.rfft(x.real.astype(np.float64))) < 5e-6
