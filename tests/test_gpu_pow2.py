"""GPU parity of the power-of-two single-CTA Stockham kernels (C2C, R2C, C2R).

Compared with the reference's own outputs (tests/golden) and with the NumPy
oracle on the same seeded inputs; tolerance rel-L2 <= 1e-5.
"""

import numpy as np
import pytest
import torch

import trnfft_b200 as trnfft
from trnfft_b200 import ComplexTensor
from oracle import trnfft_oracle as O
from tests.helpers import TOL, cplx, cuda, host, rel_l2

pytestmark = pytest.mark.gpu

POW2 = [2, 4, 8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096]


@pytest.mark.parametrize("n", POW2)
def test_c2c_vs_reference_golden(golden, n):
    g = golden("pow2_c2c")
    x = ComplexTensor(cuda(g[f"x_re_{n}"]), cuda(g[f"x_im_{n}"]))
    y = trnfft.fft(x)
    z = trnfft.ifft(x)
    assert rel_l2(cplx(y), g[f"fft_re_{n}"] + 1j * g[f"fft_im_{n}"]) < TOL
    assert rel_l2(cplx(z), g[f"ifft_re_{n}"] + 1j * g[f"ifft_im_{n}"]) < TOL


@pytest.mark.parametrize("n", POW2)
@pytest.mark.parametrize("batch", [1, 3, 257])
def test_c2c_vs_oracle_ragged_batches(n, batch):
    rng = np.random.default_rng(n * 1000 + batch)
    xr = rng.standard_normal((batch, n)).astype(np.float32)
    xi = rng.standard_normal((batch, n)).astype(np.float32)
    y = trnfft.fft(ComplexTensor(cuda(xr), cuda(xi)))
    er, ei = O.fft(xr, xi)
    assert rel_l2(cplx(y), er + 1j * ei) < TOL
    z = trnfft.ifft(ComplexTensor(cuda(xr), cuda(xi)))
    er, ei = O.ifft(xr, xi)
    assert rel_l2(cplx(z), er + 1j * ei) < TOL


def test_c2c_large_batch_roundtrip_and_fp64():
    """Config-1 shape (8192 x 1024): fft then ifft returns the input; fft vs fp64."""
    torch.manual_seed(0)
    xr = torch.randn(8192, 1024, device="cuda")
    xi = torch.randn(8192, 1024, device="cuda")
    X = trnfft.fft(ComplexTensor(xr, xi))
    ref = np.fft.fft(host(xr).astype(np.float64) + 1j * host(xi))
    assert rel_l2(cplx(X), ref) < 1e-6
    back = trnfft.ifft(X)
    assert rel_l2(cplx(back), host(xr) + 1j * host(xi)) < 1e-6


def test_known_answers():
    """The reference's known-answer tests (tests/test_fft.py:12-69)."""
    x = torch.zeros(16, device="cuda")
    x[0] = 1
    r = trnfft.fft(x)
    np.testing.assert_allclose(host(r.real), np.ones(16), atol=1e-6)
    np.testing.assert_allclose(host(r.imag), np.zeros(16), atol=1e-6)
    r = trnfft.fft(torch.ones(16, device="cuda"))
    assert abs(r.real[0].item() - 16) < 1e-5
    assert r.abs()[1:].max().item() < 1e-5
    t = torch.arange(64, dtype=torch.float32, device="cuda")
    mags = trnfft.fft(torch.cos(2 * np.pi * 5 * t / 64)).abs()
    assert mags[5].item() > 31 and mags[59].item() > 31
    r = trnfft.fft(torch.tensor([1.0, 2.0, 3.0, 4.0], device="cuda"), n=8)
    e = np.fft.fft([1, 2, 3, 4, 0, 0, 0, 0])
    np.testing.assert_allclose(host(r.real), e.real, atol=1e-5)
    np.testing.assert_allclose(host(r.imag), e.imag, atol=1e-5)


def test_cpu_tensors_roundtrip_through_device():
    x = torch.randn(4, 256)
    y = trnfft.fft(x)
    assert y.real.device.type == "cpu"
    assert rel_l2(cplx(y), np.fft.fft(x.numpy().astype(np.float64))) < 1e-6


def test_nd_batch_shape_and_n1():
    x = torch.randn(2, 3, 5, 64, device="cuda")
    y = trnfft.fft(x)
    assert y.shape == x.shape
    assert rel_l2(cplx(y), np.fft.fft(host(x).astype(np.float64))) < 1e-6
    one = torch.randn(7, 1, device="cuda")
    np.testing.assert_array_equal(host(trnfft.fft(one).real), host(one))


@pytest.mark.parametrize("n", [4, 8, 16, 64, 128, 512, 1024, 4096, 8192])
@pytest.mark.parametrize("batch", [1, 5])
def test_r2c_c2r_vs_oracle(n, batch):
    rng = np.random.default_rng(7 * n + batch)
    x = rng.standard_normal((batch, n)).astype(np.float32)
    X = trnfft.rfft(cuda(x))
    er, ei = O.rfft(x)
    assert X.shape == (batch, n // 2 + 1)
    assert rel_l2(cplx(X), er + 1j * ei) < TOL
    back = trnfft.irfft(X, n=n)
    assert rel_l2(host(back), x) < TOL
    # non-Hermitian half spectrum: imaginary parts of DC/Nyquist must not contribute
    sr = rng.standard_normal((batch, n // 2 + 1)).astype(np.float32)
    si = rng.standard_normal((batch, n // 2 + 1)).astype(np.float32)
    y = trnfft.irfft(ComplexTensor(cuda(sr), cuda(si)), n=n)
    assert rel_l2(host(y), O.irfft(sr, si, n=n)) < TOL


@pytest.mark.parametrize("n", [16, 128, 1024])
def test_real_vs_reference_golden(golden, n):
    g = golden("real")
    X = trnfft.rfft(cuda(g[f"x_{n}"]))
    assert rel_l2(cplx(X), g[f"rfft_fast_re_{n}"] + 1j * g[f"rfft_fast_im_{n}"]) < TOL
    y = trnfft.irfft(ComplexTensor(cuda(g[f"spec_re_{n}"]), cuda(g[f"spec_im_{n}"])), n=n)
    assert rel_l2(host(y), g[f"irfft_spec_fast_{n}"]) < TOL


def test_autograd_fft_and_rfft():
    """Gradients match torch.fft's (the reference checks existence and finiteness,
    tests/test_nn.py:79-88; here the values are checked too)."""
    torch.manual_seed(3)
    xr = torch.randn(4, 64, device="cuda", requires_grad=True)
    xi = torch.randn(4, 64, device="cuda", requires_grad=True)
    X = trnfft.fft(ComplexTensor(xr, xi))
    loss = (X.real ** 2 + 3 * X.imag).sum()
    loss.backward()
    zr = xr.detach().clone().requires_grad_(True)
    zi = xi.detach().clone().requires_grad_(True)
    Z = torch.fft.fft(torch.complex(zr, zi))
    (Z.real ** 2 + 3 * Z.imag).sum().backward()
    assert rel_l2(host(xr.grad), host(zr.grad)) < 1e-5
    assert rel_l2(host(xi.grad), host(zi.grad)) < 1e-5
    x = torch.randn(3, 128, device="cuda", requires_grad=True)
    R = trnfft.rfft(x)
    (R.real * 2 + R.imag ** 2).sum().backward()
    x2 = x.detach().clone().requires_grad_(True)
    R2 = torch.fft.rfft(x2)
    (R2.real * 2 + R2.imag ** 2).sum().backward()
    assert rel_l2(host(x.grad), host(x2.grad)) < 1e-5
    sr = torch.randn(3, 65, device="cuda", requires_grad=True)
    si = torch.randn(3, 65, device="cuda", requires_grad=True)
    y = trnfft.irfft(ComplexTensor(sr, si), n=128)
    (y * torch.arange(128, device="cuda")).sum().backward()
    tr = sr.detach().clone().requires_grad_(True)
    ti = si.detach().clone().requires_grad_(True)
    y2 = torch.fft.irfft(torch.complex(tr, ti), n=128)
    (y2 * torch.arange(128, device="cuda")).sum().backward()
    assert rel_l2(host(sr.grad), host(tr.grad)) < 1e-5
    assert rel_l2(host(si.grad), host(ti.grad)) < 1e-5


@pytest.mark.parametrize("n", [64, 1024, 4096])
def test_c2c_misaligned_planes_take_plain_kernel(n):
    """Planes that are not 16-byte aligned cannot feed bulk copies; the plain
    row kernel handles them with the same results."""
    from trnfft_b200 import _lib

    rng = np.random.default_rng(n)
    b = 37
    xr = rng.standard_normal((b, n)).astype(np.float32)
    xi = rng.standard_normal((b, n)).astype(np.float32)
    br = torch.empty(b * n + 1, device="cuda")[1:].view(b, n)
    bi = torch.empty(b * n + 1, device="cuda")[1:].view(b, n)
    br.copy_(cuda(xr))
    bi.copy_(cuda(xi))
    y = trnfft.fft(ComplexTensor(br, bi))
    er, ei = O.fft(xr, xi)
    assert rel_l2(cplx(y), er + 1j * ei) < TOL
    torch.cuda.synchronize()
    assert _lib.device_status(torch.cuda.current_device()) == 0
