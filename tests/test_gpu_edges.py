"""Edge cases of the public API on the GPU: empty and ragged inputs, other
dtypes and layouts, resizing, non-power-of-two axes, and the limits."""

import numpy as np
import pytest
import torch

import trnfft_b200 as trnfft
from trnfft_b200 import ComplexTensor
from tests.helpers import cplx, cuda, host, rel_l2

pytestmark = pytest.mark.gpu


def test_empty_batch():
    x = torch.zeros(0, 64, device="cuda")
    y = trnfft.fft(x)
    assert y.shape == (0, 64)
    assert trnfft.rfft(x).shape == (0, 33)
    assert trnfft.irfft(ComplexTensor(torch.zeros(0, 33, device="cuda"), torch.zeros(0, 33, device="cuda"))).shape == (0, 64)


def test_float64_and_complex_inputs_keep_dtype_semantics():
    x = torch.randn(3, 128, dtype=torch.float64, device="cuda")
    y = trnfft.fft(x)
    assert y.dtype == torch.float64
    assert rel_l2(cplx(y), np.fft.fft(x.cpu().numpy())) < 2e-6
    z = torch.randn(3, 96, dtype=torch.complex64, device="cuda")
    w = trnfft.fft(z)
    assert rel_l2(cplx(w), np.fft.fft(z.cpu().numpy().astype(np.complex128))) < 2e-6


def test_non_contiguous_input():
    x = torch.randn(64, 40, device="cuda").t()  # (40, 64) view, not contiguous
    y = trnfft.fft(x)
    assert rel_l2(cplx(y), np.fft.fft(host(x.contiguous()).astype(np.float64))) < 2e-6


@pytest.mark.parametrize("n_in,n", [(100, 128), (128, 100), (4096, 5000), (6000, 4096)])
def test_resize_n(n_in, n):
    x = torch.randn(2, n_in, device="cuda")
    y = trnfft.fft(x, n=n)
    ref = np.fft.fft(host(x).astype(np.float64), n=n)
    assert y.shape == (2, n) and rel_l2(cplx(y), ref) < 2e-6
    r = trnfft.rfft(x, n=n)
    assert rel_l2(cplx(r), np.fft.rfft(host(x).astype(np.float64), n=n)) < 2e-6


def test_non_power_of_two_axis_in_fftn():
    x = torch.randn(6, 100, 8, device="cuda")
    y = trnfft.fftn(x, dim=(1,))
    assert rel_l2(cplx(y), np.fft.fft(host(x).astype(np.float64), axis=1)) < 2e-6
    z = trnfft.fft2(torch.randn(3, 30, 50, device="cuda"))
    assert z.shape == (3, 30, 50)


def test_length_one_and_two():
    x = torch.randn(5, 1, device="cuda")
    np.testing.assert_array_equal(host(trnfft.ifft(x).real), host(x))
    x2 = torch.randn(5, 2, device="cuda")
    assert rel_l2(cplx(trnfft.fft(x2)), np.fft.fft(host(x2).astype(np.float64))) < 1e-6
    assert rel_l2(cplx(trnfft.rfft(x2)), np.fft.rfft(host(x2).astype(np.float64))) < 1e-6
    assert rel_l2(host(trnfft.irfft(trnfft.rfft(x2), n=2)), host(x2)) < 1e-6


def test_irfft_longer_spectrum_uses_hermitian_part():
    """A half spectrum with more bins than n//2+1 (the reference's irfft uses them
    directly, trnfft/api.py:58-66); the result is the real part of that inverse."""
    rng = np.random.default_rng(5)
    sr = rng.standard_normal((2, 40)).astype(np.float32)
    si = rng.standard_normal((2, 40)).astype(np.float32)
    y = trnfft.irfft(ComplexTensor(cuda(sr), cuda(si)), n=64)
    from oracle import trnfft_oracle as O

    assert rel_l2(host(y), O.irfft(sr, si, n=64)) < 2e-6
    with pytest.raises(RuntimeError):
        trnfft.irfft(ComplexTensor(cuda(sr[:, :10]), cuda(si[:, :10])), n=64)


def test_unsupported_sizes_raise_cleanly():
    """Lengths past the supported range fail with a clear error before any launch."""
    from trnfft_b200 import _lib

    dev = torch.device("cuda", torch.cuda.current_device())
    plan = _lib.DevicePlan((1 << 31) + 1, dev.index)  # Bluestein padding would be 2^33
    t = torch.zeros(4, device=dev)
    with pytest.raises(NotImplementedError):
        _lib.call("trnfft_exec_c2c", plan.handle, _lib.ptr(t), _lib.ptr(t), _lib.ptr(t), _lib.ptr(t), 1, 0,
                  None, _lib.stream_ptr(dev))
    with pytest.raises(ValueError):
        trnfft.set_small_n_algorithm("nope")
