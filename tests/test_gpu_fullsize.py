"""Parity at the full BASELINE.json sizes.

Each case runs the CUDA path on the whole configured batch and compares the
entire result with an fp64 transform of the same float32 input (torch.fft in
complex128 on the device, used only as the checker), rel-L2 <= 1e-5.  A few
sampled rows are also checked against the oracle (the reference's own
algorithm restated in NumPy), at the tolerance the suite uses everywhere.

  configs[1](a): 262144 transforms each of N = 64, 128, 256
  configs[1](b): ComplexLinear 4096 -> 4096 on a 16384 x 4096 complex input
  configs[3]:    N = 4093, 1000, 6000 at batch 4096; rfft / irfft of N = 4093
  configs[4]:    fft2 of a 16384 x 16384 field
"""

import numpy as np
import pytest
import torch

import trnfft_b200 as trnfft
from trnfft_b200 import ComplexTensor
from oracle import trnfft_oracle as O
from tests.helpers import TOL, cplx, host, rel_l2

pytestmark = pytest.mark.gpu


def _rel(y: ComplexTensor, ref: torch.Tensor) -> float:
    d = torch.complex(y.real.double(), y.imag.double()) - ref
    return float(torch.linalg.vector_norm(d) / torch.linalg.vector_norm(ref))


def _x64(xr, xi):
    return torch.complex(xr.double(), xi.double())


@pytest.mark.parametrize("n", [64, 128, 256])
def test_config1a_small_n_full_batch(n):
    g = torch.Generator(device="cuda").manual_seed(n)
    xr = torch.randn(262144, n, device="cuda", generator=g)
    xi = torch.randn(262144, n, device="cuda", generator=g)
    y = trnfft.fft(ComplexTensor(xr, xi))
    assert _rel(y, torch.fft.fft(_x64(xr, xi))) < TOL
    sel = [0, 77, 131071, 262143]
    o_r, o_i = O.fft(host(xr)[sel], host(xi)[sel])
    assert rel_l2(cplx(y)[sel], o_r + 1j * o_i) < TOL
    z = trnfft.ifft(y)
    assert _rel(z, _x64(xr, xi)) < TOL


def test_config1b_complex_linear_full_size():
    from trnfft_b200.nn import ComplexLinear

    torch.manual_seed(7)
    layer = ComplexLinear(4096, 4096, bias=True).cuda()
    with torch.no_grad():
        layer.bias_re.uniform_(-0.1, 0.1)
        layer.bias_im.uniform_(-0.1, 0.1)
    g = torch.Generator(device="cuda").manual_seed(8)
    xr = torch.randn(16384, 4096, device="cuda", generator=g)
    xi = torch.randn(16384, 4096, device="cuda", generator=g)
    with torch.no_grad():
        y = layer(ComplexTensor(xr, xi))
    wr, wi = layer.W_re.weight.double(), layer.W_im.weight.double()
    rows = torch.arange(0, 16384, 61, device="cuda")  # 269 rows spread over the batch
    a, b = xr[rows].double(), xi[rows].double()
    ref = torch.complex(a @ wr.t() - b @ wi.t() + layer.bias_re.double(),
                        a @ wi.t() + b @ wr.t() + layer.bias_im.double())
    assert _rel(ComplexTensor(y.real[rows], y.imag[rows]), ref) < TOL


@pytest.mark.parametrize("n", [4093, 1000, 6000])
def test_config3_bluestein_full_batch(n):
    g = torch.Generator(device="cuda").manual_seed(n)
    xr = torch.randn(4096, n, device="cuda", generator=g)
    xi = torch.randn(4096, n, device="cuda", generator=g)
    y = trnfft.fft(ComplexTensor(xr, xi))
    assert _rel(y, torch.fft.fft(_x64(xr, xi))) < TOL
    z = trnfft.ifft(ComplexTensor(xr, xi))
    assert _rel(z, torch.fft.ifft(_x64(xr, xi))) < TOL
    # the reference's own algorithm in its accurate mode on sampled rows
    sel = [0, 4095]
    o_r, o_i = O.fft(host(xr)[sel], host(xi)[sel], precision="double")
    assert rel_l2(cplx(y)[sel], o_r + 1j * o_i) < TOL


def test_config3_rfft_irfft_4093_full_batch():
    g = torch.Generator(device="cuda").manual_seed(4093)
    x = torch.randn(4096, 4093, device="cuda", generator=g)
    y = trnfft.rfft(x)
    assert y.shape == (4096, 2047)
    assert _rel(y, torch.fft.rfft(x.double())) < TOL
    back = trnfft.irfft(y, n=4093)
    assert float(torch.linalg.vector_norm(back.double() - x.double()) / torch.linalg.vector_norm(x.double())) < TOL
    # irfft of an arbitrary one-sided spectrum against fp64
    sr = torch.randn(4096, 2047, device="cuda", generator=g)
    si = torch.randn(4096, 2047, device="cuda", generator=g)
    r = trnfft.irfft(ComplexTensor(sr, si), n=4093)
    ref = torch.fft.irfft(_x64(sr, si), n=4093)
    assert float(torch.linalg.vector_norm(r.double() - ref) / torch.linalg.vector_norm(ref)) < TOL


def test_config4_fft2_16384_squared():
    g = torch.Generator(device="cuda").manual_seed(16384)
    xr = torch.randn(16384, 16384, device="cuda", generator=g)
    xi = torch.randn(16384, 16384, device="cuda", generator=g)
    y = trnfft.fft2(ComplexTensor(xr, xi))
    ref = torch.fft.fft2(_x64(xr, xi))
    assert _rel(y, ref) < TOL
    del ref
    torch.cuda.empty_cache()
    back = trnfft.ifft2(y) if hasattr(trnfft, "ifft2") else trnfft.ifftn(y, dim=(-2, -1))
    assert _rel(back, _x64(xr, xi)) < TOL
