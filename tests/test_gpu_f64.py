"""GPU parity of the double-precision kernels (precision="double", float64 tensors).

The reference promotes Bluestein to float64 in "double" mode
(trnfft/fft_core.py:1306-1309) and computes in float64 for float64 tensors;
the committed golden fixtures hold its "double" results.  Here:

* float64 inputs against numpy's fp64 FFT: rel-L2 <= 1e-12 (fp64 rounding);
* float32 inputs in precision="double" against the reference's "double"
  golden and the fp64 FFT of the same float32 values: rel-L2 <= 1e-6 (the
  result is rounded to float32 once, about 6e-8);
* the configs[3] shapes at full batch.
"""

import numpy as np
import pytest
import torch

import trnfft_b200 as trnfft
from trnfft_b200 import ComplexTensor
from tests.helpers import cplx, host, rel_l2

pytestmark = pytest.mark.gpu

F64_TOL = 1e-12


def _c64(a):
    return torch.as_tensor(np.ascontiguousarray(a), dtype=torch.float64).cuda()


@pytest.fixture
def double_mode():
    prev = trnfft.get_precision()
    trnfft.set_precision("double")
    yield
    trnfft.set_precision(prev)


@pytest.mark.parametrize("n", [1, 2, 4, 8, 64, 1024, 4096, 8192, 1 << 15, 1 << 20, 1 << 24,
                               3, 5, 7, 100, 1000, 4093, 6000, 8191, 40961])
def test_float64_tensors_match_numpy_fp64(n):
    batch = 3 if n <= 1 << 20 else 1
    rng = np.random.default_rng(n)
    x = rng.standard_normal((batch, n)) + 1j * rng.standard_normal((batch, n))
    X = trnfft.fft(ComplexTensor(_c64(x.real), _c64(x.imag)))
    assert X.real.dtype == torch.float64
    got = X.real.cpu().numpy() + 1j * X.imag.cpu().numpy()
    assert rel_l2(got, np.fft.fft(x)) < F64_TOL
    Y = trnfft.ifft(X)
    back = Y.real.cpu().numpy() + 1j * Y.imag.cpu().numpy()
    assert rel_l2(back, x) < F64_TOL


@pytest.mark.parametrize("n", [3, 5, 7, 11, 100, 127, 997, 1000, 4093, 6000])
def test_double_mode_matches_reference_double_golden(golden, double_mode, n):
    g = golden("bluestein")
    xr = torch.as_tensor(g[f"x_re_{n}"]).cuda()
    xi = torch.as_tensor(g[f"x_im_{n}"]).cuda()
    y = trnfft.fft(ComplexTensor(xr, xi))
    z = trnfft.ifft(ComplexTensor(xr, xi))
    assert y.real.dtype == torch.float32
    assert rel_l2(cplx(y), g[f"fft_double_re_{n}"] + 1j * g[f"fft_double_im_{n}"]) < 1e-6
    assert rel_l2(cplx(z), g[f"ifft_double_re_{n}"] + 1j * g[f"ifft_double_im_{n}"]) < 1e-6
    exact = np.fft.fft(g[f"x_re_{n}"].astype(np.float64) + 1j * g[f"x_im_{n}"])
    assert rel_l2(cplx(y), exact) < 1e-7


@pytest.mark.parametrize("n", [4093, 1000, 6000])
def test_double_mode_config3_full_batch(double_mode, n):
    g = torch.Generator(device="cuda").manual_seed(n)
    xr = torch.randn(4096, n, device="cuda", generator=g)
    xi = torch.randn(4096, n, device="cuda", generator=g)
    y = trnfft.fft(ComplexTensor(xr, xi))
    ref = torch.fft.fft(torch.complex(xr.double(), xi.double()))
    d = torch.complex(y.real.double(), y.imag.double()) - ref
    # only the final rounding to float32 remains
    assert float(torch.linalg.vector_norm(d) / torch.linalg.vector_norm(ref)) < 1e-7


def test_double_mode_rfft_irfft_and_grad(double_mode):
    rng = np.random.default_rng(2)
    x = rng.standard_normal((4, 4093))
    xt = torch.as_tensor(x, dtype=torch.float32).cuda().requires_grad_()
    y = trnfft.rfft(xt)
    assert rel_l2(cplx(y), np.fft.rfft(x.astype(np.float32).astype(np.float64))) < 1e-7
    back = trnfft.irfft(y, n=4093)
    assert rel_l2(host(back), x.astype(np.float32)) < 1e-6
    (y.real.sum() + y.imag.sum()).backward()
    xd = torch.as_tensor(x.astype(np.float32), dtype=torch.float64).requires_grad_()
    yd = torch.fft.rfft(xd)
    (yd.real.sum() + yd.imag.sum()).backward()
    assert rel_l2(host(xt.grad), xd.grad.numpy()) < 1e-6


def test_float64_fft2_matches_numpy():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((2, 96, 128)) + 1j * rng.standard_normal((2, 96, 128))
    X = trnfft.fft2(ComplexTensor(_c64(x.real), _c64(x.imag)))
    got = X.real.cpu().numpy() + 1j * X.imag.cpu().numpy()
    assert rel_l2(got, np.fft.fft2(x)) < F64_TOL


def test_convert_f32_f64_entry_point():
    """trnfft_convert_f32_f64 widens and narrows exactly like a cast (round to nearest)."""
    from trnfft_b200 import _lib

    rng = np.random.default_rng(5)
    x = torch.from_numpy(rng.standard_normal(10007).astype(np.float32)).cuda()
    d = torch.empty(x.shape, dtype=torch.float64, device="cuda")
    _lib.call("trnfft_convert_f32_f64", _lib.ptr(x), _lib.ptr(d), x.numel(), 1, 0, _lib.stream_ptr(x.device))
    assert torch.equal(d, x.double())
    d2 = torch.from_numpy(rng.standard_normal(10007)).cuda()
    f = torch.empty(d2.shape, dtype=torch.float32, device="cuda")
    _lib.call("trnfft_convert_f32_f64", _lib.ptr(d2), _lib.ptr(f), d2.numel(), 0, 0, _lib.stream_ptr(d2.device))
    assert torch.equal(f, d2.float())


@pytest.mark.parametrize("n", [1, 64, 4096, 1 << 15, 4093, 40961])
def test_f32io_entry_matches_double_entry(n):
    """trnfft_exec_c2c_f64_f32io (float32 planes in and out, fp64 inside) equals the float64 entry
    on the widened input, rounded to float32, for one-pass, two-pass, fused-Bluestein and
    chained-Bluestein plans."""
    from trnfft_b200 import _lib

    rng = np.random.default_rng(n)
    B = 3
    xr = torch.from_numpy(rng.standard_normal((B, n)).astype(np.float32)).cuda()
    xi = torch.from_numpy(rng.standard_normal((B, n)).astype(np.float32)).cuda()
    plan = _lib.device_plan(n, xr.device)
    plan.enable_f64()
    wb = plan.work_bytes_f64(B)
    work = torch.empty(max(wb, 16), dtype=torch.uint8, device="cuda")
    st = _lib.stream_ptr(xr.device)
    for inv in (0, 1):
        yr = torch.empty_like(xr)
        yi = torch.empty_like(xi)
        _lib.call("trnfft_exec_c2c_f64_f32io", plan.handle, _lib.ptr(xr), _lib.ptr(xi), _lib.ptr(yr), _lib.ptr(yi), B,
                  inv, _lib.ptr(work), st)
        ar, ai = xr.double(), xi.double()
        dr, di = torch.empty_like(ar), torch.empty_like(ai)
        _lib.call("trnfft_exec_c2c_f64", plan.handle, _lib.ptr(ar), _lib.ptr(ai), _lib.ptr(dr), _lib.ptr(di), B, inv,
                  _lib.ptr(work), st)
        assert torch.equal(yr, dr.float()) and torch.equal(yi, di.float())
