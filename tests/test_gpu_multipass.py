"""GPU parity of the large power-of-two (multi-pass) transforms, the strided-axis
transforms behind fft2/fftn, and the four-step single transform."""

import ctypes

import numpy as np
import pytest
import torch

import trnfft_b200 as trnfft
from trnfft_b200 import ComplexTensor, _lib
from trnfft_b200.nki import multicore
from oracle import trnfft_oracle as O
from tests.helpers import TOL, cplx, cuda, host, rel_l2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [8192, 16384])
def test_vs_reference_golden(golden, n):
    g = golden("pow2_large")
    y = trnfft.fft(ComplexTensor(cuda(g[f"x_re_{n}"]), cuda(g[f"x_im_{n}"])))
    assert rel_l2(cplx(y), g[f"fft_re_{n}"] + 1j * g[f"fft_im_{n}"]) < TOL


@pytest.mark.parametrize("logn", [13, 14, 16, 18, 20, 21, 22])
def test_vs_fp64(logn):
    n = 1 << logn
    b = max(1, (1 << 22) // n)
    rng = np.random.default_rng(logn)
    x = (rng.standard_normal((b, n)) + 1j * rng.standard_normal((b, n))).astype(np.complex64)
    X = trnfft.fft(ComplexTensor(cuda(x.real), cuda(x.imag)))
    assert rel_l2(cplx(X), np.fft.fft(x.astype(np.complex128))) < 2e-6
    Z = trnfft.ifft(ComplexTensor(cuda(x.real), cuda(x.imag)))
    assert rel_l2(cplx(Z), np.fft.ifft(x.astype(np.complex128))) < 2e-6


@pytest.mark.parametrize("logn", [13, 14])
@pytest.mark.parametrize("batch", [1, 3, 150, 300])
@pytest.mark.parametrize("offset", [0, 1])
def test_single_block_rows(logn, batch, offset):
    """Rows of 8192 / 16384 points: the persistent bulk-copy kernel (aligned planes; batches
    below, at and above the SM count) and the plain kernel (planes offset by one float)."""
    n = 1 << logn
    rng = np.random.default_rng(batch + logn)
    x = (rng.standard_normal((batch, n)) + 1j * rng.standard_normal((batch, n))).astype(np.complex64)
    br = torch.zeros(batch * n + 1, device="cuda")
    bi = torch.zeros(batch * n + 1, device="cuda")
    br[offset:offset + batch * n] = cuda(x.real.reshape(-1))
    bi[offset:offset + batch * n] = cuda(x.imag.reshape(-1))
    xr = br[offset:offset + batch * n].view(batch, n)
    xi = bi[offset:offset + batch * n].view(batch, n)
    X = trnfft.fft(ComplexTensor(xr, xi))
    assert rel_l2(cplx(X), np.fft.fft(x.astype(np.complex128))) < 2e-6
    Z = trnfft.ifft(X)
    assert rel_l2(cplx(Z), x.astype(np.complex128)) < 2e-6


@pytest.mark.parametrize("n", [4096, 65536])
def test_four_step_vs_reference_golden(golden, n):
    g = golden("four_step")
    x = ComplexTensor(cuda(g[f"x_re_{n}"]), cuda(g[f"x_im_{n}"]))
    multicore.set_multicore(True)
    try:
        y = multicore.multi_core_fft(x)
        z = multicore.multi_core_fft(x, inverse=True)
    finally:
        multicore.set_multicore(False)
    assert rel_l2(cplx(y), g[f"sp_re_{n}"] + 1j * g[f"sp_im_{n}"]) < TOL
    assert rel_l2(cplx(z), g[f"spi_re_{n}"] + 1j * g[f"spi_im_{n}"]) < TOL


def test_in_place_with_work_area():
    n = 1 << 15
    b = 3
    torch.manual_seed(0)
    xr = torch.randn(b, n, device="cuda")
    xi = torch.randn(b, n, device="cuda")
    ref = torch.fft.fft(torch.complex(xr, xi).to(torch.complex128))
    plan = _lib.device_plan(n, xr.device)
    wb = plan.work_bytes(b)
    assert wb == 8 * n * b
    work = torch.empty(wb, dtype=torch.uint8, device="cuda")
    _lib.call("trnfft_exec_c2c", plan.handle, _lib.ptr(xr), _lib.ptr(xi), _lib.ptr(xr), _lib.ptr(xi), b, 0,
              _lib.ptr(work), _lib.stream_ptr(xr.device))
    got = host(xr) + 1j * host(xi)
    assert rel_l2(got, ref.cpu().numpy()) < 2e-6
    with pytest.raises(ValueError, match="work area"):
        _lib.call("trnfft_exec_c2c", plan.handle, _lib.ptr(xr), _lib.ptr(xi), _lib.ptr(xr), _lib.ptr(xi), b, 0,
                  None, _lib.stream_ptr(xr.device))


def test_full_size_2_30_roundtrip_and_parseval():
    """Config 5 size (N = 2^30, 8 GiB planar): size-independent properties --
    ifft(fft(x)) == x, Parseval, and the DC bin equals the sum."""
    n = 1 << 30
    g = torch.Generator(device="cuda").manual_seed(5)
    xr = torch.randn(n, device="cuda", generator=g)
    xi = torch.randn(n, device="cuda", generator=g)
    X = trnfft.fft(ComplexTensor(xr, xi))
    dc = complex(xr.double().sum().item(), xi.double().sum().item())
    assert abs(complex(X.real[0].item(), X.imag[0].item()) - dc) < 1e-3 * np.sqrt(n)
    ex = (xr.double() ** 2).sum() + (xi.double() ** 2).sum()
    eX = ((X.real.double() ** 2).sum() + (X.imag.double() ** 2).sum()) / n
    assert abs(float(eX / ex) - 1.0) < 1e-5
    back = trnfft.ifft(X)
    del X
    err = torch.sqrt(((back.real - xr).double() ** 2).sum() + ((back.imag - xi).double() ** 2).sum())
    assert float(err / torch.sqrt(ex)) < 2e-6


def test_fft2_vs_reference_golden(golden):
    g = golden("nd")
    for key in ["16x32", "64x64", "8x256"]:
        x = ComplexTensor(cuda(g[f"x_re_{key}"]), cuda(g[f"x_im_{key}"]))
        assert rel_l2(cplx(trnfft.fft2(x)), g[f"fft2_re_{key}"] + 1j * g[f"fft2_im_{key}"]) < TOL
        z = trnfft.ifftn(x, dim=(-2, -1))
        assert rel_l2(cplx(z), g[f"ifft2_re_{key}"] + 1j * g[f"ifft2_im_{key}"]) < TOL
    x3 = cuda(g["x3"])
    assert rel_l2(cplx(trnfft.fftn(x3)), g["fftn3_re"] + 1j * g["fftn3_im"]) < TOL
    assert rel_l2(cplx(trnfft.fftn(x3, dim=(0, 2))), g["fftn3_d02_re"] + 1j * g["fftn3_d02_im"]) < TOL
    r = trnfft.rfftn(x3)
    assert rel_l2(cplx(r), g["rfftn3_re"] + 1j * g["rfftn3_im"]) < TOL
    assert rel_l2(host(trnfft.irfftn(r, s=x3.shape)), g["irfftn3"]) < TOL
    r2 = trnfft.rfft2(cuda(g["x2"]), s=(16, 32))
    assert rel_l2(cplx(r2), g["rfft2_s_re"] + 1j * g["rfft2_s_im"]) < TOL
    xh = ComplexTensor(cuda(g["h_re"]), cuda(g["h_im"]))
    assert rel_l2(host(trnfft.hfft(xh, n=16)), g["hfft_16"]) < TOL
    ih = trnfft.ihfft(cuda(g["ih_x"]))
    assert rel_l2(cplx(ih), g["ihfft_re"] + 1j * g["ihfft_im"]) < TOL


@pytest.mark.parametrize("shape,dim", [((3, 1024, 40), 1), ((2, 4096, 24), 1), ((5, 7, 9), 1),
                                       ((64, 2048), 0), ((1 << 13, 16), 0), ((6, 12, 64), 0)])
def test_axis_vs_fp64(shape, dim):
    rng = np.random.default_rng(sum(shape))
    x = (rng.standard_normal(shape) + 1j * rng.standard_normal(shape)).astype(np.complex64)
    y = trnfft.fftn(ComplexTensor(cuda(x.real), cuda(x.imag)), dim=(dim,))
    assert rel_l2(cplx(y), np.fft.fft(x.astype(np.complex128), axis=dim)) < 2e-6


def test_fft2_large_vs_fp64():
    rng = np.random.default_rng(9)
    x = (rng.standard_normal((1024, 2048)) + 1j * rng.standard_normal((1024, 2048))).astype(np.complex64)
    y = trnfft.fft2(ComplexTensor(cuda(x.real), cuda(x.imag)))
    assert rel_l2(cplx(y), np.fft.fft2(x.astype(np.complex128))) < 2e-6


def test_axis_autograd_matches_torch():
    torch.manual_seed(2)
    xr = torch.randn(4, 32, 16, device="cuda", requires_grad=True)
    xi = torch.randn(4, 32, 16, device="cuda", requires_grad=True)
    y = trnfft.fft2(ComplexTensor(xr, xi))
    (y.real * 3 + y.imag ** 2).sum().backward()
    zr = xr.detach().clone().requires_grad_(True)
    zi = xi.detach().clone().requires_grad_(True)
    z = torch.fft.fft2(torch.complex(zr, zi))
    (z.real * 3 + z.imag ** 2).sum().backward()
    assert rel_l2(host(xr.grad), host(zr.grad)) < 1e-5
    assert rel_l2(host(xi.grad), host(zi.grad)) < 1e-5


@pytest.mark.parametrize("n1,cols,col0,big", [(512, 64, 192, 1 << 16), (4096, 32, 96, 1 << 20), (32768, 16, 16384, 1 << 30)])
@pytest.mark.parametrize("inverse", [False, True])
def test_axis_with_fused_four_step_twiddle(n1, cols, col0, big, inverse):
    """trnfft_exec_c2c_axis_tw == column FFT followed by W_big^{(col0 + c) k} (fp64 reference)."""
    rng = np.random.default_rng(n1 + cols)
    x = (rng.standard_normal((n1, cols)) + 1j * rng.standard_normal((n1, cols))).astype(np.complex64)
    xr, xi = cuda(x.real), cuda(x.imag)
    yr, yi = torch.empty_like(xr), torch.empty_like(xi)
    plan = _lib.device_plan(n1, xr.device)
    twp = _lib.device_plan(big, xr.device)
    _lib.call("trnfft_exec_c2c_axis_tw", plan.handle, twp.handle, _lib.ptr(xr), _lib.ptr(xi), _lib.ptr(yr),
              _lib.ptr(yi), 1, cols, 0, 0, int(inverse), col0, _lib.stream_ptr(xr.device))
    xd = x.astype(np.complex128)
    f = np.fft.ifft(xd, axis=0) if inverse else np.fft.fft(xd, axis=0)
    k = np.arange(n1)[:, None]
    c = np.arange(cols)[None, :] + col0
    e = (k * c) % big
    w = np.exp((2j if inverse else -2j) * np.pi * e / big)
    assert rel_l2(host(yr) + 1j * host(yi), f * w) < 2e-6


@pytest.mark.parametrize("n1,work_needed", [(512, False), (1 << 16, True)])
@pytest.mark.parametrize("inverse", [False, True])
@pytest.mark.parametrize("cap", [None, "7"])
def test_fourstep_scatter_one_gpu(monkeypatch, n1, work_needed, inverse, cap):
    """trnfft_exec_fourstep_scatter with two row buffers on one GPU: output row K of the twiddled
    column FFT lands in buffer K // rows_per_peer, row K % rows_per_peer, columns peer_col0 + c.
    cap: TRNFFT_B200_SCATTER_BLOCKS (7 blocks loop over every tile)."""
    if cap is not None:
        monkeypatch.setenv("TRNFFT_B200_SCATTER_BLOCKS", cap)
    cols, big, col_offset, peer_col0, peer_ld = 64, 1 << 26, 192, 64, 160
    rpp = n1 // 2
    rng = np.random.default_rng(n1 + int(inverse))
    x = (rng.standard_normal((n1, cols)) + 1j * rng.standard_normal((n1, cols))).astype(np.complex64)
    xr, xi = cuda(x.real), cuda(x.imag)
    bufs = [torch.zeros(rpp, peer_ld, device="cuda") for _ in range(4)]  # re0, re1, im0, im1
    pre = (ctypes.c_void_p * 2)(bufs[0].data_ptr(), bufs[1].data_ptr())
    pim = (ctypes.c_void_p * 2)(bufs[2].data_ptr(), bufs[3].data_ptr())
    work = torch.empty(2 * n1 * cols, device="cuda") if work_needed else None
    plan = _lib.device_plan(n1, xr.device)
    twp = _lib.device_plan(big, xr.device)
    _lib.call("trnfft_exec_fourstep_scatter", plan.handle, twp.handle, _lib.ptr(xr), _lib.ptr(xi), cols, cols,
              int(inverse), col_offset, 2, pre, pim, rpp, peer_ld, peer_col0, _lib.ptr(work),
              _lib.stream_ptr(xr.device))
    xd = x.astype(np.complex128)
    f = np.fft.ifft(xd, axis=0) if inverse else np.fft.fft(xd, axis=0)
    k = np.arange(n1)[:, None]
    c = np.arange(cols)[None, :] + col_offset
    y = f * np.exp((2j if inverse else -2j) * np.pi * ((k * c) % big) / big)
    got = np.concatenate([host(bufs[q]) + 1j * host(bufs[2 + q]) for q in range(2)], axis=0)
    assert rel_l2(got[:, peer_col0:peer_col0 + cols], y) < 2e-6
    untouched = np.concatenate([got[:, :peer_col0], got[:, peer_col0 + cols:]], axis=1)
    assert not untouched.any()


@pytest.mark.parametrize("n", [1 << 11, 1 << 17, 1 << 21, 3 * 4096])
def test_stage_parallel_fft_vs_fp64(n):
    """multi_core_fft's four-step (fused column twiddle for powers of two) against fp64."""
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) + 1j * rng.standard_normal(n)).astype(np.complex64)
    xc = ComplexTensor(cuda(x.real), cuda(x.imag))
    multicore.set_multicore(True)
    try:
        y = multicore.multi_core_fft(xc)
        z = multicore.multi_core_fft(xc, inverse=True)
    finally:
        multicore.set_multicore(False)
    assert rel_l2(cplx(y), np.fft.fft(x.astype(np.complex128))) < TOL
    assert rel_l2(cplx(z), np.fft.ifft(x.astype(np.complex128))) < TOL
