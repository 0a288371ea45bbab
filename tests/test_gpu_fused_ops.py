"""GPU parity of the fused iSTFT kernel, the fused complex-mask kernel, the
real-input Bluestein kernels and the in-place / overlap rules of exec_c2c.

Every case compares the CUDA path with the oracle (the reference's algorithm
in NumPy) or an fp64 transform on the same seeded inputs, rel-L2 <= 1e-5.
"""

import ctypes

import numpy as np
import pytest
import torch

import trnfft_b200 as trnfft
from trnfft_b200 import ComplexTensor, _lib, _ops
from trnfft_b200.nki.dispatch import complex_mask_apply
from oracle import trnfft_oracle as O
from tests.helpers import TOL, cplx, cuda, host, rel_l2

pytestmark = pytest.mark.gpu


# -- fused iSTFT ---------------------------------------------------------------

ISTFT_CASES = [
    # n_fft, hop, center, onesided, normalized, length, win_length
    (512, 256, True, True, False, None, None),    # configs[2] parameters
    (256, 64, True, True, False, 4000, None),     # the reference's default hop n_fft/4
    (64, 16, False, True, True, None, None),
    (128, 32, True, False, False, None, None),    # two-sided spectrum
    (32, 32, True, True, False, 700, 24),         # hop == n_fft, shorter window, zero-padded tail
    (8, 3, True, True, False, None, None),        # odd hop
    (8192, 2048, True, True, False, None, None),  # largest n_fft
    (4, 1, False, True, False, None, None),       # smallest n_fft
]


@pytest.mark.parametrize("n_fft,hop,center,onesided,normalized,length,wl", ISTFT_CASES)
def test_istft_fused_vs_oracle(n_fft, hop, center, onesided, normalized, length, wl):
    rng = np.random.default_rng(n_fft * 7 + hop)
    L = max(3 * n_fft, 2000)
    x = rng.standard_normal((3, L)).astype(np.float32)
    win = np.hanning(wl or n_fft).astype(np.float32) + 0.05  # no exact zeros inside
    sr, si = O.stft(x, n_fft, hop, wl, win, center=center, normalized=normalized, onesided=onesided)
    # perturb so the spectrum is not exactly an STFT (exercises the normalisation edge)
    sr = sr + 0.01 * rng.standard_normal(sr.shape).astype(np.float32)
    si = si + 0.01 * rng.standard_normal(si.shape).astype(np.float32)
    want = O.istft(sr, si, n_fft, hop, wl, win, center=center, normalized=normalized, onesided=onesided,
                   length=length)
    got = trnfft.istft(ComplexTensor(cuda(sr), cuda(si)), n_fft, hop, wl, torch.from_numpy(win).cuda(),
                       center=center, normalized=normalized, onesided=onesided, length=length)
    assert got.shape == want.shape
    assert rel_l2(host(got), want) < TOL


def test_istft_config_roundtrip_full_size():
    """configs[2] shape: istft(stft(x)) == x for 256 x 160000 with the fused kernels."""
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(256, 160000, device="cuda", generator=g)
    w = torch.hann_window(512, device="cuda")
    S = trnfft.stft(x, 512, 256, window=w)
    back = trnfft.istft(S, 512, 256, window=w, length=160000)
    assert float(torch.linalg.vector_norm(back - x) / torch.linalg.vector_norm(x)) < TOL


def test_istft_matches_composite_path():
    rng = np.random.default_rng(11)
    sr = cuda(rng.standard_normal((2, 129, 40)))
    si = cuda(rng.standard_normal((2, 129, 40)))
    w = torch.hann_window(256, device="cuda")
    fused = _ops.istft(sr, si, 256, 64, w, True, False, True, None)
    comp = _ops._istft_composite(sr, si, 256, 64, w, True, False, True, None)
    assert rel_l2(host(fused), host(comp)) < TOL


# -- complex mask ----------------------------------------------------------------


@pytest.mark.parametrize("mshape,sshape", [((4, 257, 100), (4, 257, 100)), ((257, 100), (4, 257, 100)),
                                           ((1, 33, 7), (5, 33, 7)), ((3, 1, 7), (3, 5, 7)),
                                           ((13,), (6, 13)), ((7, 1), (7, 9))])
def test_complex_mask_apply_vs_numpy(mshape, sshape):
    rng = np.random.default_rng(len(mshape) * 100 + sshape[-1])
    m = rng.standard_normal(mshape) + 1j * rng.standard_normal(mshape)
    s = rng.standard_normal(sshape) + 1j * rng.standard_normal(sshape)
    y = complex_mask_apply(ComplexTensor(cuda(m.real), cuda(m.imag)), ComplexTensor(cuda(s.real), cuda(s.imag)))
    want = m.astype(np.complex64) * s.astype(np.complex64)
    assert y.shape == want.shape
    assert rel_l2(cplx(y), want) < TOL


def test_complex_mask_apply_grad():
    rng = np.random.default_rng(5)
    mr, mi, sr, si = (cuda(rng.standard_normal((33, 7))).requires_grad_() for _ in range(4))
    y = complex_mask_apply(ComplexTensor(mr, mi), ComplexTensor(sr, si))
    (y.real.square().sum() + 3 * y.imag.sum()).backward()
    m = torch.complex(mr.detach().double(), mi.detach().double()).requires_grad_()
    s = torch.complex(sr.detach().double(), si.detach().double()).requires_grad_()
    z = m * s
    (z.real.square().sum() + 3 * z.imag.sum()).backward()
    # torch's gradient of a real loss w.r.t. a complex leaf is dL/d(re) + i dL/d(im)
    assert rel_l2(host(mr.grad) + 1j * host(mi.grad), m.grad.cpu().numpy()) < TOL
    assert rel_l2(host(sr.grad) + 1j * host(si.grad), s.grad.cpu().numpy()) < TOL


def test_complex_mask_apply_c_abi_rejects_bad_period():
    d = torch.zeros(10, device="cuda")
    with pytest.raises(ValueError, match="not a multiple"):
        _lib.call("trnfft_complex_mask_apply", _lib.ptr(d), _lib.ptr(d), 3, _lib.ptr(d), _lib.ptr(d),
                  _lib.ptr(d), _lib.ptr(d), 10, 0, _lib.stream_ptr(d.device))


# -- real-input Bluestein (fused R2C / C2R modes) ----------------------------------


@pytest.mark.parametrize("n", [3, 5, 17, 100, 999, 1000, 4093, 6000, 8191])
def test_rfft_irfft_bluestein_kernels_vs_fp64(n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal((5, n)).astype(np.float32)
    y = trnfft.rfft(cuda(x))
    assert rel_l2(cplx(y), np.fft.rfft(x.astype(np.float64))) < TOL
    s = (rng.standard_normal((5, n // 2 + 1)) + 1j * rng.standard_normal((5, n // 2 + 1))).astype(np.complex64)
    r = trnfft.irfft(ComplexTensor(cuda(s.real), cuda(s.imag)), n=n)
    assert rel_l2(host(r), np.fft.irfft(s.astype(np.complex128), n=n)) < TOL


def test_rfft_odd_uses_real_kernel_with_grad():
    x = torch.randn(4, 1001, device="cuda", dtype=torch.float32, requires_grad=True)
    y = trnfft.rfft(x)
    (y.real.sum() + 2 * y.imag.sum()).backward()
    xd = x.detach().double().requires_grad_()
    yd = torch.fft.rfft(xd)
    (yd.real.sum() + 2 * yd.imag.sum()).backward()
    assert rel_l2(host(x.grad), xd.grad.cpu().numpy()) < TOL


# -- in place and overlapping planes ---------------------------------------------


@pytest.mark.parametrize("n", [8192, 16384])
def test_inplace_one_pass_rows_need_no_work_area(n):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal((3, n)) + 1j * rng.standard_normal((3, n))).astype(np.complex64)
    re, im = cuda(x.real), cuda(x.imag)
    plan = _lib.device_plan(n, re.device)
    _lib.call("trnfft_exec_c2c", plan.handle, _lib.ptr(re), _lib.ptr(im), _lib.ptr(re), _lib.ptr(im), 3, 0, None,
              _lib.stream_ptr(re.device))
    assert rel_l2(host(re) + 1j * host(im), np.fft.fft(x.astype(np.complex128))) < TOL


def test_partial_overlap_rejected_for_one_pass_sizes():
    buf = torch.zeros(3, 1024, device="cuda")
    plan = _lib.device_plan(1024, buf.device)
    p = buf.data_ptr()
    with pytest.raises(ValueError, match="overlap"):
        # out_re == in_im
        _lib.call("trnfft_exec_c2c", plan.handle, ctypes.c_void_p(p), ctypes.c_void_p(p + 4096),
                  ctypes.c_void_p(p + 4096), ctypes.c_void_p(p + 8192), 1, 0, None, _lib.stream_ptr(buf.device))


def test_partial_overlap_multipass_goes_through_work_area():
    n = 1 << 15
    rng = np.random.default_rng(9)
    x = (rng.standard_normal(n) + 1j * rng.standard_normal(n)).astype(np.complex64)
    buf = torch.empty(3 * n, device="cuda")
    buf[:n] = cuda(x.real)
    buf[n:2 * n] = cuda(x.imag)
    plan = _lib.device_plan(n, buf.device)
    work = torch.empty(plan.work_bytes(1), dtype=torch.uint8, device="cuda")
    p = buf.data_ptr()
    # in = (plane 0, plane 1), out = (plane 1, plane 2): out_re == in_im
    _lib.call("trnfft_exec_c2c", plan.handle, ctypes.c_void_p(p), ctypes.c_void_p(p + 4 * n),
              ctypes.c_void_p(p + 4 * n), ctypes.c_void_p(p + 8 * n), 1, 0, _lib.ptr(work),
              _lib.stream_ptr(buf.device))
    got = host(buf[n:2 * n]) + 1j * host(buf[2 * n:])
    assert rel_l2(got, np.fft.fft(x.astype(np.complex128))) < TOL
    with pytest.raises(ValueError, match="work area"):
        _lib.call("trnfft_exec_c2c", plan.handle, ctypes.c_void_p(p), ctypes.c_void_p(p + 4 * n),
                  ctypes.c_void_p(p + 4 * n), ctypes.c_void_p(p + 8 * n), 1, 0, None, _lib.stream_ptr(buf.device))
