"""GPU parity of the direct mixed-radix kernel (7-smooth n <= 8192).

The reference runs these lengths through Bluestein (trnfft/fft_core.py:44-50);
both compute the same DFT, so the kernel is checked against the reference's
"double" golden where it exists, against fp64 NumPy, and against the oracle
(the reference's algorithm in NumPy), rel-L2 <= 1e-5, for every radix the
schedule uses (2, 3, 4, 5, 7, 8, 16), forward, inverse and the real modes.
"""

import numpy as np
import pytest
import torch

import trnfft_b200 as trnfft
from trnfft_b200 import ComplexTensor, _lib
from oracle import trnfft_oracle as O
from tests.helpers import TOL, cplx, cuda, host, rel_l2

pytestmark = pytest.mark.gpu

SMOOTH = [6, 10, 12, 14, 15, 21, 35, 49, 96, 100, 105, 243, 343, 625, 1000, 1536, 2187, 3000, 4800, 6000,
          6561, 7000, 8000, 8100]


@pytest.mark.parametrize("n", SMOOTH)
def test_mixed_radix_vs_fp64(n):
    plan = _lib.device_plan(n, torch.device("cuda", torch.cuda.current_device()))
    assert plan.algorithm == _lib.ALG_MIXED
    rng = np.random.default_rng(n)
    batch = 5
    x = (rng.standard_normal((batch, n)) + 1j * rng.standard_normal((batch, n))).astype(np.complex64)
    y = trnfft.fft(ComplexTensor(cuda(x.real), cuda(x.imag)))
    assert rel_l2(cplx(y), np.fft.fft(x.astype(np.complex128))) < 2e-6
    z = trnfft.ifft(ComplexTensor(cuda(x.real), cuda(x.imag)))
    assert rel_l2(cplx(z), np.fft.ifft(x.astype(np.complex128))) < 2e-6
    r = rng.standard_normal((batch, n)).astype(np.float32)
    R = trnfft.rfft(cuda(r))
    assert rel_l2(cplx(R), np.fft.rfft(r.astype(np.float64))) < 2e-6
    back = trnfft.irfft(R, n=n)
    assert rel_l2(host(back), r) < 2e-6


@pytest.mark.parametrize("n", [100, 1000, 6000])
def test_mixed_radix_vs_reference_golden_and_oracle(golden, n):
    g = golden("bluestein")
    x = ComplexTensor(cuda(g[f"x_re_{n}"]), cuda(g[f"x_im_{n}"]))
    y = trnfft.fft(x)
    assert rel_l2(cplx(y), g[f"fft_double_re_{n}"] + 1j * g[f"fft_double_im_{n}"]) < TOL
    o_r, o_i = O.fft(g[f"x_re_{n}"], g[f"x_im_{n}"], precision="double")
    assert rel_l2(cplx(y), o_r + 1j * o_i) < TOL


def test_mixed_radix_inplace_and_batch_edges():
    n = 6000
    for batch in (1, 2, 3, 257):
        rng = np.random.default_rng(batch)
        x = (rng.standard_normal((batch, n)) + 1j * rng.standard_normal((batch, n))).astype(np.complex64)
        re, im = cuda(x.real), cuda(x.imag)
        plan = _lib.device_plan(n, re.device)
        _lib.call("trnfft_exec_c2c", plan.handle, _lib.ptr(re), _lib.ptr(im), _lib.ptr(re), _lib.ptr(im), batch, 0,
                  None, _lib.stream_ptr(re.device))
        assert rel_l2(host(re) + 1j * host(im), np.fft.fft(x.astype(np.complex128))) < 2e-6
