"""GPU parity of the tcgen05 3xTF32 complex GEMM (ComplexLinear, complex_matmul)."""

import numpy as np
import pytest
import torch

import trnfft_b200 as trnfft
from trnfft_b200 import ComplexTensor, _lib
from trnfft_b200.nn import ComplexLinear
from tests.helpers import TOL, cplx, cuda, host, rel_l2

pytestmark = pytest.mark.gpu


def test_linear_vs_reference_golden(golden):
    g = golden("linear")
    layer = ComplexLinear(96, 48).cuda()
    with torch.no_grad():
        layer.W_re.weight.copy_(cuda(g["w_re"]))
        layer.W_im.weight.copy_(cuda(g["w_im"]))
        layer.bias_re.copy_(cuda(g["b_re"]))
        layer.bias_im.copy_(cuda(g["b_im"]))
        y = layer(ComplexTensor(cuda(g["x_re"]), cuda(g["x_im"])))
    assert rel_l2(cplx(y), g["y_re"] + 1j * g["y_im"]) < TOL
    assert _lib.device_status(torch.cuda.current_device()) == 0


@pytest.mark.parametrize("M,N,K", [(128, 256, 32), (300, 200, 128), (1, 7, 5), (1000, 513, 260), (2048, 1024, 1024)])
def test_linear_vs_fp64(M, N, K):
    rng = np.random.default_rng(M + N + K)
    x = rng.standard_normal((M, K)) + 1j * rng.standard_normal((M, K))
    w = (rng.uniform(-1, 1, (N, K)) + 1j * rng.uniform(-1, 1, (N, K))) / np.sqrt(K)
    x = x.astype(np.complex64)
    w = w.astype(np.complex64)
    xr, xi = cuda(x.real), cuda(x.imag)
    y = trnfft.nki.dispatch.complex_linear(ComplexTensor(xr, xi), cuda(w.real), cuda(w.imag))
    ref = x.astype(np.complex128) @ w.astype(np.complex128).T
    assert rel_l2(cplx(y), ref) < TOL
    assert _lib.device_status(torch.cuda.current_device()) == 0


def test_complex_matmul_vs_reference_golden(golden):
    g = golden("linear")
    a = ComplexTensor(cuda(g["a_re"]), cuda(g["a_im"]))
    b = ComplexTensor(cuda(g["b2_re"]), cuda(g["b2_im"]))
    c = trnfft.complex_matmul(a, b)
    assert rel_l2(cplx(c), g["c_re"] + 1j * g["c_im"]) < TOL
    c2 = a @ b
    assert rel_l2(cplx(c2), g["c_re"] + 1j * g["c_im"]) < TOL


def test_linear_gradients_match_torch():
    torch.manual_seed(0)
    layer = ComplexLinear(64, 32).cuda()
    xr = torch.randn(8, 64, device="cuda", requires_grad=True)
    xi = torch.randn(8, 64, device="cuda", requires_grad=True)
    y = layer(ComplexTensor(xr, xi))
    (y.real ** 2 + y.imag ** 2).sum().backward()
    wr = layer.W_re.weight.detach().clone().requires_grad_(True)
    wi = layer.W_im.weight.detach().clone().requires_grad_(True)
    zr = xr.detach().clone().requires_grad_(True)
    zi = xi.detach().clone().requires_grad_(True)
    re = zr @ wr.t() - zi @ wi.t()
    im = zr @ wi.t() + zi @ wr.t()
    (re ** 2 + im ** 2).sum().backward()
    assert rel_l2(host(layer.W_re.weight.grad), host(wr.grad)) < 1e-5
    assert rel_l2(host(layer.W_im.weight.grad), host(wi.grad)) < 1e-5
    assert rel_l2(host(xr.grad), host(zr.grad)) < 1e-5


@pytest.mark.parametrize("n", [8, 64, 128, 256])
def test_dft_as_gemm_vs_reference_golden(golden, n):
    """Small-n transforms on the tensor-core DFT-GEMM path (the reference's
    NKI path for n <= 256, trnfft/fft_core.py:221-251)."""
    g = golden("pow2_c2c")
    trnfft.set_small_n_algorithm("gemm")
    try:
        x = ComplexTensor(cuda(g[f"x_re_{n}"]), cuda(g[f"x_im_{n}"]))
        y = trnfft.fft(x)
        z = trnfft.ifft(x)
    finally:
        trnfft.set_small_n_algorithm("stockham")
    assert rel_l2(cplx(y), g[f"fft_re_{n}"] + 1j * g[f"fft_im_{n}"]) < TOL
    assert rel_l2(cplx(z), g[f"ifft_re_{n}"] + 1j * g[f"ifft_im_{n}"]) < TOL


def test_dft_as_gemm_large_batch_vs_fp64():
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((4096, 256)) + 1j * rng.standard_normal((4096, 256))).astype(np.complex64)
    trnfft.set_small_n_algorithm("gemm")
    try:
        y = trnfft.fft(ComplexTensor(cuda(x.real), cuda(x.imag)))
    finally:
        trnfft.set_small_n_algorithm("stockham")
    assert rel_l2(cplx(y), np.fft.fft(x.astype(np.complex128))) < 2e-6


def test_complex_linear_on_a_second_device_after_the_first():
    """The GEMM's shared-memory opt-in is per device: a layer on cuda:1 after one on cuda:0
    (same process) must launch and agree with fp64 (needs two GPUs)."""
    import torch

    if torch.cuda.device_count() < 2:
        import pytest

        pytest.skip("needs two GPUs")
    from trnfft_b200 import ComplexTensor
    from trnfft_b200.nn import ComplexLinear

    for dev in ("cuda:0", "cuda:1"):
        torch.manual_seed(3)
        layer = ComplexLinear(512, 256).to(dev)
        x = ComplexTensor(torch.randn(300, 512, device=dev), torch.randn(300, 512, device=dev))
        with torch.no_grad():
            y = layer(x)
        wr, wi = layer.W_re.weight.double(), layer.W_im.weight.double()
        a, b = x.real.double(), x.imag.double()
        ref = torch.complex(a @ wr.t() - b @ wi.t(), a @ wi.t() + b @ wr.t())
        got = torch.complex(y.real.double(), y.imag.double())
        assert y.real.device == torch.device(dev)
        assert float(torch.linalg.vector_norm(got - ref) / torch.linalg.vector_norm(ref)) < 1e-5


_VARIANT_SCRIPT = r"""
import numpy as np, torch
import trnfft_b200 as trnfft
from trnfft_b200 import ComplexTensor, _lib
worst = 0.0
for (M, N, K) in [(1, 7, 5), (300, 200, 128), (1000, 513, 260), (512, 768, 1024)]:
    rng = np.random.default_rng(M + N + K)
    x = (rng.standard_normal((M, K)) + 1j * rng.standard_normal((M, K))).astype(np.complex64)
    w = ((rng.uniform(-1, 1, (N, K)) + 1j * rng.uniform(-1, 1, (N, K))) / np.sqrt(K)).astype(np.complex64)
    b = (rng.standard_normal(N) + 1j * rng.standard_normal(N)).astype(np.complex64)
    f = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    y = trnfft.nki.dispatch.complex_linear(ComplexTensor(f(x.real), f(x.imag)), f(w.real), f(w.imag), f(b.real), f(b.imag))
    ref = x.astype(np.complex128) @ w.astype(np.complex128).T + b.astype(np.complex128)
    got = y.real.double().cpu().numpy() + 1j * y.imag.double().cpu().numpy()
    worst = max(worst, float(np.linalg.norm(got - ref) / np.linalg.norm(ref)))
    assert _lib.device_status(torch.cuda.current_device()) == 0
print("WORST", worst)
"""


@pytest.mark.parametrize("env", [{"TRNFFT_B200_GEMM_PAIR": "1"}, {"TRNFFT_B200_LINEAR_4M": "1"}],
                         ids=["two-SM pair kernel", "four-product form"])
def test_linear_variants_vs_fp64(env):
    """The opt-in GEMM variants (selected once per process by environment variables, so each runs in
    a child process) agree with fp64 like the default three-product one-CTA path."""
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _VARIANT_SCRIPT], cwd=root, env={**os.environ, **env},
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    worst = float(r.stdout.split("WORST")[-1])
    assert worst < TOL
