"""Host-only checks (no GPU): the C-ABI library loads and exports every
declared symbol, and the pure host logic mirrors the reference."""

import ctypes
import os
import re

import pytest
import torch

import trnfft_b200 as trnfft
from trnfft_b200 import _lib
from trnfft_b200.nki import multicore

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in os.listdir(os.path.join(ROOT, "include")):
        if h.endswith(".h"):
            txt = open(os.path.join(ROOT, "include", h)).read()
            names |= set(re.findall(r"^\s*(?:const\s+)?\w[\w\s\*]*?\b(trnfft_\w+)\s*\(", txt, re.M))
    return names


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(_lib.LIB_PATH):
        from trnfft_b200 import build

        build.build()
    return ctypes.CDLL(_lib.LIB_PATH)


def test_library_exports_every_declared_symbol(lib):
    names = declared_symbols()
    assert "trnfft_exec_c2c" in names and len(names) >= 8
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/ but not exported"
    assert set(_lib.SIGNATURES) == names


def test_abi_version_and_error_string(lib):
    lib.trnfft_abi_version.restype = ctypes.c_int
    assert lib.trnfft_abi_version() == _lib.ABI_VERSION
    lib.trnfft_plan_destroy.argtypes = [ctypes.c_void_p]
    assert lib.trnfft_plan_destroy(None) == 0


def test_plan_cache_semantics():
    trnfft.clear_plan_cache()
    p = trnfft.create_plan(1024)
    assert p is trnfft.create_plan(1024) and p.is_power_of_2
    q = trnfft.create_plan(4093, inverse=True)
    assert q.padded_n == 8192 and not q.is_power_of_2 and q.inverse
    assert trnfft.create_plan(6000).padded_n == 16384
    assert trnfft.create_plan(1000).padded_n == 2048
    trnfft.clear_plan_cache()


def test_precision_and_backend_switch():
    trnfft.set_precision("double")
    assert trnfft.get_precision() == "double"
    trnfft.set_precision("fast")
    with pytest.raises(ValueError):
        trnfft.set_precision("quad")
    assert trnfft.get_backend() in ("auto", "cuda")
    with pytest.raises(RuntimeError):
        trnfft.set_backend("pytorch")
    trnfft.set_backend("cuda")
    trnfft.set_backend("auto")
    assert trnfft.HAS_NKI is False


def test_factorize_and_num_cores():
    assert multicore._factorize(1 << 30) == (32768, 32768)
    assert multicore._factorize(65536) == (256, 256)
    with pytest.raises(ValueError, match="prime"):
        multicore._factorize(65537)
    multicore._num_cores = 8
    assert multicore._resolve_num_cores(4) == 4 and multicore._resolve_num_cores(16) == 8
    multicore._num_cores = 0
    if not torch.cuda.is_available():
        assert multicore._resolve_num_cores(1) == 1
        assert multicore._resolve_num_cores(4) == 2


def test_no_cpu_fallback_without_cuda():
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is visible")
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        trnfft.fft(torch.randn(8))


def test_multicore_prime_raises_before_compute():
    multicore.set_multicore(True)
    try:
        with pytest.raises(NotImplementedError, match="prime"):
            multicore.multi_core_fft(trnfft.ComplexTensor(torch.randn(7), torch.zeros(7)))
    finally:
        multicore.set_multicore(False)


def test_complex_layers_off_the_hot_path_match_their_definitions():
    """ComplexConv1d, ComplexBatchNorm1d and ComplexModReLU (CPU, torch only) against the
    complex arithmetic they define (trnfft/nn.py:52-129)."""
    import torch

    from trnfft_b200 import ComplexTensor
    from trnfft_b200.nn import ComplexBatchNorm1d, ComplexConv1d, ComplexModReLU

    torch.manual_seed(0)
    conv = ComplexConv1d(3, 5, 4, stride=2, padding=1)
    with torch.no_grad():
        conv.bias_re.normal_()
        conv.bias_im.normal_()
    x = ComplexTensor(torch.randn(2, 3, 20), torch.randn(2, 3, 20))
    y = conv(x)
    xc = torch.complex(x.real, x.imag).to(torch.complex64)
    kc = torch.complex(conv.conv_re.weight, conv.conv_im.weight)
    bc = torch.complex(conv.bias_re, conv.bias_im)
    want = torch.nn.functional.conv1d(xc, kc, bc, stride=2, padding=1)
    assert torch.allclose(torch.complex(y.real, y.imag), want, atol=1e-5)

    relu = ComplexModReLU(7)
    with torch.no_grad():
        relu.bias.normal_()
    z = ComplexTensor(torch.randn(4, 5, 7), torch.randn(4, 5, 7))
    out = relu(z)
    zc = torch.complex(z.real, z.imag)
    r = zc.abs()
    want = torch.relu(r + relu.bias) * zc / r.clamp_min(1e-8)
    assert torch.allclose(torch.complex(out.real, out.imag), want, atol=1e-6)

    bn = ComplexBatchNorm1d(3)
    u = ComplexTensor(torch.randn(8, 3, 10), torch.randn(8, 3, 10))
    v = bn(u)
    ref = torch.nn.BatchNorm1d(3)
    assert torch.allclose(v.real, ref(u.real), atol=1e-6)
    assert torch.allclose(v.imag, torch.nn.BatchNorm1d(3)(u.imag), atol=1e-6)


def test_istft_out_len_matches_the_reference_trim_rules():
    """The fused iSTFT's output length rule (api.py:454-468) against the oracle's istft."""
    import numpy as np

    from oracle import trnfft_oracle as O
    from trnfft_b200._ops import istft_out_len

    rng = np.random.default_rng(0)
    for n_fft, hop, frames, center, length in [(16, 4, 9, True, None), (16, 4, 9, False, None),
                                                (16, 16, 3, True, None), (8, 3, 5, True, 30),
                                                (8, 3, 5, True, 2), (4, 1, 2, True, None)]:
        bins = n_fft // 2 + 1
        sr = rng.standard_normal((bins, frames)).astype(np.float32)
        si = rng.standard_normal((bins, frames)).astype(np.float32)
        want = O.istft(sr, si, n_fft, hop, window=np.ones(n_fft, np.float32), center=center, length=length)
        assert istft_out_len(n_fft, frames, hop, center, length) == want.shape[-1]


def test_mask_period_and_row_chunks():
    from trnfft_b200.nki.dispatch import _mask_period
    from trnfft_b200.streaming import _chunks

    assert _mask_period((257, 100), (4, 257, 100)) == 257 * 100
    assert _mask_period((1, 1, 7), (3, 5, 7)) == 7
    assert _mask_period((3, 1, 7), (3, 5, 7)) is None
    assert _mask_period((4, 257, 100), (257, 100)) is None
    for rows, n in [(10, 4), (3, 8), (8192, 4), (1, 1)]:
        parts = list(_chunks(rows, max(1, min(n, rows))))
        assert parts[0][0] == 0 and parts[-1][1] == rows
        assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
