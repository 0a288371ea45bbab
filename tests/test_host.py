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
