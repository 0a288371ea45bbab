"""The allocation-free in-place entry point, checked against the normal one.

trnfft_exec_c2c_inplace_noalloc serves callers that cannot allocate device
memory (they run inside another allocator or pool, in real-time callbacks, or
in runtimes that only lend fixed buffers): it uses a fixed scratch array the
library reserves per GPU instead of a caller-provided work area.  Its result
must match the out-of-place trnfft_exec_c2c within the suite's tolerance, on
two calls in a row (the second call runs on scratch left over by the first).

This file is named so that pytest collects it last.
"""

import ctypes

import numpy as np
import pytest
import torch

from trnfft_b200 import _lib
from tests.helpers import TOL, rel_l2

pytestmark = pytest.mark.gpu


def _reference(plan, xr, xi, inverse):
    yr = torch.empty_like(xr)
    yi = torch.empty_like(xi)
    _lib.call("trnfft_exec_c2c", plan.handle, _lib.ptr(xr), _lib.ptr(xi), _lib.ptr(yr), _lib.ptr(yi),
              xr.shape[0], int(inverse), None, _lib.stream_ptr(xr.device))
    return yr, yi


@pytest.mark.parametrize("n,batch", [(1 << 13, 4), (1 << 21, 1), (1 << 13, 256), (1 << 20, 2)])
def test_noalloc_matches_exec_c2c_twice(n, batch):
    dev = torch.device("cuda", torch.cuda.current_device())
    plan = _lib.device_plan(n, dev)
    st = _lib.stream_ptr(dev)
    for call, inverse in enumerate((False, True)):
        g = torch.Generator(device=dev).manual_seed(100 + call)
        xr = torch.randn(batch, n, device=dev, generator=g)
        xi = torch.randn(batch, n, device=dev, generator=g)
        want_r, want_i = _reference(plan, xr, xi, inverse)
        _lib.call("trnfft_exec_c2c_inplace_noalloc", plan.handle, _lib.ptr(xr), _lib.ptr(xi), batch,
                  int(inverse), st)
        torch.cuda.synchronize()
        got = xr.cpu().numpy() + 1j * xi.cpu().numpy()
        want = want_r.cpu().numpy() + 1j * want_i.cpu().numpy()
        assert rel_l2(got, want) < TOL


def test_noalloc_rejects_sizes_beyond_scratch():
    dev = torch.device("cuda", torch.cuda.current_device())
    n = 1 << 21
    plan = _lib.device_plan(n, dev)
    x = torch.zeros(2, n, device=dev)
    with pytest.raises(ValueError, match="exceeds the fixed scratch"):
        _lib.call("trnfft_exec_c2c_inplace_noalloc", plan.handle, _lib.ptr(x), _lib.ptr(x), 2, 0,
                  _lib.stream_ptr(dev))
    # 2^20 x 3 is one transform more than the scratch holds (2^20 x 2 fits exactly)
    mid = _lib.device_plan(1 << 20, dev)
    y = torch.zeros(3, 1 << 20, device=dev)
    with pytest.raises(ValueError, match="exceeds the fixed scratch"):
        _lib.call("trnfft_exec_c2c_inplace_noalloc", mid.handle, _lib.ptr(y), _lib.ptr(y), 3, 0,
                  _lib.stream_ptr(dev))
    small = _lib.device_plan(1024, dev)
    with pytest.raises(ValueError, match="only power-of-two n > 4096"):
        _lib.call("trnfft_exec_c2c_inplace_noalloc", small.handle, _lib.ptr(x), _lib.ptr(x), 1, 0,
                  _lib.stream_ptr(dev))
