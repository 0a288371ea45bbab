"""GPU checks of the host-streaming helper and of ComplexLinear's cached weight split."""

import numpy as np
import pytest
import torch

import trnfft_b200 as trnfft
from trnfft_b200 import ComplexTensor
from trnfft_b200.nn import ComplexLinear
from trnfft_b200.streaming import map_rows
from tests.helpers import TOL, rel_l2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,nchunks", [(1000, 8), (7, 8), (64, 1), (4097, 5)])
def test_map_rows_round_trip_matches_device_path(rows, nchunks):
    g = torch.Generator().manual_seed(rows)
    xr = torch.randn(rows, 1024, generator=g).pin_memory()
    xi = torch.randn(rows, 1024, generator=g).pin_memory()

    def step(ts):
        y = trnfft.fft(ComplexTensor(ts[0], ts[1]))
        return [y.real, y.imag]

    outs = map_rows(step, [xr, xi], nchunks=nchunks)
    torch.cuda.current_stream().synchronize()
    want = np.fft.fft(xr.double().numpy() + 1j * xi.double().numpy())
    assert rel_l2(outs[0].numpy() + 1j * outs[1].numpy(), want) < TOL


def test_complex_linear_weight_split_cache_follows_weight_updates():
    torch.manual_seed(0)
    layer = ComplexLinear(256, 128).cuda()
    x = ComplexTensor(torch.randn(64, 256, device="cuda"), torch.randn(64, 256, device="cuda"))

    def ref():
        wr, wi = layer.W_re.weight.double(), layer.W_im.weight.double()
        a, b = x.real.double(), x.imag.double()
        return torch.complex(a @ wr.t() - b @ wi.t() + layer.bias_re.double(),
                             a @ wi.t() + b @ wr.t() + layer.bias_im.double())

    for step in range(3):
        with torch.no_grad():
            y = layer(x)
        got = torch.complex(y.real.double(), y.imag.double())
        want = ref()
        assert float(torch.linalg.vector_norm(got - want) / torch.linalg.vector_norm(want)) < TOL
        with torch.no_grad():  # an in-place update bumps the version: the split must be redone
            layer.W_re.weight.mul_(1.5).add_(0.01)
            layer.W_im.weight.sub_(0.02)
    # training: gradients still match torch's
    layer.zero_grad()
    xg = ComplexTensor(x.real.clone().requires_grad_(), x.imag.clone().requires_grad_())
    y = layer(xg)
    (y.real.sum() + 2 * y.imag.sum()).backward()
    wr = layer.W_re.weight.detach().clone().requires_grad_()
    wi = layer.W_im.weight.detach().clone().requires_grad_()
    a, b = x.real.clone().requires_grad_(), x.imag.clone().requires_grad_()
    yr = a @ wr.t() - b @ wi.t()
    yi = a @ wi.t() + b @ wr.t()
    (yr.sum() + 2 * yi.sum()).backward()
    assert torch.allclose(layer.W_re.weight.grad, wr.grad, rtol=1e-4, atol=1e-4)
    assert torch.allclose(xg.real.grad, a.grad, rtol=1e-4, atol=1e-4)
