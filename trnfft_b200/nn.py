"""Complex-valued layers (same classes as trnfft/nn.py).

``ComplexLinear`` is on the hot path: its forward runs the library's complex
GEMM (``trnfft_b200.nki.dispatch.complex_linear``).  ``ComplexConv1d``,
``ComplexBatchNorm1d`` and ``ComplexModReLU`` are kept for API compatibility;
they are compositions of torch layers exactly as in the reference
(trnfft/nn.py:52-129).
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn

from .complex import ComplexTensor


class ComplexLinear(nn.Module):
    """Complex-valued linear layer y = W x + b (trnfft/nn.py:18-49).

    Parameters are ``W_re``/``W_im`` (``nn.Linear`` without bias, weight
    shape (out, in)) and ``bias_re``/``bias_im``, initialised like the
    reference (kaiming_uniform with a = sqrt(5), i.e. U(+-1/sqrt(in))).
    """

    def __init__(self, in_features: int, out_features: int, bias: bool = True):
        super().__init__()
        self.W_re = nn.Linear(in_features, out_features, bias=False)
        self.W_im = nn.Linear(in_features, out_features, bias=False)
        self.bias_re = nn.Parameter(torch.zeros(out_features)) if bias else None
        self.bias_im = nn.Parameter(torch.zeros(out_features)) if bias else None
        self._reset_parameters()

    def _reset_parameters(self):
        nn.init.kaiming_uniform_(self.W_re.weight, a=math.sqrt(5))
        nn.init.kaiming_uniform_(self.W_im.weight, a=math.sqrt(5))

    def forward(self, x: ComplexTensor) -> ComplexTensor:
        from .nki.dispatch import complex_linear

        return complex_linear(x, self.W_re.weight, self.W_im.weight, self.bias_re, self.bias_im)


class ComplexConv1d(nn.Module):
    """Complex-valued 1-D convolution (trnfft/nn.py:52-86)."""

    def __init__(self, in_channels: int, out_channels: int, kernel_size: int, stride: int = 1,
                 padding: int = 0, bias: bool = True):
        super().__init__()
        self.conv_re = nn.Conv1d(in_channels, out_channels, kernel_size, stride=stride, padding=padding, bias=False)
        self.conv_im = nn.Conv1d(in_channels, out_channels, kernel_size, stride=stride, padding=padding, bias=False)
        if bias:
            self.bias_re = nn.Parameter(torch.zeros(out_channels))
            self.bias_im = nn.Parameter(torch.zeros(out_channels))
        else:
            self.bias_re = None
            self.bias_im = None

    def forward(self, x: ComplexTensor) -> ComplexTensor:
        re = self.conv_re(x.real) - self.conv_im(x.imag)
        im = self.conv_re(x.imag) + self.conv_im(x.real)
        if self.bias_re is not None:
            re = re + self.bias_re.unsqueeze(-1)
            im = im + self.bias_im.unsqueeze(-1)
        return ComplexTensor(re, im)


class ComplexBatchNorm1d(nn.Module):
    """Independent batch norm of the real and imaginary parts (trnfft/nn.py:89-104)."""

    def __init__(self, num_features: int, eps: float = 1e-5):
        super().__init__()
        self.bn_re = nn.BatchNorm1d(num_features, eps=eps)
        self.bn_im = nn.BatchNorm1d(num_features, eps=eps)

    def forward(self, x: ComplexTensor) -> ComplexTensor:
        return ComplexTensor(self.bn_re(x.real), self.bn_im(x.imag))


class ComplexModReLU(nn.Module):
    """f(z) = ReLU(|z| + b) z / |z| (trnfft/nn.py:107-129)."""

    def __init__(self, num_features: int):
        super().__init__()
        self.bias = nn.Parameter(torch.zeros(num_features))

    def forward(self, x: ComplexTensor) -> ComplexTensor:
        mag = x.abs()
        bias = self.bias
        while bias.dim() < mag.dim():
            bias = bias.unsqueeze(0)
        if mag.dim() > bias.dim():
            bias = bias.unsqueeze(-1)
        activated = torch.relu(mag + bias)
        scale = activated / torch.clamp(mag, min=1e-8)
        return ComplexTensor(x.real * scale, x.imag * scale)
