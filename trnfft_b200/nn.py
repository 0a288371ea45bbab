"""Complex-valued layers (same classes as trnfft/nn.py).

``ComplexLinear`` is on the hot path: its forward runs the library's complex
GEMM (``trnfft_b200.nki.dispatch.complex_linear``).  ``ComplexConv1d``,
``ComplexBatchNorm1d`` and ``ComplexModReLU`` are kept for API compatibility
(same parameters and values as trnfft/nn.py:52-129); they are off the FFT hot
path and written as plain torch compositions.
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
        from . import _gemm

        # the weight's TF32 hi/lo split is cached here and redone only when the
        # weight's storage or version changes (e.g. after an optimizer step)
        if not hasattr(self, "_wsplit"):
            self._wsplit = {}
        if not (self.W_re.weight.is_cuda or x.real.is_cuda):
            self._wsplit = {}
        return _gemm.complex_linear(x, self.W_re.weight, self.W_im.weight, self.bias_re, self.bias_im,
                                    cache=self._wsplit if self.W_re.weight.is_cuda else None)


class ComplexConv1d(nn.Module):
    """Complex 1-D convolution with the reference's parameters (trnfft/nn.py:52-86).

    Parameters: ``conv_re`` / ``conv_im`` (``nn.Conv1d`` without bias, the
    real and imaginary kernel) and optional ``bias_re`` / ``bias_im``.  The
    forward pass runs ONE real convolution over the stacked channels
    [x_re; x_im] with the 2x2 block kernel [[K_re, -K_im], [K_im, K_re]], whose
    output channels are then [y_re; y_im] = [K_re*x_re - K_im*x_im;
    K_im*x_re + K_re*x_im].  Not on the FFT hot path.
    """

    def __init__(self, in_channels: int, out_channels: int, kernel_size: int, stride: int = 1,
                 padding: int = 0, bias: bool = True):
        super().__init__()
        self.conv_re = nn.Conv1d(in_channels, out_channels, kernel_size, stride=stride, padding=padding, bias=False)
        self.conv_im = nn.Conv1d(in_channels, out_channels, kernel_size, stride=stride, padding=padding, bias=False)
        self.bias_re = nn.Parameter(torch.zeros(out_channels)) if bias else None
        self.bias_im = nn.Parameter(torch.zeros(out_channels)) if bias else None

    def forward(self, x: ComplexTensor) -> ComplexTensor:
        kr, ki = self.conv_re.weight, self.conv_im.weight
        block = torch.cat([torch.cat([kr, -ki], dim=1), torch.cat([ki, kr], dim=1)], dim=0)
        b = None
        if self.bias_re is not None:
            b = torch.cat([self.bias_re, self.bias_im])
        y = torch.nn.functional.conv1d(torch.cat([x.real, x.imag], dim=-2), block, b,
                                       stride=self.conv_re.stride, padding=self.conv_re.padding)
        c = kr.shape[0]
        return ComplexTensor(y[..., :c, :], y[..., c:, :])


class ComplexBatchNorm1d(nn.Module):
    """Batch normalisation of the real and the imaginary plane as separate channels
    (trnfft/nn.py:89-104: two independent ``BatchNorm1d``; no whitening of the
    complex covariance).  Keeps the reference's ``bn_re`` / ``bn_im`` modules
    (and state-dict keys); the statistics of each plane are its own."""

    def __init__(self, num_features: int, eps: float = 1e-5):
        super().__init__()
        self.bn_re = nn.BatchNorm1d(num_features, eps=eps)
        self.bn_im = nn.BatchNorm1d(num_features, eps=eps)

    def forward(self, x: ComplexTensor) -> ComplexTensor:
        planes = [bn(p) for bn, p in ((self.bn_re, x.real), (self.bn_im, x.imag))]
        return ComplexTensor(*planes)


class ComplexModReLU(nn.Module):
    """modReLU: keeps the phase of z and maps the modulus r = |z| to max(r + b, 0)
    (trnfft/nn.py:107-129), with one learnt offset b per feature, broadcast
    along the LAST axis as the reference does.  The gain
    max(r + b, 0) / max(r, 1e-8) multiplies both planes."""

    def __init__(self, num_features: int):
        super().__init__()
        self.bias = nn.Parameter(torch.zeros(num_features))

    def forward(self, x: ComplexTensor) -> ComplexTensor:
        r = x.abs()
        gain = torch.relu(r + self.bias) / r.clamp_min(1e-8)
        return ComplexTensor(x.real * gain, x.imag * gain)
