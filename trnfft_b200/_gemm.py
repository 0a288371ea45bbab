"""Complex GEMM entry points used by complex_matmul and ComplexLinear.

Stage 1 (this file as first written): planar complex products composed from
real device matmuls, the reference's pytorch formulation
(trnfft/complex.py:142-150, trnfft/nn.py:44-48).  The tcgen05 3xTF32 kernel
replaces these bodies.
"""

from __future__ import annotations

import torch

from ._device import place
from .complex import ComplexTensor


def complex_matmul(a: ComplexTensor, b: ComplexTensor) -> ComplexTensor:
    (ar, ai, br, bi), restore = place(a.real, a.imag, b.real, b.imag)
    re = torch.matmul(ar, br) - torch.matmul(ai, bi)
    im = torch.matmul(ar, bi) + torch.matmul(ai, br)
    return ComplexTensor(restore(re), restore(im))


def complex_linear(x: ComplexTensor, w_re, w_im, b_re=None, b_im=None) -> ComplexTensor:
    (xr, xi, wr, wi), restore = place(x.real, x.imag, w_re, w_im)
    re = xr @ wr.t() - xi @ wi.t()
    im = xr @ wi.t() + xi @ wr.t()
    if b_re is not None:
        re = re + b_re.to(re.device)
        im = im + b_im.to(im.device)
    return ComplexTensor(restore(re), restore(im))
