"""Shared helpers for the GPU parity tests."""

import numpy as np
import torch

from oracle import trnfft_oracle as O

rel_l2 = O.rel_l2

# Parity tolerance against the reference's pytorch backend and against the
# oracle: relative L2 error <= 1e-5 in float32.
TOL = 1e-5


def cuda(a):
    return torch.as_tensor(np.asarray(a, dtype=np.float32)).cuda()


def host(t):
    return t.detach().float().cpu().numpy()


def cplx(ct):
    return host(ct.real) + 1j * host(ct.imag)
