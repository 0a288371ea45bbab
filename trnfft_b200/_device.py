"""Placement of inputs on the CUDA device and of results back where they came from.

The reference's API accepts CPU tensors and returns CPU tensors.  Here every
transform runs on a CUDA device: CUDA inputs stay where they are; CPU inputs
are copied to the current CUDA device, transformed there, and the results are
copied back to the CPU.  Kernels compute in float32; inputs of another
floating dtype are converted and the results converted back.  Without a CUDA
device every transform raises (there is no CPU fallback).
"""

from __future__ import annotations

import torch

from . import _lib


def place(*ts: torch.Tensor, allow_f64: bool = False):
    """Return ([CUDA tensors], restore) for the given tensors: float32, or float64 when
    ``allow_f64`` and the first tensor is float64 (the transforms that have fp64 kernels)."""
    dev = None
    for t in ts:
        if t is not None and t.is_cuda:
            dev = t.device
            break
    host = dev is None
    if host:
        _lib.require_cuda()
        dev = torch.device("cuda", torch.cuda.current_device())
    odt = ts[0].dtype
    work_dt = torch.float64 if (allow_f64 and odt == torch.float64) else torch.float32
    out = [None if t is None else t.to(device=dev, dtype=work_dt) for t in ts]

    def restore(t: torch.Tensor) -> torch.Tensor:
        if host:
            t = t.to("cpu")
        if odt.is_floating_point and odt != t.dtype:
            t = t.to(odt)
        return t

    return out, restore
