"""Backend selection and the complex GEMM / linear / mask entry points.

Replaces trnfft/nki/dispatch.py.  The reference switches between
``"auto"``, ``"pytorch"`` and ``"nki"`` (dispatch.py:50-71); here the only
backend is the CUDA library, so ``"auto"`` and ``"cuda"`` select it and
``"pytorch"`` / ``"nki"`` raise: a silent CPU or torch fallback would defeat
the point of the library.
"""

from __future__ import annotations

import torch

from ..complex import ComplexTensor

HAS_NKI = False  # no Trainium here; kept for API compatibility

_VALID = ("auto", "cuda")
_backend = "auto"


def set_backend(backend: str):
    """Select the dispatch backend.  Only ``"auto"`` and ``"cuda"`` exist on B200."""
    global _backend
    if backend in ("pytorch", "nki"):
        raise RuntimeError(
            f"backend {backend!r} is not available in trnfft_b200: transforms always run on the "
            "CUDA kernels (use 'auto' or 'cuda')"
        )
    if backend not in _VALID:
        raise AssertionError(f"backend must be one of {_VALID}, got {backend!r}")
    _backend = backend


def get_backend() -> str:
    return _backend


def _use_nki() -> bool:
    return False


def complex_gemm(a: ComplexTensor, b: ComplexTensor) -> ComplexTensor:
    """C = A @ B for planar complex matrices (trnfft/nki/dispatch.py:74-84)."""
    from .. import _gemm

    return _gemm.complex_matmul(a, b)


def complex_linear(x: ComplexTensor, w_real: torch.Tensor, w_imag: torch.Tensor,
                   b_real: torch.Tensor | None = None, b_imag: torch.Tensor | None = None) -> ComplexTensor:
    """y = x @ W^T (+ b) for planar complex x and W (trnfft/nki/dispatch.py:91-102)."""
    from .. import _gemm

    return _gemm.complex_linear(x, w_real, w_imag, b_real, b_imag)


def _mask_period(mshape, sshape):
    """Elements of the mask when it repeats along the spectrogram's leading axes
    (its shape, without leading ones, is a suffix of the spectrogram's), else None."""
    m = list(mshape)
    while m and m[0] == 1:
        m.pop(0)
    if len(m) > len(sshape) or (m and list(sshape[len(sshape) - len(m):]) != m):
        return None
    c = 1
    for d in m:
        c *= d
    return c


def _mask_raw(mr, mi, sr, si):
    """y = m * s on the fused kernel; m repeats over the leading axes of s."""
    from .. import _lib

    period = _mask_period(mr.shape, sr.shape)
    if period is None:  # general broadcast: materialise both operands at the output shape
        shape = torch.broadcast_shapes(mr.shape, sr.shape)
        mr, mi = mr.expand(shape), mi.expand(shape)
        sr, si = sr.expand(shape), si.expand(shape)
        period = sr.numel()
    mr, mi, sr, si = (t.contiguous() for t in (mr, mi, sr, si))
    yr = torch.empty(sr.shape, dtype=torch.float32, device=sr.device)
    yi = torch.empty_like(yr)
    if yr.numel():
        _lib.call("trnfft_complex_mask_apply", _lib.ptr(mr), _lib.ptr(mi), period, _lib.ptr(sr), _lib.ptr(si),
                  _lib.ptr(yr), _lib.ptr(yi), yr.numel(),
                  sr.device.index if sr.device.index is not None else torch.cuda.current_device(),
                  _lib.stream_ptr(sr.device))
    return yr, yi


def _unbroadcast(g: torch.Tensor, shape) -> torch.Tensor:
    while g.dim() > len(shape):
        g = g.sum(0)
    for i, d in enumerate(shape):
        if d == 1 and g.shape[i] != 1:
            g = g.sum(i, keepdim=True)
    return g


class _MaskFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, mr, mi, sr, si):
        ctx.save_for_backward(mr, mi, sr, si)
        return _mask_raw(mr, mi, sr, si)

    @staticmethod
    def backward(ctx, gr, gi):
        # y = m s: dL/dm = g conj(s), dL/ds = g conj(m) (planar, summed over broadcast axes)
        mr, mi, sr, si = ctx.saved_tensors
        dmr, dmi = gr * sr + gi * si, gi * sr - gr * si
        dsr, dsi = gr * mr + gi * mi, gi * mr - gr * mi
        return (_unbroadcast(dmr, mr.shape), _unbroadcast(dmi, mi.shape),
                _unbroadcast(dsr, sr.shape), _unbroadcast(dsi, si.shape))


def complex_mask_apply(mask: ComplexTensor, spec: ComplexTensor) -> ComplexTensor:
    """Complex mask times spectrogram, element-wise (trnfft/nki/dispatch.py:105-113).

    One fused kernel (trnfft_complex_mask_apply) reads the four planes once and
    writes the two output planes once; shapes broadcast like ``mask * spec``.
    """
    from .._device import place

    (mr, mi, sr, si), restore = place(mask.real, mask.imag, spec.real, spec.imag)
    if torch.is_grad_enabled() and any(t.requires_grad for t in (mr, mi, sr, si)):
        yr, yi = _MaskFn.apply(mr, mi, sr, si)
    else:
        yr, yi = _mask_raw(mr, mi, sr, si)
    return ComplexTensor(restore(yr), restore(yi))
