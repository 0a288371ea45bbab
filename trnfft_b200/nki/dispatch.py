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


def complex_mask_apply(mask: ComplexTensor, spec: ComplexTensor) -> ComplexTensor:
    """Element-wise complex mask (trnfft/nki/dispatch.py:105-113)."""
    return mask * spec
