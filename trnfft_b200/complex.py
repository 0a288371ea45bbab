"""ComplexTensor: the planar (struct-of-arrays) complex type of the API.

A value is a pair of real tensors of one shape and dtype, ``real`` and
``imag``.  This is also the memory layout every CUDA kernel of the package
reads and writes (two separate float32 planes per tensor), so handing a
ComplexTensor to a transform never needs an interleave or de-interleave pass.

Behaviour follows trnfft.ComplexTensor (trnfft/complex.py:16-139), because
user code written against the reference must get identical values:

* ``ComplexTensor(x)`` with a real ``x`` means imaginary part zero; with a
  torch complex ``x`` it splits the two parts; both planes are stored
  contiguous.
* ``+``, ``-`` and ``*`` accept another ComplexTensor, a Python number or a
  real torch tensor (which acts on the real part for ``+``/``-`` and scales
  both parts for ``*``); anything else is ``NotImplemented``.
* ``@`` is the complex matrix product, which here runs on the tcgen05 GEMM.
"""

from __future__ import annotations

import torch


def _is_real_scalar_or_tensor(v) -> bool:
    """True for operands that act as a purely real value in + - *."""
    if isinstance(v, (int, float)):
        return True
    return isinstance(v, torch.Tensor) and not torch.is_complex(v)


class ComplexTensor:
    """Two equally shaped real tensors holding the real and imaginary parts."""

    __slots__ = ("real", "imag")

    def __init__(self, real: torch.Tensor, imag: torch.Tensor | None = None):
        if imag is not None:
            if real.shape != imag.shape:
                raise AssertionError(f"Shape mismatch: {real.shape} vs {imag.shape}")
            if real.dtype != imag.dtype:
                raise AssertionError(f"Dtype mismatch: {real.dtype} vs {imag.dtype}")
            re, im = real, imag
        elif torch.is_complex(real):
            re, im = real.real, real.imag
        else:
            re, im = real, torch.zeros_like(real)
        self.real = re.contiguous()
        self.imag = im.contiguous()

    # -- metadata (taken from the real plane; both planes always agree) ------
    @property
    def shape(self) -> torch.Size:
        return self.real.shape

    @property
    def dtype(self) -> torch.dtype:
        return self.real.dtype

    @property
    def device(self) -> torch.device:
        return self.real.device

    def __repr__(self) -> str:
        return f"ComplexTensor(shape={self.shape}, dtype={self.dtype})"

    # -- conversions ----------------------------------------------------------
    @classmethod
    def from_polar(cls, magnitude: torch.Tensor, phase: torch.Tensor) -> ComplexTensor:
        """r * exp(i * phi), evaluated as (r cos phi, r sin phi)."""
        return cls(magnitude * torch.cos(phase), magnitude * torch.sin(phase))

    def to_torch_complex(self) -> torch.Tensor:
        """Interleaved torch complex copy (for interop with torch.fft and the like)."""
        return torch.complex(self.real, self.imag)

    def to(self, *args, **kwargs) -> ComplexTensor:
        return ComplexTensor(self.real.to(*args, **kwargs), self.imag.to(*args, **kwargs))

    def clone(self) -> ComplexTensor:
        return ComplexTensor(self.real.clone(), self.imag.clone())

    # -- element-wise functions -----------------------------------------------
    def abs(self) -> torch.Tensor:
        """Modulus sqrt(re^2 + im^2) (no hypot scaling, matching the reference's values)."""
        return torch.sqrt(self.real ** 2 + self.imag ** 2)

    def angle(self) -> torch.Tensor:
        """Argument in (-pi, pi]."""
        return torch.atan2(self.imag, self.real)

    def conj(self) -> ComplexTensor:
        return ComplexTensor(self.real, -self.imag)

    # -- arithmetic -------------------------------------------------------------
    def __add__(self, other):
        if isinstance(other, ComplexTensor):
            return ComplexTensor(self.real + other.real, self.imag + other.imag)
        if _is_real_scalar_or_tensor(other):
            # a real addend leaves the imaginary plane unchanged (as a copy)
            return ComplexTensor(self.real + other, self.imag.clone())
        return NotImplemented

    def __radd__(self, other):
        return self.__add__(other)

    def __sub__(self, other):
        if isinstance(other, ComplexTensor):
            return ComplexTensor(self.real - other.real, self.imag - other.imag)
        if _is_real_scalar_or_tensor(other):
            return ComplexTensor(self.real - other, self.imag.clone())
        return NotImplemented

    def __mul__(self, other):
        """Element-wise product; for two complex operands (ac - bd) + i(ad + bc)."""
        if isinstance(other, ComplexTensor):
            a, b, c, d = self.real, self.imag, other.real, other.imag
            return ComplexTensor(a * c - b * d, a * d + b * c)
        if _is_real_scalar_or_tensor(other):
            return ComplexTensor(self.real * other, self.imag * other)
        return NotImplemented

    def __rmul__(self, other):
        return self.__mul__(other)

    def __neg__(self) -> ComplexTensor:
        return ComplexTensor(-self.real, -self.imag)

    def __matmul__(self, other):
        if isinstance(other, ComplexTensor):
            return complex_matmul(self, other)
        return NotImplemented

    # -- indexing and shape ------------------------------------------------------
    def __getitem__(self, key) -> ComplexTensor:
        return ComplexTensor(self.real[key], self.imag[key])

    def __setitem__(self, key, value: ComplexTensor):
        self.real[key] = value.real
        self.imag[key] = value.imag

    def reshape(self, *shape) -> ComplexTensor:
        return ComplexTensor(self.real.reshape(*shape), self.imag.reshape(*shape))

    def transpose(self, dim0: int, dim1: int) -> ComplexTensor:
        """Swap two axes; the result is materialised contiguous, like every ComplexTensor."""
        return ComplexTensor(self.real.transpose(dim0, dim1), self.imag.transpose(dim0, dim1))

    def unsqueeze(self, dim: int) -> ComplexTensor:
        return ComplexTensor(self.real.unsqueeze(dim), self.imag.unsqueeze(dim))

    def squeeze(self, dim: int | None = None) -> ComplexTensor:
        if dim is None:
            return ComplexTensor(self.real.squeeze(), self.imag.squeeze())
        return ComplexTensor(self.real.squeeze(dim), self.imag.squeeze(dim))


def complex_matmul(a: ComplexTensor, b: ComplexTensor) -> ComplexTensor:
    """Matrix product A @ B of planar complex matrices (trnfft/complex.py:142-150).

    Runs on the library's tensor-core GEMM (3xTF32, float32 accuracy) as
    y = A W^T with W = B^T; the value is re = Ar Br - Ai Bi, im = Ar Bi + Ai Br.
    """
    from .nki.dispatch import complex_gemm

    return complex_gemm(a, b)
