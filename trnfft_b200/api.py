"""Public transform API, signature-compatible with trnfft/api.py.

Usage::

    import trnfft_b200 as trnfft

    X = trnfft.fft(x)
    x = trnfft.ifft(X)
    S = trnfft.stft(waveform, n_fft=512, hop_length=256)

Every function accepts what the reference accepts (real torch tensors,
ComplexTensor, torch complex tensors) and returns the same types and shapes.
The transforms run on CUDA kernels; CPU inputs are moved to the current CUDA
device and the results moved back.
"""

from __future__ import annotations

import torch

from . import _ops
from ._device import place
from .complex import ComplexTensor
from .fft_core import fft_core, irfft_core, rfft_core


def fft(input: torch.Tensor | ComplexTensor, n: int | None = None) -> ComplexTensor:
    """1-D discrete Fourier transform along the last dimension (trnfft/api.py:22-27)."""
    x = _to_complex(input)
    if n is not None:
        x = _resize_last(x, n)
    return fft_core(x, inverse=False)


def ifft(input: torch.Tensor | ComplexTensor, n: int | None = None) -> ComplexTensor:
    """1-D inverse discrete Fourier transform, scaled by 1/n (trnfft/api.py:30-35)."""
    x = _to_complex(input)
    if n is not None:
        x = _resize_last(x, n)
    return fft_core(x, inverse=True)


def rfft(input: torch.Tensor, n: int | None = None) -> ComplexTensor:
    """FFT of a real signal, bins 0..n//2 (trnfft/api.py:38-46)."""
    if n is not None:
        input = _resize_real(input, n)
    if input.shape[-1] == 1:
        return ComplexTensor(input.clone(), torch.zeros_like(input))
    return rfft_core(input)


def irfft(input: ComplexTensor, n: int | None = None) -> torch.Tensor:
    """Inverse FFT of a Hermitian spectrum, real result (trnfft/api.py:49-68)."""
    if n is None:
        n = 2 * (input.shape[-1] - 1)
    return irfft_core(input, n)


def hfft(input: ComplexTensor, n: int | None = None) -> torch.Tensor:
    """FFT of a Hermitian signal: irfft(conj(input), n) * n (trnfft/api.py:71-87)."""
    if n is None:
        n = 2 * (input.shape[-1] - 1)
    conj_input = ComplexTensor(input.real, -input.imag)
    return irfft(conj_input, n=n) * n


def ihfft(input: torch.Tensor, n: int | None = None) -> ComplexTensor:
    """IFFT of a real signal, one-sided: conj(rfft(input, n)) / n (trnfft/api.py:90-102)."""
    n_actual = input.shape[-1] if n is None else n
    result = rfft(input, n=n_actual)
    return ComplexTensor(result.real / n_actual, -result.imag / n_actual)


def fft2(input: torch.Tensor | ComplexTensor, s: tuple[int, int] | None = None) -> ComplexTensor:
    """2-D FFT along the last two dimensions (trnfft/api.py:105-108)."""
    s_arg = None if s is None else tuple(s)
    return fftn(input, s=s_arg, dim=(-2, -1))


def _norm_dims(ndim, s, dim):
    if dim is None:
        dim = tuple(range(-len(s), 0)) if s is not None else tuple(range(-ndim, 0))
    return tuple(d % ndim for d in dim)


def fftn(
    input: torch.Tensor | ComplexTensor,
    s: tuple[int, ...] | None = None,
    dim: tuple[int, ...] | None = None,
) -> ComplexTensor:
    """N-D FFT along the given dimensions (default all) (trnfft/api.py:111-137)."""
    return _fftn(input, s, dim, inverse=False)


def ifftn(
    input: torch.Tensor | ComplexTensor,
    s: tuple[int, ...] | None = None,
    dim: tuple[int, ...] | None = None,
) -> ComplexTensor:
    """N-D inverse FFT along the given dimensions (trnfft/api.py:140-167)."""
    return _fftn(input, s, dim, inverse=True)


def _fftn(input, s, dim, inverse):
    x = _to_complex(input)
    ndim = len(x.shape)
    dim = _norm_dims(ndim, s, dim)
    if s is not None:
        if len(s) != len(dim):
            raise AssertionError(f"len(s)={len(s)} must match len(dim)={len(dim)}")
        for size, d in zip(s, dim, strict=True):
            x = _resize_dim(x, d, size)
    for d in dim:
        x = _fft_along_dim(x, d, inverse=inverse)
    return x


def rfft2(input: torch.Tensor, s: tuple[int, int] | None = None) -> ComplexTensor:
    """2-D FFT of a real signal (trnfft/api.py:170-179)."""
    return rfftn(input, s=tuple(s) if s is not None else None, dim=(-2, -1))


def rfftn(
    input: torch.Tensor,
    s: tuple[int, ...] | None = None,
    dim: tuple[int, ...] | None = None,
) -> ComplexTensor:
    """N-D FFT of a real signal; one-sided along the last of ``dim`` (trnfft/api.py:182-225)."""
    if torch.is_complex(input):
        raise AssertionError("rfftn requires real input")
    ndim = input.dim()
    dim = _norm_dims(ndim, s, dim)
    last_dim, other_dims = dim[-1], dim[:-1]
    n_last = s[-1] if s is not None else None
    if last_dim == ndim - 1:
        x = rfft(input, n=n_last)
    else:
        x = rfft(input.transpose(last_dim, -1).contiguous(), n=n_last)
        x = x.transpose(last_dim, -1)
    if s is not None:
        for size, d in zip(s[:-1], other_dims, strict=True):
            x = _resize_dim(x, d, size)
    for d in other_dims:
        x = _fft_along_dim(x, d, inverse=False)
    return x


def irfft2(input: ComplexTensor, s: tuple[int, int] | None = None) -> torch.Tensor:
    """Inverse of rfft2 (trnfft/api.py:228-241)."""
    return irfftn(input, s=tuple(s) if s is not None else None, dim=(-2, -1))


def irfftn(
    input: ComplexTensor,
    s: tuple[int, ...] | None = None,
    dim: tuple[int, ...] | None = None,
) -> torch.Tensor:
    """Inverse of rfftn (trnfft/api.py:244-288)."""
    ndim = input.real.dim()
    dim = _norm_dims(ndim, s, dim)
    last_dim, other_dims = dim[-1], dim[:-1]
    x = input
    if s is not None:
        for size, d in zip(s[:-1], other_dims, strict=True):
            x = _resize_dim(x, d, size)
        n_last = s[-1]
    else:
        n_last = 2 * (x.shape[last_dim] - 1)
    for d in other_dims:
        x = _fft_along_dim(x, d, inverse=True)
    if last_dim == ndim - 1:
        return irfft(x, n=n_last)
    x_t = ComplexTensor(
        x.real.transpose(last_dim, -1).contiguous(), x.imag.transpose(last_dim, -1).contiguous()
    )
    return irfft(x_t, n=n_last).transpose(last_dim, -1).contiguous()


def _full_window(window, n_fft, win_length, device):
    """Window zero-padded to n_fft and centred (trnfft/api.py:329-334)."""
    w = window.to(device=device, dtype=torch.float32)
    if win_length < n_fft:
        pw = torch.zeros(n_fft, dtype=torch.float32, device=device)
        off = (n_fft - win_length) // 2
        pw[off : off + win_length] = w
        w = pw
    return w.contiguous()


def stft(
    input: torch.Tensor,
    n_fft: int,
    hop_length: int | None = None,
    win_length: int | None = None,
    window: torch.Tensor | None = None,
    center: bool = True,
    pad_mode: str = "reflect",
    normalized: bool = False,
    onesided: bool = True,
) -> ComplexTensor:
    """Short-time Fourier transform, output (..., freq, time) (trnfft/api.py:291-365)."""
    if hop_length is None:
        hop_length = n_fft // 4
    if win_length is None:
        win_length = n_fft
    if window is None:
        window = torch.hann_window(win_length, dtype=input.dtype)
    (x,), restore = place(input)
    w = _full_window(window, n_fft, win_length, x.device)
    yr, yi = _ops.stft(x, n_fft, hop_length, w, center, pad_mode, normalized, onesided)
    return ComplexTensor(restore(yr), restore(yi))


def istft(
    input: ComplexTensor,
    n_fft: int,
    hop_length: int | None = None,
    win_length: int | None = None,
    window: torch.Tensor | None = None,
    center: bool = True,
    normalized: bool = False,
    onesided: bool = True,
    length: int | None = None,
) -> torch.Tensor:
    """Inverse STFT by windowed overlap-add (trnfft/api.py:368-470)."""
    if hop_length is None:
        hop_length = n_fft // 4
    if win_length is None:
        win_length = n_fft
    if window is None:
        window = torch.hann_window(win_length, dtype=input.dtype)
    (sr, si), restore = place(input.real, input.imag)
    w = _full_window(window, n_fft, win_length, sr.device)
    y = _ops.istft(sr, si, n_fft, hop_length, w, center, normalized, onesided, length)
    return restore(y)


# --- Helpers (trnfft/api.py:476-538) ---


def _to_complex(x) -> ComplexTensor:
    if isinstance(x, ComplexTensor):
        return x
    return ComplexTensor(x)


def _resize_last(x: ComplexTensor, n: int) -> ComplexTensor:
    current = x.shape[-1]
    if current == n:
        return x
    if current < n:
        pad = torch.zeros(*x.shape[:-1], n - current, dtype=x.dtype, device=x.device)
        return ComplexTensor(torch.cat([x.real, pad], dim=-1), torch.cat([x.imag, pad], dim=-1))
    return ComplexTensor(x.real[..., :n], x.imag[..., :n])


def _fft_along_dim(x: ComplexTensor, dim: int, inverse: bool) -> ComplexTensor:
    """1-D transform along one dimension of an N-D tensor.

    Power-of-two lengths run the strided-axis kernel in place of the
    reference's transpose/copy/transform/transpose (trnfft/api.py:496-516).
    """
    ndim = len(x.shape)
    dim = dim % ndim
    if dim == ndim - 1:
        return fft_core(x, inverse=inverse)
    n = x.shape[dim]
    from .precision import get_precision

    f64 = x.real.dtype == torch.float64 or get_precision() == "double"
    if n > 1 and _ops.axis_supported(n) and not f64:  # the strided-axis kernels are float32
        (xr, xi), restore = place(x.real, x.imag)
        yr, yi = _ops.c2c_axis(xr, xi, dim, bool(inverse))
        return ComplexTensor(restore(yr), restore(yi))
    xr = x.real.movedim(dim, -1)
    xi = x.imag.movedim(dim, -1)
    y = fft_core(ComplexTensor(xr, xi), inverse=inverse)
    return ComplexTensor(y.real.movedim(-1, dim), y.imag.movedim(-1, dim))


def _resize_dim(x: ComplexTensor, dim: int, n: int) -> ComplexTensor:
    ndim = len(x.shape)
    dim = dim % ndim
    if dim != ndim - 1:
        x = x.transpose(dim, -1)
    x = _resize_last(x, n)
    if dim != ndim - 1:
        x = x.transpose(dim, -1)
    return x


def _resize_real(x: torch.Tensor, n: int) -> torch.Tensor:
    current = x.shape[-1]
    if current == n:
        return x
    if current < n:
        pad = torch.zeros(*x.shape[:-1], n - current, dtype=x.dtype, device=x.device)
        return torch.cat([x, pad], dim=-1)
    return x[..., :n]

