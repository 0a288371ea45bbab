"""Device-side transform primitives over the C ABI, with autograd.

Every function here takes CUDA float32 tensors whose last axis is the
transform axis, launches one of the library's kernels on the current torch
stream and returns new tensors (outputs are allocated with ``torch.empty`` on
the input's device, so the caching allocator owns them).

Autograd follows the reference's analytic adjoints
(trnfft/nki/autograd.py:167-205): for y = fft(x), dx = n * ifft(dy); for
y = ifft(x), dx = fft(dy) / n.  The real transforms use the matching
adjoints (derived in each backward).
"""

from __future__ import annotations

import torch

from . import _lib


def _flat(t: torch.Tensor, n: int) -> torch.Tensor:
    t = t.contiguous()
    return t.reshape(-1, n)


def _check(t: torch.Tensor, what: str, f64_ok: bool = False) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"trnfft_b200: {what} must be a CUDA tensor")
    if t.dtype != torch.float32 and not (f64_ok and t.dtype == torch.float64):
        raise TypeError(f"trnfft_b200: {what} must be float32, got {t.dtype}")


# ---------------------------------------------------------------------------
# double precision (precision="double", or float64 tensors)
# ---------------------------------------------------------------------------


def _f64_wanted(t: torch.Tensor, precision=None) -> bool:
    """fp64 kernels run for float64 tensors and, in precision="double", for float32 ones
    (every size: the reference promotes Bluestein to float64 and runs power-of-two sizes up
    to 1024 as an fp64 DFT, trnfft/fft_core.py:1108-1110, 1306-1309)."""
    from .precision import _resolve

    return t.dtype == torch.float64 or _resolve(precision) == "double"


def c2c_f64_raw(xr: torch.Tensor, xi: torch.Tensor, inverse: bool):
    """Transform along the last axis with every stage in fp64 (trnfft_exec_c2c_f64).
    float32 inputs stay float32 in memory: trnfft_exec_c2c_f64_f32io widens them in the first
    kernel's loads and narrows the result in the last kernel's stores."""
    _check(xr, "real part", True)
    _check(xi, "imaginary part", True)
    n = xr.shape[-1]
    shape, odt = xr.shape, xr.dtype
    a = _flat(xr, n)
    b = _flat(xi.to(odt), n)
    if odt not in (torch.float32, torch.float64):
        a, b = a.float(), b.float()
    batch = a.shape[0]
    yr = torch.empty_like(a)
    yi = torch.empty_like(b)
    if batch and n:
        plan = _lib.device_plan(n, a.device)
        plan.enable_f64()
        wb = plan.work_bytes_f64(batch)
        work = torch.empty(wb, dtype=torch.uint8, device=a.device) if wb else None
        entry = "trnfft_exec_c2c_f64" if a.dtype == torch.float64 else "trnfft_exec_c2c_f64_f32io"
        _lib.call(entry, plan.handle, _lib.ptr(a), _lib.ptr(b), _lib.ptr(yr), _lib.ptr(yi), batch,
                  int(bool(inverse)), _lib.ptr(work), _lib.stream_ptr(a.device))
    if yr.dtype != odt:
        yr, yi = yr.to(odt), yi.to(odt)
    return yr.reshape(shape), yi.reshape(shape)


# ---------------------------------------------------------------------------
# raw launches (no autograd)
# ---------------------------------------------------------------------------


_dft_cache: dict = {}


def _dft_matrix(n: int, inverse: bool, device: torch.device):
    """n x n DFT matrix exp(-+2 pi i j k / n) (/n for the inverse), float32 planes, cached."""
    key = (n, inverse, device)
    m = _dft_cache.get(key)
    if m is None:
        j = torch.arange(n, dtype=torch.int64)
        e = (j[:, None] * j[None, :]) % n
        ang = (2.0 * torch.pi / n) * e.to(torch.float64) * (1.0 if inverse else -1.0)
        sc = (1.0 / n) if inverse else 1.0
        m = ((torch.cos(ang) * sc).float().to(device).contiguous(), (torch.sin(ang) * sc).float().to(device).contiguous())
        _dft_cache[key] = m
    return m


def dft_gemm_raw(xr: torch.Tensor, xi: torch.Tensor, inverse: bool):
    """Power-of-two n <= 256 as X = x F on the tcgen05 3xTF32 GEMM (F symmetric, so W = F)."""
    from . import _gemm

    n = xr.shape[-1]
    shape = xr.shape
    fr, fi = _dft_matrix(n, inverse, xr.device)
    yr, yi = _gemm.linear_raw(xr.reshape(-1, n), xi.reshape(-1, n), fr, fi)
    return yr.reshape(shape), yi.reshape(shape)


def c2c_raw(xr: torch.Tensor, xi: torch.Tensor, inverse: bool, precision=None) -> tuple[torch.Tensor, torch.Tensor]:
    if _f64_wanted(xr, precision):
        return c2c_f64_raw(xr, xi, inverse)
    _check(xr, "real part")
    _check(xi, "imaginary part")
    n = xr.shape[-1]
    from .plan import DFT_GEMM_MAX_N, get_small_n_algorithm

    if get_small_n_algorithm() == "gemm" and 4 <= n <= DFT_GEMM_MAX_N and (n & (n - 1)) == 0:
        return dft_gemm_raw(xr, xi, inverse)
    shape = xr.shape
    a = _flat(xr, n)
    b = _flat(xi, n)
    yr = torch.empty_like(a)
    yi = torch.empty_like(b)
    batch = a.shape[0]
    if batch and n:
        plan = _lib.device_plan(n, a.device)
        # out-of-place calls need a work area only for multi-pass Bluestein (m > 16384)
        work = None
        if plan.algorithm == _lib.ALG_BLUESTEIN and plan.padded_n > 16384:
            work = torch.empty(plan.work_bytes(batch), dtype=torch.uint8, device=a.device)
        _lib.call("trnfft_exec_c2c", plan.handle, _lib.ptr(a), _lib.ptr(b), _lib.ptr(yr), _lib.ptr(yi),
                  batch, int(bool(inverse)), _lib.ptr(work), _lib.stream_ptr(a.device))
    return yr.reshape(shape), yi.reshape(shape)


def axis_supported(n: int) -> bool:
    """Power-of-two lengths the strided-axis kernels handle (up to 2^20)."""
    return n >= 1 and (n & (n - 1)) == 0 and n <= (1 << 20)


def c2c_axis_raw(xr: torch.Tensor, xi: torch.Tensor, dim: int, inverse: bool):
    """Transform along axis `dim` of contiguous tensors without moving it last."""
    _check(xr, "real part")
    _check(xi, "imaginary part")
    shape = xr.shape
    n = shape[dim]
    outer = 1
    for s_ in shape[:dim]:
        outer *= s_
    inner = 1
    for s_ in shape[dim + 1:]:
        inner *= s_
    a = xr.contiguous()
    b = xi.contiguous()
    yr = torch.empty_like(a)
    yi = torch.empty_like(b)
    if a.numel():
        plan = _lib.device_plan(n, a.device)
        _lib.call("trnfft_exec_c2c_axis", plan.handle, _lib.ptr(a), _lib.ptr(b), _lib.ptr(yr), _lib.ptr(yi),
                  outer, inner, int(bool(inverse)), None, _lib.stream_ptr(a.device))
    return yr, yi


class _C2CAxis(torch.autograd.Function):
    @staticmethod
    def forward(ctx, xr, xi, dim: int, inverse: bool):
        ctx.dim, ctx.inverse, ctx.n = dim, inverse, xr.shape[dim]
        return c2c_axis_raw(xr, xi, dim, inverse)

    @staticmethod
    def backward(ctx, gr, gi):
        dr, di = c2c_axis_raw(gr.contiguous(), gi.contiguous(), ctx.dim, not ctx.inverse)
        s = (1.0 / ctx.n) if ctx.inverse else float(ctx.n)
        return dr * s, di * s, None, None


def c2c_axis(xr, xi, dim: int, inverse: bool):
    if torch.is_grad_enabled() and (xr.requires_grad or xi.requires_grad):
        return _C2CAxis.apply(xr, xi, dim, inverse)
    return c2c_axis_raw(xr, xi, dim, inverse)


def _r2c_native(n: int) -> bool:
    return n >= 4 and (n & (n - 1)) == 0 and n <= 8192


def _real_kernel(n: int, device: torch.device) -> bool:
    """Whether trnfft_exec_r2c / _c2r have a direct kernel for n on this device:
    powers of two 4..8192 (packed real rows), 7-smooth lengths up to 8192 (the
    mixed-radix kernel's real modes) and Bluestein lengths whose padded size m
    fits one block (m <= 16384, the fused kernel's real-input modes)."""
    if _r2c_native(n):
        return True
    if n < 3 or (n & (n - 1)) == 0:
        return False
    plan = _lib.device_plan(n, device)
    if plan.algorithm == _lib.ALG_MIXED:
        return True
    return plan.algorithm == _lib.ALG_BLUESTEIN and plan.padded_n <= 16384


def r2c_raw(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """rfft along the last axis: (..., n) real -> (..., n//2+1) complex."""
    n = x.shape[-1]
    h = n // 2 + 1
    lead = x.shape[:-1]
    if _f64_wanted(x):  # a complex fp64 transform of the real row, as the reference does (api.py:38-46)
        yr, yi = c2c_f64_raw(x, torch.zeros_like(x), False)
        return yr[..., :h].contiguous(), yi[..., :h].contiguous()
    _check(x, "input")
    a = _flat(x, n)
    batch = a.shape[0]
    if not _real_kernel(n, a.device):
        yr, yi = c2c_raw(a, torch.zeros_like(a), False)
        return yr[:, :h].reshape(*lead, h), yi[:, :h].reshape(*lead, h)
    if _r2c_native(n) and a.data_ptr() % 8:
        a = a.clone()
    yr = torch.empty(batch, h, dtype=torch.float32, device=a.device)
    yi = torch.empty(batch, h, dtype=torch.float32, device=a.device)
    if batch:
        plan = _lib.device_plan(n, a.device)
        _lib.call("trnfft_exec_r2c", plan.handle, _lib.ptr(a), _lib.ptr(yr), _lib.ptr(yi), batch,
                  None, _lib.stream_ptr(a.device))
    return yr.reshape(*lead, h), yi.reshape(*lead, h)


def hermitian_extend(xr: torch.Tensor, xi: torch.Tensor, n: int):
    """Full length-n spectrum built the way trnfft.irfft does (trnfft/api.py:54-66)."""
    half = xr.shape[-1]
    num_neg = n - half
    if num_neg > max(half - 1, 0):
        # the reference's slice assignment fails here (trnfft/api.py:64-65)
        raise RuntimeError(
            f"irfft: cannot rebuild a length-{n} spectrum from {half} bins "
            f"(needs at least {n // 2 + 1})"
        )
    fr = torch.zeros(*xr.shape[:-1], n, dtype=xr.dtype, device=xr.device)
    fi = torch.zeros_like(fr)
    keep = min(half, n)
    fr[..., :keep] = xr[..., :keep]
    fi[..., :keep] = xi[..., :keep]
    if n > 1 and num_neg > 0:
        fr[..., half:] = torch.flip(xr[..., 1 : 1 + num_neg], dims=[-1])
        fi[..., half:] = -torch.flip(xi[..., 1 : 1 + num_neg], dims=[-1])
    return fr, fi


def c2r_raw(xr: torch.Tensor, xi: torch.Tensor, n: int) -> torch.Tensor:
    """irfft along the last axis: (..., h) complex -> (..., n) real."""
    if _f64_wanted(xr):
        fr, fi = hermitian_extend(xr, xi, n)
        yr, _ = c2c_f64_raw(fr, fi, True)
        return yr
    _check(xr, "real part")
    _check(xi, "imaginary part")
    h = xr.shape[-1]
    lead = xr.shape[:-1]
    if h == n // 2 + 1 and _real_kernel(n, xr.device):
        a = _flat(xr, h)
        b = _flat(xi, h)
        batch = a.shape[0]
        y = torch.empty(batch, n, dtype=torch.float32, device=a.device)
        if batch:
            plan = _lib.device_plan(n, a.device)
            _lib.call("trnfft_exec_c2r", plan.handle, _lib.ptr(a), _lib.ptr(b), _lib.ptr(y), batch,
                      None, _lib.stream_ptr(a.device))
        return y.reshape(*lead, n)
    fr, fi = hermitian_extend(xr, xi, n)
    yr, _ = c2c_raw(fr, fi, True)
    return yr


# ---------------------------------------------------------------------------
# autograd
# ---------------------------------------------------------------------------


class _C2C(torch.autograd.Function):
    @staticmethod
    def forward(ctx, xr, xi, inverse: bool, precision=None):
        ctx.inverse = inverse
        ctx.n = xr.shape[-1]
        ctx.precision = precision
        return c2c_raw(xr, xi, inverse, precision)

    @staticmethod
    def backward(ctx, gr, gi):
        n = ctx.n
        gr = torch.zeros_like(gr) if gr is None else gr
        gi = torch.zeros_like(gi) if gi is None else gi
        if ctx.inverse:
            dr, di = c2c_raw(gr, gi, False, ctx.precision)
            s = 1.0 / n
        else:
            dr, di = c2c_raw(gr, gi, True, ctx.precision)
            s = float(n)
        return dr * s, di * s, None, None


class _R2C(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        ctx.n = x.shape[-1]
        return r2c_raw(x)

    @staticmethod
    def backward(ctx, gr, gi):
        # y_k = sum_t x_t e^{-2 pi i k t/n} for k <= n//2, so
        # dx_t = Re sum_k (gr_k + i gi_k) e^{+2 pi i k t/n} = n * c2r(G') where
        # G'_k = G_k / 2 except at k = 0 and 2k = n (c2r counts interior bins twice).
        n = ctx.n
        gr = gr.clone()
        gi = gi.clone()
        h = gr.shape[-1]
        hi = h - 1 if n % 2 == 0 else h
        gr[..., 1:hi] *= 0.5
        gi[..., 1:hi] *= 0.5
        return c2r_raw(gr.contiguous(), gi.contiguous(), n) * float(n)


class _C2R(torch.autograd.Function):
    @staticmethod
    def forward(ctx, xr, xi, n: int):
        ctx.n = n
        ctx.h = xr.shape[-1]
        return c2r_raw(xr, xi, n)

    @staticmethod
    def backward(ctx, gy):
        # y_t = (1/n)[Re X_0 + 2 sum_{0<k<n/2} Re(X_k e^{+i theta}) + Re X_{n/2} (-1)^t],
        # so dX_k = c_k / n * rfft(dy)_k with c_k = 1 at k = 0 and 2k = n, else 2.
        n, h = ctx.n, ctx.h
        r, i = r2c_raw(gy.contiguous())
        hb = r.shape[-1]
        c = torch.full((hb,), 2.0 / n, dtype=r.dtype, device=r.device)
        c[0] = 1.0 / n
        if n % 2 == 0:
            c[-1] = 1.0 / n
        dr, di = r * c, i * c
        di[..., 0] = 0.0
        if n % 2 == 0:
            di[..., -1] = 0.0
        return dr, di, None


def _needs_grad(*ts) -> bool:
    return torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in ts)


def c2c(xr, xi, inverse: bool, precision=None):
    if _needs_grad(xr, xi):
        return _C2C.apply(xr, xi, inverse, precision)
    return c2c_raw(xr, xi, inverse, precision)


def r2c(x):
    if _needs_grad(x):
        n = x.shape[-1]
        if x.is_cuda and not _f64_wanted(x) and _real_kernel(n, x.device):
            return _R2C.apply(x)
        h = n // 2 + 1
        yr, yi = _C2C.apply(x, torch.zeros_like(x), False)
        return yr[..., :h], yi[..., :h]
    return r2c_raw(x)


def c2r(xr, xi, n: int):
    if _needs_grad(xr, xi):
        if xr.is_cuda and not _f64_wanted(xr) and xr.shape[-1] == n // 2 + 1 and _real_kernel(n, xr.device):
            return _C2R.apply(xr, xi, n)
        fr, fi = hermitian_extend(xr, xi, n)
        yr, _ = _C2C.apply(fr, fi, True)
        return yr
    return c2r_raw(xr, xi, n)


# ---------------------------------------------------------------------------
# STFT / ISTFT
# ---------------------------------------------------------------------------


def _pad_signal(x2: torch.Tensor, p: int, pad_mode: str) -> torch.Tensor:
    return torch.nn.functional.pad(x2.unsqueeze(1), (p, p), mode=pad_mode).squeeze(1)


_PAD_MODES = {"reflect": 0, "constant": 1, "replicate": 2, "circular": 3}


def _stft_composite(x, n_fft, hop, w, center, pad_mode, normalized, onesided):
    """Framing with torch ops + the library transforms; used for autograd and for
    n_fft the fused kernel does not cover."""
    lead = x.shape[:-1]
    L = x.shape[-1]
    x2 = x.reshape(-1, L)
    if center:
        x2 = _pad_signal(x2, n_fft // 2, pad_mode)
    frames = x2.unfold(-1, n_fft, hop) * w
    if onesided:
        yr, yi = r2c(frames)
    else:
        yr, yi = c2c(frames, torch.zeros_like(frames), False)
    yr = yr.transpose(-2, -1)
    yi = yi.transpose(-2, -1)
    if normalized:
        sc = 1.0 / (n_fft ** 0.5)
        yr = yr * sc
        yi = yi * sc
    nb, nf = yr.shape[-2], yr.shape[-1]
    return yr.reshape(*lead, nb, nf).contiguous(), yi.reshape(*lead, nb, nf).contiguous()


def stft(x: torch.Tensor, n_fft: int, hop: int, w: torch.Tensor, center: bool, pad_mode: str,
         normalized: bool, onesided: bool):
    """STFT with output (..., freq, time) (trnfft/api.py:291-365)."""
    _check(x, "input")
    fused = (n_fft >= 4 and (n_fft & (n_fft - 1)) == 0 and n_fft <= 8192 and pad_mode in _PAD_MODES
             and not _needs_grad(x, w))
    if not fused:
        return _stft_composite(x, n_fft, hop, w, center, pad_mode, normalized, onesided)
    lead = x.shape[:-1]
    L = x.shape[-1]
    a = x.reshape(-1, L).contiguous()
    B = a.shape[0]
    pad = n_fft // 2 if center else 0
    if center and pad_mode == "reflect" and pad >= L:
        raise RuntimeError(f"stft: reflect padding {pad} must be smaller than the signal length {L}")
    lp = L + 2 * pad
    if lp < n_fft:
        raise RuntimeError(f"stft: signal of {L} samples is shorter than n_fft={n_fft}")
    nf = 1 + (lp - n_fft) // hop
    nb = n_fft // 2 + 1 if onesided else n_fft
    yr = torch.empty(B, nb, nf, dtype=torch.float32, device=a.device)
    yi = torch.empty_like(yr)
    if B:
        plan = _lib.device_plan(n_fft, a.device)
        _lib.call("trnfft_exec_stft", plan.handle, _lib.ptr(a), B, L, hop, _lib.ptr(w.contiguous()),
                  int(bool(center)), _PAD_MODES[pad_mode], int(bool(normalized)), int(bool(onesided)), nf,
                  _lib.ptr(yr), _lib.ptr(yi), _lib.stream_ptr(a.device))
    return yr.reshape(*lead, nb, nf), yi.reshape(*lead, nb, nf)


def istft_out_len(n_fft: int, frames: int, hop: int, center: bool, length) -> int:
    """Samples istft returns (trnfft/api.py:454-468): overlap-add length, minus the centre
    padding (the tail padding only when `length` is None), or `length` itself."""
    exp_len = n_fft + (frames - 1) * hop
    cur = exp_len
    if center:
        p = n_fft // 2
        cur = exp_len - p
        if cur > p and length is None:
            cur -= p
    return cur if length is None else int(length)


def istft(sr: torch.Tensor, si: torch.Tensor, n_fft: int, hop: int, w: torch.Tensor, center: bool,
          normalized: bool, onesided: bool, length):
    """Inverse transform per frame and windowed overlap-add (trnfft/api.py:368-470).

    Power-of-two n_fft up to 8192 without autograd runs the fused kernel
    (trnfft_exec_istft); other cases compose the library's inverse transforms with a
    device overlap-add."""
    fused = (4 <= n_fft <= 8192 and (n_fft & (n_fft - 1)) == 0 and 1 <= hop <= 8192
             and not _needs_grad(sr, si, w) and sr.dtype == torch.float32
             and sr.shape[-2] == (n_fft // 2 + 1 if onesided else n_fft))
    if not fused:
        return _istft_composite(sr, si, n_fft, hop, w, center, normalized, onesided, length)
    _check(sr, "real part")
    _check(si, "imaginary part")
    lead = sr.shape[:-2]
    fb, nf = sr.shape[-2], sr.shape[-1]
    a = sr.reshape(-1, fb, nf).contiguous()
    b = si.reshape(-1, fb, nf).contiguous()
    B = a.shape[0]
    out_len = istft_out_len(n_fft, nf, hop, center, length)
    y = torch.empty(B, out_len, dtype=torch.float32, device=a.device)
    if B and out_len:
        plan = _lib.device_plan(n_fft, a.device)
        _lib.call("trnfft_exec_istft", plan.handle, _lib.ptr(a), _lib.ptr(b), B, nf, hop,
                  _lib.ptr(w.contiguous()), int(bool(center)), int(bool(normalized)), int(bool(onesided)),
                  out_len, _lib.ptr(y), _lib.stream_ptr(a.device))
    return y.reshape(*lead, out_len)


def _istft_composite(sr, si, n_fft, hop, w, center, normalized, onesided, length):
    """istft from the library's inverse transforms plus a torch overlap-add (autograd, other n_fft)."""
    if normalized:
        sc = n_fft ** 0.5
        sr = sr * sc
        si = si * sc
    lead = sr.shape[:-2]
    fb, nf = sr.shape[-2], sr.shape[-1]
    tr = sr.reshape(-1, fb, nf).transpose(-2, -1).contiguous()
    ti = si.reshape(-1, fb, nf).transpose(-2, -1).contiguous()
    if onesided:
        frames = c2r(tr, ti, n_fft)
    else:
        frames, _ = c2c(tr, ti, True)
    B = frames.shape[0]
    exp_len = n_fft + (nf - 1) * hop

    def ola(fr):  # (B, nf, n_fft) -> (B, exp_len)
        return torch.nn.functional.fold(
            fr.transpose(1, 2), output_size=(1, exp_len), kernel_size=(1, n_fft), stride=(1, hop)
        ).reshape(fr.shape[0], exp_len)

    out = ola(frames * w)
    raw = ola(frames)
    wsum = ola((w * w).expand(1, nf, n_fft).contiguous())[0]
    mask = wsum > 1e-8
    out = torch.where(mask, out / torch.where(mask, wsum, torch.ones_like(wsum)), raw)
    if center:
        p = n_fft // 2
        out = out[..., p:]
        if out.shape[-1] > p:
            out = out[..., :-p] if length is None else out
    if length is not None:
        cur = out.shape[-1]
        if cur > length:
            out = out[..., :length]
        elif cur < length:
            out = torch.cat([out, torch.zeros(B, length - cur, dtype=out.dtype, device=out.device)], -1)
    return out.reshape(*lead, out.shape[-1]).contiguous()
