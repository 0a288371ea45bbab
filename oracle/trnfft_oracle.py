"""CPU oracle for the trnfft FFT hot path -- TEST INFRASTRUCTURE ONLY.

This module restates, in NumPy, the algorithms that the reference library
trnsci/trnfft runs on its ``"pytorch"`` backend.  It is the checker for the
CUDA implementation in ``trnfft_b200`` and the CPU baseline timed by
``bench.py``; the product never imports it.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and
``--impl reference``) may use it.

Parity pin: every public function here is checked against golden vectors
produced by importing the reference itself (``tests/golden/make_golden.py``
writes ``tests/golden/*.npz``; ``tests/test_oracle_golden.py`` checks them),
and against the reference's own known-answer tests (impulse, constant, single
cosine, zero padding, (1+2i)(3+4i)).

Each function cites the reference file:line whose arithmetic it follows.
Arithmetic is float32 wherever the reference computes in float32, and the
order of operations inside a butterfly is the reference's, so results agree
with the reference to within a few float32 ulps (``cos``/``sin`` of float32
arguments may differ by one ulp between NumPy and torch).
"""

from __future__ import annotations

import math
from concurrent.futures import ThreadPoolExecutor

import numpy as np

F32 = np.float32


# ---------------------------------------------------------------------------
# power-of-2 radix-2 Cooley-Tukey (trnfft/fft_core.py:53-117)
# ---------------------------------------------------------------------------


def bit_reverse_indices(n: int, bits: int) -> np.ndarray:
    """Bit-reversal permutation (trnfft/fft_core.py:1379-1389), vectorised."""
    idx = np.arange(n, dtype=np.int64)
    rev = np.zeros(n, dtype=np.int64)
    for _ in range(bits):
        rev = (rev << 1) | (idx & 1)
        idx >>= 1
    return rev


def cooley_tukey(re: np.ndarray, im: np.ndarray, inverse: bool):
    """Iterative radix-2 DIT along the last axis (trnfft/fft_core.py:53-117).

    Stage s uses group size m = 2^(s+1), twiddles exp(sign*2*pi*i*k/m)
    computed in float32 from a float32 ``arange`` (fft_core.py:86-88), the
    butterfly ``e +/- t*o`` (fft_core.py:99-112), and a final multiply by
    float32(1/n) for the inverse (fft_core.py:114-116).  The reference loops
    over the butterfly position k in Python; here all k of a stage run at once
    with identical per-element arithmetic.
    """
    re = np.asarray(re, dtype=F32)
    im = np.asarray(im, dtype=F32)
    n = re.shape[-1]
    log2n = int(math.log2(n))
    assert 1 << log2n == n, f"Not power of 2: {n}"
    sign = 1.0 if inverse else -1.0
    idx = bit_reverse_indices(n, log2n)
    re = re[..., idx].copy()
    im = im[..., idx].copy()
    lead = re.shape[:-1]
    for s in range(log2n):
        m = 1 << (s + 1)
        half = m >> 1
        ang = (np.arange(half, dtype=F32) * F32(sign * 2.0 * math.pi)) / F32(m)
        tw_re = np.cos(ang).astype(F32)
        tw_im = np.sin(ang).astype(F32)
        r = re.reshape(*lead, n // m, m)
        i = im.reshape(*lead, n // m, m)
        e_re = r[..., :half].copy()
        e_im = i[..., :half].copy()
        o_re = r[..., half:]
        o_im = i[..., half:]
        prod_re = tw_re * o_re - tw_im * o_im
        prod_im = tw_re * o_im + tw_im * o_re
        r[..., :half] = e_re + prod_re
        i[..., :half] = e_im + prod_im
        r[..., half:] = e_re - prod_re
        i[..., half:] = e_im - prod_im
    if inverse:
        s = F32(1.0 / n)
        re = re * s
        im = im * s
    return re.astype(F32), im.astype(F32)


# ---------------------------------------------------------------------------
# plan selection (trnfft/plan.py:34-46) and Bluestein (fft_core.py:1285-1376)
# ---------------------------------------------------------------------------


def padded_length(n: int) -> int:
    """Bluestein padded length m = 2^bitlen(2n-2) (trnfft/plan.py:41-43)."""
    return 1 << (2 * n - 2).bit_length()


def bluestein(re, im, inverse: bool, precision: str = "fast"):
    """Bluestein chirp-z (trnfft/fft_core.py:1285-1376).

    ``precision="fast"`` keeps the reference's float32 chirp angle
    ``sign*pi*k*k/n`` (fft_core.py:1316-1320), whose rounding limits it to
    ~1e-4 relative error at n ~ 4000.  ``"double"`` promotes the whole chain to
    float64 (fft_core.py:1306-1309, 1372-1374); the reference runs its radix-2
    FFT in float64 then, and so does this restatement.
    """
    dt = np.float64 if precision == "double" else F32
    re = np.asarray(re).astype(dt)
    im = np.asarray(im).astype(dt)
    n = re.shape[-1]
    m = padded_length(n)
    sign = 1.0 if inverse else -1.0
    k = np.arange(n, dtype=dt)
    ang = ((dt(sign * math.pi) * k) * k) / dt(n)
    c_re = np.cos(ang).astype(dt)
    c_im = np.sin(ang).astype(dt)
    y_re = re * c_re - im * c_im
    y_im = re * c_im + im * c_re
    lead = re.shape[:-1]
    yp_re = np.zeros((*lead, m), dtype=dt)
    yp_im = np.zeros((*lead, m), dtype=dt)
    yp_re[..., :n] = y_re
    yp_im[..., :n] = y_im
    h_re = np.zeros(m, dtype=dt)
    h_im = np.zeros(m, dtype=dt)
    h_re[:n] = c_re
    h_im[:n] = -c_im
    if n > 1:
        h_re[m - np.arange(1, n)] = c_re[1:]
        h_im[m - np.arange(1, n)] = -c_im[1:]
    fft = _ct64 if dt is np.float64 else cooley_tukey
    Y_re, Y_im = fft(yp_re, yp_im, False)
    H_re, H_im = fft(h_re[None], h_im[None], False)
    p_re = Y_re * H_re - Y_im * H_im
    p_im = Y_re * H_im + Y_im * H_re
    cv_re, cv_im = fft(p_re, p_im, True)
    r_re = cv_re[..., :n]
    r_im = cv_im[..., :n]
    o_re = r_re * c_re - r_im * c_im
    o_im = r_re * c_im + r_im * c_re
    if inverse:
        s = dt(1.0 / n)
        o_re = o_re * s
        o_im = o_im * s
    return o_re.astype(F32), o_im.astype(F32)


def _ct64(re, im, inverse):
    """Float64 twin of :func:`cooley_tukey` (used by ``precision="double"``)."""
    re = np.asarray(re, dtype=np.float64)
    im = np.asarray(im, dtype=np.float64)
    n = re.shape[-1]
    log2n = int(math.log2(n))
    sign = 1.0 if inverse else -1.0
    idx = bit_reverse_indices(n, log2n)
    re = re[..., idx].copy()
    im = im[..., idx].copy()
    lead = re.shape[:-1]
    for s in range(log2n):
        m = 1 << (s + 1)
        half = m >> 1
        ang = sign * 2.0 * math.pi * np.arange(half, dtype=np.float64) / m
        tw_re, tw_im = np.cos(ang), np.sin(ang)
        r = re.reshape(*lead, n // m, m)
        i = im.reshape(*lead, n // m, m)
        e_re = r[..., :half].copy()
        e_im = i[..., :half].copy()
        o_re = r[..., half:]
        o_im = i[..., half:]
        pr = tw_re * o_re - tw_im * o_im
        pi_ = tw_re * o_im + tw_im * o_re
        r[..., :half] = e_re + pr
        i[..., :half] = e_im + pi_
        r[..., half:] = e_re - pr
        i[..., half:] = e_im - pi_
    if inverse:
        re = re / n
        im = im / n
    return re, im


def fft_core(re, im, inverse: bool = False, precision: str = "fast"):
    """Algorithm selection (trnfft/fft_core.py:22-50, plan.py:34-46)."""
    re = np.asarray(re, dtype=F32)
    im = np.asarray(im, dtype=F32)
    n = re.shape[-1]
    if n == 1:
        return re.copy(), im.copy()
    if n & (n - 1) == 0:
        return cooley_tukey(re, im, inverse)
    return bluestein(re, im, inverse, precision)


# ---------------------------------------------------------------------------
# public API restatements (trnfft/api.py)
# ---------------------------------------------------------------------------


def _resize_last(re, im, n):
    """trnfft/api.py:482-493: zero-pad or truncate the last axis."""
    cur = re.shape[-1]
    if cur == n:
        return re, im
    if cur < n:
        pad = [(0, 0)] * (re.ndim - 1) + [(0, n - cur)]
        return np.pad(re, pad), np.pad(im, pad)
    return re[..., :n], im[..., :n]


def fft(re, im=None, n=None, precision="fast"):
    """trnfft/api.py:22-27."""
    re = np.asarray(re, dtype=F32)
    im = np.zeros_like(re) if im is None else np.asarray(im, dtype=F32)
    if n is not None:
        re, im = _resize_last(re, im, n)
    return fft_core(re, im, False, precision)


def ifft(re, im=None, n=None, precision="fast"):
    """trnfft/api.py:30-35."""
    re = np.asarray(re, dtype=F32)
    im = np.zeros_like(re) if im is None else np.asarray(im, dtype=F32)
    if n is not None:
        re, im = _resize_last(re, im, n)
    return fft_core(re, im, True, precision)


def rfft(x, n=None, precision="fast"):
    """trnfft/api.py:38-46: full complex FFT of the real signal, keep n//2+1."""
    x = np.asarray(x, dtype=F32)
    if n is not None:
        x, _ = _resize_last(x, x, n)
    n = x.shape[-1]
    r, i = fft_core(x, np.zeros_like(x), False, precision)
    h = n // 2 + 1
    return r[..., :h], i[..., :h]


def hermitian_extend(re, im, n):
    """Full spectrum the reference builds in irfft (trnfft/api.py:49-68)."""
    half = re.shape[-1]
    lead = re.shape[:-1]
    fr = np.zeros((*lead, n), dtype=re.dtype)
    fi = np.zeros((*lead, n), dtype=re.dtype)
    fr[..., :half] = re
    fi[..., :half] = im
    if n > 1:
        num_neg = n - half
        if num_neg > 0:
            fr[..., half:] = np.flip(re[..., 1 : 1 + num_neg], axis=-1)
            fi[..., half:] = -np.flip(im[..., 1 : 1 + num_neg], axis=-1)
    return fr, fi


def irfft(re, im, n=None, precision="fast"):
    """trnfft/api.py:49-68: Hermitian-extend, inverse complex FFT, real part."""
    re = np.asarray(re, dtype=F32)
    im = np.asarray(im, dtype=F32)
    if n is None:
        n = 2 * (re.shape[-1] - 1)
    fr, fi = hermitian_extend(re, im, n)
    r, _ = fft_core(fr, fi, True, precision)
    return r


def _fft_along(re, im, axis, inverse, precision="fast"):
    """trnfft/api.py:496-516: move axis last, flatten, fft_core, move back."""
    re = np.moveaxis(re, axis, -1)
    im = np.moveaxis(im, axis, -1)
    r, i = fft_core(np.ascontiguousarray(re), np.ascontiguousarray(im), inverse, precision)
    return np.moveaxis(r, -1, axis), np.moveaxis(i, -1, axis)


def fftn(re, im=None, s=None, dim=None, inverse=False, precision="fast"):
    """trnfft/api.py:111-167 (fftn / ifftn)."""
    re = np.asarray(re, dtype=F32)
    im = np.zeros_like(re) if im is None else np.asarray(im, dtype=F32)
    nd = re.ndim
    if dim is None:
        dim = tuple(range(-len(s), 0)) if s is not None else tuple(range(-nd, 0))
    dim = tuple(d % nd for d in dim)
    if s is not None:
        for size, d in zip(s, dim):
            re = np.moveaxis(re, d, -1)
            im = np.moveaxis(im, d, -1)
            re, im = _resize_last(re, im, size)
            re = np.moveaxis(re, -1, d)
            im = np.moveaxis(im, -1, d)
    for d in dim:
        re, im = _fft_along(re, im, d, inverse, precision)
    return np.ascontiguousarray(re), np.ascontiguousarray(im)


def fft2(re, im=None, s=None, precision="fast"):
    """trnfft/api.py:105-108."""
    return fftn(re, im, s=s, dim=(-2, -1), precision=precision)


def ifft2(re, im=None, s=None, precision="fast"):
    return fftn(re, im, s=s, dim=(-2, -1), inverse=True, precision=precision)


def hann_window_periodic(n: int) -> np.ndarray:
    """torch.hann_window(n) (periodic=True): 0.5 - 0.5 cos(2 pi k / n)."""
    k = np.arange(n, dtype=np.float64)
    return (0.5 - 0.5 * np.cos(2.0 * math.pi * k / n)).astype(F32)


def _pad_last(x, p, mode):
    """torch.nn.functional.pad on the last axis for the modes stft accepts."""
    pw = [(0, 0)] * (x.ndim - 1) + [(p, p)]
    if mode == "reflect":
        return np.pad(x, pw, mode="reflect")
    if mode == "replicate":
        return np.pad(x, pw, mode="edge")
    if mode == "circular":
        return np.pad(x, pw, mode="wrap")
    if mode == "constant":
        return np.pad(x, pw, mode="constant")
    raise ValueError(mode)


def stft_frames(x, n_fft, hop_length, window, center=True, pad_mode="reflect"):
    """Framing and windowing of trnfft/api.py:291-336; returns (..., F, n_fft)."""
    x = np.asarray(x, dtype=F32)
    win_length = window.shape[-1]
    if center:
        x = _pad_last(x, n_fft // 2, pad_mode)
    L = x.shape[-1]
    nf = 1 + (L - n_fft) // hop_length
    idx = np.arange(n_fft)[None, :] + np.arange(nf)[:, None] * hop_length
    fr = x[..., idx]
    if win_length < n_fft:
        w = np.zeros(n_fft, dtype=F32)
        off = (n_fft - win_length) // 2
        w[off : off + win_length] = window
    else:
        w = window
    return (fr * w).astype(F32)


def stft(x, n_fft, hop_length=None, win_length=None, window=None, center=True,
         pad_mode="reflect", normalized=False, onesided=True):
    """trnfft/api.py:291-365: output (..., freq, time) planar."""
    if hop_length is None:
        hop_length = n_fft // 4
    if win_length is None:
        win_length = n_fft
    if window is None:
        window = hann_window_periodic(win_length)
    window = np.asarray(window, dtype=F32)
    fr = stft_frames(x, n_fft, hop_length, window, center, pad_mode)
    shp = fr.shape
    r, i = fft_core(fr.reshape(-1, n_fft), np.zeros((int(np.prod(shp[:-1])), n_fft), F32), False)
    r = r.reshape(shp)
    i = i.reshape(shp)
    if onesided:
        nb = n_fft // 2 + 1
        r = r[..., :nb]
        i = i[..., :nb]
    r = np.swapaxes(r, -2, -1)
    i = np.swapaxes(i, -2, -1)
    if normalized:
        sc = F32(1.0 / math.sqrt(n_fft))
        r = r * sc
        i = i * sc
    return np.ascontiguousarray(r), np.ascontiguousarray(i)


def istft(re, im, n_fft, hop_length=None, win_length=None, window=None, center=True,
          normalized=False, onesided=True, length=None):
    """trnfft/api.py:368-470: inverse FFT per frame, windowed overlap-add."""
    re = np.asarray(re, dtype=F32)
    im = np.asarray(im, dtype=F32)
    if hop_length is None:
        hop_length = n_fft // 4
    if win_length is None:
        win_length = n_fft
    if window is None:
        window = hann_window_periodic(win_length)
    window = np.asarray(window, dtype=F32)
    if normalized:
        sc = F32(math.sqrt(n_fft))
        re = re * sc
        im = im * sc
    sr = np.swapaxes(re, -2, -1)
    si = np.swapaxes(im, -2, -1)
    if onesided:
        sr, si = hermitian_extend(np.ascontiguousarray(sr), np.ascontiguousarray(si), n_fft)
    nf = sr.shape[-2]
    fr, _ = fft_core(sr.reshape(-1, n_fft), si.reshape(-1, n_fft), True)
    frames = fr.reshape(*sr.shape[:-1], n_fft)
    if win_length < n_fft:
        w = np.zeros(n_fft, dtype=F32)
        off = (n_fft - win_length) // 2
        w[off : off + win_length] = window
        window = w
    exp_len = n_fft + (nf - 1) * hop_length
    lead = frames.shape[:-2]
    out = np.zeros((*lead, exp_len), dtype=F32)
    wsum = np.zeros(exp_len, dtype=F32)
    raw = np.zeros((*lead, exp_len), dtype=F32)
    for t in range(nf):
        st = t * hop_length
        out[..., st : st + n_fft] += frames[..., t, :] * window
        wsum[st : st + n_fft] += window ** 2
        raw[..., st : st + n_fft] += frames[..., t, :]
    mask = wsum > 1e-8
    out[..., mask] = out[..., mask] / wsum[mask]
    out[..., ~mask] = raw[..., ~mask]
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
            out = np.concatenate([out, np.zeros((*lead, length - cur), F32)], axis=-1)
    return out


# ---------------------------------------------------------------------------
# multi-core decomposition (trnfft/nki/multicore.py)
# ---------------------------------------------------------------------------


def factorize(n: int):
    """trnfft/nki/multicore.py:134-148: largest divisor <= sqrt(n)."""
    n1 = int(n ** 0.5)
    while n1 > 1 and n % n1 != 0:
        n1 -= 1
    if n1 <= 1:
        raise ValueError(f"n={n} has no non-trivial divisors (prime); row-column FFT not applicable")
    return n1, n // n1


def stage_parallel_fft(re, im, inverse: bool):
    """Four-step single transform (trnfft/nki/multicore.py:151-219).

    Column DFTs of the (n1, n2) view x2d[m, l] = x[n2*m + l], float32 twiddle
    exp(sign*2*pi*i*l*k1/N), row DFTs, column-major flatten.
    """
    re = np.asarray(re, dtype=F32).reshape(-1)
    im = np.asarray(im, dtype=F32).reshape(-1)
    n = re.shape[0]
    n1, n2 = factorize(n)
    sign = 1.0 if inverse else -1.0
    cr, ci = fft_core(re.reshape(n1, n2).T.copy(), im.reshape(n1, n2).T.copy(), inverse)
    Yr, Yi = cr.T, ci.T
    k1 = np.arange(n1, dtype=F32)[:, None]
    l = np.arange(n2, dtype=F32)[None, :]
    ang = (((F32(sign * 2.0 * math.pi) * l) * k1) / F32(n)).astype(F32)
    tr, ti = np.cos(ang).astype(F32), np.sin(ang).astype(F32)
    Zr = Yr * tr - Yi * ti
    Zi = Yr * ti + Yi * tr
    Xr, Xi = fft_core(np.ascontiguousarray(Zr), np.ascontiguousarray(Zi), inverse)
    return Xr.T.reshape(n).copy(), Xi.T.reshape(n).copy()


def batch_split_fft(re, im, inverse, num_cores):
    """trnfft/nki/multicore.py:222-260: chunk the batch, transform each shard."""
    re = np.asarray(re, dtype=F32)
    im = np.asarray(im, dtype=F32)
    k = min(num_cores, re.shape[0])
    if k <= 1:
        return fft_core(re, im, inverse)
    rs = np.array_split(re, k, axis=0)
    is_ = np.array_split(im, k, axis=0)
    out = [fft_core(a, b, inverse) for a, b in zip(rs, is_)]
    return np.concatenate([o[0] for o in out]), np.concatenate([o[1] for o in out])


# ---------------------------------------------------------------------------
# complex GEMM / ComplexLinear (trnfft/complex.py:142-150, trnfft/nn.py:33-49)
# ---------------------------------------------------------------------------


def complex_matmul(ar, ai, br, bi):
    """trnfft/complex.py:142-150: four real float32 matmuls."""
    ar, ai, br, bi = (np.asarray(t, dtype=F32) for t in (ar, ai, br, bi))
    return (ar @ br - ai @ bi).astype(F32), (ar @ bi + ai @ br).astype(F32)


def complex_linear(xr, xi, wr, wi, br=None, bi=None):
    """trnfft/nn.py:33-49 (pytorch branch): y = x W^T + b, complex."""
    xr, xi, wr, wi = (np.asarray(t, dtype=F32) for t in (xr, xi, wr, wi))
    yr = xr @ wr.T - xi @ wi.T
    yi = xr @ wi.T + xi @ wr.T
    if br is not None:
        yr = yr + br
        yi = yi + bi
    return yr.astype(F32), yi.astype(F32)


# ---------------------------------------------------------------------------
# threaded driver for the CPU baseline (bench.py only)
# ---------------------------------------------------------------------------


def threaded_rows(fn, arrays, threads: int):
    """Run ``fn`` over row-chunks of ``arrays`` on ``threads`` host threads.

    NumPy releases the GIL inside its array kernels, so independent row
    chunks of a batched transform run concurrently.
    """
    b = arrays[0].shape[0]
    threads = max(1, min(threads, b))
    bounds = np.linspace(0, b, threads + 1).astype(int)
    chunks = [tuple(a[bounds[t]:bounds[t + 1]] for a in arrays) for t in range(threads)]
    with ThreadPoolExecutor(threads) as ex:
        outs = list(ex.map(lambda c: fn(*c), chunks))
    return outs


def rel_l2(a, b) -> float:
    """Relative L2 error ||a - b|| / ||b|| in float64."""
    a = np.asarray(a).astype(np.complex128)
    b = np.asarray(b).astype(np.complex128)
    den = np.linalg.norm(b.ravel())
    num = np.linalg.norm((a - b).ravel())
    return float(num / den) if den > 0 else float(num)
