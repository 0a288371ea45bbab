"""Complex GEMM entry points behind complex_matmul and ComplexLinear.

``complex_linear`` runs the library's tcgen05 tensor-core GEMM
(trnfft_complex_linear: two TF32 GEMMs with the 3xTF32 split, float32
accuracy).  ``complex_matmul`` (C = A @ B) maps onto the same kernel with
W = B^T.  Backward passes use the analytic adjoints of
trnfft/nki/autograd.py:125-159 evaluated with device matmuls, as the
reference does for its kernels' backward.
"""

from __future__ import annotations

import torch

from . import _lib
from ._device import place
from .complex import ComplexTensor


def _pad_k(t: torch.Tensor, k4: int) -> torch.Tensor:
    k = t.shape[-1]
    if k == k4:
        return t.contiguous()
    return torch.nn.functional.pad(t, (0, k4 - k)).contiguous()


def _aligned(t: torch.Tensor) -> torch.Tensor:
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


def _weight_key(wr, wi, k4):
    return (wr.data_ptr(), wi.data_ptr(), wr._version, wi._version, tuple(wr.shape), k4, wr.device)


def split_weight(wr, wi, k4: int) -> torch.Tensor:
    """The TF32 hi/lo split of a complex weight: one (6, N, k4) tensor holding
    Wr_hi, Wr_lo, Wi_hi, Wi_lo, Ws_hi, Ws_lo with Ws = Wr + Wi (trnfft_split_tf32,
    trnfft_split_tf32_sum), the operands of the three-product complex GEMM."""
    wr2, wi2 = (_aligned(_pad_k(t.float(), k4)) for t in (wr, wi))
    N = wr2.shape[0]
    out = torch.empty(6, N, k4, dtype=torch.float32, device=wr2.device)
    dev = wr2.device.index if wr2.device.index is not None else torch.cuda.current_device()
    st = _lib.stream_ptr(wr2.device)
    for i, t in enumerate((wr2, wi2)):
        _lib.call("trnfft_split_tf32", _lib.ptr(t), _lib.ptr(out[2 * i]), _lib.ptr(out[2 * i + 1]), t.numel(), dev, st)
    _lib.call("trnfft_split_tf32_sum", _lib.ptr(wr2), _lib.ptr(wi2), _lib.ptr(out[4]), _lib.ptr(out[5]), wr2.numel(),
              dev, st)
    return out


def linear_raw(xr, xi, wr, wi, br=None, bi=None, cache=None):
    """y = x W^T + b for 2-D planar complex x (M x K) and W (N x K) on CUDA.

    With `cache` (a dict owned by the caller, e.g. a ComplexLinear module), the TF32 split of
    W is kept there and reused while W's storage and version are unchanged, so a forward
    splits only x."""
    M, K = xr.shape
    N = wr.shape[0]
    k4 = (K + 3) // 4 * 4
    dev = xr.device.index if xr.device.index is not None else torch.cuda.current_device()
    if br is not None:
        br = _aligned(br.float())
        bi = _aligned(bi.float())
    yr = torch.empty(M, N, dtype=torch.float32, device=xr.device)
    yi = torch.empty_like(yr)
    if not (M and N):
        return yr, yi
    xr2, xi2 = (_aligned(_pad_k(t.float(), k4)) for t in (xr, xi))
    if cache is not None:
        key = _weight_key(wr, wi, k4)
        if cache.get("key") != key:
            cache["key"] = key
            cache["split"] = split_weight(wr, wi, k4)
        ws = cache["split"]
        work = torch.empty(6 * M * k4, dtype=torch.float32, device=xr.device)
        _lib.call("trnfft_complex_linear_presplit", _lib.ptr(xr2), _lib.ptr(xi2), _lib.ptr(ws), _lib.ptr(br),
                  _lib.ptr(bi), _lib.ptr(yr), _lib.ptr(yi), M, N, k4, _lib.ptr(work), dev, _lib.stream_ptr(xr.device))
        return yr, yi
    wr2, wi2 = (_aligned(_pad_k(t.float(), k4)) for t in (wr, wi))
    wb = _lib.load().trnfft_complex_linear_work_bytes(M, N, k4)
    work = torch.empty(wb, dtype=torch.uint8, device=xr.device)
    _lib.call("trnfft_complex_linear", _lib.ptr(xr2), _lib.ptr(xi2), _lib.ptr(wr2), _lib.ptr(wi2),
              _lib.ptr(br), _lib.ptr(bi), _lib.ptr(yr), _lib.ptr(yi), M, N, k4, _lib.ptr(work), dev,
              _lib.stream_ptr(xr.device))
    return yr, yi


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, xr, xi, wr, wi, br, bi, cache=None):
        ctx.save_for_backward(xr, xi, wr, wi)
        ctx.has_bias = br is not None
        return linear_raw(xr, xi, wr, wi, br, bi, cache)

    @staticmethod
    def backward(ctx, gr, gi):
        xr, xi, wr, wi = ctx.saved_tensors
        # dX = dY conj(W); dW = dY^T conj(X) (trnfft/nki/autograd.py:147-159)
        dxr = gr @ wr + gi @ wi
        dxi = gi @ wr - gr @ wi
        dwr = gr.t() @ xr + gi.t() @ xi
        dwi = gi.t() @ xr - gr.t() @ xi
        dbr = gr.sum(0) if ctx.has_bias else None
        dbi = gi.sum(0) if ctx.has_bias else None
        return dxr, dxi, dwr, dwi, dbr, dbi, None


def complex_linear(x: ComplexTensor, w_re, w_im, b_re=None, b_im=None, cache=None) -> ComplexTensor:
    if b_re is not None and b_im is None:
        b_im = torch.zeros_like(b_re)
    ts = [x.real, x.imag, w_re, w_im] + ([b_re, b_im] if b_re is not None else [])
    dev_ts, restore = place(*ts)
    xr, xi, wr, wi = dev_ts[:4]
    br, bi = (dev_ts[4], dev_ts[5]) if b_re is not None else (None, None)
    lead = xr.shape[:-1]
    K = xr.shape[-1]
    xr2, xi2 = xr.reshape(-1, K), xi.reshape(-1, K)
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in (xr2, xi2, wr, wi, br, bi)):
        yr, yi = _LinearFn.apply(xr2, xi2, wr, wi, br, bi, cache)
    else:
        yr, yi = linear_raw(xr2, xi2, wr, wi, br, bi, cache)
    N = wr.shape[0]
    return ComplexTensor(restore(yr.reshape(*lead, N)), restore(yi.reshape(*lead, N)))


def complex_matmul(a: ComplexTensor, b: ComplexTensor) -> ComplexTensor:
    """C = A @ B (trnfft/complex.py:142-150) as complex_linear with W = B^T."""
    if a.real.dim() != 2 or b.real.dim() != 2:
        # batched matmul: loop over the leading dims of broadcast-free inputs
        if a.real.dim() == b.real.dim() and a.real.shape[:-2] == b.real.shape[:-2]:
            lead = a.real.shape[:-2]
            ar = a.real.reshape(-1, *a.real.shape[-2:])
            ai = a.imag.reshape(-1, *a.imag.shape[-2:])
            br_ = b.real.reshape(-1, *b.real.shape[-2:])
            bi_ = b.imag.reshape(-1, *b.imag.shape[-2:])
            outs = [complex_matmul(ComplexTensor(ar[i], ai[i]), ComplexTensor(br_[i], bi_[i]))
                    for i in range(ar.shape[0])]
            re = torch.stack([o.real for o in outs]).reshape(*lead, *outs[0].shape)
            im = torch.stack([o.imag for o in outs]).reshape(*lead, *outs[0].shape)
            return ComplexTensor(re, im)
        raise ValueError("complex_matmul: expected 2-D operands or equal batch shapes")
    return complex_linear(a, b.real.t().contiguous(), b.imag.t().contiguous())
