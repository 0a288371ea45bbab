"""Generate golden input/output vectors by running the reference trnfft.

Run in a container where the reference source tree is available:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py /path/to/reference

It imports the reference package read-only, selects its ``"pytorch"``
backend (the CPU path the reference runs when no Trainium is present,
trnfft/nki/dispatch.py:50-71) and writes ``tests/golden/*.npz``: seeded
inputs and the reference's outputs.  Those fixtures pin both the NumPy oracle
(``oracle/trnfft_oracle.py``) and the CUDA implementation, and they are what
travels to machines where the reference is absent.
"""

from __future__ import annotations

import math
import os
import sys

import numpy as np


def main(ref_root: str) -> None:
    sys.dont_write_bytecode = True
    sys.path.insert(0, ref_root)
    import torch

    import trnfft
    from trnfft import ComplexTensor
    from trnfft.nki import multicore
    from trnfft.nn import ComplexLinear

    trnfft.set_backend("pytorch")
    trnfft.set_precision("fast")
    out_dir = os.path.dirname(os.path.abspath(__file__))

    def g(seed):
        return torch.Generator().manual_seed(seed)

    def save(name, **arrs):
        path = os.path.join(out_dir, name + ".npz")
        np.savez_compressed(path, **{k: np.asarray(v) for k, v in arrs.items()})
        print("wrote", path, sum(np.asarray(v).nbytes for v in arrs.values()), "bytes raw")

    # --- power-of-2 C2C forward + inverse, batch 3 (trnfft/fft_core.py:53-117)
    d = {}
    for n in [2, 4, 8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096]:
        gen = g(1000 + n)
        xr = torch.randn(3, n, generator=gen)
        xi = torch.randn(3, n, generator=gen)
        y = trnfft.fft(ComplexTensor(xr, xi))
        z = trnfft.ifft(ComplexTensor(xr, xi))
        d[f"x_re_{n}"], d[f"x_im_{n}"] = xr.numpy(), xi.numpy()
        d[f"fft_re_{n}"], d[f"fft_im_{n}"] = y.real.numpy(), y.imag.numpy()
        d[f"ifft_re_{n}"], d[f"ifft_im_{n}"] = z.real.numpy(), z.imag.numpy()
    save("pow2_c2c", **d)

    # --- larger power of 2 (single transform), forward only
    d = {}
    for n in [8192, 16384]:
        gen = g(2000 + n)
        xr = torch.randn(1, n, generator=gen)
        xi = torch.randn(1, n, generator=gen)
        y = trnfft.fft(ComplexTensor(xr, xi))
        d[f"x_re_{n}"], d[f"x_im_{n}"] = xr.numpy(), xi.numpy()
        d[f"fft_re_{n}"], d[f"fft_im_{n}"] = y.real.numpy(), y.imag.numpy()
    save("pow2_large", **d)

    # --- Bluestein, "fast" and "double" (trnfft/fft_core.py:1285-1376)
    d = {}
    for n in [3, 5, 7, 11, 100, 127, 997, 1000, 4093, 6000]:
        gen = g(3000 + n)
        b = 2 if n < 2000 else 1
        xr = torch.randn(b, n, generator=gen)
        xi = torch.randn(b, n, generator=gen)
        d[f"x_re_{n}"], d[f"x_im_{n}"] = xr.numpy(), xi.numpy()
        for prec in ["fast", "double"]:
            trnfft.set_precision(prec)
            y = trnfft.fft(ComplexTensor(xr, xi))
            z = trnfft.ifft(ComplexTensor(xr, xi))
            d[f"fft_{prec}_re_{n}"], d[f"fft_{prec}_im_{n}"] = y.real.numpy(), y.imag.numpy()
            d[f"ifft_{prec}_re_{n}"], d[f"ifft_{prec}_im_{n}"] = z.real.numpy(), z.imag.numpy()
        trnfft.set_precision("fast")
    save("bluestein", **d)

    # --- rfft / irfft (trnfft/api.py:38-68)
    d = {}
    for n in [16, 128, 1024, 100, 4093]:
        gen = g(4000 + n)
        x = torch.randn(3, n, generator=gen)
        for prec in ["fast", "double"]:
            trnfft.set_precision(prec)
            X = trnfft.rfft(x)
            xr = trnfft.irfft(X, n=n)
            d[f"rfft_{prec}_re_{n}"], d[f"rfft_{prec}_im_{n}"] = X.real.numpy(), X.imag.numpy()
            d[f"irfft_{prec}_{n}"] = xr.numpy()
        trnfft.set_precision("fast")
        d[f"x_{n}"] = x.numpy()
        # irfft of a random (non-Hermitian) half spectrum: DC/Nyquist imaginary parts
        h = n // 2 + 1
        sr = torch.randn(3, h, generator=gen)
        si = torch.randn(3, h, generator=gen)
        d[f"spec_re_{n}"], d[f"spec_im_{n}"] = sr.numpy(), si.numpy()
        trnfft.set_precision("double")
        d[f"irfft_spec_double_{n}"] = trnfft.irfft(ComplexTensor(sr, si), n=n).numpy()
        trnfft.set_precision("fast")
        d[f"irfft_spec_fast_{n}"] = trnfft.irfft(ComplexTensor(sr, si), n=n).numpy()
    save("real", **d)

    # --- fft2 / fftn / ifftn (trnfft/api.py:105-167)
    d = {}
    for shape in [(16, 32), (64, 64), (8, 256)]:
        gen = g(5000 + shape[0] * shape[1])
        xr = torch.randn(2, *shape, generator=gen)
        xi = torch.randn(2, *shape, generator=gen)
        key = f"{shape[0]}x{shape[1]}"
        y = trnfft.fft2(ComplexTensor(xr, xi))
        z = trnfft.ifftn(ComplexTensor(xr, xi), dim=(-2, -1))
        d[f"x_re_{key}"], d[f"x_im_{key}"] = xr.numpy(), xi.numpy()
        d[f"fft2_re_{key}"], d[f"fft2_im_{key}"] = y.real.numpy(), y.imag.numpy()
        d[f"ifft2_re_{key}"], d[f"ifft2_im_{key}"] = z.real.numpy(), z.imag.numpy()
    gen = g(5999)
    x3 = torch.randn(4, 8, 16, generator=gen)
    y3 = trnfft.fftn(x3)
    d["x3"], d["fftn3_re"], d["fftn3_im"] = x3.numpy(), y3.real.numpy(), y3.imag.numpy()
    ys = trnfft.fftn(x3, dim=(0, 2))
    d["fftn3_d02_re"], d["fftn3_d02_im"] = ys.real.numpy(), ys.imag.numpy()
    yr = trnfft.rfftn(x3)
    d["rfftn3_re"], d["rfftn3_im"] = yr.real.numpy(), yr.imag.numpy()
    d["irfftn3"] = trnfft.irfftn(yr, s=x3.shape).numpy()
    x2 = torch.randn(8, 16, generator=gen)
    y2 = trnfft.rfft2(x2, s=(16, 32))
    d["x2"], d["rfft2_s_re"], d["rfft2_s_im"] = x2.numpy(), y2.real.numpy(), y2.imag.numpy()
    xh = ComplexTensor(torch.randn(3, 9, generator=gen), torch.randn(3, 9, generator=gen))
    d["h_re"], d["h_im"] = xh.real.numpy(), xh.imag.numpy()
    d["hfft_16"] = trnfft.hfft(xh, n=16).numpy()
    xx = torch.randn(3, 16, generator=gen)
    ih = trnfft.ihfft(xx)
    d["ih_x"], d["ihfft_re"], d["ihfft_im"] = xx.numpy(), ih.real.numpy(), ih.imag.numpy()
    save("nd", **d)

    # --- STFT / ISTFT (trnfft/api.py:291-470)
    d = {}
    gen = g(6000)
    fs = 16000.0
    t = torch.arange(4000, dtype=torch.float32) / fs
    w = torch.randn(2, 4000, generator=gen)
    for j in range(8):
        f = 50.0 + 6950.0 * torch.rand(1, generator=gen).item()
        ph = 2 * math.pi * torch.rand(1, generator=gen).item()
        w = w + torch.sin(2 * math.pi * f * t + ph)
    d["wave"] = w.numpy()
    cases = {
        "c512": dict(n_fft=512, hop_length=256),
        "c256_64": dict(n_fft=256, hop_length=64),
        "c128_nocenter": dict(n_fft=128, hop_length=32, center=False),
        "c512_norm_two": dict(n_fft=512, hop_length=128, normalized=True, onesided=False),
        "c256_win200": dict(n_fft=256, hop_length=100, win_length=200),
        "c64_const": dict(n_fft=64, hop_length=16, pad_mode="constant"),
    }
    for name, kw in cases.items():
        S = trnfft.stft(w, **kw)
        d[f"stft_re_{name}"], d[f"stft_im_{name}"] = S.real.numpy(), S.imag.numpy()
    S = trnfft.stft(w, n_fft=256, hop_length=64)
    d["istft_256_64"] = trnfft.istft(S, n_fft=256, hop_length=64, length=4000).numpy()
    save("stft", **d)

    # --- four-step single transform (trnfft/nki/multicore.py:151-219)
    d = {}
    for n in [64, 4096, 65536]:
        gen = g(7000 + n)
        xr = torch.randn(n, generator=gen)
        xi = torch.randn(n, generator=gen)
        y = multicore._stage_parallel_fft(ComplexTensor(xr, xi), num_cores=2, inverse=False)
        z = multicore._stage_parallel_fft(ComplexTensor(xr, xi), num_cores=2, inverse=True)
        d[f"x_re_{n}"], d[f"x_im_{n}"] = xr.numpy(), xi.numpy()
        d[f"sp_re_{n}"], d[f"sp_im_{n}"] = y.real.numpy(), y.imag.numpy()
        d[f"spi_re_{n}"], d[f"spi_im_{n}"] = z.real.numpy(), z.imag.numpy()
    save("four_step", **d)

    # --- ComplexLinear / complex_matmul (trnfft/nn.py:33-49, complex.py:142-150)
    d = {}
    torch.manual_seed(8000)
    layer = ComplexLinear(96, 48)
    with torch.no_grad():
        layer.bias_re.copy_(torch.randn(48) * 0.1)
        layer.bias_im.copy_(torch.randn(48) * 0.1)
    x = ComplexTensor(torch.randn(40, 96), torch.randn(40, 96))
    with torch.no_grad():
        y = layer(x)
    d["x_re"], d["x_im"] = x.real.numpy(), x.imag.numpy()
    d["w_re"], d["w_im"] = layer.W_re.weight.detach().numpy(), layer.W_im.weight.detach().numpy()
    d["b_re"], d["b_im"] = layer.bias_re.detach().numpy(), layer.bias_im.detach().numpy()
    d["y_re"], d["y_im"] = y.real.numpy(), y.imag.numpy()
    a = ComplexTensor(torch.randn(33, 70), torch.randn(33, 70))
    b = ComplexTensor(torch.randn(70, 20), torch.randn(70, 20))
    c = trnfft.complex_matmul(a, b)
    d["a_re"], d["a_im"], d["b2_re"], d["b2_im"] = a.real.numpy(), a.imag.numpy(), b.real.numpy(), b.imag.numpy()
    d["c_re"], d["c_im"] = c.real.numpy(), c.imag.numpy()
    save("linear", **d)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <path to the reference source tree>")
    main(sys.argv[1])
