"""GPU parity of the kernel variants selected by environment variables.

Each variable is read once per process, so every case runs a short script in a child process
with the variable set and checks the result against numpy's float64 FFT (or the oracle's iSTFT):

* TRNFFT_B200_F64_BLUE_R2=1: the 512-thread radix-2 form of the fused fp64 Bluestein kernel;
* TRNFFT_B200_ISTFT_THREADS=256 / 512: 16 / 32 frames per iSTFT chunk;
* TRNFFT_B200_STFT_THREADS=256 / 512: 16 / 32 frames per STFT block;
* TRNFFT_B200_BLUE_LOGE=4 / 5: values per thread of the fp32 Bluestein kernel at m = 8192.
"""

import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

_SCRIPT = r"""
import numpy as np, torch
import trnfft_b200 as trnfft
from trnfft_b200 import ComplexTensor
from oracle import trnfft_oracle as O
rng = np.random.default_rng(11)
worst = 0.0
def rel(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))
# fp64 Bluestein (m = 8192) in precision "double" and fp32 Bluestein / packed real transforms
x = (rng.standard_normal((5, 4093)) + 1j * rng.standard_normal((5, 4093))).astype(np.complex64)
ref = np.fft.fft(x.astype(np.complex128), axis=-1)
t = ComplexTensor(torch.from_numpy(x.real.copy()).cuda(), torch.from_numpy(x.imag.copy()).cuda())
trnfft.set_precision("double")
y = trnfft.fft(t)
worst = max(worst, rel(y.real.double().cpu().numpy() + 1j * y.imag.double().cpu().numpy(), ref))
trnfft.set_precision("fast")
y = trnfft.fft(t)
worst = max(worst, rel(y.real.double().cpu().numpy() + 1j * y.imag.double().cpu().numpy(), ref))
xr = rng.standard_normal((6, 4093)).astype(np.float32)
yr = trnfft.rfft(torch.from_numpy(xr).cuda())
worst = max(worst, rel(yr.real.double().cpu().numpy() + 1j * yr.imag.double().cpu().numpy(),
                       np.fft.rfft(xr.astype(np.float64), axis=-1)))
# STFT / iSTFT (n_fft 512, hop 256)
sig = rng.standard_normal((3, 20000)).astype(np.float32)
win = (np.hanning(512) + 0.05).astype(np.float32)
S = trnfft.stft(torch.from_numpy(sig).cuda(), 512, 256, window=torch.from_numpy(win).cuda())
sr, si = O.stft(sig, 512, 256, None, win, center=True, normalized=False, onesided=True)
worst = max(worst, rel(S.real.double().cpu().numpy() + 1j * S.imag.double().cpu().numpy(),
                       sr.astype(np.float64) + 1j * si.astype(np.float64)))
back = trnfft.istft(S, 512, 256, window=torch.from_numpy(win).cuda())
want = O.istft(sr, si, 512, 256, None, win, center=True, normalized=False, onesided=True)
worst = max(worst, rel(back.double().cpu().numpy(), want.astype(np.float64)))
print("WORST", worst)
"""


@pytest.mark.parametrize("env", [
    {"TRNFFT_B200_F64_BLUE_R2": "1"},
    {"TRNFFT_B200_ISTFT_THREADS": "256", "TRNFFT_B200_STFT_THREADS": "256"},
    {"TRNFFT_B200_ISTFT_THREADS": "512", "TRNFFT_B200_STFT_THREADS": "512"},
    {"TRNFFT_B200_BLUE_LOGE": "4"},
    {"TRNFFT_B200_BLUE_LOGE": "5"},
], ids=["f64-bluestein-radix2", "stft-istft-256", "stft-istft-512", "bluestein-loge4", "bluestein-loge5"])
def test_env_selected_variants(env):
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _SCRIPT], cwd=root, env={**os.environ, **env},
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    assert float(r.stdout.split("WORST")[-1]) < 1e-5
