"""GPU parity of the fused STFT kernel and of istft."""

import numpy as np
import pytest
import torch

import trnfft_b200 as trnfft
from trnfft_b200 import ComplexTensor
from oracle import trnfft_oracle as O
from tests.helpers import TOL, cplx, cuda, host, rel_l2

pytestmark = pytest.mark.gpu

CASES = {
    "c512": dict(n_fft=512, hop_length=256),
    "c256_64": dict(n_fft=256, hop_length=64),
    "c128_nocenter": dict(n_fft=128, hop_length=32, center=False),
    "c512_norm_two": dict(n_fft=512, hop_length=128, normalized=True, onesided=False),
    "c256_win200": dict(n_fft=256, hop_length=100, win_length=200),
    "c64_const": dict(n_fft=64, hop_length=16, pad_mode="constant"),
}


@pytest.mark.parametrize("name", list(CASES))
def test_vs_reference_golden(golden, name):
    g = golden("stft")
    S = trnfft.stft(cuda(g["wave"]), **CASES[name])
    ref = g[f"stft_re_{name}"] + 1j * g[f"stft_im_{name}"]
    assert S.shape == ref.shape
    assert rel_l2(cplx(S), ref) < TOL


@pytest.mark.parametrize("n_fft,hop,mode", [(4, 1, "reflect"), (16, 5, "replicate"), (1024, 300, "circular"),
                                            (8192, 2048, "reflect"), (2048, 512, "constant")])
def test_vs_oracle_pad_modes(n_fft, hop, mode):
    rng = np.random.default_rng(n_fft)
    w = rng.standard_normal((3, 9000)).astype(np.float32)
    S = trnfft.stft(cuda(w), n_fft=n_fft, hop_length=hop, pad_mode=mode)
    r, i = O.stft(w, n_fft=n_fft, hop_length=hop, pad_mode=mode)
    assert S.shape == r.shape
    assert rel_l2(cplx(S), r + 1j * i) < TOL


def test_config3_shape_vs_torch_and_oracle():
    """Config 3: 256 waveforms of 160000 samples, n_fft 512, hop 256 -> (256, 257, 626)."""
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(256, 160000, device="cuda", generator=g)
    S = trnfft.stft(x, n_fft=512, hop_length=256)
    assert S.shape == (256, 257, 626)
    ref = torch.stft(x, 512, 256, window=torch.hann_window(512, device="cuda"), center=True,
                     pad_mode="reflect", return_complex=True)
    assert rel_l2(cplx(S), ref.cpu().numpy()) < 2e-6
    r, i = O.stft(host(x[:2]), n_fft=512, hop_length=256)
    assert rel_l2(cplx(S)[:2], r + 1j * i) < TOL


def test_1d_and_known_tone():
    sr, freq = 1000, 100
    t = torch.arange(0, 1.0, 1.0 / sr, device="cuda")
    S = trnfft.stft(torch.sin(2 * np.pi * freq * t), n_fft=256, hop_length=64, center=False)
    assert S.shape[0] == 129
    peak = S.abs().mean(dim=-1).argmax().item()
    assert abs(peak - int(freq * 256 / sr)) <= 1


def test_istft_roundtrip_and_golden(golden):
    g = golden("stft")
    w = cuda(g["wave"])
    S = trnfft.stft(w, n_fft=256, hop_length=64)
    back = trnfft.istft(S, n_fft=256, hop_length=64, length=4000)
    assert rel_l2(host(back), g["istft_256_64"]) < TOL
    np.testing.assert_allclose(host(back), g["wave"], atol=1e-3)


def test_stft_gradient_matches_torch():
    torch.manual_seed(0)
    x = torch.randn(2, 2048, device="cuda", requires_grad=True)
    S = trnfft.stft(x, n_fft=256, hop_length=64)
    (S.real * 2 + S.imag ** 2).sum().backward()
    y = x.detach().clone().requires_grad_(True)
    T = torch.stft(y, 256, 64, window=torch.hann_window(256, device="cuda"), center=True,
                   pad_mode="reflect", return_complex=True)
    (T.real * 2 + T.imag ** 2).sum().backward()
    assert rel_l2(host(x.grad), host(y.grad)) < 1e-5
