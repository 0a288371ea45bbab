"""Multi-GPU transforms over NCCL (needs >= 2 visible GPUs; skipped otherwise).

Two processes, one per GPU: the distributed four-step FFT (contiguous and
column-block inputs, natural and transposed outputs) and the row-sharded fft2,
gathered and compared with NumPy's fp64 FFT of the whole input."""

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    from trnfft_b200 import ComplexTensor
    from trnfft_b200 import distributed as D

    n = 1 << 22
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(n) + 1j * rng.standard_normal(n)).astype(np.complex64)
    xr = torch.tensor(x.real, device="cuda")
    xi = torch.tensor(x.imag, device="cuda")
    lo, hi = D.shard_rows(n, world, rank)
    res = {}
    y = D.fft_distributed(ComplexTensor(xr[lo:hi], xi[lo:hi]), n)
    res["nat"] = (y.real.cpu().numpy(), y.imag.cpu().numpy())
    cr, ci = D.column_block(xr, xi, n, world, rank)
    y = D.fft_distributed(ComplexTensor(cr, ci), n, columns_in=True)
    res["cols"] = (y.real.cpu().numpy(), y.imag.cpu().numpy())
    y = D.fft_distributed(ComplexTensor(cr, ci), n, columns_in=True, exchange="nccl")
    res["cols_nccl"] = (y.real.cpu().numpy(), y.imag.cpu().numpy())
    y = D.fft_distributed(ComplexTensor(xr[lo:hi], xi[lo:hi]), n)  # second call reuses the mapped buffers
    res["nat2"] = (y.real.cpu().numpy(), y.imag.cpu().numpy())
    z = D.fft_distributed(ComplexTensor(xr[lo:hi], xi[lo:hi]), n, inverse=True)
    res["inv"] = (z.real.cpu().numpy(), z.imag.cpu().numpy())
    H, W = 2048, 4096
    f = (rng.standard_normal((H, W)) + 1j * rng.standard_normal((H, W))).astype(np.complex64)
    h0, h1 = D.shard_rows(H, world, rank)
    g = D.fft2_distributed(ComplexTensor(torch.tensor(f.real[h0:h1].copy(), device="cuda"),
                                         torch.tensor(f.imag[h0:h1].copy(), device="cuda")))
    res["fft2"] = (g.real.cpu().numpy(), g.imag.cpu().numpy())
    fl = ComplexTensor(torch.tensor(f.real[h0:h1].copy(), device="cuda"), torch.tensor(f.imag[h0:h1].copy(), device="cuda"))
    g = D.fft2_distributed(fl, natural_order=False)  # column block [H][W/P] (peer copies)
    res["fft2_cols"] = (g.real.cpu().numpy(), g.imag.cpu().numpy())
    g = D.fft2_distributed(fl, exchange="nccl")
    res["fft2_nccl"] = (g.real.cpu().numpy(), g.imag.cpu().numpy())
    g = D.fft2_distributed(fl, chunks=1)  # unchunked exchange
    res["fft2_ch"] = (g.real.cpu().numpy(), g.imag.cpu().numpy())
    g = D.fft2_distributed(fl)  # another peer call reuses the mapped planes
    res["fft2_2"] = (g.real.cpu().numpy(), g.imag.cpu().numpy())
    torch.cuda.synchronize()
    q.put((rank, res))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gpu_four_step_and_fft2():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=600) for _ in range(world))
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    n = 1 << 22
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(n) + 1j * rng.standard_normal(n)).astype(np.complex64).astype(np.complex128)
    ref = np.fft.fft(x)

    def cat(key):
        return np.concatenate([out[r][key][0] + 1j * out[r][key][1] for r in range(world)])

    def rel(a, b):
        return np.linalg.norm(a - b) / np.linalg.norm(b)

    assert rel(cat("nat"), ref) < 2e-6
    assert rel(cat("cols"), ref) < 2e-6
    assert rel(cat("cols_nccl"), ref) < 2e-6
    assert rel(cat("nat2"), ref) < 2e-6
    assert rel(cat("inv"), np.fft.ifft(x)) < 2e-6
    H, W = 2048, 4096
    f = (rng.standard_normal((H, W)) + 1j * rng.standard_normal((H, W))).astype(np.complex64).astype(np.complex128)
    F = np.fft.fft2(f)
    assert rel(cat("fft2"), F) < 2e-6
    assert rel(cat("fft2_nccl"), F) < 2e-6
    assert rel(cat("fft2_2"), F) < 2e-6
    assert rel(cat("fft2_ch"), F) < 2e-6
    cols = np.concatenate([out[r]["fft2_cols"][0] + 1j * out[r]["fft2_cols"][1] for r in range(world)], axis=1)
    assert rel(cols, F) < 2e-6
