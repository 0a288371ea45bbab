"""Host-side logic of the multi-GPU transforms with two CPU (gloo) ranks.

The exchanges of trnfft_b200.distributed are device-agnostic; here they run on
CPU tensors with torch.fft standing in for the CUDA transforms (checker only),
and the gathered result is compared with NumPy's FFT of the whole input."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _col(re, im, inverse):
    z = torch.complex(re, im)
    z = torch.fft.ifft(z, dim=0) if inverse else torch.fft.fft(z, dim=0)
    return z.real.contiguous(), z.imag.contiguous()


def _row(re, im, inverse):
    z = torch.complex(re, im)
    z = torch.fft.ifft(z, dim=-1) if inverse else torch.fft.fft(z, dim=-1)
    return z.real.contiguous(), z.imag.contiguous()


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from trnfft_b200 import distributed as D

    res = {}
    n = 1 << 12
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(n) + 1j * rng.standard_normal(n)).astype(np.complex64)
    lo, hi = D.shard_rows(n, world, rank)
    xr = torch.tensor(x.real[lo:hi].copy())
    xi = torch.tensor(x.imag[lo:hi].copy())
    for inv in (False, True):
        for nat in (True, False):
            zr, zi = D._four_step(xr, xi, n, None, inv, nat, _col, _row)
            res[("1d", inv, nat)] = (zr.numpy(), zi.numpy())
    cr, ci = D.column_block(torch.tensor(x.real.copy()), torch.tensor(x.imag.copy()), n, world, rank)
    zr, zi = D._four_step(cr, ci, n, None, False, True, _col, _row, columns_in=True)
    res["cols"] = (zr.numpy(), zi.numpy())
    H, W = 16, 32
    f = (rng.standard_normal((H, W)) + 1j * rng.standard_normal((H, W))).astype(np.complex64)
    hr = H // world
    fr = torch.tensor(f.real[rank * hr:(rank + 1) * hr].copy())
    fi = torch.tensor(f.imag[rank * hr:(rank + 1) * hr].copy())
    zr, zi = D._fft2_exchange(fr, fi, None, False, True, _row, _col)
    res["2d"] = (zr.numpy(), zi.numpy())
    q.put((rank, res))
    dist.barrier()
    dist.destroy_process_group()


def test_four_step_and_fft2_exchanges_two_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=240) for _ in range(world))
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    n = 1 << 12
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(n) + 1j * rng.standard_normal(n)).astype(np.complex64).astype(np.complex128)
    N1, N2 = 64, 64
    for inv in (False, True):
        ref = np.fft.ifft(x) if inv else np.fft.fft(x)
        nat = np.concatenate([out[r][("1d", inv, True)][0] + 1j * out[r][("1d", inv, True)][1] for r in range(world)])
        assert np.linalg.norm(nat - ref) / np.linalg.norm(ref) < 1e-5
        # transposed layout: rank p holds X[k1 + N1*k2] for k1 in block p, stored [k1 local][k2]
        tr = np.concatenate([out[r][("1d", inv, False)][0] + 1j * out[r][("1d", inv, False)][1] for r in range(world)])
        k1, k2 = np.meshgrid(np.arange(N1), np.arange(N2), indexing="ij")
        assert np.linalg.norm(tr.reshape(N1, N2) - ref[k1 + N1 * k2]) / np.linalg.norm(ref) < 1e-5
    cols = np.concatenate([out[r]["cols"][0] + 1j * out[r]["cols"][1] for r in range(world)])
    ref = np.fft.fft(x)
    assert np.linalg.norm(cols - ref) / np.linalg.norm(ref) < 1e-5
    H, W = 16, 32
    f = (rng.standard_normal((H, W)) + 1j * rng.standard_normal((H, W))).astype(np.complex64).astype(np.complex128)
    got = np.concatenate([out[r]["2d"][0] + 1j * out[r]["2d"][1] for r in range(world)])
    ref2 = np.fft.fft2(f)
    assert np.linalg.norm(got - ref2) / np.linalg.norm(ref2) < 1e-5


def test_shard_rows_cover_everything():
    from trnfft_b200.distributed import shard_rows

    for total in (7, 8, 1000, 8192):
        for world in (1, 2, 3, 8):
            spans = [shard_rows(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


def test_split_n():
    """Rows of at most 16384 points (one row-kernel pass); the columns take the rest."""
    from trnfft_b200.distributed import _split_n

    assert _split_n(1 << 30) == (1 << 16, 1 << 14)
    assert _split_n(1 << 28) == (1 << 14, 1 << 14)
    assert _split_n(4096) == (64, 64)
    assert _split_n(1 << 13) == (64, 128)
    for lg in range(2, 33):
        n1, n2 = _split_n(1 << lg)
        assert n1 * n2 == 1 << lg
        assert n2 <= 1 << 14
        assert n2 >= n1 or n2 == 1 << 14
