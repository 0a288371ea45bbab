"""Host-to-device pipelining of batched transforms.

Batched transforms act on every row independently, so a batch that lives in
host memory can stream through the GPU in row chunks: while chunk c is being
transformed, chunk c+1 is copied in and chunk c-1 is copied out.  PCIe moves
data both ways at once, so with the copies of neighbouring chunks on
different CUDA streams the step costs less than the sum of upload, compute
and download.  Measured on the B200 hosts here (PCIe 5 x16): 55 GB/s up,
53 GB/s down, 79 GB/s both ways at once; a 64 MiB-each-way fft+ifft batch
streams in 1.94 ms with 4 chunks on 2 streams, against 1.70 ms for the bare
two-way copy and 2.6 ms with unpipelined copies.

``map_rows(fn, host_inputs)`` runs ``fn`` (a function of device tensors that
returns device tensors, such as ``lambda x: [trnfft.fft(x).real, ...]``) on
row chunks of the host tensors and returns host tensors.  It is ordered after
everything already queued on the current stream, and the current stream waits
for its completion, so CUDA events recorded on the current stream around the
call time the whole pipeline.
"""

from __future__ import annotations

import torch


def _chunks(rows: int, nchunks: int):
    base, extra = divmod(rows, nchunks)
    lo = 0
    for c in range(nchunks):
        hi = lo + base + (1 if c < extra else 0)
        if hi > lo:
            yield lo, hi
        lo = hi


_streams: dict = {}


def _side_streams(device: torch.device, n: int):
    key = (device.index, n)
    s = _streams.get(key)
    if s is None:
        s = _streams[key] = [torch.cuda.Stream(device=device) for _ in range(n)]
    return s


def map_rows(fn, host_inputs, nchunks: int = 4, nstreams: int = 2, device=None, host_outputs=None):
    """Apply `fn` to row chunks of host tensors with copies overlapped on `nstreams` streams.

    host_inputs: CPU tensors sharing their leading dimension (pinned memory makes the copies
    asynchronous; pageable inputs are pinned here first).  fn(list of device tensors) ->
    list of device tensors, each with the chunk's rows as leading dimension.  host_outputs:
    optional pinned CPU tensors to receive the results (allocated when None).  Returns the
    host outputs.
    """
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    host_inputs = [t if t.is_pinned() else t.pin_memory() for t in host_inputs]
    rows = host_inputs[0].shape[0]
    if any(t.shape[0] != rows for t in host_inputs):
        raise ValueError("map_rows: the inputs must share their leading dimension")
    parent = torch.cuda.current_stream(device)
    streams = _side_streams(device, nstreams)
    start = torch.cuda.Event()
    start.record(parent)
    outs = host_outputs
    for s in streams:
        s.wait_event(start)
    for c, (lo, hi) in enumerate(_chunks(rows, max(1, min(nchunks, rows)))):
        s = streams[c % nstreams]
        with torch.cuda.stream(s):
            dev_in = [t[lo:hi].to(device, non_blocking=True) for t in host_inputs]
            dev_out = fn(dev_in)
            if outs is None:
                outs = [torch.empty((rows,) + tuple(o.shape[1:]), dtype=o.dtype, pin_memory=True) for o in dev_out]
            for h, o in zip(outs, dev_out):
                h[lo:hi].copy_(o, non_blocking=True)
            # dev_in / dev_out were allocated on s: the caching allocator reuses their memory
            # only for later work on s, which is ordered after these copies
    for s in streams:
        parent.wait_stream(s)
    return outs
