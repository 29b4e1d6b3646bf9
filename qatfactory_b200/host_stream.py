"""Fake quantization of host-resident tensors, streamed through the GPU in row chunks.

The FP4 quantizers are row-separable (every scale block lies inside one row; NVFP4 needs its
tensor amax given up front), so a pinned host tensor can be processed chunk by chunk: the
host-to-device copy of chunk i+1, the kernels of chunk i and the device-to-host copy of
chunk i-1 run on three CUDA streams at once, which overlaps both PCIe directions with each
other and with the compute.  The results are bit-identical to one call on the whole tensor.
"""

from __future__ import annotations

from typing import Callable, Sequence

import torch

Job = tuple[Callable[[torch.Tensor], torch.Tensor], torch.Tensor, torch.Tensor]


def stream_jobs(jobs: Sequence[Job], device: torch.device | None = None, chunk_rows: int = 2048,
                buffers: int = 4) -> None:
    """For every job ``(fn, x_host, out_host)``: ``out_host[r] = fn(x_host[r].cuda())`` for each
    row chunk r, with all jobs' chunks in one pipeline (no drain between tensors).

    ``x_host`` and ``out_host`` are 2-D host tensors (pinned for asynchronous copies) with the
    same number of rows; ``fn`` maps a device chunk to a device chunk of ``out_host``'s row
    shape and must be row-separable.  Asynchronous: returns once everything is enqueued, and
    the caller's current stream waits for the last copy."""

    for _, x_host, out_host in jobs:
        if x_host.ndim != 2 or out_host.ndim != 2 or x_host.shape[0] != out_host.shape[0]:
            raise ValueError("stream_rows expects 2-D host tensors with the same number of rows")
        if x_host.is_cuda or out_host.is_cuda:
            raise ValueError("stream_rows streams host tensors; call the quantizer directly on device tensors")
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    main = torch.cuda.current_stream(device)
    h2d = torch.cuda.Stream(device)
    d2h = torch.cuda.Stream(device)
    n_buf = max(2, buffers)
    staging: dict[tuple, list[torch.Tensor]] = {}
    loaded = [torch.cuda.Event() for _ in range(n_buf)]
    consumed = [torch.cuda.Event() for _ in range(n_buf)]
    h2d.wait_stream(main)
    d2h.wait_stream(main)
    i = 0
    for fn, x_host, out_host in jobs:
        rows, cols = x_host.shape
        key = (cols, x_host.dtype)
        if key not in staging:
            staging[key] = [torch.empty((chunk_rows, cols), dtype=x_host.dtype, device=device) for _ in range(n_buf)]
        for r0 in range(0, rows, chunk_rows):
            r1 = min(rows, r0 + chunk_rows)
            b = i % n_buf
            buf = staging[key][b][: r1 - r0]
            with torch.cuda.stream(h2d):
                if i >= n_buf:
                    h2d.wait_event(consumed[b])  # the kernels of chunk i - n_buf are done with slot b
                buf.copy_(x_host[r0:r1], non_blocking=True)
                loaded[b].record(h2d)
            main.wait_event(loaded[b])
            y = fn(buf)
            done = torch.cuda.Event()
            done.record(main)
            with torch.cuda.stream(d2h):
                d2h.wait_event(done)
                out_host[r0:r1].copy_(y, non_blocking=True)
                # slot b is free once the kernels AND the copy of their result are done: fn may
                # return a view of its input chunk (an identity or in-place quantizer)
                consumed[b].record(d2h)
            y.record_stream(d2h)
            i += 1
    for bufs in staging.values():
        for t in bufs:
            t.record_stream(h2d)
    main.wait_stream(d2h)


def stream_rows(fn: Callable[[torch.Tensor], torch.Tensor], x_host: torch.Tensor, out_host: torch.Tensor,
                device: torch.device | None = None, chunk_rows: int = 2048, buffers: int = 4) -> torch.Tensor:
    """``stream_jobs`` for one tensor; returns ``out_host``."""

    stream_jobs([(fn, x_host, out_host)], device, chunk_rows, buffers)
    return out_host
