"""Streaming host batches through the block with the PCIe copies hidden behind compute.

A diffusion sampler or a serving loop that keeps activations in host memory pays, per
block call, one host->device copy of x and one device->host copy of the output (270 MB
each at config 1, ~5 ms apiece over PCIe 5).  ``HostStreamer`` runs any device callable
``fn(x_dev) -> y_dev`` (the patched ``attn.forward``, a whole model step, ...) over a
sequence of pinned host inputs so that the copy of input i+1 (copy stream) and the copy
back of output i-1 (a second copy stream) overlap the compute of step i (the caller's
stream).  Two device input buffers alternate; events order every hand-over, and each
output tensor is kept alive (``record_stream``) until its copy back has finished.

With ``chunks`` > 1 the copies also overlap the first and last steps: each input is copied
in row blocks, ``fn(x_dev, io)`` receives a :class:`StreamIO` with one event per block (the
block forward projects a block of rows as soon as it lands) and hands every finished block
of its output back through ``io.out_ready``, whose copy starts at once.  Without that, the
first input copy and the last output copy (≈ 10 ms at config 1) sit outside any compute.
The reference has no counterpart (its node runs one call at a time inside ComfyUI).
"""

from __future__ import annotations

import torch

from .hybrid import StreamIO

ROW_ALIGN = 128  # row blocks start on GEMM tile boundaries


def row_blocks(rows: int, chunks: int) -> list[tuple[int, int]]:
    """``chunks`` consecutive row blocks covering [0, rows), boundaries on multiples of 128."""
    chunks = max(1, int(chunks))
    ends = []
    for k in range(1, chunks + 1):
        e = -(-rows * k // chunks)
        e = min(rows, -(-e // ROW_ALIGN) * ROW_ALIGN)
        if not ends or e > ends[-1]:
            ends.append(e)
    ends[-1] = rows
    out, r0 = [], 0
    for e in ends:
        if e > r0:
            out.append((r0, e))
            r0 = e
    return out


class HostStreamer:
    def __init__(self, fn, device, in_shape, in_dtype=torch.bfloat16):
        self.fn = fn
        self.device = torch.device(device)
        self.h2d = torch.cuda.Stream(self.device)
        self.d2h = torch.cuda.Stream(self.device)
        self.x_dev = [torch.empty(in_shape, device=self.device, dtype=in_dtype) for _ in range(2)]
        self._in_ready = [torch.cuda.Event() for _ in range(2)]
        self._in_free = [torch.cuda.Event() for _ in range(2)]
        self._out_ready = [torch.cuda.Event() for _ in range(2)]

    def run(self, inputs, outputs, *, prepare=None, chunks: int = 1):
        """inputs[i] (pinned host) -> fn -> outputs[i] (pinned host), for every i.
        ``prepare(x_dev)``, if given, runs on the compute stream before ``fn`` (for example a
        collective that completes a row-split input; it needs the whole input, so the copies
        then go in one block).  ``chunks`` > 1: row-block copies and ``fn(x_dev, io)`` (see
        the module docstring).  Returns when every copy is queued; the caller synchronises
        (or records an event on ``self.d2h``)."""
        compute = torch.cuda.current_stream(self.device)
        n = len(inputs)
        rows = self.x_dev[0].shape[0]
        blocks = row_blocks(rows, chunks if prepare is None else 1)
        by_blocks = len(blocks) > 1
        block_events = [[torch.cuda.Event() for _ in blocks] for _ in range(2)]

        def copy_in(i, b):
            with torch.cuda.stream(self.h2d):
                if i >= 2:
                    self.h2d.wait_event(self._in_free[b])  # step i-2 is done with this buffer
                for (r0, r1), ev in zip(blocks, block_events[b]):
                    self.x_dev[b][r0:r1].copy_(inputs[i][r0:r1], non_blocking=True)
                    ev.record(self.h2d)
                self._in_ready[b].record(self.h2d)

        copy_in(0, 0)
        for i in range(n):
            b = i & 1
            if i + 1 < n:
                copy_in(i + 1, b ^ 1)  # overlaps this step's compute
            x = self.x_dev[b]
            sent = []

            def out_ready(y, r0, nrows, i=i, sent=sent):
                ev = torch.cuda.Event()
                ev.record(compute)
                with torch.cuda.stream(self.d2h):
                    self.d2h.wait_event(ev)
                    outputs[i][r0:r0 + nrows].copy_(y[r0:r0 + nrows], non_blocking=True)
                sent.append((r0, nrows))

            if by_blocks:
                io = StreamIO([(r1, ev) for (_, r1), ev in zip(blocks, block_events[b])], out_ready)
                y = self.fn(x, io)
                if not io.complete:
                    raise RuntimeError("HostStreamer: fn(x, io) must wait for every input block it reads")
            else:
                compute.wait_event(self._in_ready[b])
                if prepare is not None:
                    x = prepare(x)
                y = self.fn(x)
            self._in_free[b].record(compute)
            self._out_ready[b].record(compute)
            if sum(r for _, r in sent) < y.shape[0]:
                # fn gave no (or only part of its) output back by blocks: copy it whole
                with torch.cuda.stream(self.d2h):
                    self.d2h.wait_event(self._out_ready[b])
                    outputs[i].copy_(y, non_blocking=True)
            y.record_stream(self.d2h)
        return outputs


__all__ = ["HostStreamer", "row_blocks"]
