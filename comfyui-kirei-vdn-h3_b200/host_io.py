"""Streaming host batches through the block with the PCIe copies hidden behind compute.

A diffusion sampler or a serving loop that keeps activations in host memory pays, per
block call, one host->device copy of x and one device->host copy of the output (270 MB
each at config 1, ~5 ms apiece over PCIe 5).  ``HostStreamer`` runs any device callable
``fn(x_dev) -> y_dev`` (the patched ``attn.forward``, a whole model step, ...) over a
sequence of pinned host inputs so that the copy of input i+1 (copy stream) and the copy
back of output i-1 (a second copy stream) overlap the compute of step i (the caller's
stream).  Two device input buffers alternate; events order every hand-over, and each
output tensor is kept alive (``record_stream``) until its copy back has finished.
The reference has no counterpart (its node runs one call at a time inside ComfyUI).
"""

from __future__ import annotations

import torch


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

    def run(self, inputs, outputs, *, prepare=None):
        """inputs[i] (pinned host) -> fn -> outputs[i] (pinned host), for every i.
        ``prepare(x_dev)``, if given, runs on the compute stream before ``fn`` (for example a
        collective that completes a row-split input).  Returns when every copy is queued;
        the caller synchronises (or records an event on ``self.d2h``)."""
        compute = torch.cuda.current_stream(self.device)
        n = len(inputs)
        # first input
        with torch.cuda.stream(self.h2d):
            self.x_dev[0].copy_(inputs[0], non_blocking=True)
            self._in_ready[0].record(self.h2d)
        for i in range(n):
            b = i & 1
            # queue the next input while this step computes (its buffer was freed by step i-1)
            if i + 1 < n:
                nb = b ^ 1
                with torch.cuda.stream(self.h2d):
                    if i >= 1:
                        self.h2d.wait_event(self._in_free[nb])
                    self.x_dev[nb].copy_(inputs[i + 1], non_blocking=True)
                    self._in_ready[nb].record(self.h2d)
            compute.wait_event(self._in_ready[b])
            x = self.x_dev[b]
            if prepare is not None:
                x = prepare(x)
            y = self.fn(x)
            self._in_free[b].record(compute)
            self._out_ready[b].record(compute)
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(self._out_ready[b])
                outputs[i].copy_(y, non_blocking=True)
            y.record_stream(self.d2h)
        return outputs


__all__ = ["HostStreamer"]
