"""Host-to-host streaming of layer calls with the PCIe copies overlapped.

A serving loop that keeps its activations on the host pays, per batch, an
upload of the input, the layer, and a download of the output.  Issued on one
stream these three run back to back; the upload and the download each take as
long as the layer at prefill sizes (8 MB each way per 1024 x 4096 bf16 batch).
``HostPipeline`` runs them on three streams with double-buffered device
tensors, so batch i+1's upload and batch i-1's download overlap batch i's
layer (the B200 has separate copy engines for each direction):

    upload stream    [x0 ->][x1 ->][x2 ->]
    compute stream          [f(x0)][f(x1)][f(x2)]
    download stream                [-> y0][-> y1][-> y2]

Ordering is carried by CUDA events only (no host synchronisation inside
``run``): an upload into device buffer b waits until the layer call that last
read buffer b is done; a layer call waits for its upload and for the download
that last read its output buffer; a download waits for its layer call.  The
compute stream is the caller's current stream, so collectives and kernels the
callable issues there keep their usual ordering, and an event the caller
records on it after ``run`` returns covers every copy ``run`` issued.
"""
from __future__ import annotations

from typing import Callable, Sequence

import torch


class HostPipeline:
    """Runs ``fn(x_dev, out=y_dev)`` over pinned host batches with overlapped copies.

    ``in_shape`` / ``out_shape`` are the per-batch device shapes; ``depth``
    device buffers of each are allocated once (2 is enough to overlap both
    copies with the layer).
    """

    def __init__(self, fn: Callable, in_shape, out_shape, dtype=torch.bfloat16, device=None, depth: int = 2):
        if depth < 2:
            raise ValueError("depth must be at least 2 to overlap the copies with the layer")
        self.fn = fn
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.depth = depth
        self.x_dev = [torch.empty(in_shape, dtype=dtype, device=self.device) for _ in range(depth)]
        self.y_dev = [torch.empty(out_shape, dtype=dtype, device=self.device) for _ in range(depth)]
        self.upload = torch.cuda.Stream(self.device)
        self.download = torch.cuda.Stream(self.device)
        self._computed = [torch.cuda.Event() for _ in range(depth)]
        self._uploaded = [torch.cuda.Event() for _ in range(depth)]
        self._downloaded = [torch.cuda.Event() for _ in range(depth)]
        self._used = [False] * depth

    def run(self, inputs: Sequence[torch.Tensor], outputs: Sequence[torch.Tensor]) -> None:
        """outputs[i] <- fn(inputs[i]) for every i; returns once all work is issued.

        Host tensors should be pinned (pageable memory makes the copies
        synchronous).  On return the caller's current stream is ordered after
        the last download, so ``torch.cuda.current_stream().synchronize()`` or
        an event recorded there waits for every result.
        """
        if len(inputs) != len(outputs):
            raise ValueError("inputs and outputs must have the same length")
        compute = torch.cuda.current_stream(self.device)
        # the buffers may still be in use by work the caller issued before
        self.upload.wait_stream(compute)
        for i, (xh, yh) in enumerate(zip(inputs, outputs)):
            b = i % self.depth
            with torch.cuda.stream(self.upload):
                if self._used[b]:
                    self.upload.wait_event(self._computed[b])  # the layer call that read x_dev[b]
                self.x_dev[b].copy_(xh, non_blocking=True)
                self._uploaded[b].record(self.upload)
            compute.wait_event(self._uploaded[b])
            if self._used[b]:
                compute.wait_event(self._downloaded[b])  # the download that read y_dev[b]
            self.fn(self.x_dev[b], out=self.y_dev[b])
            self._computed[b].record(compute)
            with torch.cuda.stream(self.download):
                self.download.wait_event(self._computed[b])
                yh.copy_(self.y_dev[b], non_blocking=True)
                self._downloaded[b].record(self.download)
            self._used[b] = True
        compute.wait_stream(self.download)
